/*
 * cxm.h — C ABI of the B200-native Cosxamix decode path.
 *
 * The library (cosxamix_b200/libcxm.so) replaces, behind plain pointers and
 * sizes, the body of the reference's per-token forward and sampler. Citations
 * name the reference interface each entry point replaces (paths inside the
 * Cosxamix project).
 *
 * Conventions
 *   - Every `int` result is 0 on success and negative on error; the message is
 *     in cxm_last_error() (thread-local). This mirrors Result<_, String> ->
 *     ErrorMotor::Interno (src/engine.rs:108-122, src/engine_own.rs:183).
 *   - A model handle owns one CUDA stream and its scratch buffers. It is not
 *     re-entrant: callers serialize, exactly as MotorPropio does with its
 *     Mutex (src/engine_own.rs:62, :185).
 *   - There is no CPU fallback: without a usable sm_100a device the open
 *     calls fail.
 */
#ifndef CXM_H
#define CXM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cxm_model cxm_model;
typedef struct cxm_cache cxm_cache;
typedef struct cxm_sampler cxm_sampler;

/* Mirrors forward::Config (src/forward.rs:36-55) plus the FFN width. */
typedef struct {
    int32_t n_layer, dim, n_head, n_head_kv, head_dim, vocab, ctx, ffn;
    float eps, rope_base;
    int32_t tied;      /* output projection shares token_embd (src/forward.rs:219-227) */
    int32_t has_eos;   /* tokenizer.ggml.eos_token_id present (src/forward.rs:514-518) */
    uint32_t eos;
} cxm_config;

/* ── model ─────────────────────────────────────────────────────────────── */

/* Modelo::abrir (src/forward.rs:187-266): parse the GGUF, upload every tensor
 * to HBM once (k-quant blocks regrouped, bytes unchanged, into the decode
 * kernel's tiles of R rows x L super-blocks, R*L = 32, L chosen per matrix)
 * and build the RoPE tables (src/ops.rs:1108-1129). */
int  cxm_model_open(const char *gguf_path, int device, cxm_model **out);
int  cxm_model_config(const cxm_model *m, cxm_config *out);
/* bytes of weights resident on the device (the per-token weight stream) */
uint64_t cxm_model_weight_bytes(const cxm_model *m);
/* The prompt forward of a call of 24 tokens or more (the reference's
 * matmul_i8_bloques threshold, src/ops.rs:1013, :1073-1079) runs, by default
 * (tensor_cores = 1), as batched int8 tensor-core GEMMs with the buffered
 * path's float order; 0 replays those tokens through the decode step one by
 * one. Both give the same logits and KV rows bit for bit; the switch is for
 * comparing them, as the reference's COSXAMIX_SIN_BLOQUES compares its paths.
 * Tensor-parallel models always replay. */
int cxm_model_set_prefill(cxm_model *m, int tensor_cores);
/* Caches belong to their model: use a cache only while its model is open
 * (freeing it afterwards is allowed). */
void cxm_model_close(cxm_model *m);

/* ── tensor parallelism (one process per GPU; no counterpart in the
 * reference, whose engine runs one model on one machine) ──────────────── */

/* Rank `tp_rank` of `tp_size` (1..8): this process's GPU holds the attention
 * block whole (q/k/v of every head, the whole KV cache, o_proj), the gate/up
 * rows of its FFN slice [r*F/N, (r+1)*F/N) and the ffn_down rows of its
 * hidden slice [r*D/N, (r+1)*D/N) (each row over its whole input), its share
 * of the output rows, and the embedding and norms. Every decode step gathers
 * the FFN's hidden vector and the residual stream from the ranks' slices and
 * picks the argmax over their vocabulary slices, over peer memory inside the
 * decode kernel; each value is computed by one rank exactly as one GPU
 * computes it, so logits and tokens are those of the single-GPU model. Each
 * wait is bounded (a lost rank ends the step with an error, never a hang).
 * Greedy decode only. cxm_model_config reports the whole model. The model
 * runs after cxm_tp_connect. Hidden size and FFN width must split over the
 * ranks in multiples of 4. */
int cxm_model_open_tp(const char *gguf_path, int device, int tp_rank, int tp_size, cxm_model **out);
#define CXM_TP_HANDLE_BYTES 64
/* The CUDA IPC handle of this rank's exchange area (CXM_TP_HANDLE_BYTES). */
int cxm_tp_handle(cxm_model *m, uint8_t *handle_out);
/* Map every rank's exchange area: `handles` holds tp_size handles in rank
 * order (this rank's own included), as cxm_tp_handle returned them. */
int cxm_tp_connect(cxm_model *m, const uint8_t *handles);
/* this rank, the number of ranks, and this rank's vocabulary rows
 * [vocab_lo, vocab_lo + vocab_n): the logits cxm_forward returns when
 * tp_size > 1 (vocab_n floats) */
int cxm_model_tp_info(const cxm_model *m, int *tp_rank, int *tp_size, int *vocab_lo, int *vocab_n);

/* ── KV cache (src/forward.rs:62-137) ─────────────────────────────────── */

/* Cache::nuevo: f32 K and V per layer, [max_tokens x n_head_kv*head_dim],
 * the reference's own layout (src/forward.rs:62-66). */
int      cxm_cache_new(cxm_model *m, uint32_t max_tokens, cxm_cache **out);
void     cxm_cache_free(cxm_cache *c);
uint32_t cxm_cache_len(const cxm_cache *c);                          /* Cache::largo   :77 */
int      cxm_cache_truncate(cxm_cache *c, uint32_t n);               /* Cache::truncar :98-108 */
int      cxm_cache_clear(cxm_cache *c);                              /* Cache::limpiar :81-87 */
/* Cache::prefijo (:115-127): dst becomes a copy of the first n tokens of src
 * (device-to-device; dst must belong to the same model). */
int      cxm_cache_copy_prefix(const cxm_cache *src, uint32_t n, cxm_cache *dst);
/* The shared-prefix form of the session reuse in src/engine_own.rs:198-245
 * (which borrows a cached session's prefix by Cache::prefijo, a copy): dst
 * reads the first n (<= src len) positions from src's K/V, held once, and
 * continues with its own from position n. The lender counts its borrowers:
 * while lent it cannot be truncated or cleared below the lent positions, and
 * freeing it is deferred until its last borrower is freed or lets go (by
 * cxm_cache_clear, cxm_cache_copy_prefix or another share). A borrower lends
 * at most the positions it borrows (they come from its lender). Results are
 * those of a dst holding a copy. */
int      cxm_cache_share_prefix(cxm_cache *src, uint32_t n, cxm_cache *dst);
/* Copy layer `layer`'s K (is_v = 0) or V (is_v = 1) rows [0, len) to host:
 * len * n_head_kv * head_dim floats. Test/inspection access. */
int      cxm_cache_read(const cxm_cache *c, uint32_t layer, int is_v, float *host_out);

/* ── forward and generation ────────────────────────────────────────────── */

/* Modelo::forward (src/forward.rs:375-505): extend `c` with `n` tokens and
 * return the logits of the LAST one (vocab floats) into host memory
 * (`logits_out` may be NULL). */
int cxm_forward(cxm_model *m, cxm_cache *c, const uint32_t *tokens, uint32_t n, float *logits_out);

/* Muestreador::nuevo (src/sampler.rs:40-48): temperature <= 0 is greedy. */
int  cxm_sampler_new(uint64_t seed, float temperature, float top_p, cxm_sampler **out);
void cxm_sampler_free(cxm_sampler *s);
uint64_t cxm_sampler_state(const cxm_sampler *s);

/* Muestreador::elegir (src/sampler.rs:61-126) on the logits of the model's
 * last forward. Greedy (first maximum) reads the pick cxm_forward already
 * brought back with its error word (one host synchronisation per forward
 * and pick); with
 * temperature > 0, the reference's top-p draw with its sums in its order and
 * equal probabilities ordered by index (the reference's unstable sort leaves
 * their order unspecified). Advances the sampler's state like the reference. */
int cxm_sample(cxm_model *m, cxm_sampler *s, uint32_t *token_out);

/* Modelo::generar (src/forward.rs:533-559): forward the prompt, then
 * sample -> forward one token, up to max_new tokens, stopping at the model's
 * eos and before the context overflows. The per-token step is one launch of
 * a persistent kernel, replayed as a CUDA graph; position and token live in
 * device memory. The eos pick sets a device flag: the steps queued after it
 * return at once, and neither pick nor forward another token. */
int cxm_generate(cxm_model *m, cxm_cache *c, const uint32_t *prompt, uint32_t n_prompt, uint32_t max_new,
                 cxm_sampler *s, uint32_t *out, uint32_t *n_out);

/* Greedy Modelo::generar for n conversations at once (n <= 512), each on its
 * own cache (which may borrow a shared prefix): every prompt is forwarded as
 * its own forward call; then each step takes every conversation's next token
 * through the tensor-core GEMMs together (one read of the weights for all),
 * each row in the order of a forward call of one row, so every conversation
 * gets the tokens cxm_generate gives it alone. out: [n][max_new] tokens,
 * n_out[z] of them valid (a conversation stops at the model's eos). Every
 * cache needs room for len + prompt + max_new positions; a cache lent as a
 * prefix cannot take part. Single-GPU models. */
int cxm_generate_batch(cxm_model *m, cxm_cache *const *caches, const uint32_t *const *prompts,
                       const uint32_t *n_prompt, uint32_t n, uint32_t max_new, uint32_t *out, uint32_t *n_out);

const char *cxm_last_error(void);

/* ── kernel-level entry points (parity checks) ─────────────────────────── */

/* The reference's per-row fused-kernel ABI (src/kernels/c.rs:18-30,
 * src/kernels/q2k.rs:153: float f(blocks, xq, xe, xs, n_superblocks)) lifted
 * to the device: the integer sub-block sums of one GGUF row against an i8
 * activation, one int32 per sub-block (16 or 32 values). Host pointers. */
int cxm_debug_subblock_sums(int ggml_type, const uint8_t *row, const int8_t *xq, uint32_t n_superblocks,
                            int32_t *out);

/* ops::matmul_auto with one activation row (src/ops.rs:1056-1093):
 * y[rows] = W[rows x k] · x[k], W raw GGUF k-quant bytes. Host pointers. */
int cxm_debug_matvec(int ggml_type, const uint8_t *w, uint32_t rows, uint32_t k, const float *x, float *y);

/* ops::matmul_auto with m activation rows (src/ops.rs:1056-1093) on the
 * reference's portable backend: y[m x rows] = x[m x k] · W[rows x k]^T, each
 * output in the float order the reference's path for m rows gives it (the
 * fused kernel, or matmul_i8_directo's scaled dot and offset terms, which
 * matmul_i8_bloques also takes without AVX2). Host pointers. */
int cxm_debug_matmul(int ggml_type, const uint8_t *w, uint32_t rows, uint32_t k, const float *x, uint32_t m,
                     float *y);

/* ops::atencion for one new token (src/ops.rs:1258-1325) on the device's
 * split-K flash-decode kernel: q[heads*hd], k/v[total x heads_kv*hd]. Host
 * pointers; allocates its device buffers per call. */
int cxm_debug_attention(const float *q, const float *k, const float *v, uint32_t total, uint32_t heads,
                        uint32_t heads_kv, uint32_t head_dim, float *out);

/* No counterpart in the reference (its attention, src/ops.rs:1258-1325, runs
 * on host memory): cxm_debug_attention's kernels on caller-owned DEVICE
 * buffers, allocating nothing — no cudaMalloc, cudaFree or allocating library
 * routine. For callers that cannot allocate device memory: a serving process
 * that has already given the whole device to weights and KV caches, where a
 * cudaMalloc fails, and latency-sensitive callers that cannot take the
 * device-wide synchronisation cudaMalloc/cudaFree may imply.
 *   Limit: heads * round_up(total, 4) <= 65536 scores (a static 256 KiB device
 *   array); a larger call fails with an error and launches nothing.
 *   The scratch array is shared by every call on a device: calls whose GPU
 *   work overlaps (two host threads, or two streams) race on it.
 *   The first call on each device looks up the array's address and sets the
 *   kernels' shared-memory limits (with that device current); make that first
 *   call before any stream capture. The address is kept for the life of the
 *   process: after a cudaDeviceReset of that device (which ends the process's
 *   context there) it is stale, so this entry point must not be called on
 *   that device again in the same process.
 *   Work is enqueued on `stream` (a cudaStream_t; NULL = the default stream),
 *   which is synchronised before the call returns so the kernels' error word
 *   can be reported. */
int cxm_attention_noalloc(const float *q, const float *k, const float *v, uint32_t total, uint32_t heads,
                          uint32_t heads_kv, uint32_t head_dim, float *out, void *stream);

/* f32::exp as every exponential of the path computes it on the device
 * (softmax, SiLU): the same rounding as the host C library's expf, which the
 * reference's f32::exp calls (src/ops.rs:1221, src/kernels/scalar.rs:65). */
int cxm_debug_expf(const float *x, float *y, uint64_t n);

/* y[i] = x[0] + ... + x[i] as the reference's sequential f32 loops add them
 * (`total += *v`, src/ops.rs:1222; `acumulada += ...`, src/sampler.rs:110,
 * :144), each running sum rounded in turn: the device sampler's summation.
 * The total is also taken a second time without the running sums (the
 * summation's other path); the call fails if the two differ. */
int cxm_debug_seq_sums(const float *x, float *y, uint64_t n);

/* ── measurement hooks (no counterpart in the reference: timing only) ──── */

/* Replay the greedy decode step `steps` times for the token at the cache's
 * current end, timing on the device (CUDA events on the model's stream).
 * Inputs stay resident; the cache grows by `steps`. */
int cxm_bench_decode(cxm_model *m, cxm_cache *c, uint32_t steps, float *ms_total);

/* The same with the sampled step (decode kernel, then the device sampler,
 * Muestreador::elegir) for a sampler with temperature > 0; the sampler's
 * state advances one draw per step. NULL or temperature 0: greedy. */
int cxm_bench_decode_sampled(cxm_model *m, cxm_cache *c, cxm_sampler *s, uint32_t steps, float *ms_total);

/* The device sampler alone, `reps` times on the logits of the model's last
 * step (a forward first), device-timed. With phase_ns (nphase <= 78
 * entries), the last run's step ends on CTA 0 in ns from its start: the
 * max, the exponentials, the total, the keys, the four radix passes, the
 * gather, the cumulative sums, the end (0 where a run skips a step); then
 * the passes of its two sums; then the start of each of the total's first
 * 64 passes. */
int cxm_bench_sample(cxm_model *m, cxm_sampler *s, uint32_t reps, float *ms_total, uint64_t *phase_ns,
                     uint32_t nphase);

/* Arm the prompt GEMM's step stamps: the launch-th k_pf_gemm launch from
 * now (0-based; < 0 disarms) records on its CTA (0, 0) the %globaltimer of
 * its roles' steps. cxm_read_gemm_stamps then synchronizes the device and
 * gives n <= 100 of them in ns from the CTA's start (0: not reached): [16+b]
 * block b's MMA inputs in, [32+b] a producer's copies in, [48+b] its operands
 * out, [64+b] epilogue warp 0's accumulators in, [80+b] out (b < 16); [96]
 * offset chains done, [97] end, [98] past the CTA barrier before the chains,
 * [99] the chains' first 8 sub-blocks. */
int cxm_arm_gemm_stamps(int launch);
int cxm_read_gemm_stamps(uint64_t *out, uint32_t n);

/* Average device time of one gate|up matvec phase (the largest of a layer)
 * of the decode kernel: `reps` such phases, cycling over the layers so every
 * phase streams its own weights from HBM, run in one launch behind grid
 * barriers as in the step. `bytes_per_launch` = GGUF bytes of gate + up. */
int cxm_bench_matvec(cxm_model *m, uint32_t reps, float *ms_per_launch, uint64_t *bytes_per_launch);

/* Number of kernel launches (of this library's kernels) in one decode step. */
int cxm_step_launches(const cxm_model *m);

/* ── synthetic models (src/daiss.rs:422-586 + src/quant_kquants.rs) ────── */

/* Tensor-type recipes for the synthetic GGUF writer. */
enum {
    CXM_MIX_UNIFORM = 0,  /* every 2-D tensor in `type` */
    CXM_MIX_Q4_K_M = 1    /* Q6_K for the output projection (or tied token_embd) and
                             for attn_v / ffn_down of even layers; Q4_K elsewhere */
};

typedef struct {
    int32_t vocab, dim, n_layer, n_head, n_head_kv, ffn, ctx;
    float eps, rope_base;
    int32_t tied;       /* omit output.weight */
    int32_t mix;        /* CXM_MIX_* */
    int32_t type;       /* GGML type for CXM_MIX_UNIFORM */
    uint64_t seed;
    float sigma;        /* N(0, sigma) for every matrix */
    int32_t threads;    /* 0 = all host threads */
    int32_t has_eos;    /* write tokenizer.ggml.eos_token_id = eos (0: no eos key, generation never stops early) */
    uint32_t eos;
} cxm_synth_spec;

/* Write a seeded random-init qwen2-keyed GGUF: row r of tensor `name` draws
 * from Azar(semilla_de(seed, name, r)) (src/daiss.rs:364-379), Box-Muller
 * pairs, then the k-quant writer of its type. Norms are 1, biases 0. */
int cxm_synth_write(const cxm_synth_spec *spec, const char *path);

/* Quantize n floats (multiple of 256) to `ggml_type` with the library's
 * k-quant writers (Q2_K/Q3_K/Q4_K/Q5_K after src/quant_kquants.rs, Q6_K our
 * own); returns the number of bytes written, or <0. */
int64_t cxm_quantize(int ggml_type, const float *x, uint64_t n, uint8_t *out, uint64_t out_cap);

#ifdef __cplusplus
}
#endif
#endif
