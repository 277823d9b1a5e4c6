/*
 * cxm_oracle.h — CPU restatement of Cosxamix's decode path, used ONLY as a
 * checker (tests, smoke check, and the CPU-baseline leg of bench.py).
 *
 * TEST INFRASTRUCTURE. Nothing in the product library links or calls this.
 *
 * Every function restates the reference's scalar Rust specification; the
 * citation (file:line, paths inside the Cosxamix project) is given beside it.
 * The restatement follows the *scalar* kernels (src/kernels/scalar.rs), not the
 * AVX2 ones: those differ only in float summation order, never in the integer
 * sub-block sums.
 */
#ifndef CXM_ORACLE_H
#define CXM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type numbers, src/gguf.rs:39-54 */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6, ORC_Q5_1 = 7,
    ORC_Q8_0 = 8, ORC_Q8_1 = 9, ORC_Q2K = 10, ORC_Q3K = 11, ORC_Q4K = 12, ORC_Q5K = 13,
    ORC_Q6K = 14, ORC_Q8K = 15
};

int    orc_values_per_block(int type);          /* src/gguf.rs:83-90 */
int    orc_bytes_per_block(int type);           /* src/gguf.rs:93-111 */
int    orc_sub_block(int type);                 /* src/quant.rs:213-219; 0 = none */

float    orc_f16_to_f32(uint16_t h);            /* src/quant.rs:38-60 */
uint16_t orc_f32_to_f16(float x);               /* src/quant.rs:691-731 */

/* dequantize `n` values (multiple of the block) of `type` -> out. 0 ok, <0 err.
 * src/quant.rs:124-162 and the per-format readers :472-679 */
int orc_dequantize(int type, const uint8_t *blocks, size_t nbytes, size_t n, float *out);

/* unpack to i8 with a scale and an offset per sub-block. Returns sub size or <0.
 * src/quant.rs:238-468 */
int orc_unpack_i8(int type, const uint8_t *blocks, size_t nbytes, size_t n,
                  int8_t *q, float *scales, float *offsets);

/* per-sub-block activation quantization, src/ops.rs:178-198 (+ sums :862-879) */
void orc_quantize_i8(const float *x, size_t n, int sub, int8_t *q, float *scales, float *sums);

int32_t orc_dot_i8(const int8_t *a, const int8_t *b, size_t n);                    /* scalar.rs:80-83 */
float   orc_dot_i8_scaled(const int8_t *a, const int8_t *b, const float *ea,
                          const float *eb, size_t n, int block);                   /* scalar.rs:95-109 */
float   orc_dot_f32(const float *a, const float *b, size_t n);                     /* scalar.rs:16-23 */

/* fused k-quant row · i8 activation; nblk = 256-value super-blocks */
float orc_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* scalar.rs:132-170 */
float orc_dot_q5k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* scalar.rs:179-217 */
float orc_dot_q3k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* scalar.rs:236-275 */
float orc_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* scalar.rs:294-324 */
float orc_dot_q2k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* kernels/q2k.rs:41-69 */
float orc_dot_row(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk);

/* the integer part of the fused dots: one int32 per sub-block, exactly the
 * `entero` each scalar kernel forms before scaling (values shifted to be
 * unsigned as the reference does: Q3_K +4, Q6_K +0..63). */
int orc_subblock_sums(int type, const uint8_t *row, const int8_t *xq, size_t nblk, int32_t *out);

void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps); /* scalar.rs:36-54 */
void orc_silu(float *out, const float *in, size_t n);                               /* scalar.rs:63-67 */
void orc_rope_tables(int head_dim, float base, int ctx, float *cos_t, float *sin_t); /* ops.rs:1108-1129 */
int  orc_rope(float *x, int tokens, int heads, int head_dim, const float *cos_t,
              const float *sin_t, int ctx, int pos);                                /* ops.rs:1150-1193 */
int  orc_softmax(float *x, size_t n, size_t width);                                /* ops.rs:1206-1230 */
int  orc_attention(const float *q, const float *k, const float *v, int tokens, int total,
                   int heads, int heads_kv, int head_dim, float *out);             /* ops.rs:1258-1325 */

/* ops::matmul_auto (ops.rs:1056-1093): dst[m,n] = lhs[m,k] · W[n,k]^T by
 * the path the reference takes for (m, k, type) on this oracle's backend. */
int orc_matmul_auto(int m, int k, int n, const float *lhs, const uint8_t *w, size_t wbytes,
                    int type, float *dst);
/* The path matmul_auto takes: F32 (ops::matmul, :88-156, unquantized
 * formats), FUSED (matmul_i8_fusionado, :435-522: the per-row fused kernels),
 * BUFFERED (matmul_i8_directo, :310-414: the row unpacked to i8, then
 * dot_i8_escalado and the offset term), BLOCKED (matmul_i8_bloques,
 * :607-829: the AVX2 tile kernel; without AVX2 it is BUFFERED, :599-606).
 * m >= ORC_BLOCKED_FROM (BLOQUES_DESDE, :1013) is BLOCKED/BUFFERED;
 * otherwise FUSED when hay_fusionado (:837-858) and (Q4_K or m <= 4). */
enum { ORC_PATH_F32 = 0, ORC_PATH_FUSED = 1, ORC_PATH_BUFFERED = 2, ORC_PATH_BLOCKED = 3 };
enum { ORC_BLOCKED_FROM = 24 };
int orc_matmul_path(int m, int k, int type);
/* one path forced (the reference's tests call each path directly) */
int orc_matmul_by_path(int path, int m, int k, int n, const float *lhs, const uint8_t *w, size_t wbytes, int type,
                       float *dst);
/* One output of the buffered path (ops.rs:383-405): the row unpacked by
 * desempaquetar_i8, dot_i8_escalado on this backend, then
 * total += des[b]*xe[b]*xs[b] over the sub-blocks when any des is nonzero. */
float orc_dot_row_buffered(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs,
                           size_t nblk);

/* xorshift64* generator, src/daiss.rs:317-357 */
uint64_t orc_azar_next(uint64_t *state);
void     orc_azar_normals(uint64_t *state, float sigma, float *a, float *b);
uint64_t orc_azar_seed(uint64_t s);                                                 /* daiss.rs:322-327 */

/* sampler, src/sampler.rs:28-152 */
typedef struct orc_sampler orc_sampler;
orc_sampler *orc_sampler_new(uint64_t seed, float temperature, float top_p);
void         orc_sampler_free(orc_sampler *s);
uint32_t     orc_sampler_pick(orc_sampler *s, const float *logits, size_t n);
uint32_t     orc_argmax(const float *v, size_t n);
uint64_t     orc_sampler_state(const orc_sampler *s);

/* model + KV cache, src/forward.rs */
typedef struct orc_model orc_model;
typedef struct orc_cache orc_cache;
typedef struct {
    int n_layer, dim, n_head, n_head_kv, head_dim, vocab, ctx, ffn;
    float eps, rope_base;
    int tied;
} orc_config;

orc_model *orc_model_open(const char *path);                      /* forward.rs:187-266 */
const char *orc_last_error(void);
void        orc_model_close(orc_model *m);
void        orc_model_config(const orc_model *m, orc_config *out);
orc_cache  *orc_cache_new(const orc_model *m);                    /* forward.rs:69-75 */
void        orc_cache_free(orc_cache *c);
int         orc_cache_len(const orc_cache *c);
void        orc_cache_truncate(orc_cache *c, int n);              /* forward.rs:98-108 */
orc_cache  *orc_cache_prefix(const orc_cache *c, int n);          /* forward.rs:115-127 */
void        orc_cache_clear(orc_cache *c);                        /* forward.rs:81-87 */
/* raw access for tests: K or V of layer l, [len x kv_dim] floats */
const float *orc_cache_layer(const orc_cache *c, int layer, int is_v);
/* logits of the LAST token (vocab floats). forward.rs:375-505 */
int orc_forward(orc_model *m, orc_cache *c, const uint32_t *tokens, int n, float *logits);
/* Modelo::generar, forward.rs:533-559: greedy/sampled continuation of prompt */
int orc_generate(orc_model *m, orc_cache *c, const uint32_t *prompt, int n_prompt, int max_new,
                 orc_sampler *s, uint32_t *out, int *n_out);

void orc_cache_fill(orc_cache *c, int n, uint64_t seed);
void orc_expf(const float *x, float *y, size_t n);

/* worker threads of the row-parallel matmul (0 = one per CPU of the process's
 * affinity mask); the
 * workers persist between calls, like the reference's rayon pool */
void orc_set_threads(int n);
int  orc_get_threads(void);

/* Backend of orc_forward's kernels. SCALAR (the default) is the parity
 * target: the reference run with COSXAMIX_KERNEL=escalar (its portable
 * backend, src/kernels/mod.rs:136-163), kernels and matmul dispatch both.
 * X86 runs what the reference picks by default on an AVX2/FMA/F16C host:
 * the AVX2 kernels below for Q4_K, Q6_K, RMSNorm, attention's dot products,
 * dot_i8_escalado and the blocked prefill tiles, a registered reference
 * kernel where one is given, the fused path for all five k-quants, and a
 * prefetch of the row two ahead (src/ops.rs:45-80). Its logits differ from
 * SCALAR's in float summation order only. */
enum { ORC_BACKEND_SCALAR = 0, ORC_BACKEND_X86 = 1 };
void orc_set_backend(int backend);
int  orc_get_backend(void);

/* the reference's kernel ABI (src/kernels/c.rs:18-30) */
typedef float (*orc_dot_fn)(const uint8_t *blocks, const int8_t *xq, const float *xe, const float *xs,
                            size_t n_superblocks);
/* the reference's Q4_K assembly with the "complete" contract: two 8-float
 * accumulators out (src/kernels/q4k_asm.rs:214-235) */
typedef void (*orc_q4k_acc_fn)(const uint8_t *blocks, const int8_t *xq, const float *xe, const float *xs,
                               size_t n_superblocks, float *acc16);
/* use `f` for `type` under the X86 backend (NULL: the built-in choice) */
int  orc_set_dot_kernel(int type, orc_dot_fn f);
void orc_set_q4k_acc_kernel(orc_q4k_acc_fn f);

/* AVX2 restatements, src/kernels/x86.rs (cxm_x86.c) */
float orc_x86_dot_f32(const float *a, const float *b, size_t n);                              /* x86.rs:25-128 */
void  orc_x86_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps);      /* x86.rs:152-213 */
float orc_x86_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* :394-558 */
float orc_x86_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk); /* :760-846 */
float orc_x86_reduce_q4k_acc(const float *acc16);                                             /* q4k_asm.rs:214-235 */
void  orc_x86_q4k_scales(const uint8_t *block, const float *xe, const float *xs, float *scales8,
                         float *mins8);                                                       /* x86.rs:394-471 */
/* one row through the X86 backend's choice for `type` */
float orc_x86_dot_row(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk);
/* dot_i8_escalado_avx2 (x86.rs:315-380): one 8-lane f32 accumulator, an FMA
 * per 32 values with the sub-block scale products, one lane reduction */
float orc_x86_dot_i8_scaled(const int8_t *a, const int8_t *b, const float *ea, const float *eb, size_t n, int block);
/* One output of tesela_{i8,u8}_avx2 (x86.rs:864-948): `chunks` 32-value
 * chunks of activation x (expanded scales ex) against column w (expanded
 * scales ew); `unsig`: w holds unsigned values 0..=129 */
float orc_x86_tile_out(const int8_t *x, const float *ex, const int8_t *w, const float *ew, size_t chunks, int unsig);
/* 1 (default): with one token, q/k/v and gate/up run as one parallel region
 * with x quantized once per sub-block size (src/forward.rs:333-368,
 * src/ops.rs:895-1009); 0: one call per matrix, the reference's
 * COSXAMIX_SIN_VARIAS. Same values either way. */
void orc_set_varias(int on);

#ifdef __cplusplus
}
#endif
#endif
