// The decode step as ONE persistent kernel (one CTA per SM, co-resident by a
// cooperative launch), running a program of phases:
//
//   per layer: q|k|v matvec (norm + quantize in front; bias, RoPE, KV append
//   behind) · attention scores · softmax + attention output · o matvec
//   (+ residual) · gate|up matvec (norm in front, SwiGLU behind) · down
//   matvec (+ residual); then the final norm + output projection + argmax, and
//   the commit of the position/token.
//
// Dependent phases are separated by a grid barrier (bounded spin). Weights
// never depend on activations, so every warp streams its own weight tiles of
// the whole step, in the order it will need them, with coalesced cp.async
// copies into a private shared-memory ring that runs ahead across phase
// boundaries — while the warps sit in barriers, prologues or attention. (Many
// small 1-D bulk copies from one thread per SM top out near 4.3 TB/s on B200;
// warp-wide 16-byte copies stream at over 7.) A normed prologue loads its
// activation through L2 into registers, its norm weights before the barrier;
// a quantize-only prologue stages its activation with one 1-D bulk copy.
// With tensor parallelism the FFN is split by output rows over the ranks,
// and exchange phases gather the ranks' slices of the FFN's hidden vector and
// of the residual stream, and pick the argmax over the ranks' vocabulary
// slices, over peer memory.
//
// Weights are stored as tiles of R rows x LPR super-blocks (R*LPR = 32: one
// warp's lanes, lane = R*block + row), lane-interleaved in 16-byte chunks so
// the 32 lanes read consecutive 16-byte words. LPR ("lanes per row") is
// chosen per matrix: the fewest lanes for which the phase's row groups split
// evenly over the warps, more for the short matrices, whose rows would
// otherwise leave most warps idle (at most 16, so a tile holds both rows of
// an output pair). A warp owns a group of R rows at a time:
// lane (block, row) forms that super-block's sub-block terms, and each row's
// running total visits the blocks in order, handed from lane to lane (the
// reference's sequential sum, src/ops.rs:435-522 with
// src/kernels/scalar.rs:132-324). The rows an epilogue combines (a RoPE pair,
// gate and up) are adjacent rows of a group.
#pragma once

#include "expf_glibc.h"
#include "kernels.cuh"
#include "pipeline.cuh"
#include "step_kernels.cuh"

namespace cxm {

// ── tiled k-quant matrix ──
// Group g (rows g*R .. g*R+R-1) starts at base + g*group_stride; its tile t
// (super-blocks t*LPR .. t*LPR+nb, nb = min(LPR, nblk - t*LPR)) starts
// 32*t*bpb bytes further. Inside a tile of L = R*nb lanes (lane = R*block +
// row):
//   plane A  [chunk c][lane] 16-byte units, c < a_chunks(type)
//   plane S  [lane] s_bytes(type)        (Q6_K 16, Q3_K 12, Q2_K 16)
//   plane D  [lane] d_bytes(type)        (Q6_K 2, Q3_K 2, Q2_K 4)
// so a tile holds exactly L GGUF blocks (L*bpb bytes). group_stride rounds
// R*nblk*bpb up to 16 bytes so every tile starts 16-byte aligned.
struct QMat {
    const uint8_t *base;
    int type, rows, K, nblk, ngroup, bpb;
    int lpr, rpt;  // lanes (super-blocks) per row in a tile; rows per tile = 32 / lpr
    uint32_t group_stride;
};

__host__ __device__ inline int a_chunks(int t) { return plane_a_bytes(t) / 16; }
__host__ __device__ inline int tile_nb(int nblk, int lpr, int t) { return nblk - lpr * t < lpr ? nblk - lpr * t : lpr; }
__host__ __device__ inline uint32_t tile_copy_bytes(int rpt, int nb, int bpb) {
    return (uint32_t)((rpt * nb * bpb + 15) & ~15);
}
__host__ __device__ inline size_t tile_offset(const QMat &M, int g, int t) {
    return (size_t)g * M.group_stride + (size_t)t * 32 * (size_t)M.bpb;
}

// GGUF byte k of super-block b of tiled row r (row order as stored).
__device__ inline uint8_t qm_block_byte(const QMat &M, int r, int b, int k) {
    const int g = r / M.rpt, sl = r % M.rpt, t = b / M.lpr, bl = b % M.lpr, nb = tile_nb(M.nblk, M.lpr, t);
    const int L = M.rpt * nb, lane = M.rpt * bl + sl;
    const uint8_t *tile = M.base + tile_offset(M, g, t);
    const int pa = plane_a_bytes(M.type), ps = plane_s_bytes(M.type), pd = plane_d_bytes(M.type);
    int lo_a = 0, lo_s = pa, lo_d = pa + ps;  // GGUF offsets of the parts
    if (M.type == 10) {                        // Q2_K: scales, qs, d|dmin
        lo_s = 0;
        lo_a = 16;
        lo_d = 80;
    }
    if (k >= lo_a && k < lo_a + pa) {
        const int o = k - lo_a;
        return tile[((o >> 4) * L + lane) * 16 + (o & 15)];
    }
    if (ps && k >= lo_s && k < lo_s + ps) return tile[a_chunks(M.type) * L * 16 + lane * ps + (k - lo_s)];
    return tile[a_chunks(M.type) * L * 16 + L * ps + lane * pd + (k - lo_d)];
}

// one value of a tiled row, exactly as src/quant.rs:582-679 dequantizes it
__device__ inline float qm_dequant(const QMat &M, int r, int idx) {
    const int b = idx >> 8, i = idx & 255;
    auto B = [&](int k) -> uint32_t { return qm_block_byte(M, r, b, k); };
    auto H = [&](int k) -> float { return h2f(B(k) | (B(k + 1) << 8)); };
    switch (M.type) {
    case 12: case 13: {
        const float d = H(0), dmin = H(2);
        const uint32_t w0 = B(4) | B(5) << 8 | B(6) << 16 | B(7) << 24;
        const uint32_t w1 = B(8) | B(9) << 8 | B(10) << 16 | B(11) << 24;
        const uint32_t w2 = B(12) | B(13) << 8 | B(14) << 16 | B(15) << 24;
        const int p = i >> 6, half = (i >> 5) & 1, l = i & 31;
        int sc, mn;
        scale_min_k4(2 * p + half, w0, w1, w2, sc, mn);
        const float dl = fm(d, (float)sc), ml = fm(dmin, (float)mn);
        if (M.type == 12) {
            const uint32_t v = B(16 + 32 * p + l);
            return fs(fm(dl, (float)(half ? (v >> 4) : (v & 0xF))), ml);
        }
        const uint32_t v = B(48 + 32 * p + l);
        const int qv = half ? (int)(v >> 4) : (int)(v & 0xF);
        const float extra = (B(16 + l) >> (2 * p + half)) & 1 ? 16.0f : 0.0f;
        return fs(fm(dl, fa((float)qv, extra)), ml);
    }
    case 14: {
        const int h = i >> 7, rr = i & 127, gi = rr >> 5, l = rr & 31;
        const uint32_t qlb = B(64 * h + 32 * (gi & 1) + l);
        const int nib = gi < 2 ? (int)(qlb & 0xF) : (int)(qlb >> 4);
        const int qv = (nib | (int)(((B(128 + 32 * h + l) >> (2 * gi)) & 3) << 4)) - 32;
        const int sc = (int)(int8_t)B(192 + 8 * h + (rr >> 4));
        return fm(fm(H(208), (float)sc), (float)qv);
    }
    case 11: {
        const int h = i >> 7, rr = i & 127, r4 = rr >> 5, l = rr & 31, g = 4 * h + r4;
        const uint32_t a0 = B(96) | B(97) << 8 | B(98) << 16 | B(99) << 24;
        const uint32_t a1 = B(100) | B(101) << 8 | B(102) << 16 | B(103) << 24;
        const uint32_t tt = B(104) | B(105) << 8 | B(106) << 16 | B(107) << 24;
        const int is = 2 * g + (l >> 4), wi = is >> 2;
        const uint32_t aa = (wi & 1) ? a1 : a0;
        const uint32_t wq = ((aa >> ((wi >> 1) * 4)) & 0x0F0F0F0Fu) | (((tt >> (2 * wi)) & 0x03030303u) << 4);
        const int sc = (int)((wq >> (8 * (is & 3))) & 0xFF);
        const float dl = fm(H(108), fs((float)sc, 32.0f));
        const int hi = (B(l) >> g) & 1 ? 0 : 4;
        const int qv = (int)((B(32 + 32 * h + l) >> (2 * r4)) & 3) - hi;
        return fm(dl, (float)qv);
    }
    default: {  // Q2_K
        const int h = i >> 7, rr = i & 127, r4 = rr >> 5, l = rr & 31, g = 4 * h + r4;
        const int sc = (int)B(2 * g + (l >> 4));
        const float dl = fm(H(80), (float)(sc & 0xF)), ml = fm(H(82), (float)(sc >> 4));
        const int qv = (int)((B(16 + 32 * h + l) >> (2 * r4)) & 3);
        return fs(fm(dl, (float)qv), ml);
    }
    }
}

// ── the program ──
// PH_XGATHER / PH_XARGMAX: the tensor-parallel exchanges with the other
// ranks (GPUs) of the model, over their exchange areas mapped into this
// process
enum PhaseKind : int { PH_MATVEC = 0, PH_SCORES = 1, PH_ATTN = 2, PH_COMMIT = 3, PH_XGATHER = 4, PH_XARGMAX = 5 };

// Float order of a segment's row totals, as the reference's matmul_auto
// picks it for the number of activation rows (src/ops.rs:1056-1093):
// ORD_FUSED, the per-row fused kernel (src/ops.rs:435-522); ORD_BUFFERED,
// matmul_i8_directo (src/ops.rs:310-414): dot_i8_escalado over the row, then
// the offset terms as a second chain. The two differ only for the formats
// with a minimum (Q4_K, Q5_K, Q2_K).
enum Order : int { ORD_FUSED = 0, ORD_BUFFERED = 1 };

struct MvSeg {
    QMat M;
    int units;                // output units (row pairs); padded groups hold more
    int pairing, epi, half;   // Pairing, Epilogue; half = head_dim/2 for PAIR_ROPE
    int ord;                  // Order
    int at_pos, pos_stride;   // out += pos*pos_stride (K/V cache rows)
    int idx_off;              // EPI_LOGITS: vocabulary index of row 0 (this rank's slice)
    const float *bias;
    float *out;
    float *out2;              // EPI_RESID: a second copy of the result (a tensor-parallel rank's exported slice)
    // EPI_SWIGLU: the hidden vector also quantized for the next matvec
    // (ffn_down) as its sub-blocks of qsub values complete: qcnt[s] counts the
    // values of sub-block s written so far; the write that completes one
    // quantizes it into qout (carve_act's layout for qK values). NULL: not done.
    unsigned char *qout;
    int *qcnt;
    int qsub, qK;
};

struct MvPhase {
    MvSeg seg[3];
    int nseg, ngroup, K, ntile;  // segments share K and the tile shape (lpr)
    int prologue, need16, need32;
    uint32_t sv_off;             // region offset of the warps' offset-term spill (ORD_BUFFERED with a minimum)
    int sv_warp;                 // floats of it per warp: rows per tile x sub-blocks per row
    const float *in, *norm_w;
    float eps;
    QMat E;          // PRO_EMBED: token_embd (tiled); or e32 when it is F32
    const float *e32;
    float *x_out;    // PRO_EMBED: CTA 0 stores the embedding row (the residual)
};

struct AtPhase {
    const float *q, *k, *v;  // k/v: this layer's cache, [max_pos][KV*hd]
    const float *kp, *vp;    // a borrowed prefix's layer K/V: positions below plen are read there
    int plen;
    float *out, *scores;
    // the output quantized for the next matvec (o_proj): each item's 32 dims
    // are whole sub-blocks of 16 or 32, quantized where they are formed,
    // into the layout of a matvec activation (NULL: not done)
    unsigned char *qout;
    int qneed16, qneed32, qK;
    int H, KV, hd, score_stride, P;  // P: positions per score item
    int ring;                        // V chunks in the attention phase's ring
    float scale;
};

// an exchange: PH_XGATHER copies every other rank's slice of an n-float
// vector (rank p's slice: [p·n/tp, (p+1)·n/tp), at byte offset src_off of
// its exchange area) into dst; PH_XARGMAX takes the largest argmax key.
// `seq`: the exchange's number in the program (from 1), its flag epoch.
struct XPhase {
    float *dst;
    int n, seq;
    uint32_t src_off;
};

struct __align__(16) Phase {
    int kind, barrier;  // barrier: a grid barrier comes first
    MvPhase mv;
    AtPhase at;
    XPhase xp;
};
static_assert(sizeof(Phase) % 16 == 0, "phase descriptors are staged in 16-byte copies");

// What a warp's tile walk needs of one matvec phase. The host writes one per
// matvec phase, in program order, after the program's phases; each CTA
// stages the table in shared memory, so crossing into the next phase costs
// the walk no global-memory round trip.
struct __align__(16) FeedPhase {
    const uint8_t *b[3];  // segment bases
    uint32_t g[3];        // group strides
    int n0, n1;           // groups of segments 0 and 1 (segment 2 takes the rest)
    int ngroup;
    uint16_t p[3];        // bytes per super-block
    uint16_t ntile, nblk, lpr, rpt, pad;
};
static_assert(sizeof(FeedPhase) == 64, "FeedPhase is four 16-byte chunks");

// A rank's exchange area, mapped by its peers through CUDA IPC: the FFN's
// hidden vector [hdim] f32 (the model's own; the rank writes its slice, the
// peers read it), the exported residual slices [2][xdim] f32 (alternating by
// layer, so a peer still reading one layer's never sees the next layer's
// writes), the argmax keys [kTpMax] (slot p written by rank p), the flags
// [kTpMax] (slot p written by rank p: the epoch of its last exchange).
constexpr int kTpMax = 8;
__host__ __device__ inline size_t xch_xo_off(int hdim) { return (size_t)hdim * sizeof(float); }
__host__ __device__ inline size_t xch_keys_off(int hdim, int xdim) {
    return xch_xo_off(hdim) + (size_t)2 * xdim * sizeof(float);
}
__host__ __device__ inline size_t xch_flags_off(int hdim, int xdim) {
    return xch_keys_off(hdim, xdim) + kTpMax * sizeof(uint64_t);
}
__host__ __device__ inline size_t xch_bytes(int hdim, int xdim) {
    return xch_flags_off(hdim, xdim) + kTpMax * sizeof(unsigned);
}

struct DecodeArgs {
    const Phase *prog;
    int nphase;
    int tp, tp_rank, xdim, hdim, nx;  // ranks; this one; residual and FFN lengths; exchanges in the program
    unsigned char *xch[kTpMax];     // every rank's exchange area (this rank's own at tp_rank)
    unsigned *epoch;                // exchanges completed by earlier launches (this rank)
    const FeedPhase *feed;    // the matvec phases' walk table
    int nfeed;
    unsigned *bar;            // grid-barrier counter, zeroed before each launch
    int *err;
    int *d_len;               // position of the token; NULL: position 0, no token checks
    uint32_t *toks;
    int vocab, max_pos;
    unsigned long long *argmax_key;
    const float *rope_cos, *rope_sin;
    int write_token, commit;  // commit: toks[len+1] = argmax (write_token), len += 1
    int *d_stop;              // set: the generation met its eos and the step does nothing (NULL: never)
    int eos;                  // the token whose greedy pick sets *d_stop, or -1
    int *qcnt;                // the hidden vector's sub-block counts (MvSeg.qcnt), nqcnt of them
    int nqcnt;
    int ring_slots;           // tile slots per warp ring (2..kMaxSlots)
    uint32_t slot_bytes, region_bytes;
};

constexpr int kDW = 8;                       // warps
constexpr int kDecodeThreads = kDW * 32;
constexpr int kMaxSlots = 4;                 // tiles per warp ring
constexpr int kTermMax = 16;

__device__ __forceinline__ void dsync() { asm volatile("bar.sync 1, %0;" ::"n"(kDW * 32) : "memory"); }

// named barrier of the consumer warps that also ORs a predicate over them, so
// a decision taken after it is the same in every consumer thread
__device__ __forceinline__ bool dsync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kDW * 32)
        : "memory");
    return r != 0;
}

__host__ __device__ inline size_t act_bytes(int K, int need16, int need32) {
    size_t b = 0;
    if (need16) b += (size_t)(K / 256) * kXqStride + (size_t)K / 16 * 8;
    if (need32) b += (size_t)(K / 256) * kXqStride + (size_t)K / 32 * 8;
    return (b + 15) & ~(size_t)15;
}

struct Act {
    int8_t *q16, *q32;
    float2 *es16, *es32;  // (scale, sum) per sub-block of 16 / 32
};

__device__ inline Act carve_act(unsigned char *region, int K, int need16, int need32) {
    Act a{};
    unsigned char *p = region;
    const int nblk = K / 256;
    if (need16) { a.q16 = (int8_t *)p; p += nblk * kXqStride; }
    if (need32) { a.q32 = (int8_t *)p; p += nblk * kXqStride; }
    if (need16) { a.es16 = (float2 *)p; p += K / 16 * 8; }
    if (need32) { a.es32 = (float2 *)p; p += K / 32 * 8; }
    return a;
}

// The prologue of a matvec phase, redundantly in every CTA: its activation x
// (written by other CTAs before the barrier, read through L2; or the token's
// embedding row), RMSNorm when the phase has norm weights
// (src/kernels/scalar.rs:36-54), then i8 per sub-block of 16 and/or 32
// (src/ops.rs:178-198). The values live in registers: thread t takes, in
// round i, the 8 values of half-chunk hc = i*256 + t (a chunk is 16 values;
// a sub-block of 32 is the 4 half-chunks of 4 consecutive lanes).
// RMSNorm: scale = 1 / sqrt(Σx²/K + eps) in f64, each op correctly rounded,
// then f32(x·scale)·w. The f64 sum of f32 squares is taken per thread, then
// across lanes and warps. A normed activation has at most two rounds, and
// its norm weights are loaded before the grid barrier (they depend on
// nothing). A plain one of at most kMaxStaged values (the attention output)
// is first staged whole in shared memory by one bulk copy: a copy engine
// pulls data that every CTA reads at once faster than the threads' loads. A
// longer one (the FFN's hidden vector) is loaded straight into registers,
// four rounds at a time (staging it would take the ring's shared memory).
constexpr int kMaxActivation = 16384;         // values of a quantized activation
constexpr int kMaxNormed = 2 * kDW * 32 * 8;  // values of a normed one (4096 at 8 warps)
constexpr int kMaxStaged = kMaxActivation;    // values of a quantize-only activation staged by a bulk copy

__device__ __forceinline__ void load8(const float *src, int hc, float (&x)[8], bool cg) {
    const float4 *p = (const float4 *)src + 2 * hc;
    const float4 u = cg ? __ldcg(p) : __ldg(p), w = cg ? __ldcg(p + 1) : __ldg(p + 1);
    x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
    x[4] = w.x; x[5] = w.y; x[6] = w.z; x[7] = w.w;
}

// round hc of x from the previous phase (zeros past the end)
__device__ __forceinline__ void load_x(const MvPhase &P, int hc, float (&x)[8]) {
    if (hc < (P.K >> 3)) {
        load8(P.in, hc, x, true);
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) x[k] = 0.0f;
    }
}

// one value of a k-quant embedding row (a call: the dequantizer stays out of
// the inlined prologue)
__device__ __noinline__ float embed_value(const QMat &E, int tok, int i) { return qm_dequant(E, tok, i); }

// round hc of the token's embedding row; CTA 0 also starts the residual
// stream with it
__device__ __forceinline__ void load_embed(const MvPhase &P, uint32_t tok, int hc, float (&x)[8]) {
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = 0.0f;
    if (hc >= (P.K >> 3)) return;
    if (P.e32) {
        load8(P.e32 + (size_t)tok * P.K, hc, x, false);
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) x[k] = embed_value(P.E, (int)tok, 8 * hc + k);
    }
    if (blockIdx.x == 0) {
        ((float4 *)P.x_out)[2 * hc] = make_float4(x[0], x[1], x[2], x[3]);
        ((float4 *)P.x_out)[2 * hc + 1] = make_float4(x[4], x[5], x[6], x[7]);
    }
}

// the norm weights of this thread's two rounds, loaded before the barrier
struct NormW {
    float w[2][8];
};
__device__ __forceinline__ void load_norm_w(const MvPhase &P, NormW &nw) {
    const int tid = threadIdx.x, nh = P.K >> 3;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int hc = r * kDW * 32 + tid;
        if (hc < nh) {
            load8(P.norm_w, hc, nw.w[r], false);
        } else {
#pragma unroll
            for (int k = 0; k < 8; k++) nw.w[r][k] = 0.0f;
        }
    }
}

__device__ __forceinline__ void norm8(float (&x)[8], double scale, const float (&w)[8]) {
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = __fmul_rn(__double2float_rn(__dmul_rn((double)x[k], scale)), w[k]);
}

// i8 values of 8 elements against the sub-block's amax, packed, and their sum
__device__ __forceinline__ int quant8(const float (&x)[8], float am, uint32_t &w0, uint32_t &w1) {
    const float inv = am > 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
    int sm = 0;
    w0 = w1 = 0u;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int qv = (int)roundf(__fmul_rn(x[k], inv));
        sm += qv;
        if (k < 4) w0 |= ((uint32_t)qv & 0xFFu) << (8 * k);
        else w1 |= ((uint32_t)qv & 0xFFu) << (8 * (k - 4));
    }
    return sm;
}

// R rounds (first half-chunk hc0, then hc0 + 256, ...) quantized stage by
// stage in lockstep, so their latency chains (shuffles, divisions) overlap.
// nh (= K/8) is a multiple of 32: a warp's lanes are all in range or all
// out, and the shuffles see full warps; rounds past the end store nothing.
template <int R>
__device__ __forceinline__ void quant_rounds(const MvPhase &P, const Act &a, int hc0, const float (&x)[R][8]) {
    const int nh = P.K >> 3;
    float amax[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        amax[r] = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) amax[r] = fmaxf(amax[r], fabsf(x[r][k]));
    }
    if (P.need16) {
        float am[R];
        int sm[R];
        uint32_t w0[R], w1[R];
#pragma unroll
        for (int r = 0; r < R; r++) am[r] = fmaxf(amax[r], __shfl_xor_sync(0xffffffffu, amax[r], 1));
#pragma unroll
        for (int r = 0; r < R; r++) sm[r] = quant8(x[r], am[r], w0[r], w1[r]);
#pragma unroll
        for (int r = 0; r < R; r++) sm[r] += __shfl_xor_sync(0xffffffffu, sm[r], 1);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int hc = hc0 + r * kDW * 32, c = hc >> 1;
            if (hc < nh) {
                *(uint2 *)(a.q16 + ((16 * c) >> 8) * kXqStride + ((16 * c) & 255) + 8 * (hc & 1)) = make_uint2(w0[r], w1[r]);
                if (!(hc & 1)) {
                    a.es16[c] = make_float2(am[r] > 0.0f ? __fdiv_rn(am[r], 127.0f) : 0.0f, (float)sm[r]);
                }
            }
        }
    }
    if (P.need32) {
        float am[R];
        int sm[R];
        uint32_t w0[R], w1[R];
#pragma unroll
        for (int r = 0; r < R; r++) am[r] = fmaxf(amax[r], __shfl_xor_sync(0xffffffffu, amax[r], 1));
#pragma unroll
        for (int r = 0; r < R; r++) am[r] = fmaxf(am[r], __shfl_xor_sync(0xffffffffu, am[r], 2));
#pragma unroll
        for (int r = 0; r < R; r++) sm[r] = quant8(x[r], am[r], w0[r], w1[r]);
#pragma unroll
        for (int r = 0; r < R; r++) sm[r] += __shfl_xor_sync(0xffffffffu, sm[r], 1);
#pragma unroll
        for (int r = 0; r < R; r++) sm[r] += __shfl_xor_sync(0xffffffffu, sm[r], 2);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int hc = hc0 + r * kDW * 32, c = hc >> 1;
            if (hc < nh) {
                *(uint2 *)(a.q32 + ((16 * c) >> 8) * kXqStride + ((16 * c) & 255) + 8 * (hc & 1)) = make_uint2(w0[r], w1[r]);
                if (!(hc & 3)) {
                    a.es32[hc >> 2] = make_float2(am[r] > 0.0f ? __fdiv_rn(am[r], 127.0f) : 0.0f, (float)sm[r]);
                }
            }
        }
    }
}

__device__ __forceinline__ void quantize_act(const MvPhase &P, uint32_t tok, const NormW &nw, const float *stage,
                                             const Act &a, double *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = kDW * 32;
    const int nr = ((P.K >> 3) + nt - 1) / nt;  // rounds
    if (P.prologue != PRO_QUANT) {  // at most two rounds
        float x[2][8];
        if (P.prologue == PRO_EMBED) {
            load_embed(P, tok, tid, x[0]);
            load_embed(P, tok, nt + tid, x[1]);
        } else {
            load_x(P, tid, x[0]);
            load_x(P, nt + tid, x[1]);
        }
        double acc = 0.0;
#pragma unroll
        for (int r = 0; r < 2; r++) {
#pragma unroll
            for (int k = 0; k < 8; k++) acc = __dadd_rn(acc, __dmul_rn((double)x[r][k], (double)x[r][k]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[warp] = acc;
        dsync();
        // every thread finishes the reduction itself (same order, same result)
        double sum = 0.0;
#pragma unroll
        for (int w = 0; w < kDW; w++) sum = __dadd_rn(sum, red[w]);
        const int K = P.K;
        // Σ/K: a product by 1/K (exact) when K is a power of two
        const double ms = (K & (K - 1)) == 0 ? __dmul_rn(sum, 1.0 / (double)K) : __ddiv_rn(sum, (double)K);
        const double scale = __drcp_rn(__dsqrt_rn(__dadd_rn(ms, (double)P.eps)));
        norm8(x[0], scale, nw.w[0]);
        norm8(x[1], scale, nw.w[1]);
        if (nr == 1) quant_rounds<1>(P, a, tid, *(const float(*)[1][8])x);
        else quant_rounds<2>(P, a, tid, x);
    } else if (!stage) {  // straight from L2, four rounds at a time, each batch's loads issued first
        for (int i = 0; i < nr; i += 4) {
            float x[4][8];
#pragma unroll
            for (int r = 0; r < 4; r++) load_x(P, (i + r) * nt + tid, x[r]);
            quant_rounds<4>(P, a, i * nt + tid, x);
        }
    } else {  // from the staged copy, two rounds at a time
        const int nh = P.K >> 3;
        for (int i = 0; i < nr; i += 2) {
            float x[2][8];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int hc = (i + r) * nt + tid;
                const float4 u = hc < nh ? ((const float4 *)stage)[2 * hc] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                const float4 w = hc < nh ? ((const float4 *)stage)[2 * hc + 1] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                x[r][0] = u.x; x[r][1] = u.y; x[r][2] = u.z; x[r][3] = u.w;
                x[r][4] = w.x; x[r][5] = w.y; x[r][6] = w.z; x[r][7] = w.w;
            }
            if (i + 1 < nr) quant_rounds<2>(P, a, i * nt + tid, x);
            else quant_rounds<1>(P, a, i * nt + tid, *(const float(*)[1][8])x);
        }
    }
    dsync();
}

// rows (r0, r1) of output unit u of a segment: the pair an epilogue combines
__device__ __forceinline__ void unit_rows(const MvSeg &g, int u, int &r0, int &r1) {
    if (g.pairing == PAIR_ADJ) {
        r0 = 2 * u;
        r1 = 2 * u + 1;
    } else if (g.pairing == PAIR_ROPE) {
        const int h = u / g.half, i = u % g.half;
        r0 = h * 2 * g.half + i;
        r1 = r0 + g.half;
    } else {
        r0 = r1 = u;  // gate row u, up row u
    }
}

// the epilogue's inputs (bias, RoPE rotation, residual), loaded when a
// quad starts so their latency hides under the quad's tiles
struct EpiIn {
    float a, b, c, d;
};

__device__ __forceinline__ EpiIn epi_load(const DecodeArgs &A, const MvSeg &g, int r0, int r1, int pos) {
    EpiIn e{0.0f, 0.0f, 0.0f, 0.0f};
    if (g.at_pos && (pos < 0 || pos >= A.max_pos)) return e;
    switch (g.epi) {
    case EPI_STORE:
        if (g.bias) {
            e.a = __ldg(g.bias + r0);
            e.b = __ldg(g.bias + r1);
        }
        break;
    case EPI_ROPE: {
        const int i = r0 % (2 * g.half);
        if (g.bias) {
            e.a = __ldg(g.bias + r0);
            e.b = __ldg(g.bias + r1);
        }
        e.c = __ldg(A.rope_cos + (size_t)pos * g.half + i);
        e.d = __ldg(A.rope_sin + (size_t)pos * g.half + i);
        break;
    }
    case EPI_RESID:  // this unit's rows are written by this lane only
        e.a = __ldcg(g.out + r0);
        e.b = __ldcg(g.out + r1);
        break;
    default:
        break;
    }
    return e;
}

__device__ void unit_epilogue(const DecodeArgs &A, const MvSeg &g, int r0, int r1, float y0, float y1, int pos,
                              const EpiIn &e, unsigned long long &best) {
    if (g.at_pos && (pos < 0 || pos >= A.max_pos)) return;
    float *out = g.out + (g.at_pos ? (size_t)pos * g.pos_stride : 0);
    switch (g.epi) {
    case EPI_STORE:
        if (g.bias) {
            y0 = fa(y0, e.a);
            y1 = fa(y1, e.b);
        }
        out[r0] = y0;
        out[r1] = y1;
        break;
    case EPI_ROPE: {
        // src/ops.rs:1150-1193, split-half pair (i, i + hd/2) at pos
        const float a = g.bias ? fa(y0, e.a) : y0, b = g.bias ? fa(y1, e.b) : y1;
        out[r0] = fs(fm(a, e.c), fm(b, e.d));
        out[r1] = fa(fm(a, e.d), fm(b, e.c));
        break;
    }
    case EPI_RESID:  // src/forward.rs:467-469, :489-491
        out[r0] = fa(e.a, y0);
        out[r1] = fa(e.b, y1);
        if (g.out2) {
            g.out2[r0] = out[r0];
            g.out2[r1] = out[r1];
        }
        break;
    case EPI_SWIGLU: {
        // src/kernels/scalar.rs:63-67 then `*a *= u` (src/forward.rs:485-487)
        const float act = __fdiv_rn(y0, fa(1.0f, expf_glibc(-y0)));
        out[r0] = fm(act, y1);
        break;
    }
    case EPI_LOGITS: {
        out[r0] = y0;
        out[r1] = y1;
        const unsigned long long ka = (y0 == y0) ? argmax_key(y0, (uint32_t)(r0 + g.idx_off)) : 0ull;
        const unsigned long long kb = (y1 == y1) ? argmax_key(y1, (uint32_t)(r1 + g.idx_off)) : 0ull;
        const unsigned long long kk = ka > kb ? ka : kb;
        best = kk > best ? kk : best;
        break;
    }
    }
}

// The sub-block sb of a segment's hidden vector, complete in global memory,
// quantized exactly as quantize_act quantizes it (src/ops.rs:178-198):
// amax over the sub-block, 127/amax, round-half-away, the (scale, sum) pair.
__device__ __noinline__ void hidden_quant_block(const MvSeg &g, int sb) {
    const int sub = g.qsub;
    const float *h = g.out + (size_t)sb * sub;
    float x[32];
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        x[i] = i < sub ? __ldcg(h + i) : 0.0f;
        am = fmaxf(am, fabsf(x[i]));
    }
    const float inv = am > 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
    const Act a = carve_act(g.qout, g.qK, sub == 16, sub == 32);
    int8_t *q = (sub == 16 ? a.q16 : a.q32) + ((sb * sub) >> 8) * kXqStride + ((sb * sub) & 255);
    int sm = 0;
#pragma unroll
    for (int w4 = 0; w4 < 8; w4++) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int qv = (int)roundf(__fmul_rn(x[4 * w4 + k], inv));
            sm += qv;  // zero beyond sub
            word |= ((uint32_t)qv & 0xFFu) << (8 * k);
        }
        if (4 * w4 < sub) ((uint32_t *)q)[w4] = word;
    }
    (sub == 16 ? a.es16 : a.es32)[sb] = make_float2(am > 0.0f ? __fdiv_rn(am, 127.0f) : 0.0f, (float)sm);
}

// After a flush's epilogues (whole warp): every lane that wrote hidden value
// v of a segment with `qout` counts it into its sub-block, one atomic per
// distinct sub-block of the warp; the lane whose count completes a sub-block
// quantizes it and clears the count for the next layer.
__device__ __forceinline__ void hidden_quant_arrive(const MvSeg &g, int v, bool wrote) {
    const int lane = threadIdx.x & 31;
    const int sb = wrote ? v / g.qsub : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, sb);
    __threadfence();  // each lane's hidden value before its sub-block's count
    __syncwarp();
    if (!wrote || lane != __ffs(peers) - 1) return;
    const int n = __popc(peers);
    if (atomicAdd(&g.qcnt[sb], n) + n != g.qsub) return;
    __threadfence();  // the other CTAs' values after their counts
    hidden_quant_block(g, sb);
    g.qcnt[sb] = 0;
}

// group range of this CTA in a matvec phase: contiguous and balanced
__device__ __forceinline__ void cta_groups(int ngroup, int &qb, int &qe) {
    qb = (int)(((long long)blockIdx.x * ngroup) / gridDim.x);
    qe = (int)(((long long)(blockIdx.x + 1) * ngroup) / gridDim.x);
}

// ── a warp's walk over its weight tiles ──
// Every consumer warp streams its own tiles: matvec phases in program order;
// in each, its row groups qb + warp + 8k of the CTA's range [qb, qe), tile by
// tile. It copies them with 16-byte cp.async (a warp moves 512 contiguous
// bytes per instruction) into a private ring, running ring_slots - 1 tiles
// ahead of its compute, into the next phases too: the weights never depend
// on the activations, so the copies overlap barriers, prologues and
// attention.
struct Feed {
    int m, q, qe, t;  // next tile: matvec phase (index into the walk table), phase-global group, tile
    int ntile, nblk, lpr, rpt;
    int n0, n1;       // groups of segments 0 and 1 (segment 2 takes the rest)
    int p0, p1, p2;   // bytes per super-block
    uint32_t g0, g1, g2;  // group strides
    const uint8_t *b0, *b1, *b2;
};

// position the walk at the first group of this warp in matvec phase >= f.m
__device__ inline void feed_phase(const FeedPhase *tab, int ntab, Feed &f, int warp) {
    for (; f.m < ntab; f.m++) {
        const FeedPhase &F = tab[f.m];
        int qb, qe;
        cta_groups(F.ngroup, qb, qe);
        if (qb + warp >= qe) continue;
        f.ntile = F.ntile;
        f.nblk = F.nblk;
        f.lpr = F.lpr;
        f.rpt = F.rpt;
        f.n0 = F.n0;
        f.n1 = F.n1;
        f.p0 = F.p[0];
        f.p1 = F.p[1];
        f.p2 = F.p[2];
        f.g0 = F.g[0];
        f.g1 = F.g[1];
        f.g2 = F.g[2];
        f.b0 = F.b[0];
        f.b1 = F.b[1];
        f.b2 = F.b[2];
        f.q = qb + warp;
        f.qe = qe;
        f.t = 0;
        return;
    }
}

__device__ __forceinline__ bool feed_next(const FeedPhase *tab, int ntab, Feed &f, int warp, const uint8_t *&src,
                                          uint32_t &bytes) {
    if (f.m >= ntab) return false;
    int lq = f.q;
    const uint8_t *b;
    uint32_t gs;
    int bpb;
    if (lq < f.n0) {
        b = f.b0; gs = f.g0; bpb = f.p0;
    } else if ((lq -= f.n0) < f.n1) {
        b = f.b1; gs = f.g1; bpb = f.p1;
    } else {
        lq -= f.n1;
        b = f.b2; gs = f.g2; bpb = f.p2;
    }
    const int nb = tile_nb(f.nblk, f.lpr, f.t);
    src = b + (size_t)lq * gs + (size_t)f.t * 32 * bpb;
    bytes = tile_copy_bytes(f.rpt, nb, bpb);
    if (++f.t == f.ntile) {
        f.t = 0;
        f.q += kDW;
        if (f.q >= f.qe) {
            f.m++;
            feed_phase(tab, ntab, f, warp);
        }
    }
    return true;
}

// one tile into a ring slot: the warp's lanes copy 16-byte chunks, one group
__device__ __forceinline__ void issue_tile(unsigned char *slot, const uint8_t *src, uint32_t bytes, int lane) {
    const uint32_t o0 = (uint32_t)lane * 16;
#pragma unroll 4
    for (uint32_t o = o0; o < bytes; o += 512) cp_async16(slot + o, src + o);
    cp_async_commit();
}

// wait until at most n of this thread's newest cp.async groups are pending
__device__ __forceinline__ void cp_async_wait_n(int n) {
    switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    case 7: cp_async_wait<7>(); break;
    case 8: cp_async_wait<8>(); break;
    case 9: cp_async_wait<9>(); break;
    case 10: cp_async_wait<10>(); break;
    case 11: cp_async_wait<11>(); break;
    case 12: cp_async_wait<12>(); break;
    case 13: cp_async_wait<13>(); break;
    case 14: cp_async_wait<14>(); break;
    default: cp_async_wait<15>(); break;
    }
}

// ── grid barrier among the consumer warps of all CTAs (bounded) ──
// each poll is an L2 round trip (~0.5 us): 2^21 polls bound a wait near 1 s
constexpr uint32_t kBarrierSpins = 1u << 21;

__device__ bool grid_sync(const DecodeArgs &A, unsigned target, volatile int *abort_flag, int *ok_s) {
    dsync();
    if (threadIdx.x == 0) {
        int ok = 1;
        // release this CTA's writes (made visible to thread 0 by the named
        // barrier) and arrive, without waiting for the atomic's reply
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(A.bar) : "memory");
        for (uint32_t i = 0;; i++) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.bar) : "memory");
            if ((int)(v - target) >= 0) break;
            if (i >= kBarrierSpins) {
                atomicOr(A.err, ERR_TIMEOUT);
                ok = 0;
                break;
            }
            if ((i & 255) == 255) {
                if (*(volatile int *)A.err & ERR_TIMEOUT) {  // another CTA gave up
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        if (!ok) *abort_flag = 1;
        *ok_s = ok;
    }
    dsync();
    return *ok_s != 0;
}

// ── tensor-parallel exchanges over the peers' exchange areas ──
// A flag store is a release at system scope after a system-scope fence, so a
// peer that acquires the flag sees this rank's partial vector (or key). Every
// wait is bounded like the grid barrier's; a timeout raises ERR_TIMEOUT here
// and stops the kernel, so a lost peer never hangs this GPU.
__device__ __forceinline__ unsigned *xch_flags(unsigned char *area, int hdim, int xdim) {
    return (unsigned *)(area + xch_flags_off(hdim, xdim));
}
__device__ __forceinline__ void flag_store(unsigned *f, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned flag_load(const unsigned *f) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_sys4(const float4 *p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Every other rank's flag in this rank's area reaches `ep` (thread 0). The
// ranks are separate processes whose launches can drift apart by host-side
// delays (a graph capture), so this wait is bounded by time, 10 s on the
// global timer (and, as a backstop, by a count of polls), not by the grid
// barrier's poll count.
constexpr unsigned long long kXchWaitNs = 10ull * 1000 * 1000 * 1000;
constexpr uint32_t kXchSpins = 1u << 26;
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ bool wait_peers(const DecodeArgs &A, unsigned ep) {
    const unsigned *mine = xch_flags(A.xch[A.tp_rank], A.hdim, A.xdim);
    const unsigned long long t0 = global_ns();
    for (int p = 0; p < A.tp; p++) {
        if (p == A.tp_rank) continue;
        for (uint32_t i = 0;; i++) {
            if ((int)(flag_load(mine + p) - ep) >= 0) break;
            if ((i & 255) == 255) {
                if (*(volatile int *)A.err & ERR_TIMEOUT) return false;
                if (global_ns() - t0 > kXchWaitNs || i >= kXchSpins) {
                    atomicOr(A.err, ERR_TIMEOUT);
                    return false;
                }
                __nanosleep(128);
            }
        }
    }
    return true;
}

// this rank's flag `ep` into every peer's area (after its data)
__device__ void signal_peers(const DecodeArgs &A, unsigned ep) {
    __threadfence_system();
    for (int p = 0; p < A.tp; p++)
        if (p != A.tp_rank) flag_store(xch_flags(A.xch[p], A.hdim, A.xdim) + A.tp_rank, ep);
}

// The other ranks' slices of an n-float vector into this rank's copy: CTA
// 0 publishes this rank's slice (complete: a grid barrier precedes this
// phase), every CTA waits for the peers', then copies its share of their
// slices out of their exchange areas. Each value is the one the rank that
// owns it computed, so the gathered vector is exactly the single-GPU one.
__device__ void phase_xgather(const DecodeArgs &A, const XPhase &X, unsigned ep, volatile int *abort_flag,
                              int *ok_s) {
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) signal_peers(A, ep);
        const bool ok = wait_peers(A, ep);
        if (!ok) *abort_flag = 1;
        *ok_s = ok;
    }
    dsync();
    if (!*ok_s) return;
    const int s4 = X.n / A.tp / 4;      // float4s per slice
    const int n4 = s4 * (A.tp - 1);     // the other ranks' float4s
    const int per = (n4 + gridDim.x - 1) / gridDim.x;
    const int i0 = blockIdx.x * per, i1 = min(n4, i0 + per);
    for (int i = i0 + threadIdx.x; i < i1; i += kDW * 32) {
        int p = i / s4;
        p += p >= A.tp_rank;            // skip this rank's own slice
        const int j = p * s4 + i % s4;  // float4 index in the vector
        ((float4 *)X.dst)[j] = ld_sys4((const float4 *)(A.xch[p] + X.src_off) + j);
    }
}

// the greedy pick over the ranks' vocabulary slices: CTA 0 publishes this
// rank's argmax key (its slice's first maximum), takes every peer's, and
// leaves the largest (the first maximum of the whole vocabulary) in
// *argmax_key for the commit
__device__ void phase_xargmax(const DecodeArgs &A, unsigned ep, volatile int *abort_flag) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    const unsigned long long mine = __ldcg(A.argmax_key);
    for (int p = 0; p < A.tp; p++)
        if (p != A.tp_rank) {
            unsigned long long *k = (unsigned long long *)(A.xch[p] + xch_keys_off(A.hdim, A.xdim)) + A.tp_rank;
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(k), "l"(mine) : "memory");
        }
    signal_peers(A, ep);
    if (!wait_peers(A, ep)) {
        *abort_flag = 1;
        return;
    }
    unsigned long long best = mine;
    const unsigned long long *keys = (const unsigned long long *)(A.xch[A.tp_rank] + xch_keys_off(A.hdim, A.xdim));
    for (int p = 0; p < A.tp; p++) {
        if (p == A.tp_rank) continue;
        unsigned long long v;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(keys + p) : "memory");
        best = v > best ? v : best;
    }
    *A.argmax_key = best;
}

// ── attention phases (src/ops.rs:1258-1325), reference order ──
// An attention item is one head and 32 of its output dims. Its region: the
// head's probabilities (max_pos rounded to 4 floats), then a ring of `ring`
// V chunks, each kAttnPos positions of the item's 32 dims ([position][dim]:
// a position's 128 bytes arrive in eight 16-byte copies, and the 32 lanes of
// the position-by-position sums read one position's 32 consecutive floats,
// free of bank conflicts).
constexpr int kAttnPos = 128, kAttnMinRing = 3, kAttnMaxRing = 8;
constexpr int kAttnChunkFloats = 32 * kAttnPos;
__host__ __device__ inline size_t scores_region(int P, int G, int hd) {
    return ((size_t)P * (hd + 4) + (size_t)G * hd) * sizeof(float);
}
__host__ __device__ inline size_t attn_region(int max_pos, int ring) {
    return ((size_t)((max_pos + 3) & ~3) + (size_t)ring * kAttnChunkFloats) * sizeof(float);
}

// positions per score item of a step over n positions: enough items for
// every CTA, at most at.P (the region's capacity)
__device__ __forceinline__ int score_span(const AtPhase &at, int n) {
    const int want = (at.KV * n + gridDim.x - 1) / gridDim.x;
    return want < 1 ? 1 : (want > at.P ? at.P : want);
}

// Before the scores phase's grid barrier: the K rows of this CTA's first
// item that are already in the cache (every position but the step's own,
// which the q|k|v phase is writing), as one cp.async group.
__device__ __forceinline__ void scores_prefetch(const AtPhase &at, int n, float *region) {
    const int tid = threadIdx.x, hd = at.hd, kvd = at.KV * hd, c4 = hd / 4;
    const int P = score_span(at, n), nchunk = (n + P - 1) / P, items = at.KV * nchunk;
    const int item = blockIdx.x;
    if (item < items) {
        const int g = item / nchunk, p0 = (item % nchunk) * P, cnt = min(P, n - 1 - p0);  // not position n-1
        for (int i = tid; i < cnt * c4; i += kDW * 32) {
            const int r = i / c4, c = i - r * c4;
            cp_async16(region + r * (hd + 4) + 4 * c, kv_row(at.k, at.kp, at.plen, p0 + r, kvd, (size_t)g * hd + 4 * c));
        }
    }
    cp_async_commit();
}

// score[h][p] = (sequential dot of q_h and k_p over the head dim) · scale; an
// item is one kv head and P positions, shared by the G query heads on it
// (the first item's cached K rows were staged by scores_prefetch)
__device__ __forceinline__ void phase_scores(const AtPhase &at, int n, float *region) {
    const int tid = threadIdx.x, hd = at.hd, G = at.H / at.KV, kvd = at.KV * hd, c4 = hd / 4;
    const int P = score_span(at, n), nchunk = (n + P - 1) / P, items = at.KV * nchunk;
    float *ks = region, *qs = region + (size_t)at.P * (hd + 4);
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int g = item / nchunk, p0 = (item % nchunk) * P, cnt = min(P, n - p0);
        const bool first = item == (int)blockIdx.x;
        for (int i = tid; i < G * c4; i += kDW * 32) {
            const int hq = i / c4, c = i - hq * c4;
            cp_async16(qs + hq * hd + 4 * c, at.q + (size_t)(g * G + hq) * hd + 4 * c);
        }
        // the rows the prefetch did not stage: the step's own position (the
        // first item), or all (a later item)
        const int r0 = first ? (n - 1 >= p0 && n - 1 < p0 + cnt ? n - 1 - p0 : cnt) : 0;
        for (int i = tid; i < (cnt - r0) * c4; i += kDW * 32) {
            const int r = r0 + i / c4, c = i % c4;
            cp_async16(ks + r * (hd + 4) + 4 * c, kv_row(at.k, at.kp, at.plen, p0 + r, kvd, (size_t)g * hd + 4 * c));
        }
        cp_async_commit();
        cp_async_wait<0>();
        dsync();
        if (tid < G * P) {
            const int hq = tid / P, pp = tid - hq * P;
            if (pp < cnt) {
                const float4 *kr = (const float4 *)(ks + pp * (hd + 4));
                const float4 *q4 = (const float4 *)(qs + hq * hd);
                float acc = 0.0f;
                for (int c = 0; c < c4; c++) {
                    const float4 kv = kr[c], qv = q4[c];
                    acc = fa(acc, fm(qv.x, kv.x));
                    acc = fa(acc, fm(qv.y, kv.y));
                    acc = fa(acc, fm(qv.z, kv.z));
                    acc = fa(acc, fm(qv.w, kv.w));
                }
                at.scores[(size_t)(g * G + hq) * at.score_stride + p0 + pp] = fm(acc, at.scale);
            }
        }
        dsync();
    }
}

// the sum of p[0..n) added one value after another from 0.0f (one thread):
// 16 values per step, the next step's loads in flight during this step's adds
__device__ __forceinline__ float seq_sum(const float *p, int n) {
    float acc = 0.0f;
    int i = 0;
    float4 n0 = make_float4(0.f, 0.f, 0.f, 0.f), n1 = n0, n2 = n0, n3 = n0;
    if (16 <= n) {
        n0 = ((const float4 *)p)[0];
        n1 = ((const float4 *)p)[1];
        n2 = ((const float4 *)p)[2];
        n3 = ((const float4 *)p)[3];
    }
    for (; i + 16 <= n; i += 16) {
        const float4 q0 = n0, q1 = n1, q2 = n2, q3 = n3;
        if (i + 32 <= n) {
            const float4 *c4 = (const float4 *)(p + i + 16);
            n0 = c4[0];
            n1 = c4[1];
            n2 = c4[2];
            n3 = c4[3];
        }
        acc = fa(fa(fa(fa(acc, q0.x), q0.y), q0.z), q0.w);
        acc = fa(fa(fa(fa(acc, q1.x), q1.y), q1.z), q1.w);
        acc = fa(fa(fa(fa(acc, q2.x), q2.y), q2.z), q2.w);
        acc = fa(fa(fa(fa(acc, q3.x), q3.y), q3.z), q3.w);
    }
    for (; i < n; i++) acc = fa(acc, p[i]);
    return acc;
}

// One attention item: head h and dims [d0, d0 + 32) (src/ops.rs:1258-1325).
// The head's scores staged in shared memory; their max and exp(s - max)
// (src/ops.rs:1206-1230) across the CTA; the sum position by position by
// thread 0; then warp 0 adds prob_p·v_p[d] position by position, lane d for
// dim d0 + d, over the staged V chunks.

// V chunk c of an item into its ring slot (the caller commits the cp.async
// group)
__device__ __forceinline__ void attn_stage(const AtPhase &at, int n, size_t voff, float *ring, int c) {
    const int tid = threadIdx.x, kvd = at.KV * at.hd;
    if (c * kAttnPos >= n) return;
    const int base = c * kAttnPos, cnt = min(kAttnPos, n - base);
    float *dst = ring + (c % at.ring) * kAttnChunkFloats;
    for (int i = tid; i < cnt * 8; i += kDW * 32) {
        const int p = i >> 3, q = i & 7;
        cp_async16(dst + p * 32 + 4 * q, kv_row(at.v, at.vp, at.plen, base + p, kvd, voff + 4 * q));
    }
}

// the item's 32 dims of a V row: their offset in the row
__device__ __forceinline__ size_t attn_voff(const AtPhase &at, int item) {
    const int ns = at.hd / 32, h = item / ns, G = at.H / at.KV;
    return (size_t)(h / G) * at.hd + (item % ns) * 32;
}

// Before the attention phase's grid barrier: the first ring - 1 V chunks of
// this CTA's first item (the V rows of every position are in the cache once
// the scores phase began), one cp.async group each.
__device__ __forceinline__ void attn_prefetch(const AtPhase &at, int n, int max_pos, float *region) {
    const int items = at.H * (at.hd / 32), item = blockIdx.x;
    float *ring = region + ((max_pos + 3) & ~3);
    for (int c = 0; c < at.ring - 1; c++) {
        if (item < items) attn_stage(at, n, attn_voff(at, item), ring, c);
        cp_async_commit();
    }
}

// acc + Σ (e[r]·inv)·v[r] over the cnt positions of a chunk, one position
// after another (lane d: vt points at dim d of the chunk's first position,
// positions 32 floats apart)
__device__ __forceinline__ void pv_chunk(const float *vt, const float *pp, int cnt, float inv, float &acc) {
    int r = 0;
    for (; r + 16 <= cnt; r += 16) {
        float4 q[4];
        float w[16];
#pragma unroll
        for (int k = 0; k < 4; k++) q[k] = ((const float4 *)(pp + r))[k];
#pragma unroll
        for (int k = 0; k < 16; k++) w[k] = vt[(r + k) * 32];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            acc = fa(acc, fm(fm(q[k].x, inv), w[4 * k]));
            acc = fa(acc, fm(fm(q[k].y, inv), w[4 * k + 1]));
            acc = fa(acc, fm(fm(q[k].z, inv), w[4 * k + 2]));
            acc = fa(acc, fm(fm(q[k].w, inv), w[4 * k + 3]));
        }
    }
    for (; r < cnt; r++) acc = fa(acc, fm(fm(pp[r], inv), vt[r * 32]));
}

// The 32 outputs of an attention item (one per lane of warp 0, dims d0..d0+31
// of the concatenated heads) quantized as quantize_act quantizes them
// (src/ops.rs:178-198: amax per sub-block, 127/amax, round half away, the
// scale amax/127 and the integer sum), written into the global activation
// buffer in carve_act's layout: the next phase copies it instead of
// quantizing the whole vector in every CTA.
__device__ __forceinline__ void attn_quant_out(const AtPhase &at, int d, float v) {
    const int lane = threadIdx.x & 31;
    const Act a = carve_act(at.qout, at.qK, at.qneed16, at.qneed32);
    const float av = fabsf(v);
    for (int sz = 16; sz <= 32; sz += 16) {
        if ((sz == 16 && !at.qneed16) || (sz == 32 && !at.qneed32)) continue;
        float am = av;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
            if (o < sz) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float inv = am > 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
        const int qv = (int)roundf(__fmul_rn(v, inv));
        int sm = qv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
            if (o < sz) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        int8_t *q = sz == 16 ? a.q16 : a.q32;
        q[(d >> 8) * kXqStride + (d & 255)] = (int8_t)qv;
        if ((lane & (sz - 1)) == 0)
            (sz == 16 ? a.es16 : a.es32)[d / sz] = make_float2(am > 0.0f ? __fdiv_rn(am, 127.0f) : 0.0f, (float)sm);
    }
}

// The head's scores come in from L2 with each thread's running max; every
// thread then takes exp(s - max) of the same values (no barrier between);
// thread 0 adds them in order and forms 1/total; warp 0 adds (e·inv)·v
// position by position — e·inv is the reference's probability, formed where
// it is used. When the prefetch before the barrier staged every V chunk (a
// context up to (ring - 1)·kAttnPos positions), the PV runs without a
// barrier per chunk.
__device__ __forceinline__ void phase_attn(const AtPhase &at, int n, int max_pos, float *region, float *red,
                                           float *bc) {
    const int tid = threadIdx.x, nt = kDW * 32, lane = tid & 31, warp = tid >> 5, hd = at.hd, ns = hd / 32;
    const int items = at.H * ns, R = at.ring;
    float *pr = region;
    float *ring = region + ((max_pos + 3) & ~3);
    const int nchunks = (n + kAttnPos - 1) / kAttnPos;
    const bool staged = nchunks <= R - 1;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int h = item / ns, d0 = (item % ns) * 32;
        const size_t vb = attn_voff(at, item);
        if (item != (int)blockIdx.x)  // the first item's first chunks were staged before the barrier
            for (int c = 0; c < R - 1; c++) {
                attn_stage(at, n, vb, ring, c);
                cp_async_commit();
            }
        const int n4 = (n + 3) / 4;
        const float4 *sc = (const float4 *)(at.scores + (size_t)h * at.score_stride);
        float m = -INFINITY;
        for (int i = tid; i < n4; i += nt) {
            const float4 v = __ldcg(sc + i);
            ((float4 *)pr)[i] = v;
            const int p = 4 * i;
            m = fmaxf(m, v.x);
            if (p + 1 < n) m = fmaxf(m, v.y);
            if (p + 2 < n) m = fmaxf(m, v.z);
            if (p + 3 < n) m = fmaxf(m, v.w);
        }
        if (staged) cp_async_wait<0>();  // the barrier below publishes every thread's V copies
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp] = m;
        dsync();
        float mx = red[0];
        for (int w = 1; w < kDW; w++) mx = fmaxf(mx, red[w]);
        float inv = 1.0f;
        if (!isfinite(mx)) {  // every score -inf (or NaN): uniform (src/ops.rs:1213-1218); u·1 = u
            const float u = __fdiv_rn(1.0f, (float)n);
            for (int i = tid; i < n; i += nt) pr[i] = u;
            dsync();
        } else {
            for (int i = tid; i < n4; i += nt) {
                const int p = 4 * i;
                float4 v = ((const float4 *)pr)[i];
                v.x = expf_glibc(fs(v.x, mx));
                if (p + 1 < n) v.y = expf_glibc(fs(v.y, mx));
                if (p + 2 < n) v.z = expf_glibc(fs(v.z, mx));
                if (p + 3 < n) v.w = expf_glibc(fs(v.w, mx));
                ((float4 *)pr)[i] = v;
            }
            dsync();
            if (tid == 0) *bc = __fdiv_rn(1.0f, seq_sum(pr, n));
            dsync();
            inv = *bc;
        }
        float acc = 0.0f;
        if (staged) {
            if (warp == 0)
                for (int c = 0; c < nchunks; c++)
                    pv_chunk(ring + (c % R) * kAttnChunkFloats + lane, pr + c * kAttnPos,
                             min(kAttnPos, n - c * kAttnPos), inv, acc);
        } else {
            for (int c = 0; c < nchunks; c++) {
                attn_stage(at, n, vb, ring, c + R - 1);
                cp_async_commit();
                cp_async_wait_n(R - 1);
                dsync();
                if (warp == 0)
                    pv_chunk(ring + (c % R) * kAttnChunkFloats + lane, pr + c * kAttnPos,
                             min(kAttnPos, n - c * kAttnPos), inv, acc);
                dsync();
            }
        }
        if (warp == 0) {
            at.out[(size_t)h * hd + d0 + lane] = acc;
            if (at.qout) attn_quant_out(at, h * hd + d0 + lane, acc);
        }
        cp_async_wait<0>();
        dsync();
    }
    cp_async_wait<0>();  // a CTA without an item drains its (empty) prefetch groups
}

// ── a warp's tile ring ──
struct Ring {
    unsigned char *base;
    uint32_t slot_bytes;
    int ns;
    uint32_t issued, consumed;
    int islot, cslot;  // slots of the next copy and of the next compute
    const FeedPhase *tab;  // the walk table, in shared memory
    int ntab;
    Feed feed;
};

// refill the slot freed last (keeping ns - 1 tiles in flight), then wait for
// the next tile in this warp's sequence and return its slot
__device__ __forceinline__ const unsigned char *ring_next(const DecodeArgs &A, Ring &R, int warp, int lane) {
    const uint8_t *src;
    uint32_t bytes;
    if (R.issued < R.consumed + (uint32_t)R.ns && feed_next(R.tab, R.ntab, R.feed, warp, src, bytes)) {
        issue_tile(R.base + (size_t)R.islot * R.slot_bytes, src, bytes, lane);
        R.issued++;
        if (++R.islot == R.ns) R.islot = 0;
    }
    cp_async_wait_n((int)(R.issued - R.consumed - 1));
    __syncwarp();
    const unsigned char *tile = R.base + (size_t)R.cslot * R.slot_bytes;
    R.consumed++;
    if (++R.cslot == R.ns) R.cslot = 0;
    return tile;
}

// the sub-block terms of this lane's super-block in a tile of L lanes (BUF:
// the buffered path's dot terms in tv and offset terms in sv)
template <int T, bool BUF>
__device__ __forceinline__ void tile_terms(const unsigned char *tile, int lane, int L, const XB &xb, float *tv,
                                           float *sv, bool *anyd) {
    const int cs = L * 16;
    const uint8_t *pa = tile + lane * 16;
    const uint8_t *pss = tile + a_chunks(T) * cs + lane * plane_s_bytes(T);
    const uint8_t *pd = tile + a_chunks(T) * cs + L * plane_s_bytes(T) + lane * plane_d_bytes(T);
    if (T == 12) block_k4<false, BUF>(pa, cs, xb, tv, sv, anyd);
    else if (T == 13) block_k4<true, BUF>(pa, cs, xb, tv, sv, anyd);
    else if (T == 14) block_q6k(pa, cs, pss, pd, xb, tv);
    else if (T == 11) block_q3k(pa, cs, pss, pd, xb, tv);
    else block_q2k<BUF>(pa, cs, pss, pd, xb, tv, sv, anyd);
}

__host__ __device__ constexpr bool has_minimum(int T) { return T == 12 || T == 13 || T == 10; }

// One row group (rpt = 32/lpr rows x nblk super-blocks) of type T: returns,
// in every lane, the total of row (lane mod rpt), each added term by term in
// block and sub-block order (the lane of block j holds its terms until the
// row's running total reaches it).
struct Lanes {  // a lane's place in this phase's tiles: lane = rpt*bl + sl
    int lpr, rpt, bl, sl, ntile;
};

// BUF (ORD_BUFFERED on a format with a minimum): the lanes also form each
// block's offset terms and spill them to `sv` (this warp's area:
// [row of the group][sub-block of the row]); after the row's dot chain, the
// row's lane adds them in sub-block order when any of the row's offsets is
// nonzero (src/ops.rs:395-401).
template <int T, bool BUF>
__device__ __forceinline__ float group_dot(const DecodeArgs &A, Ring &R, int warp, int lane, int nblk, const Lanes &g,
                                           const Act &act, float *sv) {
    constexpr bool S32 = (T == 12 || T == 13);
    constexpr int NSUB = S32 ? 8 : 16;
    const int lpr = g.lpr, rpt = g.rpt, bl = g.bl, sl = g.sl;
    const int8_t *xq = S32 ? act.q32 : act.q16;
    const float2 *xes = S32 ? act.es32 : act.es16;
    float acc = 0.0f;
    bool anyd = false;
    for (int t = 0; t < g.ntile; t++) {
        const unsigned char *tile = ring_next(A, R, warp, lane);
        const int nb = nblk - lpr * t < lpr ? nblk - lpr * t : lpr;
        float tv[NSUB];
        if (bl < nb) {
            const int b = lpr * t + bl;
            const XB xb{xq + b * kXqStride, xes + b * NSUB};
            if (BUF) {
                float svt[NSUB];
                tile_terms<T, true>(tile, lane, rpt * nb, xb, tv, svt, &anyd);
                float *dst = sv + (sl * nblk + b) * NSUB;
#pragma unroll
                for (int k = 0; k < NSUB; k++) dst[k] = svt[k];
            } else {
                tile_terms<T, false>(tile, lane, rpt * nb, xb, tv, nullptr, nullptr);
            }
        } else {
#pragma unroll
            for (int k = 0; k < NSUB; k++) tv[k] = 0.0f;  // a lane past the tile's last block: its sums are dropped
        }
        __syncwarp();  // the slot may be refilled from here on
        // each row's running total visits the tile's blocks in order: at hop
        // jb every lane adds its own terms to the total it was handed, and
        // the lane of block jb passes its result on (the others' results are
        // dropped), so no lane waits on a divergent branch
        float run = acc;
        for (int jb = 0; jb < nb; jb++) {
            float v = run;
#pragma unroll
            for (int k = 0; k < NSUB; k++) v = fa(v, tv[k]);
            run = __shfl_sync(0xffffffffu, v, jb * rpt + sl);
        }
        acc = run;
    }
    if (BUF) {
        // lanes of row sl: sl, sl + rpt, sl + 2 rpt, ...
        const uint32_t rows_of = rpt == 32 ? 1u : 0xFFFFFFFFu / ((1u << rpt) - 1u);
        const uint32_t any = __ballot_sync(0xffffffffu, anyd);
        __syncwarp();  // the spilled offset terms are visible to the row's lane
        if (lane < rpt && (any & (rows_of << sl))) {
            const float *src = sv + sl * nblk * NSUB;
            for (int i = 0; i < nblk * NSUB; i++) acc = fa(acc, src[i]);
        }
        __syncwarp();  // the next group may overwrite the spill
    }
    return acc;
}

// ── the kernel ──
__global__ void __launch_bounds__(kDecodeThreads, 1) k_decode(const __grid_constant__ DecodeArgs A) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    // aligned by an offset from the shared array itself (not a round trip
    // through an integer), so every pointer derived from it stays a
    // shared-memory pointer to the compiler
    unsigned char *smem = smem_raw + ((128u - ((uint32_t)(uintptr_t)smem_raw & 127u)) & 127u);
    const int ns = A.ring_slots;
    unsigned char *region = smem + (size_t)kDW * ns * A.slot_bytes;
    Phase *phbuf = (Phase *)(region + A.region_bytes);  // two staged phase descriptors
    FeedPhase *ftab = (FeedPhase *)(phbuf + 2);         // the walk table
    __shared__ __align__(8) uint64_t act_bar;  // the bulk copy of a quantize-only prologue's input
    __shared__ volatile int abort_flag;
    __shared__ int sync_ok;
    __shared__ double red[kDW];
    __shared__ unsigned long long best_s[kDW];
    __shared__ float fred[kDW];
    __shared__ float fbc;
    __shared__ int pos_s, tok_s, bad_s, stopped_s;
    __shared__ unsigned xbase_s;  // exchanges completed before this launch
    // deferred epilogues: (segment, unit, y0, y1) per output unit, per warp
    __shared__ int2 epi_su[kDW][32];
    __shared__ float2 epi_y[kDW][32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kDescWords = (int)(sizeof(Phase) / 16);
    if (tid == 0) {
        mbar_init(&act_bar, 1);
        abort_flag = 0;
        mbar_fence_init();
        // The step's position and token, read once here: thread 0 of every CTA
        // reads them before its first grid barrier, so before the commit of
        // CTA 0 (after the last barrier) rewrites them.
        int p = 0, bad = 0;
        uint32_t t = 0;
        if (A.d_len) {
            p = *(volatile int *)A.d_len;
            const bool pos_ok = p >= 0 && p < A.max_pos;
            t = pos_ok ? A.toks[p] : 0u;
            if (!pos_ok) bad = ERR_POSITION;
            else if (t >= (uint32_t)A.vocab) bad = ERR_TOKEN;
        }
        pos_s = p;
        tok_s = (int)t;
        bad_s = bad;
        // a generation that met its eos: read before the first grid barrier,
        // so before this launch's own commit can set it
        stopped_s = A.d_stop ? *(volatile int *)A.d_stop : 0;
        // read before the first grid barrier, so before CTA 0's commit updates it
        xbase_s = A.epoch ? *(volatile unsigned *)A.epoch : 0u;
    }
    if (blockIdx.x == 0 && A.qcnt)  // the hidden-vector sub-block counts start at zero every step
        for (int i = tid; i < A.nqcnt; i += kDecodeThreads) A.qcnt[i] = 0;
    if (tid < kDescWords) ((uint4 *)&phbuf[0])[tid] = __ldg((const uint4 *)&A.prog[0] + tid);
    for (int i = tid; i < A.nfeed * 4; i += kDecodeThreads) ((uint4 *)ftab)[i] = __ldg((const uint4 *)A.feed + i);
    __syncthreads();

    // an invalid position or token stops every CTA before any work; so does
    // a generation that already met its eos (src/forward.rs:544-547)
    const int pos = pos_s;
    const uint32_t tok = (uint32_t)tok_s;
    if (stopped_s) return;
    if (bad_s) {
        if (blockIdx.x == 0 && tid == 0) atomicOr(A.err, bad_s);
        return;
    }

    // this warp's tile ring, primed ns - 1 tiles ahead
    Ring R;
    R.base = smem + (size_t)warp * ns * A.slot_bytes;
    R.slot_bytes = A.slot_bytes;
    R.ns = ns;
    R.issued = R.consumed = 0;
    R.islot = R.cslot = 0;
    R.tab = ftab;
    R.ntab = A.nfeed;
    R.feed.m = 0;
    feed_phase(R.tab, R.ntab, R.feed, warp);
    {
        const uint8_t *src;
        uint32_t bytes;
        while (R.issued < (uint32_t)ns - 1 && feed_next(R.tab, R.ntab, R.feed, warp, src, bytes)) {
            issue_tile(R.base + (size_t)R.islot * R.slot_bytes, src, bytes, lane);
            R.issued++;
            if (++R.islot == ns) R.islot = 0;
        }
    }
    unsigned nbar = 0;
    uint32_t act_phase = 0;
    bool stop = false;
    for (int pi = 0; pi < A.nphase && !stop; pi++) {
        const Phase &ph = phbuf[pi & 1];
        uint4 nextd = make_uint4(0, 0, 0, 0);  // the next descriptor, stored at the end of this phase
        if (pi + 1 < A.nphase && tid < kDescWords) nextd = __ldg((const uint4 *)&A.prog[pi + 1] + tid);
        // a normed matvec's weights depend on nothing: loaded before the barrier
        NormW nw;
        if (ph.kind == PH_MATVEC && (ph.mv.prologue == PRO_NORM || ph.mv.prologue == PRO_EMBED)) load_norm_w(ph.mv, nw);
        const int n = pos + 1;
        // what an attention phase reads from before this step lands in shared
        // memory while the CTA waits at the barrier
        if (ph.kind == PH_SCORES) scores_prefetch(ph.at, n, (float *)region);
        else if (ph.kind == PH_ATTN) attn_prefetch(ph.at, n, A.max_pos, (float *)region);
        if (ph.barrier) {
            nbar++;
            if (!grid_sync(A, nbar * gridDim.x, &abort_flag, &sync_ok)) break;  // uniform
        }
        if (ph.kind == PH_MATVEC) {
            const MvPhase &P = ph.mv;
            const Act act = carve_act(region, P.K, P.need16, P.need32);
            if (P.prologue == PRO_EMBED && blockIdx.x == 0 && tid == 0 && A.argmax_key) *A.argmax_key = 0ull;
            if (P.prologue == PRO_COPYQ) {  // the whole quantized activation in one bulk copy
                const uint32_t nb = (uint32_t)act_bytes(P.K, P.need16, P.need32);
                if (tid == 0) {
                    // the region was last read through the generic proxy
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_expect_tx(&act_bar, nb);
                    bulk_g2s(region, P.in, nb, &act_bar);
                }
                const bool landed = mbar_wait_bounded(&act_bar, act_phase, &abort_flag);
                act_phase ^= 1u;
                if (!landed) abort_flag = 1;
            }
            float *stage = P.prologue == PRO_QUANT && P.K <= kMaxStaged
                               ? (float *)(region + act_bytes(P.K, P.need16, P.need32))
                               : nullptr;
            if (stage) {
                const uint32_t kbytes = (uint32_t)P.K * 4u;
                if (tid == 0) {
                    // the staging area was last read through the generic proxy
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_expect_tx(&act_bar, kbytes);
                    bulk_g2s(stage, P.in, kbytes, &act_bar);
                }
                const bool landed = mbar_wait_bounded(&act_bar, act_phase, &abort_flag);
                act_phase ^= 1u;
                if (!landed) abort_flag = 1;
            }
            if (P.prologue != PRO_COPYQ) quantize_act(P, tok, nw, stage, act, red);
            unsigned long long best = 0ull;
            int qb, qe;
            cta_groups(P.ngroup, qb, qe);
            Lanes g;
            g.lpr = P.seg[0].M.lpr;
            g.rpt = P.seg[0].M.rpt;
            const int lg = 31 - __clz(g.rpt);
            g.bl = lane >> lg;
            g.sl = lane & (g.rpt - 1);
            g.ntile = P.ntile;
            const int upg = g.rpt >> 1;  // output units per group
            int nepi = 0;
            // The epilogues run 32 units at a time, one per lane, so their
            // latency (exp, division, loads) is paid once per 32 units.
            auto flush = [&]() {
                __syncwarp();
                const int2 su = lane < nepi ? epi_su[warp][lane] : make_int2(0, -1);
                int r0 = 0, r1 = 0;
                if (su.y >= 0) {
                    const float2 y = epi_y[warp][lane];
                    const MvSeg &sg = P.seg[su.x];
                    unit_rows(sg, su.y, r0, r1);
                    const EpiIn ein = epi_load(A, sg, r0, r1, pos);
                    unit_epilogue(A, sg, r0, r1, y.x, y.y, pos, ein, best);
                }
                if (P.seg[0].qout) hidden_quant_arrive(P.seg[0], r0, su.y >= 0);  // uniform: one segment
                __syncwarp();
                nepi = 0;
            };
            // the segments' fields, in registers: the descriptor lives in shared
            // memory, which every asm memory clobber in the tile loop would
            // otherwise make the group loop load again
            const int nseg = P.nseg;
            const int sn0 = P.seg[0].M.ngroup, sn1 = nseg > 1 ? P.seg[1].M.ngroup : 0;
            const int sT0 = P.seg[0].M.type, sT1 = nseg > 1 ? P.seg[1].M.type : 0, sT2 = nseg > 2 ? P.seg[2].M.type : 0;
            const int sb0 = P.seg[0].M.nblk, sb1 = nseg > 1 ? P.seg[1].M.nblk : 0, sb2 = nseg > 2 ? P.seg[2].M.nblk : 0;
            const int su0 = P.seg[0].units, su1 = nseg > 1 ? P.seg[1].units : 0, su2 = nseg > 2 ? P.seg[2].units : 0;
            const int so0 = P.seg[0].ord, so1 = nseg > 1 ? P.seg[1].ord : 0, so2 = nseg > 2 ? P.seg[2].ord : 0;
            float *svw = (float *)(region + P.sv_off) + (size_t)warp * P.sv_warp;
            for (int q0 = qb + warp; q0 < qe; q0 += kDW) {
                // phase-global group index -> segment j, local group lq
                int j = 0, lq = q0;
                if (nseg > 1 && lq >= sn0) {
                    lq -= sn0;
                    j = 1;
                    if (nseg > 2 && lq >= sn1) {
                        lq -= sn1;
                        j = 2;
                    }
                }
                const int T = j == 0 ? sT0 : (j == 1 ? sT1 : sT2);
                const int nblk = j == 0 ? sb0 : (j == 1 ? sb1 : sb2);
                const int units = j == 0 ? su0 : (j == 1 ? su1 : su2);
                const int ord = j == 0 ? so0 : (j == 1 ? so1 : so2);
                float acc;
                // Q6_K and Q3_K have one order; Q5_K and Q2_K are buffered
                // whenever the reference's portable backend multiplies them
                switch (T) {
                case 12:
                    acc = ord == ORD_BUFFERED ? group_dot<12, true>(A, R, warp, lane, nblk, g, act, svw)
                                              : group_dot<12, false>(A, R, warp, lane, nblk, g, act, nullptr);
                    break;
                case 13: acc = group_dot<13, true>(A, R, warp, lane, nblk, g, act, svw); break;
                case 14: acc = group_dot<14, false>(A, R, warp, lane, nblk, g, act, nullptr); break;
                case 11: acc = group_dot<11, false>(A, R, warp, lane, nblk, g, act, nullptr); break;
                default: acc = group_dot<10, true>(A, R, warp, lane, nblk, g, act, svw); break;
                }
                // lanes 0..rpt-1 hold the group's row totals; an even one owns
                // the unit of rows (sl, sl+1)
                const float other = __shfl_down_sync(0xffffffffu, acc, 1);
                if (nepi + upg > 32) flush();
                const int u = (lq * g.rpt + g.sl) >> 1;
                if (lane < g.rpt && !(g.sl & 1) && u < units) {
                    epi_su[warp][nepi + (g.sl >> 1)] = make_int2(j, u);
                    epi_y[warp][nepi + (g.sl >> 1)] = make_float2(acc, other);
                }
                // units past the segment's end (zero rows of a padded group)
                // are left in place with their unit index and skipped below
                if (lane < g.rpt && !(g.sl & 1) && u >= units) epi_su[warp][nepi + (g.sl >> 1)] = make_int2(j, -1);
                nepi += upg;
            }
            if (nepi) flush();
            if (A.argmax_key && P.seg[0].epi == EPI_LOGITS) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
                    best = v > best ? v : best;
                }
                if (lane == 0) best_s[warp] = best;
                dsync();
                if (tid == 0) {
                    unsigned long long bb = 0;
                    for (int w = 0; w < kDW; w++) bb = best_s[w] > bb ? best_s[w] : bb;
                    if (bb) atomicMax(A.argmax_key, bb);
                }
            }
        } else if (ph.kind == PH_SCORES) {
            phase_scores(ph.at, n, (float *)region);
        } else if (ph.kind == PH_ATTN) {
            phase_attn(ph.at, n, A.max_pos, (float *)region, fred, &fbc);
        } else if (ph.kind == PH_XGATHER) {
            phase_xgather(A, ph.xp, xbase_s + (unsigned)ph.xp.seq, &abort_flag, &sync_ok);
        } else if (ph.kind == PH_XARGMAX) {
            phase_xargmax(A, xbase_s + (unsigned)ph.xp.seq, &abort_flag);
        } else if (ph.kind == PH_COMMIT) {
            if (blockIdx.x == 0 && tid == 0) {
                if (A.d_len) {
                    if (A.write_token && A.argmax_key && pos + 1 < A.max_pos + 1) {
                        const uint32_t pick = argmax_index(__ldcg(A.argmax_key));
                        A.toks[pos + 1] = pick;
                        if (A.d_stop && A.eos >= 0 && pick == (uint32_t)A.eos) *A.d_stop = 1;
                    }
                    if (A.commit) *(volatile int *)A.d_len = pos + 1;
                }
                if (A.epoch) *A.epoch = xbase_s + (unsigned)A.nx;
            }
        }
        stop = dsync_or(abort_flag != 0);  // every reader of this phase's descriptor is done
        if (pi + 1 < A.nphase && tid < kDescWords) ((uint4 *)&phbuf[(pi + 1) & 1])[tid] = nextd;
        dsync();
    }
    cp_async_wait<0>();  // tiles still in flight land before the CTA exits
    if (stop && tid == 0) atomicOr(A.err, ERR_TIMEOUT);
}

}  // namespace cxm
