// Definitions shared by the decode kernels, and the standalone kernels of the
// kernel-level entry points (attention on caller buffers, integer sub-block
// sums, exp). The per-token step itself is the persistent kernel of
// decode.cuh.
//
// Numerics: every float operation reproduces the reference's scalar
// specification in value AND order — per-sub-block terms summed sequentially
// per row, attention dot products, softmax sum and the probability-weighted
// value sum accumulated sequentially, and exp computed as the host libm
// computes it. On the random-init models of the benchmark a single 1-ulp
// difference flips an i8 activation rounding and moves the logits by more than
// the 1e-3 parity bar, so nothing less than identical rounding passes it.
#pragma once

#include "expf_glibc.h"
#include "kernels.cuh"
#include "pipeline.cuh"

namespace cxm {

// error flags written by kernels (never a trap); read by the host after sync
enum : int { ERR_TOKEN = 1, ERR_POSITION = 2, ERR_TIMEOUT = 4 };

enum Pairing : int {
    PAIR_ADJ = 0,   // unit u = rows (2u, 2u+1) of A
    PAIR_ROPE = 1,  // unit u = rows (h*hd + i, h*hd + i + hd/2) of A, for RoPE
    PAIR_TWO = 2    // unit u = row u of A and row u of B (gate, up)
};

enum Prologue : int {
    PRO_NORM = 0,   // RMSNorm then quantize (src/kernels/scalar.rs:36-54, src/ops.rs:178-198)
    PRO_QUANT = 1,  // quantize only
    PRO_EMBED = 2,  // embedding row of the step's token, then RMSNorm + quantize
    PRO_COPYQ = 3   // the activation arrives quantized (by the phase that produced it): one bulk copy
};

enum Epilogue : int {
    EPI_STORE = 0,     // out[r] = y (+ bias)
    EPI_ROPE = 1,      // bias, rotate the pair, store (q buffer, or K cache at pos)
    EPI_RESID = 2,     // out[r] += y (residual add, src/forward.rs:467-469)
    EPI_SWIGLU = 3,    // out[u] = silu(gate)·up (src/forward.rs:482-487)
    EPI_LOGITS = 4     // out[r] = y and the running argmax (src/sampler.rs:129-137)
};

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Orderable key of (value, index): larger value first, then smaller index.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_index(unsigned long long key) {
    return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// ── attention for one new token (src/ops.rs:1258-1325) in the reference's
// order, in two kernels over many SMs:
//   scores: score[h][p] = (sequential dot of q_h and k_p over the head dim)·scale
//   output: softmax over the head's scores (subtract the max, libm exp, sum the
//           exponentials position by position, multiply by 1/total;
//           src/ops.rs:1206-1230), then out[d] = Σ_p prob_p·v_p[d] added
//           position by position.
struct AttnParams {
    const float *q;      // [H*hd] per token, rotated
    const float *k, *v;  // layer base, [max_tokens][KV*hd]
    float *out;          // [H*hd] per token
    float *scores;       // scratch [H][score_stride] per token
    const int *d_len;    // position of the (first) token; NULL: pos0
    int H, KV, hd, max_pos, score_stride;
    float scale;
    int *err;
    // several consecutive tokens (grid z): token z at position pos + z reads
    // q + z·qs, writes out + z·os and its scores at scores + z·H·score_stride
    int pos0, qs, os;
    // a cache that borrows a shared prefix: its positions below plen are read
    // from the prefix's K/V (kp, vp: the prefix's layer base)
    const float *kp, *vp;
    int plen;
    // a batch of conversations (grid z = conversation; kz non-NULL): each
    // with its own layer bases, token position and prefix
    const float *const *kz, *const *vz, *const *kpz, *const *vpz;
    const int *posz, *plenz;
    // the output kernel's tokens per CTA (several only without kz: they
    // share the K/V rows) and the number of tokens
    int tpc, ntok;
};
// the grid-z slice's cache view: K/V bases, prefix, positions attended
struct AttnView {
    const float *k, *v, *kp, *vp;
    int plen, n;
};
__device__ __forceinline__ AttnView attn_view(const AttnParams &p) {
    const int z = (int)blockIdx.z;
    if (p.kz) return AttnView{p.kz[z], p.vz[z], p.kpz[z], p.vpz[z], p.plenz[z], p.posz[z] + 1};
    return AttnView{p.k, p.v, p.kp, p.vp, p.plen, (p.d_len ? *p.d_len : p.pos0) + 1 + z};
}
// the K (or V) row of position `pos`, `off` floats in (the head's slice)
__device__ __forceinline__ const float *kv_row(const float *own, const float *pre, int plen, int pos, size_t kvd,
                                               size_t off) {
    return (pos < plen ? pre : own) + (size_t)pos * kvd + off;
}

constexpr int kScoreThreads = 128;   // positions per score CTA
constexpr int kKRow = 132;           // smem row stride (floats) of staged K rows
constexpr int kOutThreads = 128;     // one thread per head dim (head_dim <= 128)

// One CTA per (token, KV head, 128 positions): the K rows of the positions
// are staged once for all the query heads of the group; thread = position,
// each score q_h·k a sequential sum over the dims (src/ops.rs), up to eight
// heads' chains side by side.
__global__ void __launch_bounds__(kScoreThreads) k_attn_scores(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float ks[];  // [kScoreThreads][kKRow] then q [G][hd]
    griddep_launch_dependents();
    griddep_wait();
    const int g = blockIdx.x, split = blockIdx.y, tid = threadIdx.x, z = blockIdx.z;
    const AttnView w = attn_view(p);
    const int n = w.n;
    if (n > p.max_pos || n <= 0) {
        if (tid == 0 && g == 0 && split == 0) atomicOr(p.err, ERR_POSITION);
        return;
    }
    const int p0 = split * kScoreThreads;
    if (p0 >= n) return;
    const int cnt = min(kScoreThreads, n - p0);
    const int hd = p.hd, G = p.H / p.KV, kvd = p.KV * hd, c4 = hd / 4;
    float *qs = ks + kScoreThreads * kKRow;
    // stage the group's q rows and the K rows of these positions: all 16-byte copies in flight
    for (int i = tid; i < G * c4; i += kScoreThreads) {
        const int hq = i / c4, c = i - hq * c4;
        cp_async16(qs + hq * hd + 4 * c, p.q + (size_t)z * p.qs + (size_t)(g * G + hq) * hd + 4 * c);
    }
    for (int i = tid; i < cnt * c4; i += kScoreThreads) {
        const int r = i / c4, c = i - r * c4;
        cp_async16(ks + r * kKRow + 4 * c, kv_row(w.k, w.kp, w.plen, p0 + r, kvd, (size_t)g * hd + 4 * c));
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid >= cnt) return;
    const float4 *kr = (const float4 *)(ks + tid * kKRow);
    for (int h0 = 0; h0 < G; h0 += 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = 0.0f;
        for (int c = 0; c < c4; c++) {
            const float4 kv = kr[c];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (h0 + j >= G) break;
                const float4 qv = ((const float4 *)(qs + (h0 + j) * hd))[c];
                acc[j] = fa(acc[j], fm(qv.x, kv.x));
                acc[j] = fa(acc[j], fm(qv.y, kv.y));
                acc[j] = fa(acc[j], fm(qv.z, kv.z));
                acc[j] = fa(acc[j], fm(qv.w, kv.w));
            }
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (h0 + j >= G) break;
            p.scores[((size_t)z * p.H + g * G + h0 + j) * p.score_stride + p0 + tid] = fm(acc[j], p.scale);
        }
    }
}

// One CTA per (head, tpc consecutive tokens): each token's softmax of the
// head's scores (a warp per token: max, exps, the total added position by
// position by one lane, ×1/total), then thread d adds prob_p·v_p[d] over the
// positions in order, one sequential chain per (token, dim), the tokens'
// chains side by side so each V value is read once for all of them. A warp
// reads 32 consecutive dims of a position (128 bytes) from L2, eight
// positions' loads in flight ahead of their additions.
constexpr int kOutTok = 8;  // tokens per CTA at most
// out[t][d] = Σ_p prob_t,p·v_p[d] for TT (or nt <= TT) tokens, position by
// position, V values loaded UB positions ahead of their additions
template <int TT, int UB>
__device__ __forceinline__ void attn_pv(const AttnParams &p, const AttnView &w, const float *pr, int stride, int n0, int nt,
                                        int kvd, size_t voff, int z0, int h, int hd, int tid) {
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; t++) acc[t] = 0.0f;
    const int nmax = n0 + nt - 1;
    int r = 0;
    for (; r + UB <= nmax; r += UB) {
        float v[UB];
#pragma unroll
        for (int k = 0; k < UB; k++) v[k] = __ldcg(kv_row(w.v, w.vp, w.plen, r + k, kvd, voff));
#pragma unroll
        for (int k = 0; k < UB; k++) {
#pragma unroll
            for (int t = 0; t < TT; t++)
                if (TT == 1 || (t < nt && r + k < n0 + t)) acc[t] = fa(acc[t], fm(pr[t * stride + r + k], v[k]));
        }
    }
    for (; r < nmax; r++) {
        const float v = __ldcg(kv_row(w.v, w.vp, w.plen, r, kvd, voff));
#pragma unroll
        for (int t = 0; t < TT; t++)
            if (TT == 1 || (t < nt && r < n0 + t)) acc[t] = fa(acc[t], fm(pr[t * stride + r], v));
    }
#pragma unroll
    for (int t = 0; t < TT; t++)
        if (t < nt) p.out[(size_t)(z0 + t) * p.os + (size_t)h * hd + tid] = acc[t];
}

__global__ void __launch_bounds__(kOutThreads) k_attn_out(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float pr[];  // the probabilities [tpc][max_pos rounded to 4]
    griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = p.kz ? 1 : p.tpc, z0 = (int)blockIdx.z * T, nt = min(T, p.ntok - z0);
    const AttnView w = attn_view(p);  // (z = blockIdx.z: with several tokens per CTA only its n differs)
    const int n0 = p.kz ? w.n : (p.d_len ? *p.d_len : p.pos0) + 1 + z0;  // positions of the first token
    const int stride = (p.max_pos + 3) & ~3;
    if (n0 + nt - 1 > p.max_pos || n0 <= 0) return;  // k_attn_scores reported it
    const int hd = p.hd, G = p.H / p.KV, g = h / G, kvd = p.KV * hd;
    for (int t = 0; t < nt; t++) {
        const float *sc = p.scores + ((size_t)(z0 + t) * p.H + h) * p.score_stride;
        for (int i = tid; i < (n0 + t + 3) / 4; i += kOutThreads) cp_async16(pr + t * stride + 4 * i, sc + 4 * i);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int t = warp; t < nt; t += kOutThreads / 32) {  // a warp per token
        float *q = pr + t * stride;
        const int n = n0 + t;
        float m = -INFINITY;
        for (int i = lane; i < n; i += 32) m = fmaxf(m, q[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (!isfinite(m)) {
            const float u = __fdiv_rn(1.0f, (float)n);
            for (int i = lane; i < n; i += 32) q[i] = u;
            continue;
        }
        for (int i = lane; i < n; i += 32) q[i] = expf_glibc(fs(q[i], m));
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) {  // the total in position order (src/ops.rs:1219-1223)
            float total = 0.0f;
            int i = 0;
            for (; i + 4 <= n; i += 4) {
                const float4 v = *(const float4 *)(q + i);
                total = fa(fa(fa(fa(total, v.x), v.y), v.z), v.w);
            }
            for (; i < n; i++) total = fa(total, q[i]);
            inv = __fdiv_rn(1.0f, total);
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int i = lane; i < n; i += 32) q[i] = fm(q[i], inv);
    }
    __syncthreads();
    if (tid >= hd) return;
    const size_t voff = (size_t)g * hd + tid;
    if (nt == 1) attn_pv<1, 16>(p, w, pr, stride, n0, 1, kvd, voff, z0, h, hd, tid);
    else attn_pv<kOutTok, 8>(p, w, pr, stride, n0, nt, kvd, voff, z0, h, hd, tid);
}

// ── kernel-level parity: integer sub-block sums of one row against an xq ──
__global__ void k_subblock_sums(DMat W, const int8_t *xq_g, int32_t *out) {
    extern __shared__ __align__(16) unsigned char smem[];
    int8_t *xq = (int8_t *)smem;
    for (int i = threadIdx.x; i < W.K; i += blockDim.x) xq[i] = xq_g[i];
    float *zero_e = (float *)(smem + ((W.K + 15) & ~15));
    float *zero_s = zero_e + W.K / 16;
    for (int i = threadIdx.x; i < W.K / 16; i += blockDim.x) {
        zero_e[i] = 0.0f;
        zero_s[i] = 0.0f;
    }
    __syncthreads();
    const XQ x{xq, zero_e, zero_s};
    for (int qt = threadIdx.x; qt < W.nblk * 4; qt += blockDim.x) {
        int is[4];
        float t[4];
        switch (W.type) {
        case 12: quarter<12>(W, 0, qt, x, t, is); break;
        case 13: quarter<13>(W, 0, qt, x, t, is); break;
        case 14: quarter<14>(W, 0, qt, x, t, is); break;
        case 11: quarter<11>(W, 0, qt, x, t, is); break;
        default: quarter<10>(W, 0, qt, x, t, is); break;
        }
        const int b = qt >> 2, q = qt & 3;
        for (int k = 0; k < terms_per_quarter(W.type); k++)
            out[b * subs_per_block(W.type) + term_sub(W.type, q, k)] = is[k];
    }
}

// ── expf parity probe: the device exp against the host libm ──
__global__ void k_expf(const float *x, float *y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = expf_glibc(x[i]);
}

}  // namespace cxm
