// The kernels of one decode step. Launched by model.cu, each step captured
// once into a CUDA graph and replayed; the position and the token are read
// from device memory so the same graph serves every step of a conversation.
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

namespace cxm {

constexpr int kThreads = 256;  // matvec CTA: 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kBatch = 8;          // row pairs per warp batch (16 sequential chains)
constexpr int kTileStride = 132;   // floats per row of a warp's term tile (128 terms + pad)
constexpr int kTileFloats = 2 * kBatch * kTileStride;

// error flags written by kernels (never a trap); read by the host after sync
enum : int { ERR_TOKEN = 1, ERR_POSITION = 2 };

enum Pairing : int {
    PAIR_ADJ = 0,   // unit u = rows (2u, 2u+1) of A
    PAIR_ROPE = 1,  // unit u = rows (h*hd + i, h*hd + i + hd/2) of A, for RoPE
    PAIR_TWO = 2    // unit u = row u of A and row u of B (gate, up)
};

enum Epilogue : int {
    EPI_STORE = 0,     // out[r] = y (+ bias)
    EPI_ROPE = 1,      // bias, rotate the pair, store (q buffer, or K cache at pos)
    EPI_RESID = 2,     // out[r] += y (residual add, src/forward.rs:467-469)
    EPI_SWIGLU = 3,    // out[u] = silu(gate)·up (src/forward.rs:482-487)
    EPI_LOGITS = 4     // out[r] = y and the running argmax (src/sampler.rs:129-137)
};

struct Seg {
    DMat A, B;
    int pairing, epi, units, half;
    const float *bias;
    float *out;
    int at_pos;      // out += pos * pos_stride (K/V cache rows)
    int pos_stride;
};

enum Prologue : int { PRO_NORM = 0, PRO_QUANT = 1 };

struct MatvecParams {
    Seg seg[3];
    int nseg, total_units;
    int K, prologue, need16, need32;
    const float *in, *norm_w;
    float eps;
    const int *d_len;
    int max_pos;
    const float *rope_cos, *rope_sin;
    unsigned long long *argmax_key;
    int *err;
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

// Activation quantization into shared memory, redundantly per CTA:
// optional RMSNorm (src/kernels/scalar.rs:36-54, f64 sum of squares), then
// i8 per sub-block of 16 and/or 32 (src/ops.rs:178-198).
__device__ void prologue_quantize(const MatvecParams &p, int8_t *xq16, float *xe16, float *xs16, int8_t *xq32,
                                  float *xe32, float *xs32, double *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.K;
    double scale = 0.0;
    if (p.prologue == PRO_NORM) {
        double acc = 0.0;
        for (int i = tid; i < K; i += blockDim.x) {
            double v = (double)p.in[i];
            acc = __dadd_rn(acc, __dmul_rn(v, v));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        if (tid == 0) {
            double s = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) s = __dadd_rn(s, red[w]);
            red[0] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s, (double)K), (double)p.eps)));
        }
        __syncthreads();
        scale = red[0];
    }
    const int nchunk = K >> 5;
    for (int c = warp; c < nchunk; c += (blockDim.x >> 5)) {
        const int i = c * 32 + lane;
        float v = p.in[i];
        if (p.prologue == PRO_NORM) v = __fmul_rn(__double2float_rn(__dmul_rn((double)v, scale)), p.norm_w[i]);
        const float av = fabsf(v);
        if (p.need32) {
            float amax = av;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            int qv = (int)roundf(__fmul_rn(v, inv));
            xq32[i] = (int8_t)qv;
            int s = warp_sum_i((int)(int8_t)qv);
            if (lane == 0) {
                xe32[c] = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
                xs32[c] = (float)s;
            }
        }
        if (p.need16) {
            float amax = av;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            int qv = (int)roundf(__fmul_rn(v, inv));
            xq16[i] = (int8_t)qv;
            int s = (int)(int8_t)qv;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if ((lane & 15) == 0) {
                xe16[2 * c + (lane >> 4)] = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
                xs16[2 * c + (lane >> 4)] = (float)s;
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ void quarter_any(const DMat &W, int row, int qt, const XQ &x, float *t) {
    switch (W.type) {
    case 12: quarter<12>(W, row, qt, x, t, nullptr); break;
    case 13: quarter<13>(W, row, qt, x, t, nullptr); break;
    case 14: quarter<14>(W, row, qt, x, t, nullptr); break;
    case 11: quarter<11>(W, row, qt, x, t, nullptr); break;
    default: quarter<10>(W, row, qt, x, t, nullptr); break;
    }
}

// Terms of quarter qt of rows r0 (of A) and r1 (of B), stored in the tile at
// their sub-block positions relative to the iteration's first block.
template <int T>
__device__ __forceinline__ void pair_terms(const DMat &A, int r0, const DMat &B, int r1, int qt, int it, const XQ &x,
                                           float *row0, float *row1) {
    float t0[4], t1[4];
    quarter<T>(A, r0, qt, x, t0, nullptr);
    quarter<T>(B, r1, qt, x, t1, nullptr);
    const int q = qt & 3, bl = (qt >> 2) - it * 8;
    constexpr int tpq = (T == 12 || T == 13) ? 2 : 4, spb = (T == 12 || T == 13) ? 8 : 16;
#pragma unroll
    for (int k = 0; k < tpq; k++) {
        const int pos = bl * spb + term_sub(T, q, k);
        row0[pos] = t0[k];
        row1[pos] = t1[k];
    }
}

struct Unit {
    int seg, r0, r1;
};

__device__ __forceinline__ Unit decode_unit(const MatvecParams &p, int u) {
    int s = 0;
    while (s < p.nseg - 1 && u >= p.seg[s].units) {
        u -= p.seg[s].units;
        s++;
    }
    const Seg &g = p.seg[s];
    Unit r;
    r.seg = s;
    if (g.pairing == PAIR_ADJ) {
        r.r0 = 2 * u;
        r.r1 = 2 * u + 1;
    } else if (g.pairing == PAIR_ROPE) {
        const int h = u / g.half, i = u - h * g.half;
        r.r0 = h * 2 * g.half + i;
        r.r1 = r.r0 + g.half;
    } else {
        r.r0 = u;
        r.r1 = u;
    }
    return r;
}

// k-quant matvec, several matrices per launch (q|k|v, gate|up), activation
// quantization fused in front and the consumer fused behind. A warp takes
// batches of up to 8 row pairs; per 32-quarter iteration its lanes produce the
// sub-block terms of every row into a shared-memory tile, then 16 lanes — one
// per row — add their row's terms in sub-block order onto a running f32 total.
__global__ void __launch_bounds__(kThreads) k_matvec(const __grid_constant__ MatvecParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = p.K;
    float *tiles = (float *)smem;
    int8_t *xq16 = (int8_t *)(tiles + kWarps * kTileFloats);
    int8_t *xq32 = xq16 + (p.need16 ? K : 0);
    float *xe16 = (float *)(xq32 + (p.need32 ? K : 0));
    float *xs16 = xe16 + (p.need16 ? K / 16 : 0);
    float *xe32 = xs16 + (p.need16 ? K / 16 : 0);
    float *xs32 = xe32 + (p.need32 ? K / 32 : 0);
    __shared__ double red[kWarps];
    __shared__ unsigned long long best_s[kWarps];

    prologue_quantize(p, xq16, xe16, xs16, xq32, xe32, xs32, red);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gwarp = blockIdx.x * kWarps + warp, nwarps = gridDim.x * kWarps;
    const int pos = p.d_len ? *p.d_len : 0;
    const int nq = (K / 256) * 4;
    float *tile = tiles + warp * kTileFloats;
    const XQ x16{xq16, xe16, xs16}, x32{xq32, xe32, xs32};
    unsigned long long best = 0ull;

    for (int k0 = 0;; k0 += kBatch) {
        const int first = gwarp + k0 * nwarps;
        if (first >= p.total_units) break;
        const int nb = min(kBatch, (p.total_units - first + nwarps - 1) / nwarps);
        // lane L < 2*nb owns the chain of row slot L (unit L/2, row L%2)
        int my_type = 0;
        if (lane < 2 * nb) {
            const Unit mu = decode_unit(p, first + (lane >> 1) * nwarps);
            const Seg &mg = p.seg[mu.seg];
            my_type = (lane & 1) && mg.pairing == PAIR_TWO ? mg.B.type : mg.A.type;
        }
        float total = 0.0f;
        for (int it = 0; it * 32 < nq; it++) {
            const int qt = it * 32 + lane;
            for (int j = 0; j < nb; j++) {
                const Unit un = decode_unit(p, first + j * nwarps);
                const Seg &g = p.seg[un.seg];
                const DMat &A = g.A;
                const DMat &B = (g.pairing == PAIR_TWO) ? g.B : g.A;
                float *row0 = tile + (2 * j) * kTileStride, *row1 = row0 + kTileStride;
                if (qt < nq) {
                    const XQ &xa = (A.type == 12 || A.type == 13) ? x32 : x16;
                    if (A.type == B.type) {
                        switch (A.type) {
                        case 12: pair_terms<12>(A, un.r0, B, un.r1, qt, it, xa, row0, row1); break;
                        case 13: pair_terms<13>(A, un.r0, B, un.r1, qt, it, xa, row0, row1); break;
                        case 14: pair_terms<14>(A, un.r0, B, un.r1, qt, it, xa, row0, row1); break;
                        case 11: pair_terms<11>(A, un.r0, B, un.r1, qt, it, xa, row0, row1); break;
                        default: pair_terms<10>(A, un.r0, B, un.r1, qt, it, xa, row0, row1); break;
                        }
                    } else {
                        const XQ &xb = (B.type == 12 || B.type == 13) ? x32 : x16;
                        float t0[4], t1[4];
                        quarter_any(A, un.r0, qt, xa, t0);
                        quarter_any(B, un.r1, qt, xb, t1);
                        const int q = qt & 3, bl = (qt >> 2) - it * 8;
                        for (int k = 0; k < terms_per_quarter(A.type); k++)
                            row0[bl * subs_per_block(A.type) + term_sub(A.type, q, k)] = t0[k];
                        for (int k = 0; k < terms_per_quarter(B.type); k++)
                            row1[bl * subs_per_block(B.type) + term_sub(B.type, q, k)] = t1[k];
                    }
                }
            }
            __syncwarp();
            if (lane < 2 * nb) {
                const int blocks = min(8, (nq - it * 32) >> 2);
                const int nterms = blocks * subs_per_block(my_type);
                const float4 *src = (const float4 *)(tile + lane * kTileStride);
                for (int c = 0; c < (nterms >> 2); c++) {
                    const float4 v = src[c];
                    total = fa(fa(fa(fa(total, v.x), v.y), v.z), v.w);
                }
            }
            __syncwarp();
        }
        const float other = __shfl_down_sync(0xffffffffu, total, 1);
        if (lane < 2 * nb && !(lane & 1)) {
            const Unit un = decode_unit(p, first + (lane >> 1) * nwarps);
            const Seg &g = p.seg[un.seg];
            const int r0 = un.r0, r1 = un.r1;
            float y0 = total, y1 = other;
            if (!(g.at_pos && (pos < 0 || pos >= p.max_pos))) {
                float *out = g.out + (g.at_pos ? (size_t)pos * g.pos_stride : 0);
                switch (g.epi) {
                case EPI_STORE:
                    if (g.bias) {
                        y0 = fa(y0, g.bias[r0]);
                        y1 = fa(y1, g.bias[r1]);
                    }
                    out[r0] = y0;
                    out[r1] = y1;
                    break;
                case EPI_ROPE: {
                    // src/ops.rs:1150-1193, split-half pair (i, i + hd/2) at pos
                    const int i = r0 % (2 * g.half);
                    const float c = p.rope_cos[(size_t)pos * g.half + i], sn = p.rope_sin[(size_t)pos * g.half + i];
                    const float a = fa(y0, g.bias[r0]), b = fa(y1, g.bias[r1]);
                    out[r0] = fs(fm(a, c), fm(b, sn));
                    out[r1] = fa(fm(a, sn), fm(b, c));
                    break;
                }
                case EPI_RESID:
                    out[r0] = fa(out[r0], y0);
                    out[r1] = fa(out[r1], y1);
                    break;
                case EPI_SWIGLU: {
                    // src/kernels/scalar.rs:63-67 then `*a *= u`
                    const float act = __fdiv_rn(y0, fa(1.0f, expf_glibc(-y0)));
                    out[r0] = fm(act, y1);
                    break;
                }
                case EPI_LOGITS: {
                    out[r0] = y0;
                    out[r1] = y1;
                    unsigned long long ka = (y0 == y0) ? argmax_key(y0, (uint32_t)r0) : 0ull;
                    unsigned long long kb = (y1 == y1) ? argmax_key(y1, (uint32_t)r1) : 0ull;
                    unsigned long long kk = ka > kb ? ka : kb;
                    best = kk > best ? kk : best;
                    break;
                }
                }
            }
        }
    }
    if (p.argmax_key) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if (lane == 0) best_s[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = 0;
            for (int w = 0; w < kWarps; w++) b = best_s[w] > b ? best_s[w] : b;
            if (b) atomicMax(p.argmax_key, b);
        }
    }
}

// ── attention for one new token (src/ops.rs:1258-1325), one CTA per query
// head, in the reference's order: each score is the sequential dot over the
// head dimension times 1/sqrt(hd); softmax subtracts the max, exponentiates,
// adds the exponentials position by position and multiplies by 1/total
// (src/ops.rs:1206-1230); the output adds p·v position by position per dim.
struct AttnParams {
    const float *q;      // [H*hd], rotated
    const float *k, *v;  // layer base, [max_tokens][KV*hd]
    float *out;          // [H*hd]
    const int *d_len;
    int H, KV, hd, max_pos;
    float scale;
    int *err;
};

constexpr int kAttnThreads = 512;

__global__ void __launch_bounds__(kAttnThreads) k_attention(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const int h = blockIdx.x, G = p.H / p.KV, g = h / G, hd = p.hd, tid = threadIdx.x;
    const int n = *p.d_len + 1;
    if (n > p.max_pos || n <= 0) {
        if (tid == 0 && h == 0) atomicOr(p.err, ERR_POSITION);
        return;
    }
    const int kvd = p.KV * hd;
    float *qs = sm;              // [hd]
    float *sc = sm + hd;         // [n]
    __shared__ float red[kAttnThreads / 32];
    __shared__ float bcast;
    for (int i = tid; i < hd; i += kAttnThreads) qs[i] = p.q[(size_t)h * hd + i];
    __syncthreads();
    const float4 *q4 = (const float4 *)qs;
    for (int pp = tid; pp < n; pp += kAttnThreads) {
        const float4 *kr = (const float4 *)(p.k + (size_t)pp * kvd + (size_t)g * hd);
        float acc = 0.0f;
        for (int c = 0; c < hd / 4; c++) {
            const float4 kv = __ldg(kr + c), qv = q4[c];
            acc = fa(acc, fm(qv.x, kv.x));
            acc = fa(acc, fm(qv.y, kv.y));
            acc = fa(acc, fm(qv.z, kv.z));
            acc = fa(acc, fm(qv.w, kv.w));
        }
        sc[pp] = fm(acc, p.scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int i = tid; i < n; i += kAttnThreads) m = fmaxf(m, sc[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < kAttnThreads / 32; w++) mm = fmaxf(mm, red[w]);
        bcast = mm;
    }
    __syncthreads();
    const float mx = bcast;
    if (!isfinite(mx)) {
        const float u = __fdiv_rn(1.0f, (float)n);
        for (int i = tid; i < n; i += kAttnThreads) sc[i] = u;
    } else {
        for (int i = tid; i < n; i += kAttnThreads) sc[i] = expf_glibc(fs(sc[i], mx));
        __syncthreads();
        if (tid == 0) {
            float total = 0.0f;
            int i = 0;
            for (; i + 4 <= n; i += 4) {
                const float4 v = *(const float4 *)(sc + i);
                total = fa(fa(fa(fa(total, v.x), v.y), v.z), v.w);
            }
            for (; i < n; i++) total = fa(total, sc[i]);
            bcast = __fdiv_rn(1.0f, total);
        }
        __syncthreads();
        const float inv = bcast;
        for (int i = tid; i < n; i += kAttnThreads) sc[i] = fm(sc[i], inv);
    }
    __syncthreads();
    for (int d = tid; d < hd; d += kAttnThreads) {
        const float *vb = p.v + (size_t)g * hd + d;
        float acc = 0.0f;
        int pp = 0;
        for (; pp + 4 <= n; pp += 4) {
            const float v0 = __ldg(vb + (size_t)pp * kvd), v1 = __ldg(vb + (size_t)(pp + 1) * kvd);
            const float v2 = __ldg(vb + (size_t)(pp + 2) * kvd), v3 = __ldg(vb + (size_t)(pp + 3) * kvd);
            acc = fa(acc, fm(sc[pp], v0));
            acc = fa(acc, fm(sc[pp + 1], v1));
            acc = fa(acc, fm(sc[pp + 2], v2));
            acc = fa(acc, fm(sc[pp + 3], v3));
        }
        for (; pp < n; pp++) acc = fa(acc, fm(sc[pp], __ldg(vb + (size_t)pp * kvd)));
        p.out[(size_t)h * hd + d] = acc;
    }
}

// ── embedding row (src/forward.rs:389-405): x = dequant(token_embd[tok]) ──
struct EmbedParams {
    DMat E;
    const float *e32;      // F32 table (when E.type == 0)
    const uint32_t *toks;
    const int *d_len;
    int dim, vocab, max_pos;
    float *x;
    unsigned long long *argmax_key;
    int *err;
};

__global__ void k_embed(const __grid_constant__ EmbedParams p) {
    const int pos = *p.d_len;
    if (pos >= p.max_pos) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, ERR_POSITION);
        return;
    }
    const uint32_t tok = p.toks[pos];
    if (tok >= (uint32_t)p.vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, ERR_TOKEN);
        return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && p.argmax_key) *p.argmax_key = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.dim; i += gridDim.x * blockDim.x)
        p.x[i] = p.E.type == 0 ? p.e32[(size_t)tok * p.dim + i] : dequant_value(p.E, (int)tok, i);
}

// ── end of step: append the chosen token, advance the position ──
__global__ void k_commit(int *d_len, uint32_t *toks, const unsigned long long *argmax_key, int write_token,
                         int max_pos) {
    if (threadIdx.x || blockIdx.x) return;
    const int len = *d_len;
    if (write_token && argmax_key && len + 1 < max_pos) toks[len + 1] = argmax_index(*argmax_key);
    *d_len = len + 1;
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
