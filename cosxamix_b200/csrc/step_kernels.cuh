// The kernels of one decode step. Launched by model.cu, each step captured
// once into a CUDA graph and replayed; the position and the token are read
// from device memory so the same graph serves every step of a conversation.
#pragma once

#include "kernels.cuh"

namespace cxm {

constexpr int kThreads = 256;  // matvec CTA: 8 warps
constexpr int kWarps = kThreads / 32;

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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
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
            acc += v * v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        if (tid == 0) {
            double s = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
            red[0] = 1.0 / sqrt(s / (double)K + (double)p.eps);
        }
        __syncthreads();
        scale = red[0];
    }
    const int nchunk = K >> 5;
    for (int c = warp; c < nchunk; c += (blockDim.x >> 5)) {
        const int i = c * 32 + lane;
        float v = p.in[i];
        if (p.prologue == PRO_NORM) v = __fmul_rn((float)((double)v * scale), p.norm_w[i]);
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

template <int T>
__device__ __forceinline__ void pair_dot(const DMat &A, int r0, const DMat &B, int r1, int lane, const XQ &x,
                                         float &y0, float &y1) {
    const int nq = A.nblk * 4;
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 2
    for (int qt = lane; qt < nq; qt += 32) {
        float t0 = quarter<T>(A, r0, qt, x, nullptr);
        float t1 = quarter<T>(B, r1, qt, x, nullptr);
        a0 += t0;
        a1 += t1;
    }
    y0 = a0;
    y1 = a1;
}

__device__ __forceinline__ float row_dot_any(const DMat &W, int r, int lane, const XQ &x) {
    const int nq = W.nblk * 4;
    float a = 0.0f;
    for (int qt = lane; qt < nq; qt += 32) {
        switch (W.type) {
        case 12: a += quarter<12>(W, r, qt, x, nullptr); break;
        case 13: a += quarter<13>(W, r, qt, x, nullptr); break;
        case 14: a += quarter<14>(W, r, qt, x, nullptr); break;
        case 11: a += quarter<11>(W, r, qt, x, nullptr); break;
        default: a += quarter<10>(W, r, qt, x, nullptr); break;
        }
    }
    return a;
}

__global__ void __launch_bounds__(kThreads) k_matvec(const __grid_constant__ MatvecParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = p.K;
    int8_t *xq16 = (int8_t *)smem;
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
    unsigned long long best = 0ull;

    for (int u = gwarp; u < p.total_units; u += nwarps) {
        int s = 0, uu = u;
        while (s < p.nseg - 1 && uu >= p.seg[s].units) {
            uu -= p.seg[s].units;
            s++;
        }
        const Seg &g = p.seg[s];
        int r0, r1;
        if (g.pairing == PAIR_ADJ) {
            r0 = 2 * uu;
            r1 = 2 * uu + 1;
        } else if (g.pairing == PAIR_ROPE) {
            const int h = uu / g.half, i = uu - h * g.half;
            r0 = h * 2 * g.half + i;
            r1 = r0 + g.half;
        } else {
            r0 = uu;
            r1 = uu;
        }
        const DMat &A = g.A;
        const DMat &B = (g.pairing == PAIR_TWO) ? g.B : g.A;
        const int sub = (A.type == 12 || A.type == 13) ? 32 : 16;
        const XQ x = sub == 32 ? XQ{xq32, xe32, xs32} : XQ{xq16, xe16, xs16};
        float y0, y1;
        if (A.type == B.type) {
            switch (A.type) {
            case 12: pair_dot<12>(A, r0, B, r1, lane, x, y0, y1); break;
            case 13: pair_dot<13>(A, r0, B, r1, lane, x, y0, y1); break;
            case 14: pair_dot<14>(A, r0, B, r1, lane, x, y0, y1); break;
            case 11: pair_dot<11>(A, r0, B, r1, lane, x, y0, y1); break;
            default: pair_dot<10>(A, r0, B, r1, lane, x, y0, y1); break;
            }
        } else {
            const int subB = (B.type == 12 || B.type == 13) ? 32 : 16;
            const XQ xb = subB == 32 ? XQ{xq32, xe32, xs32} : XQ{xq16, xe16, xs16};
            y0 = row_dot_any(A, r0, lane, x);
            y1 = row_dot_any(B, r1, lane, xb);
        }
        y0 = warp_sum(y0);
        y1 = warp_sum(y1);
        if (lane == 0 && !(g.at_pos && (pos < 0 || pos >= p.max_pos))) {
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
                const float act = __fdiv_rn(y0, fa(1.0f, expf(-y0)));
                out[r0] = fm(act, y1);
                break;
            }
            case EPI_LOGITS: {
                out[r0] = y0;
                out[r1] = y1;
                unsigned long long k0 = (y0 == y0) ? argmax_key(y0, (uint32_t)r0) : 0ull;
                unsigned long long k1 = (y1 == y1) ? argmax_key(y1, (uint32_t)r1) : 0ull;
                unsigned long long k = k0 > k1 ? k0 : k1;
                best = k > best ? k : best;
                break;
            }
            }
        }
    }
    if (p.argmax_key) {
        if (lane == 0) best_s[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = 0;
            for (int w = 0; w < kWarps; w++) b = best_s[w] > b ? best_s[w] : b;
            if (b) atomicMax(p.argmax_key, b);
        }
    }
}

// ── split-K flash-decode attention (src/ops.rs:1258-1325 for one new token)
// grid (n_head_kv, S_max): CTA (g, s) handles positions [s*P, min((s+1)*P, n))
// for the G = H/KV query heads of kv head g, writes (m, l, o) partials, and
// the last CTA of each kv head to arrive merges them. n = *d_len + 1.
struct AttnParams {
    const float *q;   // [H*hd], rotated
    const float *k, *v;  // layer base, [max_tokens][KV*hd]
    float *out;       // [H*hd]
    float *part;      // [H][S_max][hd + 2]
    int *counter;     // [KV], zero between launches
    const int *d_len;
    int H, KV, P, S_max, max_pos;
    float scale;
    int *err;
};

constexpr int kAttnThreads = 128;
constexpr int kGMax = 8;

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attention(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const int G = p.H / p.KV, kvh = blockIdx.x, s = blockIdx.y;
    const int n = *p.d_len + 1;
    if (n > p.max_pos) {
        if (threadIdx.x == 0 && s == 0 && kvh == 0) atomicOr(p.err, ERR_POSITION);
        return;
    }
    const int nsplit = (n + p.P - 1) / p.P;
    if (s >= nsplit) return;
    const int start = s * p.P, cnt = min(p.P, n - start);
    const int kvd = p.KV * HD;
    float *qs = sm;                  // [G][HD]
    float *sc = qs + G * HD;         // [G][P]
    float *red = sc + G * p.P;       // [G][2] (m, l)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < G * HD; i += kAttnThreads) qs[i] = p.q[(size_t)kvh * G * HD + i];
    __syncthreads();

    // scores: C lanes per position, 4 dims each
    constexpr int C = HD / 4, PPW = 32 / C;
    const int pl = lane / C, c = lane % C;
    const float *kb = p.k + (size_t)kvh * HD;
    for (int p0 = warp * PPW; p0 < cnt; p0 += (kAttnThreads / 32) * PPW) {
        const int pp = p0 + pl;
        const bool valid = pp < cnt;
        float4 kv4 = valid ? __ldg((const float4 *)(kb + (size_t)(start + pp) * kvd) + c) : make_float4(0, 0, 0, 0);
        for (int g = 0; g < G; g++) {
            float4 q4 = ((const float4 *)(qs + g * HD))[c];
            float part = q4.x * kv4.x + q4.y * kv4.y + q4.z * kv4.z + q4.w * kv4.w;
#pragma unroll
            for (int o = C / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (c == 0 && valid) sc[g * p.P + pp] = fm(part, p.scale);
        }
    }
    __syncthreads();
    // softmax numerators per head (src/ops.rs:1206-1230: subtract the max, exp)
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int i = lane; i < cnt; i += 32) m = fmaxf(m, sc[g * p.P + i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int i = lane; i < cnt; i += 32) {
            float e = expf(sc[g * p.P + i] - m);
            sc[g * p.P + i] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            red[2 * g] = m;
            red[2 * g + 1] = l;
        }
    }
    __syncthreads();
    // o = Σ e·v ; TPD threads share one dim over interleaved positions
    constexpr int TPD = kAttnThreads / HD;
    const int d = tid % HD, pg = tid / HD;
    const float *vb = p.v + (size_t)kvh * HD + d;
    float acc[kGMax];
    float *accs = sc + G * p.P + 2 * G + 8;  // [TPD][G][HD] reduction scratch (TPD > 1)
    for (int g0 = 0; g0 < G; g0 += kGMax) {
        const int gn = min(kGMax, G - g0);
#pragma unroll
        for (int j = 0; j < kGMax; j++) acc[j] = 0.0f;
        for (int i = pg; i < cnt; i += TPD) {
            const float vv = __ldg(vb + (size_t)(start + i) * kvd);
#pragma unroll
            for (int j = 0; j < kGMax; j++)
                if (j < gn) acc[j] += sc[(g0 + j) * p.P + i] * vv;
        }
        if (TPD > 1) {
#pragma unroll
            for (int j = 0; j < kGMax; j++)
                if (j < gn) accs[(pg * kGMax + j) * HD + d] = acc[j];
            __syncthreads();
            if (pg == 0) {
                for (int t = 1; t < TPD; t++)
#pragma unroll
                    for (int j = 0; j < kGMax; j++)
                        if (j < gn) acc[j] += accs[(t * kGMax + j) * HD + d];
            }
            __syncthreads();
        }
        if (pg == 0) {
            for (int j = 0; j < gn; j++) {
                const int h = kvh * G + g0 + j;
                float *pp = p.part + ((size_t)h * p.S_max + s) * (HD + 2);
                pp[d] = acc[j];
                if (d == 0) {
                    pp[HD] = red[2 * (g0 + j)];
                    pp[HD + 1] = red[2 * (g0 + j) + 1];
                }
            }
        }
    }
    // last CTA of this kv head merges the splits
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(p.counter + kvh, 1) == nsplit - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < G * HD; i += kAttnThreads) {
        const int g = i / HD, dd = i % HD, h = kvh * G + g;
        const float *base = p.part + (size_t)h * p.S_max * (HD + 2);
        float M = -INFINITY;
        for (int t = 0; t < nsplit; t++) M = fmaxf(M, __ldcg(base + (size_t)t * (HD + 2) + HD));
        float L = 0.0f, o = 0.0f;
        for (int t = 0; t < nsplit; t++) {
            const float *pp = base + (size_t)t * (HD + 2);
            const float w = expf(__ldcg(pp + HD) - M);
            L += __ldcg(pp + HD + 1) * w;
            o += __ldcg(pp + dd) * w;
        }
        p.out[(size_t)h * HD + dd] = o / L;
    }
    if (tid == 0) p.counter[kvh] = 0;
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

// ── kernel-level parity: integer sub-block sums of rows against an xq ──
__global__ void k_subblock_sums(DMat W, const int8_t *xq_g, int32_t *out) {
    extern __shared__ __align__(16) unsigned char smem[];
    int8_t *xq = (int8_t *)smem;
    for (int i = threadIdx.x; i < W.K; i += blockDim.x) xq[i] = xq_g[i];
    __syncthreads();
    const int sub = (W.type == 12 || W.type == 13) ? 32 : 16;
    const int per_quarter = 64 / sub;
    XQ x{xq, nullptr, nullptr};
    // one thread per quarter; the float part is not needed
    float *dummy_e = (float *)(smem + ((W.K + 15) & ~15));
    float *dummy_s = dummy_e + W.K / 16;
    for (int i = threadIdx.x; i < W.K / 16; i += blockDim.x) {
        dummy_e[i] = 0.0f;
        dummy_s[i] = 0.0f;
    }
    __syncthreads();
    x.e = dummy_e;
    x.s = dummy_s;
    for (int qt = threadIdx.x; qt < W.nblk * 4; qt += blockDim.x) {
        int is[4];
        switch (W.type) {
        case 12: quarter<12>(W, 0, qt, x, is); break;
        case 13: quarter<13>(W, 0, qt, x, is); break;
        case 14: quarter<14>(W, 0, qt, x, is); break;
        case 11: quarter<11>(W, 0, qt, x, is); break;
        default: quarter<10>(W, 0, qt, x, is); break;
        }
        const int b = qt >> 2, q = qt & 3;
        if (sub == 32) {
            out[b * 8 + 2 * q] = is[0];
            out[b * 8 + 2 * q + 1] = is[1];
        } else if (W.type == 14) {
            // quarter q of Q6_K covers groups 4h+par and 4h+par+2
            const int h = q >> 1, par = q & 1, glo = 4 * h + par, ghi = glo + 2;
            out[b * 16 + 2 * glo] = is[0];
            out[b * 16 + 2 * glo + 1] = is[1];
            out[b * 16 + 2 * ghi] = is[2];
            out[b * 16 + 2 * ghi + 1] = is[3];
        } else {
            for (int k = 0; k < 4; k++) out[b * 16 + 4 * q + k] = is[k];
        }
        (void)per_quarter;
    }
}

}  // namespace cxm
