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
#include "pipeline.cuh"

namespace cxm {

// error flags written by kernels (never a trap); read by the host after sync
enum : int { ERR_TOKEN = 1, ERR_POSITION = 2, ERR_TIMEOUT = 4 };

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

// ── matvec geometry ──
constexpr int kCW = 8;                          // consumer warps
constexpr int kMvThreads = (kCW + 1) * 32;      // + one producer warp
constexpr int kStages = 3;                      // smem ring depth
constexpr int kSlots = 32;                      // row slots per stage (16 row pairs)
constexpr int kChunk = 8;                       // super-blocks per stage (2048 values)
// slot strides padded so the 8 lanes of a shared-memory phase hit distinct banks
constexpr int kSlotA = kChunk * 192 + 32, kSlotS = kChunk * 16 + 32, kSlotD = kChunk * 4;
constexpr int kStageA = kSlots * kSlotA, kStageS = kSlots * kSlotS, kStageD = kSlots * kSlotD;
constexpr int kStageBytes = kStageA + kStageS + kStageD;  // 55 KB
constexpr int kSlotsPerWarp = kSlots / kCW;     // 4

__host__ __device__ inline size_t matvec_act_bytes(int K, int need16, int need32) {
    size_t b = 0;
    if (need16) b += (size_t)(K / 256) * kXqStride + (size_t)K / 16 * 8;
    if (need32) b += (size_t)(K / 256) * kXqStride + (size_t)K / 32 * 8;
    return (b + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t matvec_smem_bytes(int K, int need16, int need32) {
    return (size_t)kStages * kStageBytes + matvec_act_bytes(K, need16, need32) + 128;
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory"); }

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

// Activation quantization into shared memory, redundantly per CTA, by the
// consumer warps: optional RMSNorm (src/kernels/scalar.rs:36-54, f64 sum of
// squares), then i8 per sub-block of 16 and/or 32 (src/ops.rs:178-198).
__device__ void prologue_quantize(const MatvecParams &p, int8_t *xq16, float *xe16, float *xs16, int8_t *xq32,
                                  float *xe32, float *xs32, double *red, double *scale_s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = kCW * 32;
    const int K = p.K;
    double scale = 0.0;
    if (p.prologue == PRO_NORM) {
        // sum of squares: 16-byte loads, 4 in flight per thread
        const float4 *in4 = (const float4 *)p.in;
        const int K4 = K >> 2;
        double acc = 0.0;
        for (int i0 = tid; i0 < K4; i0 += 4 * nt) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = (i0 + u * nt < K4) ? in4[i0 + u * nt] : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const double a = v[u].x, b = v[u].y, c = v[u].z, d = v[u].w;
                acc = __dadd_rn(acc, __dmul_rn(a, a));
                acc = __dadd_rn(acc, __dmul_rn(b, b));
                acc = __dadd_rn(acc, __dmul_rn(c, c));
                acc = __dadd_rn(acc, __dmul_rn(d, d));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[warp] = acc;
        consumers_sync();
        if (tid == 0) {
            double s = 0.0;
            for (int w = 0; w < kCW; w++) s = __dadd_rn(s, red[w]);
            *scale_s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s, (double)K), (double)p.eps)));
        }
        consumers_sync();
        scale = *scale_s;
    }
    // quantize: a warp per 32-value chunk, 8 chunks' loads in flight per lane
    const int nchunk = K >> 5;
    for (int c0 = warp; c0 < nchunk; c0 += 8 * kCW) {
        float vals[8], ws[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int c = c0 + u * kCW;
            vals[u] = c < nchunk ? p.in[c * 32 + lane] : 0.0f;
            ws[u] = (c < nchunk && p.prologue == PRO_NORM) ? p.norm_w[c * 32 + lane] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int c = c0 + u * kCW;
            if (c >= nchunk) break;
            const int i = c * 32 + lane;
            float v = vals[u];
            if (p.prologue == PRO_NORM) v = __fmul_rn(__double2float_rn(__dmul_rn((double)v, scale)), ws[u]);
            const float av = fabsf(v);
            if (p.need32) {
                float amax = av;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                const int qv = (int)roundf(__fmul_rn(v, inv));
                xq32[(i >> 8) * kXqStride + (i & 255)] = (int8_t)qv;
                const int s = warp_sum_i((int)(int8_t)qv);
                if (lane == 0) {
                    xe32[c] = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
                    xs32[c] = (float)s;
                }
            }
            if (p.need16) {
                float amax = av;
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                const int qv = (int)roundf(__fmul_rn(v, inv));
                xq16[(i >> 8) * kXqStride + (i & 255)] = (int8_t)qv;
                int s = (int)(int8_t)qv;
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if ((lane & 15) == 0) {
                    xe16[2 * c + (lane >> 4)] = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
                    xs16[2 * c + (lane >> 4)] = (float)s;
                }
            }
        }
    }
    consumers_sync();
}

// ── work decomposition ──
// A CTA owns a contiguous, balanced range of units. It walks them in groups of
// at most 16 units (rows of one segment), and each group in k-chunks of 8
// super-blocks: one chunk of a group is one pipeline stage. Unit j of a group
// occupies slots 2j (its first row) and 2j+1 (its second row), so both rows of
// a unit land in the same consumer warp.
struct Grp {
    int seg, local, n;
};

__device__ __forceinline__ bool grp_next(const MatvecParams &p, int &gu, int ue, Grp &g) {
    if (gu >= ue) return false;
    int s = 0, u = gu;
    while (s < p.nseg - 1 && u >= p.seg[s].units) {
        u -= p.seg[s].units;
        s++;
    }
    const Seg &sg = p.seg[s];
    int n = min(16, min(ue - gu, sg.units - u));
    if (sg.pairing == PAIR_ROPE) n = min(n, sg.half - u % sg.half);
    g.seg = s;
    g.local = u;
    g.n = n;
    gu += n;
    return true;
}

// matrix and row of a slot; false when the slot is empty
__device__ __forceinline__ bool slot_row(const MatvecParams &p, const Grp &g, int slot, const DMat *&M, int &row) {
    const Seg &s = p.seg[g.seg];
    if (slot >= 2 * g.n) return false;
    if (s.pairing == PAIR_ADJ) {
        M = &s.A;
        row = 2 * g.local + slot;
        return true;
    }
    const int j = slot >> 1, hi = slot & 1;
    if (s.pairing == PAIR_ROPE) {
        const int h = g.local / s.half, i = g.local % s.half;
        M = &s.A;
        row = h * 2 * s.half + i + j + (hi ? s.half : 0);
    } else {
        M = hi ? &s.B : &s.A;
        row = g.local + j;
    }
    return true;
}

template <int T>
__device__ __forceinline__ void chunk_terms(const uint8_t *sa, const uint8_t *ss, const uint8_t *sd, int b0, int lane,
                                            const XQ &x, float *tile_row) {
    float t[4];
    const int bl = lane >> 2, q = lane & 3;
    quarter_at<T, false>(sa + bl * plane_a_bytes(T), ss + bl * plane_s_bytes(T), sd + bl * plane_d_bytes(T), b0 + bl,
                         q, x, t, nullptr);
    constexpr int tpq = (T == 12 || T == 13) ? 2 : 4, spb = (T == 12 || T == 13) ? 8 : 16;
#pragma unroll
    for (int k = 0; k < tpq; k++) tile_row[bl * spb + term_sub(T, q, k)] = t[k];
}

__device__ void unit_epilogue(const MatvecParams &p, const Seg &g, int r0, int r1, float y0, float y1, int pos,
                              unsigned long long &best) {
    if (g.at_pos && (pos < 0 || pos >= p.max_pos)) return;
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
        // src/kernels/scalar.rs:63-67 then `*a *= u` (src/forward.rs:485-487)
        const float act = __fdiv_rn(y0, fa(1.0f, expf_glibc(-y0)));
        out[r0] = fm(act, y1);
        break;
    }
    case EPI_LOGITS: {
        out[r0] = y0;
        out[r1] = y1;
        const unsigned long long ka = (y0 == y0) ? argmax_key(y0, (uint32_t)r0) : 0ull;
        const unsigned long long kb = (y1 == y1) ? argmax_key(y1, (uint32_t)r1) : 0ull;
        const unsigned long long kk = ka > kb ? ka : kb;
        best = kk > best ? kk : best;
        break;
    }
    }
}

// k-quant matvec, several matrices per launch (q|k|v, gate|up), activation
// quantization fused in front and the consumer fused behind. Persistent: one
// CTA per SM. A producer warp streams each stage's weight planes with bulk
// copies (the TMA unit) into a 3-deep shared-memory ring; in the 8 consumer
// warps a lane takes one super-block of one row (lane = 4*block + slot) and
// forms all its sub-block terms, then the terms of each row are added in
// sub-block order onto the row's running total, handed from block to block
// by warp shuffles.
__global__ void __launch_bounds__(kMvThreads, 1) k_matvec(const __grid_constant__ MatvecParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    unsigned char *stages = smem;
    const int K = p.K, nblk = K / 256, nkc = (nblk + kChunk - 1) / kChunk;
    int8_t *xq16 = (int8_t *)(smem + (size_t)kStages * kStageBytes);
    int8_t *xq32 = xq16 + (p.need16 ? nblk * kXqStride : 0);
    float *xe16 = (float *)(xq32 + (p.need32 ? nblk * kXqStride : 0));
    float *xs16 = xe16 + (p.need16 ? K / 16 : 0);
    float *xe32 = xs16 + (p.need16 ? K / 16 : 0);
    float *xs32 = xe32 + (p.need32 ? K / 32 : 0);
    __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
    __shared__ volatile int abort_flag;
    __shared__ double red[kCW];
    __shared__ double scale_s;
    __shared__ unsigned long long best_s[kCW];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    griddep_launch_dependents();

    const int U = p.total_units, G = gridDim.x;
    const int ub = (int)(((long long)blockIdx.x * U) / G), ue = (int)(((long long)(blockIdx.x + 1) * U) / G);

    if (warp == kCW) {
        // ── producer: weights never depend on the previous kernel, so they
        // start streaming before the dependency wait ──
        uint32_t it = 0;
        int gu = ub;
        Grp g;
        bool ok = true;
        while (ok && grp_next(p, gu, ue, g)) {
            for (int kc = 0; kc < nkc && ok; kc++, it++) {
                const int s = it % kStages;
                const uint32_t ph = (it / kStages) & 1;
                int got = 1;
                if (lane == 0) got = mbar_wait_bounded(&empty[s], ph ^ 1, &abort_flag) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);  // warp-uniform, and orders the copies after the wait
                if (!got) {
                    ok = false;
                    break;
                }
                const int b0 = kc * kChunk, nb = min(kChunk, nblk - b0);
                // each lane streams one slot's row chunk
                const DMat *M = nullptr;
                int row = 0;
                const bool valid = slot_row(p, g, lane, M, row);
                uint32_t ba = 0, bs = 0, bd = 0;
                if (valid) {
                    ba = (uint32_t)(nb * plane_a_bytes(M->type));
                    bs = plane_s_bytes(M->type) ? pitch16((uint32_t)(nb * plane_s_bytes(M->type))) : 0;
                    bd = plane_d_bytes(M->type) ? pitch16((uint32_t)(nb * plane_d_bytes(M->type))) : 0;
                }
                uint32_t bytes = ba + bs + bd;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
                if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
                __syncwarp();
                if (valid) {
                    unsigned char *st = stages + (size_t)s * kStageBytes;
                    bulk_g2s(st + lane * kSlotA, M->a + (size_t)row * M->a_row + (size_t)b0 * plane_a_bytes(M->type),
                             ba, &full[s]);
                    if (bs)
                        bulk_g2s(st + kStageA + lane * kSlotS,
                                 M->s + (size_t)row * M->s_row + (size_t)b0 * plane_s_bytes(M->type), bs, &full[s]);
                    if (bd)
                        bulk_g2s(st + kStageA + kStageS + lane * kSlotD,
                                 M->d + (size_t)row * M->d_row + (size_t)b0 * plane_d_bytes(M->type), bd, &full[s]);
                }
            }
        }
        if (!ok && lane == 0) {
            abort_flag = 1;
            atomicOr(p.err, ERR_TIMEOUT);
        }
        // drain: the last stages issued must have landed before the CTA exits
        if (lane == 0) {
            const uint32_t last = it;
            for (uint32_t j = last > (uint32_t)kStages ? last - kStages : 0; j < last; j++)
                mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1, &abort_flag, 1u << 14);
        }
        return;
    }

    // ── consumers ──
    griddep_wait();  // activations, caches and the residual come from earlier kernels
    prologue_quantize(p, xq16, xe16, xs16, xq32, xe32, xs32, red, &scale_s);
    const int pos = p.d_len ? *p.d_len : 0;
    const int bl = lane >> 2, sl = lane & 3, slot = warp * kSlotsPerWarp + sl;
    unsigned long long best = 0ull;
    uint32_t it = 0;
    int gu = ub;
    Grp g;
    bool ok = true;
    while (ok && grp_next(p, gu, ue, g)) {
        const DMat *M = nullptr;
        int row = 0;
        const bool valid = slot_row(p, g, slot, M, row);
        const int T = valid ? M->type : 0;
        const bool s32 = (T == 12 || T == 13);
        const int nsub = s32 ? 8 : 16;
        const int8_t *xq = s32 ? xq32 : xq16;
        const float *xe = s32 ? xe32 : xe16, *xs = s32 ? xs32 : xs16;
        float acc = 0.0f;
        for (int kc = 0; kc < nkc; kc++, it++) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1;
            const bool got = mbar_wait_bounded(&full[s], ph, &abort_flag);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            const int b0 = kc * kChunk, nb = min(kChunk, nblk - b0);
            float t[16];
            if (valid && bl < nb) {
                const unsigned char *st = stages + (size_t)s * kStageBytes;
                const uint8_t *pa = st + slot * kSlotA + bl * plane_a_bytes(T);
                const uint8_t *ps = st + kStageA + slot * kSlotS + bl * plane_s_bytes(T);
                const uint8_t *pd = st + kStageA + kStageS + slot * kSlotD + bl * plane_d_bytes(T);
                const int b = b0 + bl;
                const XB xb{xq + b * kXqStride, xe + b * nsub, xs + b * nsub};
                switch (T) {
                case 12: block_k4<false>(pa, xb, t); break;
                case 13: block_k4<true>(pa, xb, t); break;
                case 14: block_q6k(pa, ps, pd, xb, t); break;
                case 11: block_q3k(pa, ps, pd, xb, t); break;
                default: block_q2k(pa, ps, pd, xb, t); break;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // the stage's weights are consumed
            // the row's running total visits the blocks in order
            float run = acc;
            for (int j = 0; j < nb; j++) {
                float v = run;
                if (valid && bl == j) {
#pragma unroll
                    for (int k = 0; k < 16; k++)
                        if (k < nsub) v = fa(v, t[k]);
                }
                run = __shfl_sync(0xffffffffu, v, j * 4 + sl);
            }
            acc = run;
        }
        if (!ok) break;
        // slots sl = 0,1 hold row pair 2*warp; sl = 2,3 row pair 2*warp+1
        const float other = __shfl_down_sync(0xffffffffu, acc, 1);
        if (bl == 0 && !(sl & 1)) {
            const DMat *M1 = nullptr;
            int row1 = 0;
            if (valid && slot_row(p, g, slot + 1, M1, row1))
                unit_epilogue(p, p.seg[g.seg], row, row1, acc, other, pos, best);
        }
    }
    if (!ok && lane == 0) {
        abort_flag = 1;
        atomicOr(p.err, ERR_TIMEOUT);
    }
    if (p.argmax_key) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if (lane == 0) best_s[warp] = best;
        consumers_sync();
        if (tid == 0) {
            unsigned long long b = 0;
            for (int w = 0; w < kCW; w++) b = best_s[w] > b ? best_s[w] : b;
            if (b) atomicMax(p.argmax_key, b);
        }
    }
}

// ── attention for one new token (src/ops.rs:1258-1325) in the reference's
// order, in two kernels over many SMs:
//   scores: score[h][p] = (sequential dot of q_h and k_p over the head dim)·scale
//   output: softmax over the head's scores (subtract the max, libm exp, sum the
//           exponentials position by position, multiply by 1/total;
//           src/ops.rs:1206-1230), then out[d] = Σ_p prob_p·v_p[d] added
//           position by position.
struct AttnParams {
    const float *q;      // [H*hd], rotated
    const float *k, *v;  // layer base, [max_tokens][KV*hd]
    float *out;          // [H*hd]
    float *scores;       // scratch [H][max_pos]
    const int *d_len;
    int H, KV, hd, max_pos, score_stride;
    float scale;
    int *err;
};

constexpr int kScoreThreads = 128;   // positions per score CTA
constexpr int kKRow = 132;           // smem row stride (floats) of staged K rows
constexpr int kOutThreads = 128;
constexpr int kOutDims = 16;         // head dims per output CTA
constexpr int kVChunk = 64;          // positions per staged V chunk
constexpr int kVRing = 8;            // V chunks in flight

__global__ void __launch_bounds__(kScoreThreads) k_attn_scores(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float ks[];  // [kScoreThreads][kKRow] then q [hd]
    griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x, split = blockIdx.y, tid = threadIdx.x;
    const int n = *p.d_len + 1;
    if (n > p.max_pos || n <= 0) {
        if (tid == 0 && h == 0 && split == 0) atomicOr(p.err, ERR_POSITION);
        return;
    }
    const int p0 = split * kScoreThreads;
    if (p0 >= n) return;
    const int cnt = min(kScoreThreads, n - p0);
    const int hd = p.hd, G = p.H / p.KV, g = h / G, kvd = p.KV * hd, c4 = hd / 4;
    float *qs = ks + kScoreThreads * kKRow;
    // stage q and the K rows of these positions: all 16-byte copies in flight
    for (int i = tid; i < c4; i += kScoreThreads) cp_async16(qs + 4 * i, p.q + (size_t)h * hd + 4 * i);
    for (int i = tid; i < cnt * c4; i += kScoreThreads) {
        const int r = i / c4, c = i - r * c4;
        cp_async16(ks + r * kKRow + 4 * c, p.k + (size_t)(p0 + r) * kvd + (size_t)g * hd + 4 * c);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid < cnt) {
        const float4 *kr = (const float4 *)(ks + tid * kKRow);
        const float4 *q4 = (const float4 *)qs;
        float acc = 0.0f;
        for (int c = 0; c < c4; c++) {
            const float4 kv = kr[c], qv = q4[c];
            acc = fa(acc, fm(qv.x, kv.x));
            acc = fa(acc, fm(qv.y, kv.y));
            acc = fa(acc, fm(qv.z, kv.z));
            acc = fa(acc, fm(qv.w, kv.w));
        }
        p.scores[(size_t)h * p.score_stride + p0 + tid] = fm(acc, p.scale);
    }
}

__global__ void __launch_bounds__(kOutThreads) k_attn_out(const __grid_constant__ AttnParams p) {
    // smem: probs [max_pos rounded to 4] then a ring of kVRing V chunks [kVChunk][kOutDims]
    extern __shared__ __align__(16) float so[];
    __shared__ float red[kOutThreads / 32];
    __shared__ float bcast;
    griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x, dslice = blockIdx.y, tid = threadIdx.x;
    const int n = *p.d_len + 1;
    if (n > p.max_pos || n <= 0) return;  // k_attn_scores reported it
    const int hd = p.hd, G = p.H / p.KV, g = h / G, kvd = p.KV * hd;
    const int d0 = dslice * kOutDims;
    if (d0 >= hd) return;
    float *pr = so;
    float *vs = so + ((p.max_pos + 3) & ~3);
    const float *sc = p.scores + (size_t)h * p.score_stride;
    const float *vb = p.v + (size_t)g * hd + d0;
    const int nchunks = (n + kVChunk - 1) / kVChunk;
    auto stage = [&](int c) {
        if (c >= nchunks) return;
        const int base = c * kVChunk, cnt = min(kVChunk, n - base);
        float *dst = vs + (c % kVRing) * kVChunk * kOutDims;
        for (int i = tid; i < cnt * (kOutDims / 4); i += kOutThreads) {
            const int r = i / (kOutDims / 4), q = i - r * (kOutDims / 4);
            cp_async16(dst + r * kOutDims + 4 * q, vb + (size_t)(base + r) * kvd + 4 * q);
        }
    };
    // the scores and the first V chunks all in flight at once; the softmax
    // runs while V streams in
    for (int i = tid; i < (n + 3) / 4; i += kOutThreads) cp_async16(pr + 4 * i, sc + 4 * i);
    cp_async_commit();
    for (int c = 0; c < kVRing - 1; c++) {
        stage(c);
        cp_async_commit();
    }
    cp_async_wait<kVRing - 1>();
    __syncthreads();
    float m = -INFINITY;
    for (int i = tid; i < n; i += kOutThreads) m = fmaxf(m, pr[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < kOutThreads / 32; w++) mm = fmaxf(mm, red[w]);
        bcast = mm;
    }
    __syncthreads();
    const float mx = bcast;
    __syncthreads();
    if (!isfinite(mx)) {
        const float u = __fdiv_rn(1.0f, (float)n);
        for (int i = tid; i < n; i += kOutThreads) pr[i] = u;
    } else {
        for (int i = tid; i < n; i += kOutThreads) pr[i] = expf_glibc(fs(pr[i], mx));
        __syncthreads();
        if (tid == 0) {
            float total = 0.0f;
            int i = 0;
            for (; i + 4 <= n; i += 4) {
                const float4 v = *(const float4 *)(pr + i);
                total = fa(fa(fa(fa(total, v.x), v.y), v.z), v.w);
            }
            for (; i < n; i++) total = fa(total, pr[i]);
            bcast = __fdiv_rn(1.0f, total);
        }
        __syncthreads();
        const float inv = bcast;
        for (int i = tid; i < n; i += kOutThreads) pr[i] = fm(pr[i], inv);
    }
    __syncthreads();
    // out[d] = Σ_p prob_p·v_p[d], one sequential chain per dim
    float acc = 0.0f;
    for (int c = 0; c < nchunks; c++) {
        stage(c + kVRing - 1);
        cp_async_commit();
        cp_async_wait<kVRing - 1>();
        __syncthreads();
        if (tid < kOutDims && d0 + tid < hd) {
            const float *src = vs + (c % kVRing) * kVChunk * kOutDims + tid;
            const int base = c * kVChunk, cnt = min(kVChunk, n - base);
            for (int r = 0; r < cnt; r++) acc = fa(acc, fm(pr[base + r], src[r * kOutDims]));
        }
        __syncthreads();
    }
    if (tid < kOutDims && d0 + tid < hd) p.out[(size_t)h * hd + d0 + tid] = acc;
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
    griddep_launch_dependents();
    griddep_wait();
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
    griddep_wait();
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
