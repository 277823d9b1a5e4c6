// Device code shared by the decode kernels: the weight planes, the k-quant
// super-block arithmetic of the five layouts, and the dequantization of a
// single value (embedding rows).
//
// Weights live in HBM as "planes" (see DMat): the GGUF super-block bytes are
// split once at load into 16-byte-aligned per-row arrays so every weight load
// is an aligned 128-bit load or bulk copy, without changing a single bit of
// the values.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace cxm {

// ── repacked weight matrix ──
// Plane A per super-block: Q4_K 144 B (whole block), Q5_K 176 B (whole block),
// Q6_K 192 B (ql|qh), Q3_K 96 B (hmask|qs), Q2_K 64 B (qs).
// Plane S: Q6_K 16 B int8 scales, Q3_K 12 B packed 6-bit scales, Q2_K 16 B.
// Plane D: Q6_K 2 B (d), Q3_K 2 B (d), Q2_K 4 B (d, dmin).
// Row pitches are multiples of 16 bytes (S and D rows padded).
struct DMat {
    int type, rows, K, nblk;
    const uint8_t *a, *s, *d;
    uint32_t a_row, s_row, d_row;  // bytes per row of each plane (pitch)
};

__host__ __device__ inline int plane_a_bytes(int t) {
    return t == 12 ? 144 : t == 13 ? 176 : t == 14 ? 192 : t == 11 ? 96 : t == 10 ? 64 : 0;
}
__host__ __device__ inline int plane_s_bytes(int t) { return t == 14 ? 16 : t == 11 ? 12 : t == 10 ? 16 : 0; }
__host__ __device__ inline int plane_d_bytes(int t) { return t == 14 ? 2 : t == 11 ? 2 : t == 10 ? 4 : 0; }
__host__ __device__ inline uint32_t pitch16(uint32_t b) { return (b + 15u) & ~15u; }

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// Exact IEEE single-precision operations, never contracted into FMA, so every
// term keeps the reference's rounding.
__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }

__device__ __forceinline__ uint32_t byte_of(uint32_t w0, uint32_t w1, uint32_t w2, int i) {
    uint32_t w = i < 4 ? w0 : (i < 8 ? w1 : w2);
    return (w >> (8 * (i & 3))) & 0xFF;
}

// 6-bit scale/min of sub-block j from the 12 packed bytes (words w0..w2 hold
// bytes 0..11). src/quant.rs:108-117.
__device__ __forceinline__ void scale_min_k4(int j, uint32_t w0, uint32_t w1, uint32_t w2, int &sc, int &mn) {
    if (j < 4) {
        sc = byte_of(w0, w1, w2, j) & 63;
        mn = byte_of(w0, w1, w2, j + 4) & 63;
    } else {
        sc = (byte_of(w0, w1, w2, j + 4) & 0xF) | ((byte_of(w0, w1, w2, j - 4) >> 6) << 4);
        mn = (byte_of(w0, w1, w2, j + 4) >> 4) | ((byte_of(w0, w1, w2, j) >> 6) << 4);
    }
}

struct XQ {  // the quantized activation, in shared memory
    const int8_t *q;
    const float *e, *s;
};

__device__ __forceinline__ int dot4w(const uint32_t *w, int4 a) {
    int s = 0;
    s = __dp4a((int)w[0], a.x, s);
    s = __dp4a((int)w[1], a.y, s);
    s = __dp4a((int)w[2], a.z, s);
    s = __dp4a((int)w[3], a.w, s);
    return s;
}

// loads from global memory (read-only path) or from shared memory (plain)
template <bool G>
__device__ __forceinline__ uint4 ld16(const uint8_t *p) {
    if (G) return __ldg((const uint4 *)p);
    return *(const uint4 *)p;
}
template <bool G>
__device__ __forceinline__ uint32_t ld4(const uint8_t *p) {
    if (G) return __ldg((const uint32_t *)p);
    return *(const uint32_t *)p;
}
template <bool G>
__device__ __forceinline__ uint32_t ld2(const uint8_t *p) {
    if (G) return __ldg((const unsigned short *)p);
    return *(const unsigned short *)p;
}
template <bool G>
__device__ __forceinline__ void ld32(const uint8_t *p, uint32_t w[8]) {
    uint4 a = ld16<G>(p), b = ld16<G>(p + 16);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}

// ── one "quarter" (64 values) of a super-block ──
// A lane works on quarter q (0..3) of super-block b (the block's index along
// the row, which addresses the activation). `pa`, `ps`, `pd` point at this
// block's bytes in planes A, S and D. Writes the quarter's sub-block terms
// t[0..tpq) in the order of term_sub(); `isum` (optional) gets the integer
// sub-block sums.

// Q4_K: src/kernels/scalar.rs:132-170
template <bool G>
__device__ __forceinline__ void q_q4k(const uint8_t *pa, int b, int q, const XQ &x, float *t, int *isum) {
    const uint4 hdr = ld16<G>(pa);
    uint32_t w[8];
    ld32<G>(pa + 16 + 32 * q, w);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    int sc0, m0, sc1, m1;
    scale_min_k4(2 * q, hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4(2 * q + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        lo[i] = w[i] & 0x0F0F0F0Fu;
        hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
    }
    const int4 *xp = (const int4 *)(x.q + b * 256 + q * 64);
    const int s0 = dot4w(lo, xp[0]) + dot4w(lo + 4, xp[1]);
    const int s1 = dot4w(hi, xp[2]) + dot4w(hi + 4, xp[3]);
    const int j0 = b * 8 + 2 * q;
    if (isum) { isum[0] = s0; isum[1] = s1; }
    t[0] = fm(x.e[j0], fs(fm(fm(d, (float)sc0), (float)s0), fm(fm(dmin, (float)m0), x.s[j0])));
    t[1] = fm(x.e[j0 + 1], fs(fm(fm(d, (float)sc1), (float)s1), fm(fm(dmin, (float)m1), x.s[j0 + 1])));
}

// Q5_K: src/kernels/scalar.rs:179-217
template <bool G>
__device__ __forceinline__ void q_q5k(const uint8_t *pa, int b, int q, const XQ &x, float *t, int *isum) {
    const uint4 hdr = ld16<G>(pa);
    uint32_t qh[8], w[8];
    ld32<G>(pa + 16, qh);
    ld32<G>(pa + 48 + 32 * q, w);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    int sc0, m0, sc1, m1;
    const int j0 = 2 * q, j1 = 2 * q + 1;
    scale_min_k4(j0, hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4(j1, hdr.y, hdr.z, hdr.w, sc1, m1);
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        lo[i] = (w[i] & 0x0F0F0F0Fu) | (((qh[i] >> j0) & 0x01010101u) << 4);
        hi[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> j1) & 0x01010101u) << 4);
    }
    const int4 *xp = (const int4 *)(x.q + b * 256 + q * 64);
    const int s0 = dot4w(lo, xp[0]) + dot4w(lo + 4, xp[1]);
    const int s1 = dot4w(hi, xp[2]) + dot4w(hi + 4, xp[3]);
    const int k0 = b * 8 + j0;
    if (isum) { isum[0] = s0; isum[1] = s1; }
    t[0] = fm(x.e[k0], fs(fm(fm(d, (float)sc0), (float)s0), fm(fm(dmin, (float)m0), x.s[k0])));
    t[1] = fm(x.e[k0 + 1], fs(fm(fm(d, (float)sc1), (float)s1), fm(fm(dmin, (float)m1), x.s[k0 + 1])));
}

// Q6_K: src/kernels/scalar.rs:294-324. Quarter q = half h (q>>1) and ql
// column par (q&1): groups gi = par (low nibbles) and gi = par+2 (high).
template <bool G>
__device__ __forceinline__ void q_q6k(const uint8_t *pa, const uint8_t *ps, const uint8_t *pd, int b, int q,
                                      const XQ &x, float *t, int *isum) {
    const int h = q >> 1, par = q & 1;
    uint32_t ql[8], qh[8];
    ld32<G>(pa + 64 * h + 32 * par, ql);
    ld32<G>(pa + 128 + 32 * h, qh);
    const uint4 scv = ld16<G>(ps);
    const float d = h2f(ld2<G>(pd));
    uint32_t vlo[8], vhi[8];
    const int slo = 2 * par, shi = 2 * (par + 2);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        vlo[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> slo) & 0x03030303u) << 4);
        vhi[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> shi) & 0x03030303u) << 4);
    }
    const int glo = 4 * h + par, ghi = glo + 2;
    const int4 *xlo = (const int4 *)(x.q + b * 256 + 32 * glo);
    const int4 *xhi = (const int4 *)(x.q + b * 256 + 32 * ghi);
    int s[4];
    s[0] = dot4w(vlo, xlo[0]);
    s[1] = dot4w(vlo + 4, xlo[1]);
    s[2] = dot4w(vhi, xhi[0]);
    s[3] = dot4w(vhi + 4, xhi[1]);
    if (isum) { isum[0] = s[0]; isum[1] = s[1]; isum[2] = s[2]; isum[3] = s[3]; }
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int g = k < 2 ? glo : ghi, md = k & 1;
        const int si = 2 * g + md;
        const int sc = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xFF);
        const int sub = b * 16 + si;
        const float esc = fm(d, (float)sc);
        t[k] = fm(fm(x.e[sub], esc), fs((float)s[k], fm(32.0f, x.s[sub])));
    }
}

// Q3_K: src/kernels/scalar.rs:236-275. Quarter q = groups 2q and 2q+1.
template <bool G>
__device__ __forceinline__ void q_q3k(const uint8_t *pa, const uint8_t *ps, const uint8_t *pd, int b, int q,
                                      const XQ &x, float *t, int *isum) {
    uint32_t hm[8], qs[8];
    ld32<G>(pa, hm);
    ld32<G>(pa + 32 + 32 * (q >> 1), qs);
    const uint32_t a0 = ld4<G>(ps), a1 = ld4<G>(ps + 4), tt = ld4<G>(ps + 8);
    const float d = h2f(ld2<G>(pd));
    // scales of sub-blocks 4q..4q+3 (src/quant.rs:87-106)
    const uint32_t aa = (q & 1) ? a1 : a0;
    const uint32_t wq = ((aa >> ((q >> 1) * 4)) & 0x0F0F0F0Fu) | (((tt >> (2 * q)) & 0x03030303u) << 4);
    int s[4];
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
        const int g = 2 * q + gg, sh = 2 * (g & 3);
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = ((qs[i] >> sh) & 0x03030303u) | (((hm[i] >> g) & 0x01010101u) << 2);
        const int4 *xp = (const int4 *)(x.q + b * 256 + 32 * g);
        s[2 * gg] = dot4w(v, xp[0]);
        s[2 * gg + 1] = dot4w(v + 4, xp[1]);
    }
    if (isum) { isum[0] = s[0]; isum[1] = s[1]; isum[2] = s[2]; isum[3] = s[3]; }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int sc = (int)((wq >> (8 * k)) & 0xFF);
        const int sub = b * 16 + 4 * q + k;
        const float esc = fm(d, fs((float)sc, 32.0f));
        t[k] = fm(fm(x.e[sub], esc), fs((float)s[k], fm(4.0f, x.s[sub])));
    }
}

// Q2_K: src/kernels/q2k.rs:41-69. Quarter q = groups 2q and 2q+1.
template <bool G>
__device__ __forceinline__ void q_q2k(const uint8_t *pa, const uint8_t *ps, const uint8_t *pd, int b, int q,
                                      const XQ &x, float *t, int *isum) {
    uint32_t qs[8];
    ld32<G>(pa + 32 * (q >> 1), qs);
    const uint32_t scw = ld4<G>(ps + 4 * q);
    const uint32_t dd = ld4<G>(pd);
    const float d = h2f(dd), dm = h2f(dd >> 16);
    int s[4];
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
        const int g = 2 * q + gg, sh = 2 * (g & 3);
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = (qs[i] >> sh) & 0x03030303u;
        const int4 *xp = (const int4 *)(x.q + b * 256 + 32 * g);
        s[2 * gg] = dot4w(v, xp[0]);
        s[2 * gg + 1] = dot4w(v + 4, xp[1]);
    }
    if (isum) { isum[0] = s[0]; isum[1] = s[1]; isum[2] = s[2]; isum[3] = s[3]; }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int sc = (int)((scw >> (8 * k)) & 0xFF);
        const int sub = b * 16 + 4 * q + k;
        const float ev = fm(d, (float)(sc & 0xF)), mv = fm(dm, (float)(sc >> 4));
        t[k] = fm(x.e[sub], fs(fm(ev, (float)s[k]), fm(mv, x.s[sub])));
    }
}

// One quarter of format T. The row total of the reference is the sequential
// f32 sum of all terms in sub-block order (src/kernels/scalar.rs, `total +=`
// per sub-block); callers reproduce it exactly.
template <int T, bool G>
__device__ __forceinline__ void quarter_at(const uint8_t *pa, const uint8_t *ps, const uint8_t *pd, int b, int q,
                                           const XQ &x, float *t, int *isum) {
    if (T == 12) q_q4k<G>(pa, b, q, x, t, isum);
    else if (T == 13) q_q5k<G>(pa, b, q, x, t, isum);
    else if (T == 14) q_q6k<G>(pa, ps, pd, b, q, x, t, isum);
    else if (T == 11) q_q3k<G>(pa, ps, pd, b, q, x, t, isum);
    else q_q2k<G>(pa, ps, pd, b, q, x, t, isum);
}

// quarter qt (block qt/4, quarter qt%4) of row `row` of a matrix in HBM
template <int T>
__device__ __forceinline__ void quarter(const DMat &W, int row, int qt, const XQ &x, float *t, int *isum) {
    const int b = qt >> 2;
    const uint8_t *pa = W.a + (size_t)row * W.a_row + (size_t)b * plane_a_bytes(T);
    const uint8_t *ps = W.s + (size_t)row * W.s_row + (size_t)b * plane_s_bytes(T);
    const uint8_t *pd = W.d + (size_t)row * W.d_row + (size_t)b * plane_d_bytes(T);
    quarter_at<T, true>(pa, ps, pd, b, qt & 3, x, t, isum);
}

__host__ __device__ __forceinline__ int terms_per_quarter(int type) { return (type == 12 || type == 13) ? 2 : 4; }
__host__ __device__ __forceinline__ int subs_per_block(int type) { return (type == 12 || type == 13) ? 8 : 16; }
__device__ __forceinline__ int term_sub(int type, int q, int k) {
    if (type == 12 || type == 13) return 2 * q + k;
    if (type == 14) {
        const int g = 4 * (q >> 1) + (q & 1) + (k >= 2 ? 2 : 0);
        return 2 * g + (k & 1);
    }
    return 4 * q + k;
}

// ── a whole super-block from shared memory ──
// The streaming matvec gives each lane one super-block of one row: it forms
// all of the block's sub-block terms t[0..nsub) in sub-block order. The
// block's plane-A bytes are 16-byte chunks `cs` bytes apart (16 when they are
// contiguous; the lane count x 16 in a quad tile, where the lanes' chunks are
// interleaved). `xq` is the activation with each 256-value block padded to
// kXqStride bytes (bank spread); `xe`/`xs` hold 8 (sub-blocks of 32) or 16
// (of 16) floats per block.
constexpr int kXqStride = 272;

struct XB {  // one block of the quantized activation
    const int8_t *q;      // 256 values
    const float2 *es;     // (scale, sum) of each of its nsub sub-blocks: one 8-byte load per sub-block
};

__device__ __forceinline__ int dot16(uint4 w, int4 a) {
    int s = __dp4a((int)w.x, a.x, 0);
    s = __dp4a((int)w.y, a.y, s);
    s = __dp4a((int)w.z, a.z, s);
    return __dp4a((int)w.w, a.w, s);
}

// unsigned bytes of w times signed bytes of a, accumulated (dp4a.u32.s32)
__device__ __forceinline__ int dp4a_us(uint32_t w, int a, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(a), "r"(c));
    return d;
}
// the same over 16 bytes: w's bytes are high nibbles left in place (n·16),
// so the sum is 16 times the nibbles' sum, exactly
__device__ __forceinline__ int dot16_hi(uint4 w, int4 a, int c) {
    int s = dp4a_us(w.x, a.x, c);
    s = dp4a_us(w.y, a.y, s);
    s = dp4a_us(w.z, a.z, s);
    return dp4a_us(w.w, a.w, s);
}
__device__ __forceinline__ uint4 and4(uint4 v, uint32_t m) { return make_uint4(v.x & m, v.y & m, v.z & m, v.w & m); }
__device__ __forceinline__ uint4 shr4(uint4 v, int n) { return make_uint4(v.x >> n, v.y >> n, v.z >> n, v.w >> n); }
__device__ __forceinline__ uint4 or4(uint4 a, uint4 b) { return make_uint4(a.x | b.x, a.y | b.y, a.z | b.z, a.w | b.w); }
__device__ __forceinline__ uint4 shl4(uint4 v, int n) { return make_uint4(v.x << n, v.y << n, v.z << n, v.w << n); }

// Q4_K / Q5_K: 8 terms.
// BUF = false: the fused kernel's term per sub-block,
//   xe·(d·sc·Σxq·q − dmin·m·xs)            (src/kernels/scalar.rs:132-217)
// BUF = true: the buffered path's two terms per sub-block (src/ops.rs:383-405
// over src/quant.rs:276-300): t = (d·sc)·xe·Σxq·q for dot_i8_escalado
// (src/kernels/scalar.rs:95-109) and sv = (−dmin·m)·xe·xs for the offset
// chain that follows it; `anyd` gets whether any −dmin·m is nonzero.
template <bool Q5, bool BUF = false>
__device__ __forceinline__ void block_k4(const uint8_t *pa, int cs, const XB &x, float *t, float *sv = nullptr,
                                         bool *anyd = nullptr) {
    const uint4 hdr = *(const uint4 *)pa;
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    const int4 *xp = (const int4 *)x.q;
    const int c0 = Q5 ? 3 : 1;  // first qs chunk
    uint4 qh0 = make_uint4(0, 0, 0, 0), qh1 = qh0;
    if (Q5) {
        qh0 = *(const uint4 *)(pa + cs);
        qh1 = *(const uint4 *)(pa + 2 * cs);
    }
#pragma unroll
    for (int p = 0; p < 4; p++) {
        const uint4 wa = *(const uint4 *)(pa + (c0 + 2 * p) * cs), wb = *(const uint4 *)(pa + (c0 + 2 * p + 1) * cs);
        uint4 la = and4(wa, 0x0F0F0F0Fu), lb = and4(wb, 0x0F0F0F0Fu);
        uint4 ha = make_uint4(0, 0, 0, 0), hb = ha;
        if (Q5) {
            ha = and4(shr4(wa, 4), 0x0F0F0F0Fu);
            hb = and4(shr4(wb, 4), 0x0F0F0F0Fu);
            la = or4(la, shl4(and4(shr4(qh0, 2 * p), 0x01010101u), 4));
            lb = or4(lb, shl4(and4(shr4(qh1, 2 * p), 0x01010101u), 4));
            ha = or4(ha, shl4(and4(shr4(qh0, 2 * p + 1), 0x01010101u), 4));
            hb = or4(hb, shl4(and4(shr4(qh1, 2 * p + 1), 0x01010101u), 4));
        }
        const int s0 = dot16(la, xp[4 * p]) + dot16(lb, xp[4 * p + 1]);
        int s1;
        if (Q5) {
            s1 = dot16(ha, xp[4 * p + 2]) + dot16(hb, xp[4 * p + 3]);
        } else {  // the high nibbles in place: one mask per word instead of a shift and a mask
            s1 = dot16_hi(and4(wb, 0xF0F0F0F0u), xp[4 * p + 3], dot16_hi(and4(wa, 0xF0F0F0F0u), xp[4 * p + 2], 0)) >> 4;
        }
        int sc0, m0, sc1, m1;
        scale_min_k4(2 * p, hdr.y, hdr.z, hdr.w, sc0, m0);
        scale_min_k4(2 * p + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
        const int j0 = 2 * p;
        const float2 es0 = x.es[j0], es1 = x.es[j0 + 1];
        if (BUF) {
            const float mn0 = fm(dmin, (float)m0), mn1 = fm(dmin, (float)m1);
            t[j0] = fm(fm(fm(d, (float)sc0), es0.x), (float)s0);
            t[j0 + 1] = fm(fm(fm(d, (float)sc1), es1.x), (float)s1);
            sv[j0] = fm(fm(-mn0, es0.x), es0.y);
            sv[j0 + 1] = fm(fm(-mn1, es1.x), es1.y);
            *anyd = *anyd || mn0 != 0.0f || mn1 != 0.0f;
        } else {
            t[j0] = fm(es0.x, fs(fm(fm(d, (float)sc0), (float)s0), fm(fm(dmin, (float)m0), es0.y)));
            t[j0 + 1] = fm(es1.x, fs(fm(fm(d, (float)sc1), (float)s1), fm(fm(dmin, (float)m1), es1.y)));
        }
    }
}

// Q6_K: 16 terms (src/kernels/scalar.rs:294-324). The buffered path's term
// (d·sc)·xe·Σxq·(q−32) (src/ops.rs:383-405, src/quant.rs:432-463) is the
// same value bit for bit: the product of two factors does not depend on
// their order, Σxq·q − 32·xs is an exact integer in f32, and the format has
// no offset term. Q3_K likewise.
__device__ __forceinline__ void block_q6k(const uint8_t *pa, int cs, const uint8_t *ps, const uint8_t *pd,
                                          const XB &x, float *t) {
    const float d = h2f(*(const unsigned short *)pd);
    const uint4 scv = *(const uint4 *)ps;
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
    const int4 *xp = (const int4 *)x.q;
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int md = 0; md < 2; md++) {
            // 16 positions: ql columns 0 (groups gi 0, 2) and 1 (gi 1, 3), qh bits
            const uint4 q0 = *(const uint4 *)(pa + (4 * h + md) * cs), q1 = *(const uint4 *)(pa + (4 * h + 2 + md) * cs);
            const uint4 qh = *(const uint4 *)(pa + (8 + 2 * h + md) * cs);
#pragma unroll
            for (int gi = 0; gi < 4; gi++) {
                const uint4 ql = (gi & 1) ? q1 : q0;
                const uint4 nib = (gi < 2) ? and4(ql, 0x0F0F0F0Fu) : and4(shr4(ql, 4), 0x0F0F0F0Fu);
                const uint4 v = or4(nib, shl4(and4(shr4(qh, 2 * gi), 0x03030303u), 4));
                const int g = 4 * h + gi, si = 2 * g + md;
                const int s = dot16(v, xp[si]);
                const int sc = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xFF);
                const float2 es = x.es[si];
                t[si] = fm(fm(es.x, fm(d, (float)sc)), fs((float)s, fm(32.0f, es.y)));
            }
        }
    }
}

// Q3_K: 16 terms (src/kernels/scalar.rs:236-275)
__device__ __forceinline__ void block_q3k(const uint8_t *pa, int cs, const uint8_t *ps, const uint8_t *pd,
                                          const XB &x, float *t) {
    const float d = h2f(*(const unsigned short *)pd);
    const uint32_t a0 = *(const uint32_t *)ps, a1 = *(const uint32_t *)(ps + 4), tt = *(const uint32_t *)(ps + 8);
    const int4 *xp = (const int4 *)x.q;
#pragma unroll
    for (int md = 0; md < 2; md++) {
        const uint4 hm = *(const uint4 *)(pa + md * cs);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 qs = *(const uint4 *)(pa + (2 + 2 * h + md) * cs);
#pragma unroll
            for (int r4 = 0; r4 < 4; r4++) {
                const int g = 4 * h + r4, si = 2 * g + md, wi = si >> 2;
                const uint4 v = or4(and4(shr4(qs, 2 * r4), 0x03030303u), shl4(and4(shr4(hm, g), 0x01010101u), 2));
                const int s = dot16(v, xp[si]);
                const uint32_t aa = (wi & 1) ? a1 : a0;
                const uint32_t wq = ((aa >> ((wi >> 1) * 4)) & 0x0F0F0F0Fu) | (((tt >> (2 * wi)) & 0x03030303u) << 4);
                const int sc = (int)((wq >> (8 * (si & 3))) & 0xFF);
                const float2 es = x.es[si];
                t[si] = fm(fm(es.x, fm(d, fs((float)sc, 32.0f))), fs((float)s, fm(4.0f, es.y)));
            }
        }
    }
}

// Q2_K: 16 terms. BUF = false: the fused kernel's xe·(d·sc·Σxq·q − dmin·m·xs)
// (src/kernels/q2k.rs:41-69); BUF = true: the buffered path's two terms, as
// in block_k4 (src/quant.rs:367-399 unpacks scale d·(sc&15), offset
// −dmin·(sc>>4)).
template <bool BUF = false>
__device__ __forceinline__ void block_q2k(const uint8_t *pa, int cs, const uint8_t *ps, const uint8_t *pd,
                                          const XB &x, float *t, float *sv = nullptr, bool *anyd = nullptr) {
    const uint32_t dd = *(const uint32_t *)pd;
    const float d = h2f(dd), dm = h2f(dd >> 16);
    const uint4 scv = *(const uint4 *)ps;
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
    const int4 *xp = (const int4 *)x.q;
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int md = 0; md < 2; md++) {
            const uint4 qs = *(const uint4 *)(pa + (2 * h + md) * cs);
#pragma unroll
            for (int r4 = 0; r4 < 4; r4++) {
                const int g = 4 * h + r4, si = 2 * g + md;
                const uint4 v = and4(shr4(qs, 2 * r4), 0x03030303u);
                const int s = dot16(v, xp[si]);
                const int sc = (int)((scw[si >> 2] >> (8 * (si & 3))) & 0xFF);
                const float ev = fm(d, (float)(sc & 0xF)), mv = fm(dm, (float)(sc >> 4));
                const float2 es = x.es[si];
                if (BUF) {
                    t[si] = fm(fm(ev, es.x), (float)s);
                    sv[si] = fm(fm(-mv, es.x), es.y);
                    *anyd = *anyd || mv != 0.0f;
                } else {
                    t[si] = fm(es.x, fs(fm(ev, (float)s), fm(mv, es.y)));
                }
            }
        }
    }
}

// ── dequantize one value from the planes (src/quant.rs:582-679) ──
__device__ inline float dequant_value(const DMat &W, int row, int idx) {
    const int b = idx >> 8, r = idx & 255;
    const uint8_t *A = W.a + (size_t)row * W.a_row + (size_t)b * plane_a_bytes(W.type);
    switch (W.type) {
    case 12: case 13: {
        const uint8_t *blk = A;
        float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
        uint32_t w0 = blk[4] | (blk[5] << 8) | (blk[6] << 16) | ((uint32_t)blk[7] << 24);
        uint32_t w1 = blk[8] | (blk[9] << 8) | (blk[10] << 16) | ((uint32_t)blk[11] << 24);
        uint32_t w2 = blk[12] | (blk[13] << 8) | (blk[14] << 16) | ((uint32_t)blk[15] << 24);
        const int p = r >> 6, half = (r >> 5) & 1, l = r & 31;
        int sc, mn;
        scale_min_k4(2 * p + half, w0, w1, w2, sc, mn);
        float dl = fm(d, (float)sc), ml = fm(dmin, (float)mn);
        if (W.type == 12) {
            uint8_t v = blk[16 + 32 * p + l];
            int qv = half ? (v >> 4) : (v & 0xF);
            return fs(fm(dl, (float)qv), ml);
        }
        uint8_t v = blk[48 + 32 * p + l];
        int qv = half ? (v >> 4) : (v & 0xF);
        float extra = (blk[16 + l] >> (2 * p + half)) & 1 ? 16.0f : 0.0f;
        return fs(fm(dl, fa((float)qv, extra)), ml);
    }
    case 14: {
        const int h = r >> 7, rr = r & 127, gi = rr >> 5, l = rr & 31;
        uint8_t qlb = A[64 * h + 32 * (gi & 1) + l];
        int nib = gi < 2 ? (qlb & 0xF) : (qlb >> 4);
        int qv = (nib | (((A[128 + 32 * h + l] >> (2 * gi)) & 3) << 4)) - 32;
        const uint8_t *S = W.s + (size_t)row * W.s_row + (size_t)b * 16;
        const uint8_t *Dp = W.d + (size_t)row * W.d_row + (size_t)b * 2;
        float d = h2f(Dp[0] | (Dp[1] << 8));
        int sc = (int)(int8_t)S[8 * h + (rr >> 4)];
        return fm(fm(d, (float)sc), (float)qv);
    }
    case 11: {
        const int h = r >> 7, rr = r & 127, r4 = rr >> 5, l = rr & 31, g = 4 * h + r4;
        const uint8_t *S = W.s + (size_t)row * W.s_row + (size_t)b * 12;
        const uint8_t *Dp = W.d + (size_t)row * W.d_row + (size_t)b * 2;
        uint32_t a0 = S[0] | (S[1] << 8) | (S[2] << 16) | ((uint32_t)S[3] << 24);
        uint32_t a1 = S[4] | (S[5] << 8) | (S[6] << 16) | ((uint32_t)S[7] << 24);
        uint32_t tt = S[8] | (S[9] << 8) | (S[10] << 16) | ((uint32_t)S[11] << 24);
        const int is = 2 * g + (l >> 4), wi = is >> 2;
        uint32_t aa = (wi & 1) ? a1 : a0;
        uint32_t wq = ((aa >> ((wi >> 1) * 4)) & 0x0F0F0F0Fu) | (((tt >> (2 * wi)) & 0x03030303u) << 4);
        int sc = (int)((wq >> (8 * (is & 3))) & 0xFF);
        float d = h2f(Dp[0] | (Dp[1] << 8));
        float dl = fm(d, fs((float)sc, 32.0f));
        int hi = (A[l] >> g) & 1 ? 0 : 4;
        int qv = ((A[32 + 32 * h + l] >> (2 * r4)) & 3) - hi;
        return fm(dl, (float)qv);
    }
    default: {  // 10
        const int h = r >> 7, rr = r & 127, r4 = rr >> 5, l = rr & 31, g = 4 * h + r4;
        const uint8_t *S = W.s + (size_t)row * W.s_row + (size_t)b * 16;
        const uint8_t *Dp = W.d + (size_t)row * W.d_row + (size_t)b * 4;
        float d = h2f(Dp[0] | (Dp[1] << 8)), dm = h2f(Dp[2] | (Dp[3] << 8));
        int sc = S[2 * g + (l >> 4)];
        float dl = fm(d, (float)(sc & 0xF)), ml = fm(dm, (float)(sc >> 4));
        int qv = (A[32 * h + l] >> (2 * r4)) & 3;
        return fs(fm(dl, (float)qv), ml);
    }
    }
}

}  // namespace cxm
