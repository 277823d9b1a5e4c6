/*
 * cxm_x86.c — AVX2 restatement of the kernels the reference runs on an x86-64
 * host with AVX2, FMA and F16C (src/kernels/x86.rs; the backend is picked by
 * src/kernels/mod.rs:136-163, and every CPU of that class takes it).
 *
 * TEST INFRASTRUCTURE ONLY. These kernels make the timed CPU baseline of
 * bench.py run at the reference's own speed on its own instruction set; the
 * parity checks use the scalar restatement in cxm_oracle.c, which stays the
 * default backend. Each kernel forms the same integer products as its scalar
 * twin and differs from it only in the order of the float additions (several
 * vector accumulators, FMA, one horizontal reduction at the end), exactly as
 * the reference's AVX2 kernels differ from its scalar ones.
 */
#include "cxm_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <string.h>

/* Sum of the eight lanes, halving 256 -> 128 -> 64 -> 32 bits
 * (src/kernels/x86.rs:132-146 and its twin `reducir_f32`). */
static inline float lanes_sum(__m256 v) {
    __m128 q = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    __m128 h = _mm_add_ps(q, _mm_movehl_ps(q, q));
    return _mm_cvtss_f32(_mm_add_ss(h, _mm_shuffle_ps(h, h, 0x55)));
}

/* x86.rs:25-128: four 8-wide FMA chains over 32 values, a tail of whole
 * vectors into the first chain, the chains summed pairwise and reduced, and
 * the last n % 8 products added one by one. */
float orc_x86_dot_f32(const float *a, const float *b, size_t n) {
    __m256 c0 = _mm256_setzero_ps(), c1 = _mm256_setzero_ps();
    __m256 c2 = _mm256_setzero_ps(), c3 = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 32 <= n; i += 32) {
        c0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), c0);
        c1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), c1);
        c2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16), c2);
        c3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24), c3);
    }
    for (; i + 8 <= n; i += 8) c0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), c0);
    float t = lanes_sum(_mm256_add_ps(_mm256_add_ps(c0, c1), _mm256_add_ps(c2, c3)));
    for (; i < n; i++) t += a[i] * b[i];
    return t;
}

/* x86.rs:152-213: the sum of squares in f32 over two FMA chains, one scalar
 * 1/sqrt, then x * scale * w eight at a time. */
void orc_x86_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps) {
    if (n == 0) return;
    __m256 c0 = _mm256_setzero_ps(), c1 = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 16 <= n; i += 16) {
        __m256 u = _mm256_loadu_ps(in + i), v = _mm256_loadu_ps(in + i + 8);
        c0 = _mm256_fmadd_ps(u, u, c0);
        c1 = _mm256_fmadd_ps(v, v, c1);
    }
    for (; i + 8 <= n; i += 8) {
        __m256 u = _mm256_loadu_ps(in + i);
        c0 = _mm256_fmadd_ps(u, u, c0);
    }
    float sum = lanes_sum(_mm256_add_ps(c0, c1));
    for (; i < n; i++) sum += in[i] * in[i];
    const float scale = 1.0f / sqrtf(sum / (float)n + eps);
    const __m256 vs = _mm256_set1_ps(scale);
    for (i = 0; i + 8 <= n; i += 8)
        _mm256_storeu_ps(out + i, _mm256_mul_ps(_mm256_mul_ps(_mm256_loadu_ps(in + i), vs), _mm256_loadu_ps(w + i)));
    for (; i < n; i++) out[i] = in[i] * scale * w[i];
}

static inline __m256 bytes8_to_ps(uint64_t v) {
    return _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_cvtsi64_si128((long long)v)));
}

static inline uint32_t rd32(const uint8_t *p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}

/* Q4_K row · i8 activation, x86.rs:394-558.
 *
 * Per super-block: d and dmin through the F16C conversion; the eight 6-bit
 * scales and mins unpacked at once from three little-endian words of the
 * 12 scale bytes (scales 0-3 / mins 0-3: low six bits of bytes 0-3 / 4-7;
 * scales 4-7 / mins 4-7: low / high nibble of bytes 8-11 with the top two bits
 * of bytes 0-3 / 4-7 above them); xe*d*scale for the eight sub-blocks, and the
 * dmin*min*xe*xs term gathered in a second accumulator. The unsigned nibbles
 * meet the signed activation in vpmaddubsw (at most 2*15*127, no saturation),
 * vpmaddwd widens the pairs to i32, and one FMA per 32 values adds the
 * sub-block's products times its scale. The row total is one reduction of
 * each accumulator. */
static inline void q4k_block_scales(const uint8_t *b, const float *xe, const float *xs, float s[8], __m256 *mins) {
    const __m128 h = _mm_cvtph_ps(_mm_cvtsi32_si128((int)rd32(b)));
    const float d = _mm_cvtss_f32(h), dmin = _mm_cvtss_f32(_mm_movehdup_ps(h));
    const uint32_t w0 = rd32(b + 4), w1 = rd32(b + 8), w2 = rd32(b + 12);
    const uint64_t sc = (uint64_t)(w0 & 0x3F3F3F3Fu) |
                        (uint64_t)((w2 & 0x0F0F0F0Fu) | (((w0 >> 6) & 0x03030303u) << 4)) << 32;
    const uint64_t mn = (uint64_t)(w1 & 0x3F3F3F3Fu) |
                        (uint64_t)(((w2 >> 4) & 0x0F0F0F0Fu) | (((w1 >> 6) & 0x03030303u) << 4)) << 32;
    const __m256 xe8 = _mm256_loadu_ps(xe);
    _mm256_storeu_ps(s, _mm256_mul_ps(_mm256_mul_ps(_mm256_set1_ps(d), bytes8_to_ps(sc)), xe8));
    *mins = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_mul_ps(_mm256_set1_ps(dmin), bytes8_to_ps(mn)), xe8),
                            _mm256_loadu_ps(xs), *mins);
}

/* One block's scale step alone (test access): xe*d*scale of its 8
 * sub-blocks, and the 8 lanes of dmin*min*xe*xs from a zero accumulator. */
void orc_x86_q4k_scales(const uint8_t *block, const float *xe, const float *xs, float *scales8, float *mins8) {
    __m256 mins = _mm256_setzero_ps();
    q4k_block_scales(block, xe, xs, scales8, &mins);
    _mm256_storeu_ps(mins8, mins);
}

float orc_x86_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    const __m256i ones = _mm256_set1_epi16(1), low4 = _mm256_set1_epi8(0x0F);
    __m256 acc = _mm256_setzero_ps(), mins = _mm256_setzero_ps();
    for (size_t bl = 0; bl < nblk; bl++) {
        const uint8_t *b = row + bl * 144;
        float s[8];
        q4k_block_scales(b, xe + bl * 8, xs + bl * 8, s, &mins);
        const uint8_t *qs = b + 16;
        const int8_t *x = xq + bl * 256;
        for (int p = 0; p < 4; p++) {
            const __m256i w = _mm256_loadu_si256((const __m256i *)(qs + 32 * p));
            const __m256i lo = _mm256_and_si256(w, low4);
            const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(w, 4), low4);
            const __m256i p0 = _mm256_madd_epi16(
                _mm256_maddubs_epi16(lo, _mm256_loadu_si256((const __m256i *)(x + 64 * p))), ones);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p0), _mm256_set1_ps(s[2 * p]), acc);
            const __m256i p1 = _mm256_madd_epi16(
                _mm256_maddubs_epi16(hi, _mm256_loadu_si256((const __m256i *)(x + 64 * p + 32))), ones);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p1), _mm256_set1_ps(s[2 * p + 1]), acc);
        }
    }
    return lanes_sum(acc) - lanes_sum(mins);
}

/* The reference's assembly Q4_K kernel with the "complete" contract writes
 * its two accumulators (products, mins) as 16 floats; the Rust side reduces
 * each and subtracts (src/kernels/q4k_asm.rs:214-235). */
float orc_x86_reduce_q4k_acc(const float *acc) {
    return lanes_sum(_mm256_loadu_ps(acc)) - lanes_sum(_mm256_loadu_ps(acc + 8));
}

/* Q6_K row · i8 activation, x86.rs:760-846.
 *
 * Per super-block: the 16 signed scale bytes widened to f32 in two halves,
 * d*scale*xe for each sub-block of 16, and d*scale*xe*xs gathered in a
 * correction accumulator (the values are built unsigned, 0..63, and their
 * offset of 32 is taken off at the end through the activation sums). Each
 * group of 32 values takes its low four bits from a nibble of ql and its top
 * two from qh, shifted into bits 4-5 (16-bit shifts carry bits in from the
 * neighbouring byte, which the masks drop); vpmaddubsw / vpmaddwd give eight
 * i32 lanes, four per sub-block, and a lane permutation spreads the pair of
 * sub-block scales across them. Two product accumulators alternate by group. */
float orc_x86_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    const __m256i ones = _mm256_set1_epi16(1), low4 = _mm256_set1_epi8(0x0F), top2 = _mm256_set1_epi8(0x30);
    const __m256i pick[4] = {_mm256_setr_epi32(0, 0, 0, 0, 1, 1, 1, 1), _mm256_setr_epi32(2, 2, 2, 2, 3, 3, 3, 3),
                             _mm256_setr_epi32(4, 4, 4, 4, 5, 5, 5, 5), _mm256_setr_epi32(6, 6, 6, 6, 7, 7, 7, 7)};
    __m256 acc[2] = {_mm256_setzero_ps(), _mm256_setzero_ps()};
    __m256 corr = _mm256_setzero_ps();
    for (size_t bl = 0; bl < nblk; bl++) {
        const uint8_t *b = row + bl * 210;
        const int8_t *x = xq + bl * 256;
        const __m128i sc16 = _mm_loadu_si128((const __m128i *)(b + 192));
        uint16_t dh;
        memcpy(&dh, b + 208, 2);
        const __m256 d = _mm256_broadcastss_ps(_mm_cvtph_ps(_mm_cvtsi32_si128((int)dh)));
        __m256 v[2];
        v[0] = _mm256_mul_ps(_mm256_mul_ps(d, _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(sc16))),
                             _mm256_loadu_ps(xe + bl * 16));
        v[1] = _mm256_mul_ps(_mm256_mul_ps(d, _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(sc16, 8)))),
                             _mm256_loadu_ps(xe + bl * 16 + 8));
        corr = _mm256_fmadd_ps(v[0], _mm256_loadu_ps(xs + bl * 16), corr);
        corr = _mm256_fmadd_ps(v[1], _mm256_loadu_ps(xs + bl * 16 + 8), corr);
        for (int half = 0; half < 2; half++) {
            const __m256i ql0 = _mm256_loadu_si256((const __m256i *)(b + 64 * half));
            const __m256i ql1 = _mm256_loadu_si256((const __m256i *)(b + 64 * half + 32));
            const __m256i qh = _mm256_loadu_si256((const __m256i *)(b + 128 + 32 * half));
            const __m256i low[4] = {ql0, ql1, _mm256_srli_epi16(ql0, 4), _mm256_srli_epi16(ql1, 4)};
            const __m256i high[4] = {_mm256_slli_epi16(qh, 4), _mm256_slli_epi16(qh, 2), qh, _mm256_srli_epi16(qh, 2)};
            for (int g = 0; g < 4; g++) {
                const __m256i q = _mm256_or_si256(_mm256_and_si256(low[g], low4), _mm256_and_si256(high[g], top2));
                const __m256i xv = _mm256_loadu_si256((const __m256i *)(x + (4 * half + g) * 32));
                const __m256i p32 = _mm256_madd_epi16(_mm256_maddubs_epi16(q, xv), ones);
                acc[g & 1] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p32), _mm256_permutevar8x32_ps(v[half], pick[g]),
                                             acc[g & 1]);
            }
        }
    }
    return lanes_sum(_mm256_add_ps(acc[0], acc[1])) - 32.0f * lanes_sum(corr);
}

/* dot_i8_escalado_avx2, x86.rs:315-380. The eight i32 lanes of a 32-byte
 * chunk (lane l = bytes 4l..4l+3, from vpmaddubsw on |a| and sign(b, a), then
 * vpmaddwd with ones) are converted to f32 and FMA'd into one accumulator with
 * the chunk's scale product: [e0 x4, e1 x4] for sub-blocks of 16 (two per
 * chunk), ea*eb on all lanes for sub-blocks of 32k; one lane reduction. */
float orc_x86_dot_i8_scaled(const int8_t *a, const int8_t *b, const float *ea, const float *eb, size_t n, int block) {
    const __m256i ones = _mm256_set1_epi16(1);
    __m256 acc = _mm256_setzero_ps();
    if (block == 16) {
        const size_t pairs = n / 32;
        for (size_t i = 0; i < pairs; i++) {
            const float e0 = ea[2 * i] * eb[2 * i], e1 = ea[2 * i + 1] * eb[2 * i + 1];
            const __m256 sc = _mm256_setr_ps(e0, e0, e0, e0, e1, e1, e1, e1);
            const __m256i va = _mm256_loadu_si256((const __m256i *)(a + 32 * i));
            const __m256i vb = _mm256_loadu_si256((const __m256i *)(b + 32 * i));
            const __m256i p32 = _mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_sign_epi8(va, va), _mm256_sign_epi8(vb, va)), ones);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p32), sc, acc);
        }
        return lanes_sum(acc);
    }
    const size_t per = (size_t)block / 32, nb = n / (size_t)block;
    for (size_t i = 0; i < nb; i++) {
        const __m256 sc = _mm256_set1_ps(ea[i] * eb[i]);
        for (size_t t = 0; t < per; t++) {
            const size_t idx = i * per + t;
            const __m256i va = _mm256_loadu_si256((const __m256i *)(a + 32 * idx));
            const __m256i vb = _mm256_loadu_si256((const __m256i *)(b + 32 * idx));
            const __m256i p32 = _mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_sign_epi8(va, va), _mm256_sign_epi8(vb, va)), ones);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p32), sc, acc);
        }
    }
    return lanes_sum(acc);
}

/* One (row, column) output of the tile kernels, x86.rs:864-948: per chunk,
 * the column's eight lane sums (vpmaddubsw of unsigned column bytes and
 * signed row bytes when `unsig`, else the sign trick of the i8 kernel),
 * converted, times the column's expanded scales, FMA'd with the row's
 * expanded scales into the accumulator; one lane reduction at the end. */
float orc_x86_tile_out(const int8_t *x, const float *ex, const int8_t *w, const float *ew, size_t chunks, int unsig) {
    const __m256i ones = _mm256_set1_epi16(1);
    __m256 acc = _mm256_setzero_ps();
    for (size_t t = 0; t < chunks; t++) {
        const __m256i col = _mm256_loadu_si256((const __m256i *)(w + 32 * t));
        const __m256i xv = _mm256_loadu_si256((const __m256i *)(x + 32 * t));
        const __m256 ec = _mm256_loadu_ps(ew + 8 * t), ef = _mm256_loadu_ps(ex + 8 * t);
        const __m256i p32 = unsig ? _mm256_madd_epi16(_mm256_maddubs_epi16(col, xv), ones)
                                  : _mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_sign_epi8(col, col), _mm256_sign_epi8(xv, col)), ones);
        const __m256 v = _mm256_mul_ps(_mm256_cvtepi32_ps(p32), ec);
        acc = _mm256_fmadd_ps(v, ef, acc);
    }
    return lanes_sum(acc);
}
