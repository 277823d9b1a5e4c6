// Muestreador::elegir (src/sampler.rs:61-126) on the device: one
// cooperative launch over up to one CTA per SM.
//
// The reference's arithmetic, in its order:
//   u      = (xorshift64*(state) >> 40) / 2^24, drawn first      (:56-59, :73)
//   probs  = softmax(logits * (1/T)): subtract the max, exp, a sequential
//            sum in index order, multiply by 1/total         (src/ops.rs:1206-1230)
//   top_p >= 1: walk the index order, accumulating, first > u   (:84-86, :140-152)
//   else:  the 1024 most probable, sorted by probability (descending); if
//          their mass (a sequential sum in that order) is below top_p, the
//          whole vocabulary sorted instead; cut at the first cumulative sum
//          >= top_p; walk the nucleus against u * (its sequential sum).
// Every sum is the reference's sequential f32 sum, value for value: in the
// flat distributions of a random-init model consecutive cumulative sums are
// ~1/vocab apart, so any other rounding changes the sampled token. The sums
// are nevertheless taken in parallel (exact_scan below): while the running
// sum stays inside one binade, each addition rounds to a multiple of that
// binade's ulp, so the sequence is an integer prefix sum; only the terms
// that leave the binade or round to even (ties) are added one at a time.
// The candidates' mass and the nucleus's sum are entries of the sorted
// order's cumulative sums (they add the same values in the same order from
// zero), and the walks over cumulative sums, which never decrease, are
// searches. The sort is a stable LSD radix sort over all CTAs whose ties
// (equal probabilities; the reference's unstable sort leaves their order
// unspecified) come out by ascending index. CTAs meet at bounded grid
// barriers: a wait that runs out raises ERR_TIMEOUT and the launch returns.
#pragma once

#include "expf_glibc.h"
#include "kernels.cuh"
#include "step_kernels.cuh"

namespace cxm {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kCandidates = 1024;  // src/sampler.rs:25
constexpr int kScanPer = 8;        // terms per thread in a window of exact_scan
constexpr int kScanWin = kScanPer * kSampThreads;
constexpr int kHistRow = 257;      // radix counts: warp-major rows, padded
// dynamic shared memory of k_sample: the radix counts
constexpr int kSampSmem = kSampWarps * kHistRow * 4;

struct SampleArgs {
    const float *logits;
    int n;
    const float *params;      // 1/T, top_p
    unsigned long long *rng;  // xorshift64* state, advanced once
    const int *d_len;         // token goes to toks[*d_len] (or `out` when toks is null)
    uint32_t *toks;
    uint32_t *out;
    int *d_stop;              // set: a generation met its eos; the sampler then does nothing
    int eos;                  // the model's eos token (its pick sets *d_stop), or -1
    float *probs, *prefix;    // scratch [n]
    uint32_t *key0, *val0, *key1, *val1;  // scratch [n]
    uint32_t *ghist;          // scratch [grid * 256]: each CTA's digit counts
    float *gred;              // scratch [grid + 1]: each CTA's max, then 1/total
    unsigned *bar;            // grid-barrier counter, zeroed before each launch
    int *err;                 // ERR_TIMEOUT when a grid barrier's wait runs out
    unsigned long long *stamps;  // measurement only: CTA 0's %globaltimer at its steps' ends [kSampStamps], or NULL
};

constexpr int kSampStamps = 14 + 64;  // 12 step ends, the two sums' pass counts, the total's first 64 passes' starts
__device__ __forceinline__ void samp_stamp(const SampleArgs &a, int k) {
    if (a.stamps && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.stamps[k] = t;
    }
}

__device__ __forceinline__ unsigned long long azar_next(unsigned long long &st) {
    // src/daiss.rs:317-337
    unsigned long long x = st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    st = x;
    return x * 0x2545F4914F6CDD1Dull;
}

__device__ __forceinline__ float block_max(float v, float *red) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    if (tid < 32) {
        float w = tid < kSampWarps ? red[tid] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (tid == 0) red[0] = w;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}


// ── grid barrier (bounded) ──
// `target` counts the arrivals every CTA has made so far; each poll is an L2
// round trip, and 2^21 polls bound a wait near one second.
constexpr uint32_t kSampBarrierSpins = 1u << 21;

__device__ bool samp_sync(const SampleArgs &a, unsigned &target, int *ok_s) {
    target += gridDim.x;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
        for (uint32_t i = 0;; i++) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
            if ((int)(v - target) >= 0) break;
            if (i >= kSampBarrierSpins) {
                atomicOr(a.err, ERR_TIMEOUT);
                ok = 0;
                break;
            }
            if ((i & 255) == 255) {
                if (*(volatile int *)a.err & ERR_TIMEOUT) {  // another CTA gave up
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        *ok_s = ok;
    }
    __syncthreads();
    return *ok_s != 0;
}

// ── the reference's sequential f32 sum, exactly, in parallel ──
// A running sum s in the binade of biased exponent eb (s < 2^(eb-126); the
// subnormals share the binade eb = 1) is M·u with u = 2^(eb-150) and M an
// integer below 2^24. Adding x >= 0 whose exact sum stays below the binade's
// top rounds to the nearest multiple of u: M' = M + round(x/u), ties to an
// even M'. So, from one state, a window of terms is classified at once:
// kf = floor(x/u) and kr = round(x/u) (a tie rounds down here); the running
// M is an integer prefix sum of kr; the first term that is a tie, or whose
// exact sum reaches the binade's top (M + kf >= 2^24), or that is negative,
// infinite or NaN, is an event, added as an f32 addition to the exact sum
// before it, and the next window starts after it. Each window therefore adds
// its terms exactly as the sequential loop does. A sum from zero crosses a
// few dozen binades at most; ties need the bits of x below u/2 to be zero.
// kr = round(x/u) for the binade eb (saturated at 2^25: beyond its top),
// rounded up or not, and whether x is an event by itself (a tie, negative,
// infinite or NaN)
struct ScanTerm {
    uint32_t kr;
    bool up, ev;
};

__device__ __forceinline__ ScanTerm scan_term(float x, int eb) {
    ScanTerm t;
    if (eb >= 24) {  // u >= 2^-126: x/u = x·2^(150-eb), exact below 2^25 (the scale is a normal power of two)
        const float q = __fmul_rn(x, __int_as_float((277 - eb) << 23));
        if (!(x >= 0.0f) || !(q < 33554432.0f)) {  // negative or NaN; or past the binade (infinity too)
            t.kr = 1u << 25;
            t.up = false;
            t.ev = !(x >= 0.0f) || !(x <= 3.4028235e38f);
            return t;
        }
        const float fl = floorf(q), fr = __fsub_rn(q, fl);  // both exact
        t.up = fr > 0.5f;
        t.kr = (uint32_t)fl + (t.up ? 1u : 0u);
        t.ev = fr == 0.5f;
        return t;
    }
    const uint32_t xb = __float_as_uint(x);
    const int xe = (int)(xb >> 23);  // sign and exponent
    const uint32_t xm = (xb & 0x7fffffu) | (xe ? 0x800000u : 0u);
    const int sh = eb - (xe > 1 ? xe : 1);  // x/u = xm / 2^sh
    if (sh <= 0) {  // x >= u: an integer multiple of u
        t.kr = sh < -1 ? (1u << 25) : (xm << (-sh));
        t.up = false;
        t.ev = xe >= 255;
    } else {  // sh > 25 leaves kr = 0 and no tie: xm < 2^24 <= half
        const int s2 = sh < 31 ? sh : 31;
        const uint32_t kf = xm >> s2, rem = xm - (kf << s2), half = 1u << (s2 - 1);
        t.up = rem > half;
        t.kr = kf + (t.up ? 1u : 0u);
        t.ev = rem == half || xe >= 255;
    }
    return t;
}

// M·2^(eb-150) as an f32 (exact: M <= 2^24)
__device__ __forceinline__ float scan_value(uint32_t M, int eb) {
    const float f = (float)M;
    const int e = eb - 150;
    if (e >= -126) return __fmul_rn(f, __int_as_float((e + 127) << 23));
    return __fmul_rn(__fmul_rn(f, __int_as_float(1 << 23)), __int_as_float((e + 253) << 23));
}

struct ScanShared {
    uint32_t wtot[2][kSampWarps];  // by pass parity
    int ev[3], tie[3];             // by pass mod 3: the first event; a tie among the pass's terms
    float s;
    float cand[kSampThreads];  // each thread's first event's sum
    int passes;                // passes of the last exact_scan (measurement)
};

enum : int { SCAN_ALL = 0, SCAN_UNTIL_GE = 1, SCAN_UNTIL_GT = 2 };

// the 8 terms [i0, i0 + 8) of a thread in a window (zeros past len); src is
// 16-byte aligned and i0 a multiple of 8
__device__ __forceinline__ void scan_load8(const float *src, int len, int i0, float (&x)[8]) {
    if (i0 + 8 <= len) {
        const float4 a = __ldcg((const float4 *)(src + i0)), b = __ldcg((const float4 *)(src + i0 + 4));
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) x[k] = i0 + k < len ? __ldcg(src + i0 + k) : 0.0f;
    }
}

constexpr uint32_t kScanCap = 1u << 30;  // saturation of the integer prefix sums (>= 2^24 is all that matters)
__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) { return min(a + b, kScanCap); }

// One CTA: the running sums of src[0..len) from 0.0f, each written to
// dst[i] when dst is set. With SCAN_UNTIL_GE / _GT it stops after the pass
// in which the running sum first reaches >= / > `stop` (entries of dst past
// the returned count are unspecified). Returns the number of leading terms
// summed (uniform); *sum is their sum.
// Windows are aligned runs of kScanWin terms, thread t holding terms
// 8t..8t+7 of each in registers, classified once per binade; the next
// window's loads are in flight while one is summed. A pass covers `span`
// terms from the running position: after an event it restarts there with a
// span as long as the terms summed so far (sums from zero double between
// binade crossings), and it doubles after a pass without one. Every thread
// writes the sums of its terms up to its own first event; a later pass
// rewrites those past the CTA's first event. Without dst, a pass whose block
// sum stays inside the binade and holds no tie skips that walk. Warps whose
// terms are all outside a pass only join its barriers. `pass_stamps`
// (measurement only): the start time of each of the first 64 passes. src and
// dst are 16-byte aligned.
__device__ int exact_scan(const float *src, int len, float *dst, int mode, float stop, ScanShared &sh, float *sum,
                          unsigned long long *pass_stamps = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float x[8], xn[8];
    uint32_t kr[8], up = 0, evm = 0;
    int cur = 0, ceb = -1;  // the window held in x; the binade of its classification
    scan_load8(src, len, 8 * tid, x);
    scan_load8(src, len, kScanWin + 8 * tid, xn);
    if (tid == 0)
        for (int i = 0; i < 3; i++) {
            sh.ev[i] = INT_MAX;
            sh.tie[i] = 0;
        }
    __syncthreads();
    float s = 0.0f;
    int pos = 0, span = kSampThreads, it = 0;
    for (;; it++) {
        const int e3 = it % 3;
        if (tid == 0) {  // the next pass's slots: their last readers (two passes back) are past this pass's first barrier
            sh.ev[(it + 1) % 3] = INT_MAX;
            sh.tie[(it + 1) % 3] = 0;
        }
        if (pass_stamps && tid == 0 && it < 64) {  // measurement only
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            pass_stamps[it] = t;
        }
        if (pos >= len || (pos > 0 && ((mode == SCAN_UNTIL_GE && s >= stop) || (mode == SCAN_UNTIL_GT && s > stop))))
            break;  // (no term summed yet: the stop is tested after the first)
        if (!(s <= 3.4028235e38f)) {  // infinite or NaN: the rest in order, on one thread
            if (tid == 0) {
                float r = s;
                for (int i = pos; i < len; i++) {
                    r = __fadd_rn(r, src[i]);
                    if (dst) dst[i] = r;
                }
                sh.s = r;
            }
            __syncthreads();
            s = sh.s;
            pos = len;
            break;
        }
        if (pos / kScanWin != cur) {  // the next window (uniform): its terms are loaded
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = xn[k];
            cur++;
            ceb = -1;
            scan_load8(src, len, (cur + 1) * kScanWin + 8 * tid, xn);
        }
        const uint32_t sb = __float_as_uint(s);
        const int eb = (int)(sb >> 23) > 1 ? (int)(sb >> 23) : 1;
        const uint32_t M0 = (sb & 0x7fffffu) | ((sb >> 23) ? 0x800000u : 0u);
        const int wbase = cur * kScanWin, base = wbase + 8 * tid;
        const int end = min(min(len, wbase + kScanWin), pos + span);  // this pass: terms [pos, end)
        // warps whose 256 terms are all outside the pass skip to the barriers
        const bool wact = wbase + 256 * warp + 256 > pos && wbase + 256 * warp < end;
        if (wact && eb != ceb) {
            up = evm = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const ScanTerm t = scan_term(x[k], eb);
                kr[k] = t.kr;
                up |= (t.up ? 1u : 0u) << k;
                evm |= (t.ev ? 1u : 0u) << k;
            }
            ceb = eb;
        }
        uint32_t act = 0, loc = 0, inc = 0;  // active terms of this thread, their sum (< 2^28), the warp's prefix
        if (wact) {
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (base + k >= pos && base + k < end) {
                    act |= 1u << k;
                    loc += kr[k];
                }
            // inclusive prefix of loc over the warp, saturating
            inc = loc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc = sat_add(inc, v);
            }
        }
        if (lane == 31) sh.wtot[it & 1][warp] = inc;
        if (act & evm) sh.tie[e3] = 1;
        __syncthreads();
        uint32_t wi = sh.wtot[it & 1][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi = sat_add(wi, v);
        }
        const uint32_t total = __shfl_sync(0xffffffffu, wi, 31);
        const uint32_t wex = warp ? __shfl_sync(0xffffffffu, wi, warp - 1) : 0u;
        const uint32_t tex = __shfl_up_sync(0xffffffffu, inc, 1);
        uint32_t P = sat_add(M0, sat_add(wex, lane ? tex : 0u));  // (inactive warps: unused)
        if (!dst && !sh.tie[e3] && M0 + total < (1u << 24)) {  // no event in the pass, no sums to write
            s = scan_value(M0 + total, eb);
            pos = end;
            span = min(kScanWin, 2 * span);
            continue;
        }
        // the sums of this thread's terms, up to its first event (the sums
        // after it are rewritten by a later pass)
        int eloc = INT_MAX;
        if (act) {
            float out[8];
            bool done = false;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                out[k] = 0.0f;
                if (done || !((act >> k) & 1)) continue;
                const uint32_t kf = kr[k] - ((up >> k) & 1);
                if (((evm >> k) & 1) || P + kf >= (1u << 24)) {  // an f32 addition to the exact sum before it
                    out[k] = __fadd_rn(scan_value(P, eb), x[k]);
                    sh.cand[tid] = out[k];
                    eloc = base + k;
                    done = true;
                } else {
                    P += kr[k];
                    out[k] = scan_value(P, eb);
                }
            }
            if (dst) {
                if (act == 0xFFu) {
                    ((float4 *)(dst + base))[0] = make_float4(out[0], out[1], out[2], out[3]);
                    ((float4 *)(dst + base))[1] = make_float4(out[4], out[5], out[6], out[7]);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        if ((act >> k) & 1) dst[base + k] = out[k];
                }
            }
        }
        // one shared atomic per warp: past a crossing every later thread has an event
        const int wmin = __reduce_min_sync(0xffffffffu, eloc);
        if (lane == 0 && wmin != INT_MAX) atomicMin(&sh.ev[e3], wmin);
        __syncthreads();
        const int E = sh.ev[e3];
        if (E != INT_MAX) {
            s = sh.cand[(E - wbase) >> 3];
            pos = E + 1;
            span = min(kScanWin, max(kSampThreads, pos));
        } else {
            s = scan_value(M0 + total, eb);
            pos = end;
            span = min(kScanWin, 2 * span);
        }
    }
    if (sum) *sum = s;
    if (tid == 0) sh.passes = it;
    __syncthreads();
    return pos;
}

// first i in [0, len) with p[i] > t (gt) or >= t, over values that never
// decrease; len if none. One CTA, uniform result.
__device__ int block_first(const float *p, int len, float t, bool gt) {
    const int tid = threadIdx.x;
    int lo = 0, hi = len;  // the answer is in [lo, hi]
    while (hi > lo) {
        const int span = hi - lo;
        const int stride = span <= kSampThreads ? 1 : (span + kSampThreads - 1) / kSampThreads;
        const int i = lo + tid * stride;
        bool below = false;
        if (i < hi) {
            const float v = __ldcg(p + i);
            below = gt ? !(v > t) : !(v >= t);
        }
        const int nf = __syncthreads_count(below);  // the samples below t come first
        if (stride == 1) return lo + nf;
        if (nf == 0) return lo;
        const int nlo = lo + (nf - 1) * stride + 1;
        hi = min(hi, lo + nf * stride);
        lo = nlo;
    }
    return lo;
}

// ── one stable LSD radix pass over all CTAs, on 8 key bits ──
// A CTA owns the contiguous tile [lo, hi) and its warps contiguous chunks of
// it. Counts per (digit, warp) give each chunk's place inside the tile; the
// CTAs' digit counts (through ghist, across a grid barrier) give the tile's
// place among the CTAs, so equal digits keep their (CTA, warp, lane) order.
__device__ __forceinline__ int hidx(int d, int w) { return w * kHistRow + d; }

__device__ bool radix_pass(const SampleArgs &a, const uint32_t *kin, const uint32_t *vin, uint32_t *kout,
                           uint32_t *vout, int lo, int hi, int shift, uint32_t *hist, unsigned &target, int *ok_s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (hi - lo + kSampWarps - 1) / kSampWarps;
    const int wlo = lo + warp * chunk, whi = min(hi, wlo + chunk);
    __shared__ uint32_t dall[4][256], dbef[4][256], gadj[256];
    __shared__ uint32_t wsum[kSampWarps];
    for (int i = tid; i < kHistRow * kSampWarps; i += kSampThreads) hist[i] = 0;
    __syncthreads();
    for (int b = wlo; b < whi; b += 128) {
        uint32_t k[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = b + 32 * u + lane;
            k[u] = i < whi ? __ldcg(kin + i) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (b + 32 * u + lane < whi) atomicAdd(&hist[hidx((k[u] >> shift) & 255, warp)], 1u);
    }
    __syncthreads();
    // this CTA's digit counts, published for the others
    if (tid < 256) {
        uint32_t c = 0;
        for (int w = 0; w < kSampWarps; w++) c += hist[hidx(tid, w)];
        a.ghist[blockIdx.x * 256 + tid] = c;
    }
    // exclusive scan over (digit, warp), digit-major: a thread per 8 entries
    {
        constexpr int kPer = 256 * kSampWarps / kSampThreads;
        uint32_t c[kPer], loc = 0;
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int e = tid * kPer + j;
            c[j] = hist[hidx(e / kSampWarps, e % kSampWarps)];
            loc += c[j];
        }
        uint32_t inc = loc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        if (lane == 31) wsum[warp] = inc;
        __syncthreads();
        uint32_t wt = wsum[lane], wi = wt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += v;
        }
        uint32_t run = __shfl_sync(0xffffffffu, wi - wt, warp) + inc - loc;
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int e = tid * kPer + j;
            hist[hidx(e / kSampWarps, e % kSampWarps)] = run;  // offset inside the tile
            run += c[j];
        }
    }
    if (!samp_sync(a, target, ok_s)) return false;
    // the tile's place: digit d starts after the counts of all smaller
    // digits and of d in the CTAs before this one; four threads per digit,
    // a quarter of the CTAs each
    {
        const int d = tid & 255, part = tid >> 8, G = gridDim.x;
        const int q = (G + 3) / 4, c0 = part * q, c1 = min(G, c0 + q);
        uint32_t all = 0, before = 0;
        for (int c = c0; c < c1; c++) {
            const uint32_t v = __ldcg(a.ghist + c * 256 + d);
            all += v;
            before += c < (int)blockIdx.x ? v : 0u;
        }
        dall[part][d] = all;
        dbef[part][d] = before;
        __syncthreads();
        uint32_t tot = 0, inc = 0;
        if (tid < 256) {  // warps 0-7: an exclusive scan of the 256 digit totals
            tot = dall[0][d] + dall[1][d] + dall[2][d] + dall[3][d];
            inc = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += v;
            }
            if (lane == 31) wsum[warp] = inc;
        }
        __syncthreads();
        if (tid < 256) {
            uint32_t woff = 0;
            for (int w = 0; w < warp; w++) woff += wsum[w];
            const uint32_t bef = dbef[0][d] + dbef[1][d] + dbef[2][d] + dbef[3][d];
            gadj[d] = woff + inc - tot + bef - hist[hidx(d, 0)];
        }
        __syncthreads();
        for (int e = tid; e < 256 * kSampWarps; e += kSampThreads) hist[hidx(e & 255, e >> 8)] += gadj[e & 255];
        __syncthreads();
    }
    // the scatter keeps each chunk's order, 32 keys at a time; the next 32
    // keys and values are loaded while this 32 is placed
    uint32_t kn = wlo + lane < whi ? __ldcg(kin + wlo + lane) : 0u;
    uint32_t vn = wlo + lane < whi ? __ldcg(vin + wlo + lane) : 0u;
    for (int b = wlo; b < whi; b += 32) {
        const int i = b + lane;
        const bool ok = i < whi;
        const uint32_t k = kn, vv = vn, dg = (k >> shift) & 255;
        if (b + 32 + lane < whi) {
            kn = __ldcg(kin + b + 32 + lane);
            vn = __ldcg(vin + b + 32 + lane);
        }
        const unsigned same = __match_any_sync(0xffffffffu, ok ? dg : 0x100u + lane);
        const int rank = __popc(same & ((1u << lane) - 1));
        const int leader = __ffs(same) - 1;
        uint32_t base = 0;
        if (ok && lane == leader) base = hist[hidx(dg, warp)];
        base = __shfl_sync(0xffffffffu, base, leader);
        if (ok) {
            kout[base + rank] = k;
            vout[base + rank] = vv;
        }
        __syncwarp();
        if (ok && lane == leader) hist[hidx(dg, warp)] = base + __popc(same);
        __syncwarp();
    }
    return samp_sync(a, target, ok_s);
}

__global__ void __launch_bounds__(kSampThreads, 1) k_sample(const __grid_constant__ SampleArgs a) {
    if (a.d_stop && *(volatile const int *)a.d_stop) return;  // the generation already met its eos (uniform)
    extern __shared__ __align__(16) unsigned char samp_smem[];
    uint32_t *hist = (uint32_t *)samp_smem;                          // [kSampWarps][kHistRow]
    __shared__ float red[kSampWarps];
    __shared__ ScanShared sh;
    __shared__ float u_s, sum_s;
    __shared__ int ok_s;
    const int tid = threadIdx.x, n = a.n, G = gridDim.x, cta = blockIdx.x;
    const int tile = (n + G - 1) / G, lo = min(n, cta * tile), hi = min(n, lo + tile);
    const float inv_t = a.params[0], top_p = a.params[1];
    unsigned target = 0;
    samp_stamp(a, 0);
    if (cta == 0 && tid == 0) {
        unsigned long long st = *a.rng;
        u_s = (float)(azar_next(st) >> 40) / 16777216.0f;
        *a.rng = st;
    }
    // temperature, then softmax (src/ops.rs:1206-1230), each CTA on its tile
    float m = -INFINITY;
    for (int i = lo + tid; i < hi; i += kSampThreads) {
        const float t = __fmul_rn(__ldcg(a.logits + i), inv_t);
        a.probs[i] = t;
        m = fmaxf(m, t);
    }
    m = block_max(m, red);
    if (tid == 0) a.gred[cta] = m;
    if (!samp_sync(a, target, &ok_s)) return;
    samp_stamp(a, 1);
    float gm = -INFINITY;
    for (int c = tid; c < G; c += kSampThreads) gm = fmaxf(gm, __ldcg(a.gred + c));
    gm = block_max(gm, red);
    if (!isfinite(gm)) {  // all -inf, or +inf present: the uniform distribution
        const float p = __fdiv_rn(1.0f, (float)n);
        for (int i = lo + tid; i < hi; i += kSampThreads) a.probs[i] = p;
    } else {
        for (int i = lo + tid; i < hi; i += kSampThreads) a.probs[i] = expf_glibc(__fsub_rn(a.probs[i], gm));
        if (!samp_sync(a, target, &ok_s)) return;
        samp_stamp(a, 2);
        if (cta == 0) {  // the total, in index order
            exact_scan(a.probs, n, nullptr, SCAN_ALL, 0.0f, sh, &sum_s, a.stamps ? a.stamps + 14 : nullptr);
            if (a.stamps && tid == 0) a.stamps[12] = (unsigned long long)sh.passes;
            if (tid == 0) a.gred[G] = __fdiv_rn(1.0f, sum_s);
        }
        if (!samp_sync(a, target, &ok_s)) return;
        samp_stamp(a, 3);
        const float inv = __ldcg(a.gred + G);
        for (int i = lo + tid; i < hi; i += kSampThreads) a.probs[i] = __fmul_rn(a.probs[i], inv);
    }
    uint32_t tok;
    if (top_p >= 1.0f) {
        // the whole vocabulary in index order (src/sampler.rs:84-86)
        if (!samp_sync(a, target, &ok_s) || cta != 0) return;
        const float u = u_s;
        const int len = exact_scan(a.probs, n, a.prefix, SCAN_UNTIL_GT, u, sh, nullptr);
        const int i = block_first(a.prefix, len, u, true);
        tok = (uint32_t)(i < len ? i : n - 1);
    } else {
        // descending probability, ties by ascending index: ascending key
        // 0x7fffffff - bits (probabilities are >= 0) on an index-ordered start
        for (int i = lo + tid; i < hi; i += kSampThreads) {
            a.key0[i] = 0x7fffffffu - __float_as_uint(a.probs[i]);
            a.val0[i] = (uint32_t)i;
        }
        __syncthreads();
        samp_stamp(a, 4);
        if (!radix_pass(a, a.key0, a.val0, a.key1, a.val1, lo, hi, 0, hist, target, &ok_s)) return;
        samp_stamp(a, 5);
        if (!radix_pass(a, a.key1, a.val1, a.key0, a.val0, lo, hi, 8, hist, target, &ok_s)) return;
        samp_stamp(a, 6);
        if (!radix_pass(a, a.key0, a.val0, a.key1, a.val1, lo, hi, 16, hist, target, &ok_s)) return;
        samp_stamp(a, 7);
        if (!radix_pass(a, a.key1, a.val1, a.key0, a.val0, lo, hi, 24, hist, target, &ok_s)) return;
        samp_stamp(a, 8);
        const uint32_t *order = a.val0;
        float *sorted = (float *)a.key1;  // probabilities in sorted order
        for (int i = lo + tid; i < hi; i += kSampThreads) sorted[i] = __ldcg(a.probs + __ldcg(order + i));
        if (!samp_sync(a, target, &ok_s) || cta != 0) return;
        samp_stamp(a, 9);
        const float u = u_s;
        // The cumulative sums of the sorted probabilities. The candidates'
        // mass is the one at k - 1; below top_p (with k < n) the whole order
        // is the nucleus, else the candidates, whose first sum >= top_p then
        // comes before k: either way the cut is after the first sum >= top_p,
        // or at n (src/sampler.rs:96-117).
        const int len = exact_scan(sorted, n, a.prefix, SCAN_UNTIL_GE, top_p, sh, nullptr);
        samp_stamp(a, 10);
        if (a.stamps && tid == 0) a.stamps[13] = (unsigned long long)sh.passes;
        const int first = block_first(a.prefix, len, top_p, false);
        const int cut = first < len ? first + 1 : n;
        const float total = __ldcg(a.prefix + cut - 1);
        const int i = block_first(a.prefix, cut, __fmul_rn(u, total), true);
        tok = __ldcg(order + (i < cut ? i : cut - 1));
    }
    samp_stamp(a, 11);
    if (tid == 0) {
        if (a.toks) a.toks[*a.d_len] = tok;
        if (a.out) *a.out = tok;
        if (a.d_stop && a.eos >= 0 && tok == (uint32_t)a.eos) *a.d_stop = 1;
    }
}

}  // namespace cxm
