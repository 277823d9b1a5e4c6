// Muestreador::elegir (src/sampler.rs:61-126) on the device, one CTA.
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
// Every sum is sequential in the reference's order, on one thread: in the
// flat distributions of a random-init model consecutive cumulative sums are
// ~1/vocab apart, so any other order changes the sampled token. The rest is
// parallel: exps, and a stable LSD radix sort whose ties (equal
// probabilities; the reference's unstable sort leaves their order
// unspecified) come out by ascending index. The walk over the cumulative
// sums, which never decrease, is a binary search.
#pragma once

#include "expf_glibc.h"
#include "kernels.cuh"

namespace cxm {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kCandidates = 1024;  // src/sampler.rs:25

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
};

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

// the count of digit d in warp w's chunk: warp-major with a padded row, so
// a warp's lanes with different digits hit different banks
constexpr int kHistRow = 257;
__device__ __forceinline__ int hidx(int d, int w) { return w * kHistRow + d; }

// one stable counting pass of an LSD radix sort on 8 key bits; a warp owns a
// contiguous chunk and keeps its elements' order
__device__ __forceinline__ void radix_pass(const uint32_t *kin, const uint32_t *vin, uint32_t *kout, uint32_t *vout, int n, int shift,
                           uint32_t *hist /* [kSampWarps][kHistRow] */) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (n + kSampWarps - 1) / kSampWarps;
    const int lo = warp * chunk, hi = min(n, lo + chunk);
    for (int i = tid; i < kHistRow * kSampWarps; i += kSampThreads) hist[i] = 0;
    __syncthreads();
    // four keys per lane in flight before their counts
    for (int b = lo; b < hi; b += 128) {
        uint32_t k[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = b + 32 * u + lane;
            k[u] = i < hi ? __ldcg(kin + i) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (b + 32 * u + lane < hi) atomicAdd(&hist[hidx((k[u] >> shift) & 255, warp)], 1u);
    }
    __syncthreads();
    // exclusive scan over (digit, warp): digit-major, so equal digits keep
    // warp (= position) order; a thread per 8 entries, then the warps' sums
    {
        constexpr int kPer = 256 * kSampWarps / kSampThreads;
        uint32_t c[kPer], loc = 0;
#pragma unroll
        for (int j = 0; j < kPer; j++) {  // entry e = digit * kSampWarps + warp
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
        __shared__ uint32_t wsum[kSampWarps];
        if (lane == 31) wsum[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            uint32_t w = lane < kSampWarps ? wsum[lane] : 0u, wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += v;
            }
            if (lane < kSampWarps) wsum[lane] = wi - w;
        }
        __syncthreads();
        uint32_t run = wsum[warp] + inc - loc;
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int e = tid * kPer + j;
            hist[hidx(e / kSampWarps, e % kSampWarps)] = run;
            run += c[j];
        }
    }
    __syncthreads();
    // the scatter keeps the chunk's order, 32 keys at a time; the next 32
    // keys and values are loaded while this 32 is placed
    uint32_t kn = lo + lane < hi ? __ldcg(kin + lo + lane) : 0u;
    uint32_t vn = lo + lane < hi ? __ldcg(vin + lo + lane) : 0u;
    for (int b = lo; b < hi; b += 32) {
        const int i = b + lane;
        const bool ok = i < hi;
        const uint32_t k = kn, vv = vn, d = (k >> shift) & 255;
        if (b + 32 + lane < hi) {
            kn = __ldcg(kin + b + 32 + lane);
            vn = __ldcg(vin + b + 32 + lane);
        }
        const unsigned same = __match_any_sync(0xffffffffu, ok ? d : 0x100u + lane);
        const int rank = __popc(same & ((1u << lane) - 1));
        const int leader = __ffs(same) - 1;
        uint32_t base = 0;
        if (ok && lane == leader) base = hist[hidx(d, warp)];
        base = __shfl_sync(0xffffffffu, base, leader);
        if (ok) {
            kout[base + rank] = k;
            vout[base + rank] = vv;
        }
        __syncwarp();
        if (ok && lane == leader) hist[hidx(d, warp)] = base + __popc(same);
        __syncwarp();
    }
    __syncthreads();
}

constexpr int kScanChunk = 8192;  // floats per shared-memory stage of a sequential scan

// Thread 0 adds src[0..len) in order, from 0.0f, writing each running sum to
// dst[i] when dst is set and stopping after the first i with sum >= stop when
// use_stop. The other threads stage the next chunk of src into shared memory
// meanwhile. Returns the number of terms added (uniform).
__device__ __forceinline__ int seq_scan(const float *src, int len, float *dst, bool use_stop, float stop, float *stage,
                        float *sum_out, int *flag) {
    const int tid = threadIdx.x;
    float acc = 0.0f;
    int done = len;
    const int nchunk = (len + kScanChunk - 1) / kScanChunk;
    if (tid == 0) *flag = 0;
    for (int i = tid; i < min(len, kScanChunk); i += kSampThreads) stage[i] = src[i];
    __syncthreads();
    for (int c = 0; c < nchunk; c++) {
        const float *cur = stage + (c & 1) * kScanChunk;
        float *nxt = stage + ((c + 1) & 1) * kScanChunk;
        const int base = c * kScanChunk, cnt = min(kScanChunk, len - base);
        if (tid == 0) {
            // 16 values per step: four vector loads in flight, then the adds
            // in order; the running sums never decrease (probabilities are
            // >= 0), so the step's last one tells whether the stop is inside
            int i = 0;
            // the next step's four loads are issued before this step's adds
            float4 n0 = make_float4(0.f, 0.f, 0.f, 0.f), n1 = n0, n2 = n0, n3 = n0;
            if (16 <= cnt) {
                const float4 *c4 = (const float4 *)cur;
                n0 = c4[0];
                n1 = c4[1];
                n2 = c4[2];
                n3 = c4[3];
            }
            for (; i + 16 <= cnt; i += 16) {
                const float4 q0 = n0, q1 = n1, q2 = n2, q3 = n3;
                if (i + 32 <= cnt) {
                    const float4 *c4 = (const float4 *)(cur + i + 16);
                    n0 = c4[0];
                    n1 = c4[1];
                    n2 = c4[2];
                    n3 = c4[3];
                }
                float r[16];
                r[0] = __fadd_rn(acc, q0.x);
                r[1] = __fadd_rn(r[0], q0.y);
                r[2] = __fadd_rn(r[1], q0.z);
                r[3] = __fadd_rn(r[2], q0.w);
                r[4] = __fadd_rn(r[3], q1.x);
                r[5] = __fadd_rn(r[4], q1.y);
                r[6] = __fadd_rn(r[5], q1.z);
                r[7] = __fadd_rn(r[6], q1.w);
                r[8] = __fadd_rn(r[7], q2.x);
                r[9] = __fadd_rn(r[8], q2.y);
                r[10] = __fadd_rn(r[9], q2.z);
                r[11] = __fadd_rn(r[10], q2.w);
                r[12] = __fadd_rn(r[11], q3.x);
                r[13] = __fadd_rn(r[12], q3.y);
                r[14] = __fadd_rn(r[13], q3.z);
                r[15] = __fadd_rn(r[14], q3.w);
                if (dst) {
                    float4 *d4 = (float4 *)(dst + base + i);
                    d4[0] = make_float4(r[0], r[1], r[2], r[3]);
                    d4[1] = make_float4(r[4], r[5], r[6], r[7]);
                    d4[2] = make_float4(r[8], r[9], r[10], r[11]);
                    d4[3] = make_float4(r[12], r[13], r[14], r[15]);
                }
                if (use_stop && r[15] >= stop) {
                    int j = 0;
                    while (r[j] < stop) j++;
                    acc = r[j];
                    done = base + i + j + 1;
                    *flag = 1;
                    break;
                }
                acc = r[15];
            }
            if (!(use_stop && done < len)) {
                for (; i < cnt; i++) {
                    acc = __fadd_rn(acc, cur[i]);
                    if (dst) dst[base + i] = acc;
                    if (use_stop && acc >= stop) {
                        done = base + i + 1;
                        *flag = 1;
                        break;
                    }
                }
            }
        } else if (c + 1 < nchunk) {
            const int nb = base + kScanChunk, ncnt = min(kScanChunk, len - nb);
            for (int i = tid - 1; i < ncnt; i += kSampThreads - 1) nxt[i] = src[nb + i];
        }
        __syncthreads();
        if (*flag) break;
    }
    if (tid == 0) {
        *sum_out = acc;
        *flag = done;
    }
    __syncthreads();
    const int r = *flag;
    __syncthreads();
    return r;
}

// first i in [0, len) with prefix[i] > t (prefix never decreases); len if none
__device__ __forceinline__ int first_above(const float *prefix, int len, float t) {
    int lo = 0, hi = len;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] > t) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

__global__ void __launch_bounds__(kSampThreads, 1) k_sample(const __grid_constant__ SampleArgs a) {
    if (a.d_stop && *(volatile const int *)a.d_stop) return;  // the generation already met its eos (uniform)
    extern __shared__ __align__(16) float stage[];  // 2 x kScanChunk
    __shared__ float red[kSampWarps];
    __shared__ uint32_t hist[kHistRow * kSampWarps];
    __shared__ float u_s, sum_s;
    __shared__ int flag_s;
    const int tid = threadIdx.x, n = a.n;
    const float inv_t = a.params[0], top_p = a.params[1];
    if (tid == 0) {
        unsigned long long st = *a.rng;
        u_s = (float)(azar_next(st) >> 40) / 16777216.0f;
        *a.rng = st;
    }
    // temperature, then softmax (src/ops.rs:1206-1230). The element-wise
    // loops take four elements per thread per step, loads first, so their
    // L2 round trips overlap.
    constexpr int kU = 4, kStep = kU * kSampThreads;
    float m = -INFINITY;
    for (int i0 = tid; i0 < n; i0 += kStep) {
        float v[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) v[u] = i0 + u * kSampThreads < n ? __ldcg(a.logits + i0 + u * kSampThreads) : 0.0f;
#pragma unroll
        for (int u = 0; u < kU; u++)
            if (i0 + u * kSampThreads < n) {
                const float t = __fmul_rn(v[u], inv_t);
                a.probs[i0 + u * kSampThreads] = t;
                m = fmaxf(m, t);
            }
    }
    m = block_max(m, red);
    if (!isfinite(m)) {
        const float p = __fdiv_rn(1.0f, (float)n);
        for (int i = tid; i < n; i += kSampThreads) a.probs[i] = p;
    } else {
        for (int i0 = tid; i0 < n; i0 += kStep) {
            float v[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) v[u] = i0 + u * kSampThreads < n ? a.probs[i0 + u * kSampThreads] : 0.0f;
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (i0 + u * kSampThreads < n) a.probs[i0 + u * kSampThreads] = expf_glibc(__fsub_rn(v[u], m));
        }
        __syncthreads();
        seq_scan(a.probs, n, nullptr, false, 0.0f, stage, &sum_s, &flag_s);  // the total, in index order
        const float inv = __fdiv_rn(1.0f, sum_s);
        for (int i0 = tid; i0 < n; i0 += kStep) {
            float v[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) v[u] = i0 + u * kSampThreads < n ? a.probs[i0 + u * kSampThreads] : 0.0f;
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (i0 + u * kSampThreads < n) a.probs[i0 + u * kSampThreads] = __fmul_rn(v[u], inv);
        }
    }
    __syncthreads();
    const float u = u_s;
    uint32_t tok;
    if (top_p >= 1.0f) {
        // the whole vocabulary in index order (src/sampler.rs:84-86)
        seq_scan(a.probs, n, a.prefix, false, 0.0f, stage, &sum_s, &flag_s);
        const int i = first_above(a.prefix, n, u);
        tok = (uint32_t)(i < n ? i : n - 1);
    } else {
        // descending probability, ties by ascending index: ascending key
        // 0x7fffffff - bits (probabilities are >= 0) on an index-ordered start
        for (int i0 = tid; i0 < n; i0 += kStep) {
            float v[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) v[u] = i0 + u * kSampThreads < n ? a.probs[i0 + u * kSampThreads] : 0.0f;
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (i0 + u * kSampThreads < n) {
                    a.key0[i0 + u * kSampThreads] = 0x7fffffffu - __float_as_uint(v[u]);
                    a.val0[i0 + u * kSampThreads] = (uint32_t)(i0 + u * kSampThreads);
                }
        }
        __syncthreads();
        radix_pass(a.key0, a.val0, a.key1, a.val1, n, 0, hist);
        radix_pass(a.key1, a.val1, a.key0, a.val0, n, 8, hist);
        radix_pass(a.key0, a.val0, a.key1, a.val1, n, 16, hist);
        radix_pass(a.key1, a.val1, a.key0, a.val0, n, 24, hist);
        const uint32_t *order = a.val0;
        float *sorted = a.key1 ? (float *)a.key1 : nullptr;  // probabilities in sorted order
        for (int i0 = tid; i0 < n; i0 += kStep) {
            uint32_t o[kU];
            float v[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) o[u] = i0 + u * kSampThreads < n ? __ldcg(order + i0 + u * kSampThreads) : 0u;
#pragma unroll
            for (int u = 0; u < kU; u++) v[u] = i0 + u * kSampThreads < n ? a.probs[o[u]] : 0.0f;
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (i0 + u * kSampThreads < n) sorted[i0 + u * kSampThreads] = v[u];
        }
        __syncthreads();
        const int k = n < kCandidates ? n : kCandidates;
        seq_scan(sorted, k, nullptr, false, 0.0f, stage, &sum_s, &flag_s);  // the candidates' mass
        const int len = (sum_s < top_p && k < n) ? n : k;
        // cut at the first cumulative sum >= top_p (the crossing token is in);
        // the nucleus's sum is the cumulative sum there
        const int cut = seq_scan(sorted, len, a.prefix, true, top_p, stage, &sum_s, &flag_s);
        const int i = first_above(a.prefix, cut, __fmul_rn(u, sum_s));
        tok = order[i < cut ? i : cut - 1];
    }
    if (tid == 0) {
        if (a.toks) a.toks[*a.d_len] = tok;
        if (a.out) *a.out = tok;
        if (a.d_stop && a.eos >= 0 && tok == (uint32_t)a.eos) *a.d_stop = 1;
    }
}

}  // namespace cxm
