// The prompt forward of 24 tokens and more on the tensor cores.
//
// The reference multiplies all the tokens of one forward call at once, and
// from BLOQUES_DESDE = 24 rows every matrix takes its buffered path
// (src/ops.rs:1073-1079, :599-606 on the portable backend): per output,
// dot_i8_escalado over the row's sub-blocks, total += (esc·xe)·Σxq·q, then,
// when any offset of the row is nonzero, total += (des·xe)·xs sub-block by
// sub-block (src/ops.rs:372-405, src/kernels/scalar.rs:95-109). The integer
// sums Σxq·q are exact and do not depend on their order, so they come from
// int8 tensor-core MMAs (tcgen05.mma kind::i8, s32 accumulators in tensor
// memory), one accumulator per sub-block; the float chain then runs on the
// CUDA cores in the reference's order. The results are those of the decode
// kernel replaying the tokens one by one with ROWS_MANY orders, bit for bit.
//
// Kernels:
//   k_pf_embed  the tokens' embedding rows
//   k_pf_rows   RMSNorm (optional) + i8 quantization of each token's row, into
//               the MMA's K-major operand tiles and per-sub-block scale/sum
//   k_pf_gemm   one 128-token x N-row tile of out = W·x over the whole row
//               (warp-specialized: 8 epilogue warps own the TMEM lanes =
//               tokens, two per lane quarter, each for half of the rows;
//               3 producer warps copy the k-quant blocks a few ahead and
//               unpack them to int8 operand tiles; one thread copies the
//               activation tiles and issues the MMAs), then the segment's
//               epilogue (bias, RoPE + K/V append, residual, SwiGLU)
// Attention over the new tokens uses the standalone attention kernels with a
// token dimension (step_kernels.cuh).
#pragma once

#include "decode.cuh"

namespace cxm {

// ── tcgen05 (5th-generation tensor core) primitives, sm_100a ──
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes made visible to the tensor core's reads
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (=|+=) A[smem desc] · B[smem desc]^T, int8 x int8 -> s32
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// the mbarrier gets one arrival when every MMA this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes (one per thread)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 8 consecutive 32-bit columns of this warp's 32 TMEM lanes (into r[0..7])
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand without swizzle: 8-row
// x 16-byte core matrices, rows 16 bytes apart; `lbo` bytes from a core matrix
// to the next along K, `sbo` bytes to the next 8 rows (sm_100 format: address
// and offsets in 16-byte units, version 1 in bits 46-47, layout type 0).
__device__ __forceinline__ uint64_t umma_desc(const void *smem, uint32_t lbo, uint32_t sbo) {
    const uint64_t a = (smem_u32(smem) >> 4) & 0x3FFFu;
    return a | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: s32 accumulator, signed A and B, both
// K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ── the activation operand ──
// M-tiles of 128 token rows; each tile holds its K-steps of 32 values one
// after another, 4 KB each, in the canonical K-major layout (LBO 128, SBO 256):
// byte (m, k) of a step at (m/8)·256 + (k/16)·128 + (m%8)·16 + k%16.
constexpr int kPfM = 128;
__host__ __device__ inline size_t pfa_bytes(int tokens, int K) {
    return (size_t)((tokens + kPfM - 1) / kPfM) * (size_t)(K / 32) * 4096;
}
__device__ __forceinline__ size_t pfa_offset(int m, int k, int K) {
    const int mt = m >> 7, mm = m & 127, s = k >> 5, kk = k & 31;
    return ((size_t)mt * (K >> 5) + s) * 4096 + (mm >> 3) * 256 + (kk >> 4) * 128 + (mm & 7) * 16 + (kk & 15);
}

// Per-sub-block activation scale and sum of token m, sub-block sb: tiles of
// the M-tiles' 128 tokens, token-minor, so a warp of consecutive tokens reads
// one sub-block's values with one 128-byte access. Sized for whole M-tiles.
__host__ __device__ inline size_t pf_es_index(int m, int sb, int nsub) {
    return ((size_t)(m >> 7) * nsub + sb) * 128 + (m & 127);
}
__host__ __device__ inline size_t pf_es_floats(int tokens, int nsub) {
    return (size_t)((tokens + kPfM - 1) / kPfM) * kPfM * nsub;
}

struct PfRows {
    const float *in;        // [tokens][ld_in]
    int ld_in;
    const float *norm_w;    // RMSNorm weights, or null (quantize only)
    float eps;
    int K, tokens, need16, need32;
    int8_t *a16, *a32;      // tiled operands (sub-blocks of 16 / 32)
    float *e16, *s16, *e32, *s32;  // scale and sum per sub-block of 16 / 32 (pf_es_index)
};

// One token row per CTA of kDecodeThreads threads, with exactly the
// arithmetic of the decode kernel's prologue (quantize_act): the f64 sum of
// squares per thread over its two rounds of 8 values, across the warp by
// xor-shuffles, across the warps in order; then per sub-block the i8
// quantization of src/ops.rs:178-198.
__global__ void __launch_bounds__(kDecodeThreads) k_pf_rows(const __grid_constant__ PfRows P) {
    __shared__ double red[kDW];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = kDecodeThreads;
    const float *x = P.in + (size_t)row * P.ld_in;
    const int nh = P.K >> 3;
    double scale = 0.0;
    if (P.norm_w) {
        double acc = 0.0;
        for (int r = 0; r < 2; r++) {
            const int hc = r * nt + tid;
            for (int k = 0; k < 8; k++) {
                const float v = hc < nh ? x[8 * hc + k] : 0.0f;
                acc = __dadd_rn(acc, __dmul_rn((double)v, (double)v));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        double sum = 0.0;
        for (int w = 0; w < kDW; w++) sum = __dadd_rn(sum, red[w]);
        const int K = P.K;
        const double ms = (K & (K - 1)) == 0 ? __dmul_rn(sum, 1.0 / (double)K) : __ddiv_rn(sum, (double)K);
        scale = __drcp_rn(__dsqrt_rn(__dadd_rn(ms, (double)P.eps)));
    }
    for (int hc0 = 0; hc0 < nh; hc0 += nt) {
        const int hc = hc0 + tid;  // nh is a multiple of 32: warps are all in range or all out
        if (hc0 + warp * 32 >= nh) continue;
        float v[8];
        for (int k = 0; k < 8; k++) {
            v[k] = x[8 * hc + k];
            if (P.norm_w) v[k] = __fmul_rn(__double2float_rn(__dmul_rn((double)v[k], scale)), P.norm_w[8 * hc + k]);
        }
        float amax = 0.0f;
        for (int k = 0; k < 8; k++) amax = fmaxf(amax, fabsf(v[k]));
        for (int sz = 16; sz <= 32; sz += 16) {
            if ((sz == 16 && !P.need16) || (sz == 32 && !P.need32)) continue;
            float am = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            if (sz == 32) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            uint32_t w0, w1;
            int sm = quant8(v, am, w0, w1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            if (sz == 32) sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            int8_t *a = sz == 16 ? P.a16 : P.a32;
            *(uint2 *)(a + pfa_offset(row, 8 * hc, P.K)) = make_uint2(w0, w1);
            const int per = sz / 8;  // half-chunks per sub-block
            if (hc % per == 0) {
                const int nsub = P.K / sz, sb = hc / per;
                float *e = sz == 16 ? P.e16 : P.e32, *s = sz == 16 ? P.s16 : P.s32;
                e[pf_es_index(row, sb, nsub)] = am > 0.0f ? __fdiv_rn(am, 127.0f) : 0.0f;
                s[pf_es_index(row, sb, nsub)] = (float)sm;
            }
        }
    }
}

// The tokens' embedding rows (src/forward.rs:389-405), dequantized as the
// decode kernel's first prologue does.
__global__ void k_pf_embed(QMat E, const float *e32, const uint32_t *toks, int D, float *x) {
    const int row = blockIdx.y;
    const uint32_t t = toks[row];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
        x[(size_t)row * D + i] = e32 ? e32[(size_t)t * D + i] : embed_value(E, (int)t, i);
}

// ── the GEMM ──
struct PfGemm {
    MvSeg seg;              // weights (tiled), units, pairing, epilogue, bias
    int tokens, pos0;       // rows of the activation; position of the first token
    const int8_t *a;        // tiled activation operand (sub-blocks of seg's format)
    const float *xe, *xs;   // [tokens][nsub]
    int nsub;               // K / sub
    int ld_out;             // floats between tokens' rows of seg.out (not for cache rows: pos_stride)
    const float *rope_cos, *rope_sin;
    int *err;
    // rows of several conversations (batched decode): row m's position, and
    // the base its cache rows (seg.at_pos) go to; NULL: pos0 + m, seg.out
    const int *row_pos;
    float *const *row_out;
    // each row in the order of a forward call of one row (ORD_FUSED: the
    // fused per-row kernel's terms, src/kernels/scalar.rs:132-217) instead
    // of the buffered path's; the same values for the formats without a
    // minimum
    int fused;
    // measurement only: CTA (0, 0)'s %globaltimer at its roles' steps (kPfStampSlots), or NULL
    unsigned long long *stamps;
};

constexpr int kPfThreads = 384;  // warps 0-7: epilogue (TMEM lanes, two halves of the rows); 8-10: producers; 11: copies and MMAs
constexpr int kPfProducers = 96;
constexpr int kPfStages = 2;     // operand tiles of the weights and accumulator buffers in TMEM
constexpr int kPfAStages = 3;    // activation tiles in flight
constexpr int kPfRaw = 4;        // weight blocks in flight (GGUF bytes)
constexpr uint32_t kPfTmemCols = 512;  // two accumulator buffers of 256 columns

// rows per CTA tile: every sub-block of a super-block gets its own accumulator
// of N columns, two super-blocks in flight: 2 · subs · N = 512 columns
__host__ __device__ constexpr int pf_rows_per_tile(int sub) { return sub == 32 ? 32 : 16; }

// stamp slots: [0] start; per block b < 16: [16+b] MMA inputs in, [32+b] a
// producer's copies in, [48+b] its operands out, [64+b] epilogue warp 0's
// accumulators in, [80+b] out; [96] offset chains done, [97] end; [98] the
// epilogue past the CTA barrier, [99] the first 8 sub-blocks of its chains
constexpr int kPfStampSlots = 100;
__device__ __forceinline__ void pf_stamp(const PfGemm &G, int slot) {
    if (G.stamps && blockIdx.x == 0 && blockIdx.y == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        G.stamps[slot] = t;
    }
}

struct PfSmem {  // byte offsets in the dynamic shared memory
    uint32_t a[kPfAStages], b[kPfStages], esc[kPfStages], raw, des, anyd, total;
};
__host__ __device__ inline PfSmem pf_smem(int type, int K) {
    const int sub = type == 12 || type == 13 ? 32 : 16, N = pf_rows_per_tile(sub), nsb = 256 / sub;
    const uint32_t bbytes = sub == 32 ? (uint32_t)(8 * N * 32) : (uint32_t)(N * 16 * 18);  // + two zero blocks
    PfSmem s{};
    uint32_t o = 0;
    for (int i = 0; i < kPfAStages; i++) {
        s.a[i] = o;
        o += 32768;
    }
    for (int i = 0; i < kPfStages; i++) {
        s.b[i] = o;
        o += (bbytes + 127) & ~127u;
    }
    for (int i = 0; i < kPfStages; i++) {
        s.esc[i] = o;
        o += (uint32_t)(nsb * N * 4);
    }
    s.raw = o;
    o += (uint32_t)(kPfRaw * N * 224);  // kPfRaw super-blocks per row, GGUF bytes (<= 210) in 224-byte slots
    s.des = o;
    const bool mins = type == 12 || type == 13 || type == 10;
    o += mins ? (uint32_t)(N * (K / sub) * 4) : 0u;
    s.anyd = o;
    o += 128;
    s.total = (o + 127) & ~127u;
    return s;
}

// A producer thread's share of a block's copies (at most 4 pieces at 96
// producers: 32 rows x 11 chunks for Q5_K), planned once per CTA: the byte
// offset in the row's slot, the source offset in the matrix for block 0's
// tile position, and the piece kind (0-31: plane-A chunk k; 32: plane S
// 16 bytes; 33-35: plane S 4 bytes; 36: plane D word; 37: zeros).
constexpr int kPfCopyMax = 4;
// pieces of one row's block: plane-A chunks, plane-S pieces, the plane-D word
__host__ __device__ inline int pf_copy_pieces(int type) {
    const int ps = plane_s_bytes(type), pd = plane_d_bytes(type);
    return plane_a_bytes(type) / 16 + (ps == 16 ? 1 : ps / 4) + (pd ? 1 : 0);
}
struct PfCopyPlan {
    int cnt;
    uint32_t dst[kPfCopyMax], src[kPfCopyMax];
    uint8_t kind[kPfCopyMax], sl[kPfCopyMax];
};
__device__ __forceinline__ void pf_copy_plan(const QMat &M, int r0, int N, int i0, int step, PfCopyPlan &P) {
    const int T = M.type, pa = plane_a_bytes(T), ps = plane_s_bytes(T), pd = plane_d_bytes(T), ach = pa / 16;
    const int rows = M.ngroup * M.rpt;  // rows allocated (padded groups)
    int lo_a = 0, lo_s = pa, lo_d = pa + ps;
    if (T == 10) {  // Q2_K: scales, qs, d|dmin
        lo_s = 0;
        lo_a = 16;
        lo_d = 80;
    }
    const int sp = ps == 16 ? 1 : ps / 4, per = pf_copy_pieces(T);
    P.cnt = 0;
#pragma unroll
    for (int c = 0; c < kPfCopyMax; c++) {
        const int i = i0 + c * step;
        P.kind[c] = 38;  // nothing
        P.dst[c] = P.src[c] = 0;
        P.sl[c] = 0;
        if (i >= N * per) continue;
        P.cnt = c + 1;
        const int n = i / per, k = i - n * per, r = r0 + n;
        const int g = r / M.rpt, sl = r % M.rpt;
        P.sl[c] = (uint8_t)sl;
        P.src[c] = (uint32_t)g * M.group_stride;
        if (r >= rows) {
            P.kind[c] = k < ach ? 37 : 38;  // 38: nothing
            P.dst[c] = (uint32_t)(n * 224 + lo_a + 16 * k);
        } else if (k < ach) {
            P.kind[c] = (uint8_t)k;
            P.dst[c] = (uint32_t)(n * 224 + lo_a + 16 * k);
        } else if (k < ach + sp) {
            P.kind[c] = ps == 16 ? 32 : (uint8_t)(33 + (k - ach));
            P.dst[c] = (uint32_t)(n * 224 + lo_s + (ps == 16 ? 0 : 4 * (k - ach)));
        } else {
            P.kind[c] = 36;
            P.dst[c] = (uint32_t)(n * 224 + lo_d);
        }
    }
}
// Asynchronous copies of super-block b of the tile's rows into `raw` (one
// 224-byte slot per row in the GGUF block layout pf_unpack_quarter reads):
// plane A in 16-byte chunks, plane S in one 16-byte or three 4-byte pieces,
// plane D as the aligned 4-byte word that holds it. A 2-byte d (Q6_K, Q3_K)
// then sits 2·(row & 1) bytes into its word: the rows of a tile group are its
// lanes, tile groups have an even number of rows and the plane starts 4-byte
// aligned. Rows past the matrix get zeros.
__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void pf_copy(const QMat &M, const PfCopyPlan &P, int b, uint8_t *raw) {
    const int T = M.type, ps = plane_s_bytes(T), pd = plane_d_bytes(T), ach = plane_a_bytes(T) / 16;
    const int t = b / M.lpr, bl = b - t * M.lpr, nb = tile_nb(M.nblk, M.lpr, t), L = M.rpt * nb;
    const uint8_t *tb = M.base + (size_t)t * 32 * (size_t)M.bpb;
    const uint32_t sofs = (uint32_t)(ach * L * 16), dofs = sofs + (uint32_t)(L * ps);
#pragma unroll
    for (int c = 0; c < kPfCopyMax; c++) {
        if (c >= P.cnt) break;
        const int kind = P.kind[c], lane = M.rpt * bl + P.sl[c];
        const uint8_t *tile = tb + P.src[c];
        uint8_t *d = raw + P.dst[c];
        if (kind < 32) cp_async16(d, tile + ((size_t)kind * L + lane) * 16);
        else if (kind == 32) cp_async16(d, tile + sofs + (size_t)lane * 16);
        else if (kind < 36) cp_async4(d, tile + sofs + (size_t)lane * ps + 4 * (kind - 33));
        else if (kind == 36) cp_async4(d, tile + ((dofs + (uint32_t)lane * pd) & ~3u));
        else if (kind == 37) cp_async16_zfill(d, M.base, 0);
    }
}

__device__ __forceinline__ float rd_h(const uint8_t *p) { return h2f((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

// Quarter q (values 64q..64q+63) of one super-block as desempaquetar_i8
// unpacks it (src/quant.rs:238-468): the int8 values four to a word, w[i]
// holding values 4i..4i+3 (the byte order of the operand tile), and the
// scale (e[k]) and offset (o[k], formats with a minimum) of each of the
// quarter's sub-blocks k. Whole words at a time, as the decode kernel reads
// the same bytes: a nibble or 2-bit field of four values per mask, the -32
// (Q6_K) and -4 (Q3_K) bias per byte. `doff`: where the 2-byte d of Q6_K
// and Q3_K sits past its GGUF offset (pf_copy's aligned word).
__device__ __forceinline__ uint32_t ld_w(const uint8_t *p) { return *(const uint32_t *)p; }

__device__ __forceinline__ void pf_unpack_quarter(int T, const uint8_t *blk, int q, uint32_t (&w)[16], float (&e)[4],
                                                  float (&o)[4], int doff) {
    switch (T) {
    case 12: case 13: {  // Q4_K / Q5_K: sub-blocks 2q (low nibbles) and 2q+1 (high)
        const float d = rd_h(blk), dmin = rd_h(blk + 2);
        const uint32_t w0 = ld_w(blk + 4), w1 = ld_w(blk + 8), w2 = ld_w(blk + 12);
#pragma unroll
        for (int t = 0; t < 2; t++) {
            int sc, mn;
            scale_min_k4(2 * q + t, w0, w1, w2, sc, mn);
            e[t] = fm(d, (float)sc);
            o[t] = -fm(dmin, (float)mn);
        }
        const uint8_t *qs = blk + (T == 12 ? 16 : 48) + 32 * q;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t x = ld_w(qs + 4 * i);
            uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
            if (T == 13) {
                const uint32_t h = ld_w(blk + 16 + 4 * i);
                lo |= ((h >> (2 * q)) & 0x01010101u) << 4;
                hi |= ((h >> (2 * q + 1)) & 0x01010101u) << 4;
            }
            w[i] = lo;
            w[8 + i] = hi;
        }
        break;
    }
    case 14: {  // Q6_K: half h = q/2; q%2 = 0: groups primera, segunda; 1: tercera, cuarta
        const int h = q >> 1, odd = q & 1;
        const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h, *sc = blk + 192 + 8 * h;
        const float d = rd_h(blk + 208 + doff);
#pragma unroll
        for (int p = 0; p < 4; p++) e[p] = fm(d, (float)(int8_t)sc[4 * odd + p]);
        const int sl = odd ? 4 : 0, sh0 = odd ? 4 : 0, sh1 = odd ? 6 : 2;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t a = ld_w(ql + 4 * i), c = ld_w(ql + 32 + 4 * i), hb = ld_w(qh + 4 * i);
            w[i] = __vsub4(((a >> sl) & 0x0F0F0F0Fu) | (((hb >> sh0) & 0x03030303u) << 4), 0x20202020u);
            w[8 + i] = __vsub4(((c >> sl) & 0x0F0F0F0Fu) | (((hb >> sh1) & 0x03030303u) << 4), 0x20202020u);
        }
        break;
    }
    case 11: {  // Q3_K: half m2 = q/2, shifts 2it for it = 2(q%2), 2(q%2)+1
        const int m2 = q >> 1;
        const uint8_t *hm = blk, *qs = blk + 32 + 32 * m2;
        const float d = rd_h(blk + 108 + doff);
        const uint32_t a0 = ld_w(blk + 96), a1 = ld_w(blk + 100), tt = ld_w(blk + 104);
#pragma unroll
        for (int ii = 0; ii < 2; ii++) {
            const int it = 2 * (q & 1) + ii, g = 4 * m2 + it;
#pragma unroll
            for (int t = 0; t < 2; t++) {
                const int is = 2 * g + t, wi = is >> 2;
                const uint32_t aa = (wi & 1) ? a1 : a0;
                const uint32_t wq = ((aa >> ((wi >> 1) * 4)) & 0x0F0F0F0Fu) | (((tt >> (2 * wi)) & 0x03030303u) << 4);
                const int s6 = (int)((wq >> (8 * (is & 3))) & 0xFF);
                e[2 * ii + t] = fm(d, fs((float)s6, 32.0f));
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t x = ld_w(qs + 4 * i), hb = ld_w(hm + 4 * i);
                w[8 * ii + i] = __vsub4(((x >> (2 * it)) & 0x03030303u) | (((hb >> g) & 0x01010101u) << 2), 0x04040404u);
            }
        }
        break;
    }
    default: {  // Q2_K
        const int m2 = q >> 1;
        const uint8_t *sc = blk, *qs = blk + 16 + 32 * m2;
        const float d = rd_h(blk + 80), dmin = rd_h(blk + 82);
#pragma unroll
        for (int ii = 0; ii < 2; ii++) {
            const int it = 2 * (q & 1) + ii, g = 4 * m2 + it;
#pragma unroll
            for (int t = 0; t < 2; t++) {
                const int is = 2 * g + t;
                e[2 * ii + t] = fm(d, (float)(sc[is] & 0xF));
                o[2 * ii + t] = -fm(dmin, (float)(sc[is] >> 4));
            }
#pragma unroll
            for (int i = 0; i < 8; i++) w[8 * ii + i] = (ld_w(qs + 4 * i) >> (2 * it)) & 0x03030303u;
        }
        break;
    }
    }
}

// bounded mbarrier wait of a role: on a timeout it raises ERR_TIMEOUT and the
// CTA's abort flag, so every other role's wait ends too
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    if (mbar_wait_bounded(bar, parity, abort)) return true;
    *abort = 1;
    atomicOr(err, ERR_TIMEOUT);
    return false;
}

// AND of `ok` over the 96 producer threads (named barrier 2), so they leave
// their loop together and none is left waiting at a barrier of the group
__device__ __forceinline__ bool producers_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 2, 96, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}

// An epilogue warp's whole main loop, for HN rows per warp (sub-blocks of
// 32: 16 rows, 8 sub-blocks a block; of 16: 8 rows, 16 sub-blocks) and the
// buffered or the fused order. Per block: wait for its accumulators, then
// 64 TMEM columns behind each wait; each row's chain advances sub-block by
// sub-block: acc += (esc·xe)·Σ (buffered), or the fused kernel's
// xe·((d·sc)·Σ − (dmin·m)·xs). The token's xe (xs) of the next block are
// loaded while a block is summed. `cb0`: column of this warp's rows in
// buffer 0; `esc0`, `db0`: their scale rows (buffer 0) and offsets.
template <int HN, bool FUSED>
__device__ __forceinline__ bool pf_epi_loop(const PfGemm &G, const float *xe, const float *xs, int nblk, int N,
                                            uint32_t cb0, const unsigned char *sm, const PfSmem &L, int c0,
                                            const float *db0, uint64_t *mma_done, uint64_t *tmem_empty,
                                            volatile int *abort_s, float (&acc)[16]) {
    constexpr int NSB = 128 / HN, JB = 64 / HN, NX = FUSED ? NSB : 1;
    const int lane = threadIdx.x & 31;
    float ev[NSB], xv[NX];
#pragma unroll
    for (int k = 0; k < NSB; k++) ev[k] = __ldg(xe + (size_t)k * 128);
#pragma unroll
    for (int k = 0; k < NX; k++) xv[k] = FUSED ? __ldg(xs + (size_t)k * 128) : 0.0f;
    for (int b = 0; b < nblk; b++) {
        const int st = b & 1, bn = b + 1 < nblk ? b + 1 : b;
        float en[NSB], xn[NX];
#pragma unroll
        for (int k = 0; k < NSB; k++) en[k] = __ldg(xe + (size_t)(bn * NSB + k) * 128);
#pragma unroll
        for (int k = 0; k < NX; k++) xn[k] = FUSED ? __ldg(xs + (size_t)(bn * NSB + k) * 128) : 0.0f;
        // warp-uniform: the TMEM loads below are collective over the warp
        if (!__all_sync(0xffffffffu, pf_wait(&mma_done[st], (b >> 1) & 1, abort_s, G.err) && !*abort_s)) return false;
        tc_fence_after();
        if (threadIdx.x == 0 && b < 16) pf_stamp(G, 64 + b);
        const float *esc = (const float *)(sm + L.esc[st]) + c0;
        const uint32_t cb = cb0 + (uint32_t)(st * 256);
        const float *db = db0 + b * NSB;
#pragma unroll
        for (int j0 = 0; j0 < NSB; j0 += JB) {
            uint32_t sv[64];
#pragma unroll
            for (int jj = 0; jj < JB; jj++) {
                const uint32_t col = cb + (uint32_t)((j0 + jj) * N);
                if (HN == 16) tmem_ld16(col, sv + 16 * jj);
                else tmem_ld8(col, sv + 8 * jj);
            }
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < JB; jj++) {
                const int j = j0 + jj;
                if (FUSED) {
#pragma unroll
                    for (int n = 0; n < HN; n++)
                        acc[n] = fa(acc[n], fm(ev[j], fs(fm(esc[j * N + n], (float)(int)sv[HN * jj + n]),
                                                         fm(-db[(size_t)n * G.nsub + j], xv[FUSED ? j : 0]))));
                } else {
#pragma unroll
                    for (int n = 0; n < HN; n++)
                        acc[n] = fa(acc[n], fm(fm(esc[j * N + n], ev[j]), (float)(int)sv[HN * jj + n]));
                }
            }
        }
#pragma unroll
        for (int k = 0; k < NSB; k++) ev[k] = en[k];
#pragma unroll
        for (int k = 0; k < NX; k++) xv[k] = xn[k];
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[st]);
        if (threadIdx.x == 0 && b < 16) pf_stamp(G, 80 + b);
    }
    return true;
}

// The offset chains of an epilogue thread's HN rows, after the whole rows
// (src/ops.rs:395-401): each row with a nonzero offset adds its terms
// (des·xe)·xs in sub-block order; the rows' chains advance side by side
// (sub-block outer), eight sub-blocks' xe/xs loads in flight at a time
// (nsub is a multiple of 8). `anyd`, `des`: this warp's rows.
template <int HN>
__device__ __forceinline__ void pf_offset_chains(const PfGemm &G, int m, const unsigned char *anyd, const float *des,
                                                 float (&acc)[16]) {
    const int nsub = G.nsub;
    const float *xe = G.xe + pf_es_index(m, 0, nsub), *xs = G.xs + pf_es_index(m, 0, nsub);
    uint32_t live = 0;  // rows with a nonzero offset
#pragma unroll
    for (int n = 0; n < HN; n++)
        if (anyd[n]) live |= 1u << n;
    if (!live) return;
    for (int s0 = 0; s0 < nsub; s0 += 8) {
        float e8[8], x8[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            e8[k] = __ldg(xe + (size_t)(s0 + k) * 128);
            x8[k] = __ldg(xs + (size_t)(s0 + k) * 128);
        }
        // each row's 8 offsets of the group: two 16-byte shared loads (des is
        // 16-byte aligned, nsub and s0 multiples of 8)
        float d8[HN][8];
#pragma unroll
        for (int n = 0; n < HN; n++) {
            const float4 lo = *(const float4 *)(des + n * nsub + s0), hi = *(const float4 *)(des + n * nsub + s0 + 4);
            d8[n][0] = lo.x; d8[n][1] = lo.y; d8[n][2] = lo.z; d8[n][3] = lo.w;
            d8[n][4] = hi.x; d8[n][5] = hi.y; d8[n][6] = hi.z; d8[n][7] = hi.w;
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
#pragma unroll
            for (int n = 0; n < HN; n++) {
                const float t = fm(fm(d8[n][k], e8[k]), x8[k]);
                acc[n] = (live >> n) & 1u ? fa(acc[n], t) : acc[n];
            }
        }
        if (threadIdx.x == 0 && s0 == 0) pf_stamp(G, 99);
    }
}

__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(const __grid_constant__ PfGemm G) {
    extern __shared__ __align__(128) unsigned char pf_smem_raw[];
    // 128-byte aligned by an offset from the array itself (the operand tiles
    // need 16; the descriptors address 16-byte units)
    unsigned char *sm = pf_smem_raw + ((128u - ((uint32_t)(uintptr_t)pf_smem_raw & 127u)) & 127u);
    __shared__ __align__(8) uint64_t full_a[kPfAStages], full_b[kPfStages], mma_done[kPfStages], tmem_empty[kPfStages];
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_s;
    const QMat &M = G.seg.M;
    const int T = M.type, sub = (T == 12 || T == 13) ? 32 : 16, N = pf_rows_per_tile(sub), nsb = 256 / sub;
    const bool mins = has_minimum(T);
    const PfSmem L = pf_smem(T, M.K);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = blockIdx.x * N, mt = blockIdx.y, nblk = M.nblk;
    float *des_all = (float *)(sm + L.des);
    unsigned char *anyd = sm + L.anyd;

    if (tid == 0) {
        for (int i = 0; i < kPfAStages; i++) mbar_init(&full_a[i], 1);
        for (int i = 0; i < kPfStages; i++) {
            mbar_init(&full_b[i], kPfProducers);
            mbar_init(&mma_done[i], 1);
            mbar_init(&tmem_empty[i], 8);  // the epilogue warps
        }
        abort_s = 0;
        mbar_fence_init();
    }
    if (tid < N) anyd[tid] = 0;
    if (warp == 0) {
        tmem_alloc(&tmem_base_s, kPfTmemCols);
        tmem_relinquish();
    }
    // the two zero core-matrix columns of the sub-16 operand tiles
    if (sub == 16)
        for (int s = 0; s < kPfStages; s++)
            for (int i = tid; i < N; i += kPfThreads) {
                *(uint4 *)(sm + L.b[s] + 16 * i) = make_uint4(0, 0, 0, 0);
                *(uint4 *)(sm + L.b[s] + 17 * N * 16 + 16 * i) = make_uint4(0, 0, 0, 0);
            }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) pf_stamp(G, 0);
    const uint32_t tmem = tmem_base_s;
    const uint32_t idesc = umma_idesc_i8(kPfM, N);

    float acc[16];
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0.0f;
    const int m = mt * kPfM + (tid & 127);  // the epilogue thread's token (its TMEM lane)
    const int HN = N / 2, c0 = (warp >> 2) * HN;  // an epilogue warp's half of the tile's rows
    const int groups = min(16, (G.tokens - mt * kPfM + 7) / 8);  // 8-token row groups of this tile

    if (warp == 11) {
        // ── copies of the activation tiles and the MMAs (one thread) ──
        // the activation tile of block bb into stage bb % kPfAStages: the
        // tile's token rows in groups of 8 (256 bytes per K-step); a tile of
        // few tokens (a decode batch) copies only its groups, and the MMA rows
        // past them hold stale bytes whose sums no epilogue thread stores
        auto copy_a = [&](int bb) {
            const int sa = bb % kPfAStages;
            const uint8_t *src = (const uint8_t *)(G.a + ((size_t)mt * (M.K / 32) + 8 * bb) * 4096);
            if (groups == 16) {
                mbar_arrive_expect_tx(&full_a[sa], 32768);
                bulk_g2s(sm + L.a[sa], src, 32768, &full_a[sa]);
            } else {
                mbar_arrive_expect_tx(&full_a[sa], (uint32_t)(8 * groups * 256));
                for (int k8 = 0; k8 < 8; k8++)
                    bulk_g2s(sm + L.a[sa] + k8 * 4096, src + k8 * 4096, (uint32_t)(groups * 256), &full_a[sa]);
            }
        };
        if (lane == 0) {
            int last_issued = -1;
            for (int bb = 0; bb < kPfAStages - 1 && bb < nblk; bb++) copy_a(bb);
            for (int b = 0; b < nblk; b++) {
                const int st = b & 1, sa = b % kPfAStages;
                if (!pf_wait(&full_b[st], (b >> 1) & 1, &abort_s, G.err) ||
                    !pf_wait(&full_a[sa], (b / kPfAStages) & 1, &abort_s, G.err))
                    break;
                if (b < 16) pf_stamp(G, 16 + b);
                tc_fence_after();
                const uint32_t dcol = tmem + (uint32_t)st * 256;
                for (int j = 0; j < nsb; j++) {
                    const int step = sub == 32 ? j : j >> 1;
                    const uint64_t ad = umma_desc(sm + L.a[sa] + step * 4096, 128, 256);
                    uint64_t bd;
                    if (sub == 32) {
                        bd = umma_desc(sm + L.b[st] + j * N * 32, 128, 256);
                    } else {
                        const uint32_t data = L.b[st] + N * 16 + j * N * 16;
                        if (!(j & 1)) bd = umma_desc(sm + data, (L.b[st] + 17 * N * 16) - data, 128);
                        else bd = umma_desc(sm + L.b[st], data - L.b[st], 128);
                    }
                    umma_i8(dcol + (uint32_t)(j * N), ad, bd, idesc, 0);
                }
                umma_commit(&mma_done[st]);
                last_issued = b;
                // the activation tile kPfAStages - 1 blocks ahead, into the
                // stage block b-1's MMAs read: once they are done
                const int nx = b + kPfAStages - 1;
                if (nx < nblk) {
                    if (b >= 1 && !pf_wait(&mma_done[(b - 1) & 1], ((b - 1) >> 1) & 1, &abort_s, G.err)) break;
                    copy_a(nx);
                }
            }
            // every MMA has completed before the accumulators are released
            if (last_issued >= 0) pf_wait(&mma_done[last_issued & 1], (last_issued >> 1) & 1, &abort_s, G.err);
        }
        __syncwarp();
    } else if (warp >= 8) {
        // ── producers: copy the N rows' super-blocks kPfRaw - 1 blocks ahead
        // (cp.async), unpack each to the int8 operand tile of its stage ──
        const int ptid = tid - 256;  // warps 8-10
        uint8_t *raw = sm + L.raw;
        const int slot_bytes = N * 224;
        PfCopyPlan plan;
        pf_copy_plan(M, r0, N, ptid, kPfProducers, plan);
        for (int bb = 0; bb < kPfRaw - 1; bb++) {  // one commit group per block, empty past the end
            if (bb < nblk) pf_copy(M, plan, bb, raw + (bb % kPfRaw) * slot_bytes);
            cp_async_commit();
        }
        for (int b = 0; b < nblk; b++) {
            const int st = b & 1;
            const int nx = b + kPfRaw - 1;  // its slot was unpacked at block b-1, before that block's last barrier
            if (nx < nblk) pf_copy(M, plan, nx, raw + (nx % kPfRaw) * slot_bytes);
            cp_async_commit();
            cp_async_wait<kPfRaw - 1>();  // this thread's copies of block b
            bool w = true;
            if (b >= kPfStages) w = pf_wait(&tmem_empty[st], ((b - kPfStages) >> 1) & 1, &abort_s, G.err);
            // every producer's copies of block b are in; the epilogue is done with stage st
            if (!producers_all(w && !abort_s)) break;
            if (ptid == 0 && b < 16) pf_stamp(G, 32 + b);
            const uint8_t *blkraw = raw + (b % kPfRaw) * slot_bytes;
            float *esc = (float *)(sm + L.esc[st]);  // [sub-block in block][row]
            for (int i = ptid; i < N * 4; i += kPfProducers) {
                const int n = i >> 2, q = i & 3;
                uint32_t w[16];
                float e[4], o[4];
                pf_unpack_quarter(T, blkraw + n * 224, q, w, e, o, 2 * (n & 1));
                const int per = 64 / sub, j0 = q * per;  // the quarter's sub-blocks
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    if (k >= per) break;
                    esc[(j0 + k) * N + n] = e[k];
                    if (mins) {
                        des_all[(size_t)n * G.nsub + b * nsb + j0 + k] = o[k];
                        if (o[k] != 0.0f) anyd[n] = 1;
                    }
                }
                // 16 values at a time into the operand tile of their sub-block
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int k = 64 * q + 16 * c, j = k / sub, kk = k % sub;
                    uint32_t off;
                    if (sub == 32) off = (uint32_t)(j * N * 32 + (n >> 3) * 256 + (kk >> 4) * 128 + (n & 7) * 16);
                    else off = (uint32_t)(N * 16 + j * N * 16 + (n >> 3) * 128 + (n & 7) * 16);
                    *(uint4 *)(sm + L.b[st] + off) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                }
            }
            fence_async_smem();
            asm volatile("bar.sync 2, 96;" ::: "memory");  // every producer is done with slot b % kPfRaw
            mbar_arrive(&full_b[st]);
            if (ptid == 0 && b < 16) pf_stamp(G, 48 + b);
        }
        cp_async_wait<0>();  // no copy outlives the loop
    } else {
        // ── epilogue: thread = token m (TMEM lane), rows c0..c0+HN-1; the
        // buffered path's dot chain, sub-block by sub-block in row order ──
        // (a token past the rows reads the tile's unused entries; its sums are never stored)
        const float *xe = G.xe + pf_es_index(m, 0, G.nsub), *xs = G.xs + pf_es_index(m, 0, G.nsub);
        const bool fused = G.fused && mins;
        const uint32_t cb0 = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)c0;
        const float *db0 = des_all + (size_t)c0 * G.nsub;
        if (HN == 16) {
            if (fused) pf_epi_loop<16, true>(G, xe, xs, nblk, N, cb0, sm, L, c0, db0, mma_done, tmem_empty, &abort_s, acc);
            else pf_epi_loop<16, false>(G, xe, xs, nblk, N, cb0, sm, L, c0, db0, mma_done, tmem_empty, &abort_s, acc);
        } else {
            if (fused) pf_epi_loop<8, true>(G, xe, xs, nblk, N, cb0, sm, L, c0, db0, mma_done, tmem_empty, &abort_s, acc);
            else pf_epi_loop<8, false>(G, xe, xs, nblk, N, cb0, sm, L, c0, db0, mma_done, tmem_empty, &abort_s, acc);
        }
    }
    __syncthreads();
    if (tid == 0) pf_stamp(G, 98);
    if (warp < 8 && !abort_s && m < G.tokens) {
        // the offset chain, after the whole row (src/ops.rs:395-401): each
        // row with a nonzero offset adds its terms in sub-block order; the
        // rows' chains advance side by side (sub-block outer), so the token's
        // xe/xs are read once per sub-block and the rows' chains overlap
        if (mins && !G.fused) {
            if (HN == 16) pf_offset_chains<16>(G, m, anyd + c0, des_all + (size_t)c0 * G.nsub, acc);
            else pf_offset_chains<8>(G, m, anyd + c0, des_all + (size_t)c0 * G.nsub, acc);
        }
        if (tid == 0) pf_stamp(G, 96);
        // the segment's epilogue, one output unit (two tiled rows) at a time:
        // every unit's inputs (bias, rotation, residual) loaded first, then
        // the results stored
        const MvSeg &g = G.seg;
        const int pos = G.row_pos ? G.row_pos[m] : G.pos0 + m;
        float *cache_base = G.row_out ? G.row_out[m] : g.out;
        float *out = g.at_pos ? cache_base + (size_t)pos * g.pos_stride : g.out + (size_t)m * G.ld_out;
        int ua[8], ub[8];
        float ia[8], ib[8], ic[8], id[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {  // constant indices: everything stays in registers
            const int n = 2 * k, u = (r0 + c0 + n) >> 1;
            ua[k] = -1;
            ub[k] = 0;
            ia[k] = ib[k] = ic[k] = id[k] = 0.0f;
            if (n >= HN || u >= g.units) continue;
            unit_rows(g, u, ua[k], ub[k]);
            const int ra = ua[k], rb = ub[k];
            if (g.epi == EPI_RESID) {
                ia[k] = out[ra];
                ib[k] = out[rb];
            } else if (g.bias && (g.epi == EPI_STORE || g.epi == EPI_ROPE)) {
                ia[k] = __ldg(g.bias + ra);
                ib[k] = __ldg(g.bias + rb);
            }
            if (g.epi == EPI_ROPE) {
                const int i = ra % (2 * g.half);
                ic[k] = __ldg(G.rope_cos + (size_t)pos * g.half + i);
                id[k] = __ldg(G.rope_sin + (size_t)pos * g.half + i);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int ra = ua[k], rb = ub[k];
            if (ra < 0) continue;
            const float y0 = acc[2 * k], y1 = acc[2 * k + 1];
            switch (g.epi) {
            case EPI_STORE:
                out[ra] = g.bias ? fa(y0, ia[k]) : y0;
                out[rb] = g.bias ? fa(y1, ib[k]) : y1;
                break;
            case EPI_ROPE: {  // src/ops.rs:1150-1193
                const float a = g.bias ? fa(y0, ia[k]) : y0, bb = g.bias ? fa(y1, ib[k]) : y1;
                out[ra] = fs(fm(a, ic[k]), fm(bb, id[k]));
                out[rb] = fa(fm(a, id[k]), fm(bb, ic[k]));
                break;
            }
            case EPI_RESID:  // src/forward.rs:467-469, :489-491
                out[ra] = fa(ia[k], y0);
                out[rb] = fa(ib[k], y1);
                break;
            case EPI_SWIGLU: {  // src/kernels/scalar.rs:63-67, src/forward.rs:485-487
                const float act = __fdiv_rn(y0, fa(1.0f, expf_glibc(-y0)));
                out[ra] = fm(act, y1);
                break;
            }
            default:
                break;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) pf_stamp(G, 97);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kPfTmemCols);
    }
}

}  // namespace cxm
