// Host orchestration of the decode path: model upload (k-quant quad tiles in
// HBM), KV caches, the per-token step (one persistent kernel running a
// program of phases, captured as a CUDA graph), and the C ABI of
// include/cxm.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/cxm.h"
#include "cxm_internal.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "sampler.cuh"

using namespace cxm;

#define CU(call)                                                                             \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) {                                                             \
            set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return -1;                                                                       \
        }                                                                                    \
    } while (0)

namespace {

struct Layer {
    QMat q, k, v, o, gu, down;  // gu: gate and up interleaved (PAIR_TWO quads)
    float *attn_norm, *ffn_norm, *bq, *bk, *bv;
};

}  // namespace

struct cxm_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    cxm_config cfg{};
    std::vector<Layer> layers;
    QMat embd{}, out{};
    float *embd_f32 = nullptr;
    float *out_norm = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    std::vector<void *> allocs;
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    unsigned char *attq = nullptr;  // the attention output quantized for o_proj (carve_act layout)
    unsigned char *hq = nullptr;    // the FFN hidden vector quantized for ffn_down (carve_act layout)
    int *hcnt = nullptr;            // its per-sub-block counts of written values (zero between steps)
    float *scores = nullptr;  // attention scratch [n_head][ctx]
    int *err = nullptr;
    unsigned *bar = nullptr;  // grid-barrier counter of the decode kernel
    unsigned long long *argmax_key = nullptr;
    // sampler (src/sampler.rs): xorshift64* state, (1/T, top_p), picked
    // token, scratch of the device Muestreador::elegir
    unsigned long long *rng = nullptr;
    float *samp_params = nullptr;
    uint32_t *samp_tok = nullptr;
    float *samp_probs = nullptr, *samp_prefix = nullptr;
    uint32_t *samp_k0 = nullptr, *samp_v0 = nullptr, *samp_k1 = nullptr, *samp_v1 = nullptr;
    uint32_t *samp_ghist = nullptr;  // the sampler's per-CTA digit counts [sms * 256]
    float *samp_gred = nullptr;      // its per-CTA maxima and 1/total [sms + 1]
    unsigned *samp_bar = nullptr;    // its grid-barrier counter
    int sms = 148;
    // tensor parallelism: this rank's heads, KV heads, FFN rows and
    // vocabulary rows (all of them at tp = 1); the exchange areas (own, and
    // the peers' mapped through CUDA IPC by cxm_tp_connect)
    int tp = 1, tp_rank = 0;
    int h_loc = 0, kv_loc = 0, f_loc = 0, v_loc = 0, v_off = 0;
    unsigned char *xch = nullptr;
    unsigned char *peer[kTpMax] = {};
    bool peer_mapped[kTpMax] = {};
    bool connected = true;  // false from open until cxm_tp_connect when tp > 1
    unsigned *epoch = nullptr;
    uint32_t slot_bytes = 0;  // largest quad tile of the model
    uint64_t weight_bytes = 0;
    bool logits_valid = false;
    // pinned host copies of the error word and the argmax key, read back
    // together after each step sequence (one host synchronisation)
    struct HostWords {
        int err, pad;
        unsigned long long key;
    } *hw = nullptr;
    bool key_valid = false;  // hw->key holds the last forward's greedy pick
    // the prompt forward on the tensor cores (forward calls of 24+ tokens);
    // off: those tokens replay the decode step one by one, with the same results
    bool prefill_tc = true;
    struct Prefill {  // its scratch, allocated at the first such call
        int cap = 0;  // tokens per chunk
        float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *scores = nullptr;
        int8_t *a16 = nullptr, *a32 = nullptr;
        float *e16 = nullptr, *s16 = nullptr, *e32 = nullptr, *s32 = nullptr;
        size_t score_floats = 0;
    } pf;
    struct Batch {  // batched forward: rows of many conversations, allocated at the first such call
        int cap = 0, pcap = 0;  // rows; picked rows
        int rows = 0, picks = 0;
        void *mem = nullptr;  // one allocation for all of it
        float *logits = nullptr;           // [pcap][vocab]
        float *xo = nullptr;               // [pcap][dim] the picked rows' hidden states, packed
        uint32_t *tok = nullptr;           // [cap] the rows' tokens
        int *pos = nullptr;                // [cap] their positions
        float **kz = nullptr, **vz = nullptr;            // [n_layer][rows] layer bases of each row's cache
        const float **kpz = nullptr, **vpz = nullptr;    // [n_layer][rows] of its borrowed prefix
        int *plenz = nullptr;              // [cap]
        int *sel = nullptr, *ppos = nullptr;  // [pcap] the picked rows, their positions
        uint32_t **toks = nullptr;         // [pcap] each picked row's cache: token array,
        int **len = nullptr, **stop = nullptr;  // position and eos flag
        cudaGraphExec_t graph = nullptr;   // one decode step over the current views
        int graph_n = 0;
    } bt;

    ~cxm_model() {
        if (device >= 0) cudaSetDevice(device);
        for (int p = 0; p < kTpMax; p++)
            if (peer_mapped[p]) cudaIpcCloseMemHandle(peer[p]);
        for (void *p : allocs) cudaFree(p);
        for (void *p : {(void *)pf.x, (void *)pf.q, (void *)pf.att, (void *)pf.h, (void *)pf.scores, (void *)pf.a16,
                        (void *)pf.a32, (void *)pf.e16, (void *)pf.s16, (void *)pf.e32, (void *)pf.s32})
            cudaFree(p);
        if (bt.graph) cudaGraphExecDestroy(bt.graph);
        cudaFree(bt.mem);
        if (hw) cudaFreeHost(hw);
        if (stream) cudaStreamDestroy(stream);
    }
    template <class T>
    int alloc(T **p, size_t n) {
        void *v = nullptr;
        cudaError_t e = cudaMalloc(&v, std::max<size_t>(n * sizeof(T), 256));
        if (e != cudaSuccess) {
            set_error("cudaMalloc of %zu bytes failed: %s", n * sizeof(T), cudaGetErrorString(e));
            return -1;
        }
        allocs.push_back(v);
        *p = (T *)v;
        return 0;
    }
};

// a decode program on the device and the launch geometry it needs
struct Program {
    Phase *d = nullptr;  // the phases, then the walk table (one allocation)
    int n = 0;
    int nx = 0;          // tensor-parallel exchanges
    const FeedPhase *feed = nullptr;
    int nfeed = 0;
    size_t region = 0;
};

struct cxm_cache {
    cxm_model *m = nullptr;
    int device = -1;                   // the model's, kept so freeing never reads the model
    uint32_t max_tokens = 0, len = 0;
    float *k = nullptr, *v = nullptr;  // [n_layer][max_tokens][kvd]
    uint32_t *toks = nullptr;          // [max_tokens + 2]
    int *d_len = nullptr;
    int *d_stop = nullptr;             // set by a step whose pick is the model's eos
    // A shared prefix (src/engine_own.rs:198-245 borrows a session's cache by
    // copy; here it is held once): positions below plen are read from
    // prefix's K/V, never copied. A cache that lends keeps the positions below
    // `lent` as they are while `borrowers` > 0; freed while lent, it lives on
    // (orphan) until its last borrower lets go.
    cxm_cache *prefix = nullptr;
    uint32_t plen = 0;
    int borrowers = 0;
    uint32_t lent = 0;
    bool orphan = false;
    // one program and one graph per step mode and row class (RowClass)
    Program prog[4][3];
    cudaGraphExec_t graph[4][3] = {};
    void drop_programs() {  // the programs bake in the cache's prefix
        if (device >= 0) cudaSetDevice(device);
        for (auto &gm : graph)
            for (auto &g : gm) {
                if (g) cudaGraphExecDestroy(g);
                g = nullptr;
            }
        for (auto &pm : prog)
            for (auto &p : pm) {
                cudaFree(p.d);
                p = Program{};
            }
    }
    ~cxm_cache() {
        drop_programs();
        cudaFree(k);
        cudaFree(v);
        cudaFree(toks);
        cudaFree(d_len);
        cudaFree(d_stop);
    }
};

// the layer base of a cache's borrowed prefix (nullptr without one)
static const float *prefix_k(const cxm_cache *c, int l, size_t kvd) {
    return c->prefix ? c->prefix->k + (size_t)l * c->prefix->max_tokens * kvd : nullptr;
}
static const float *prefix_v(const cxm_cache *c, int l, size_t kvd) {
    return c->prefix ? c->prefix->v + (size_t)l * c->prefix->max_tokens * kvd : nullptr;
}

// c stops borrowing its prefix; an orphaned lender goes with its last borrower
static void release_prefix(cxm_cache *c) {
    cxm_cache *p = c->prefix;
    if (!p) return;
    c->prefix = nullptr;
    c->plen = 0;
    c->drop_programs();
    if (--p->borrowers == 0) {
        p->lent = 0;
        if (p->orphan) delete p;
    }
}

struct cxm_sampler {
    uint64_t state;
    float temperature, top_p;
};

namespace {

// STEP_SAMPLE: the STEP_LOGITS step, then the sampler writes the next token
enum StepMode { STEP_PREFILL = 0, STEP_GREEDY = 1, STEP_LOGITS = 2, STEP_SAMPLE = 3 };

// The reference multiplies all the tokens of one forward call at once, and
// matmul_auto picks each matrix's path by their number m
// (src/ops.rs:1056-1093). This library's parity target is the reference's
// portable backend (COSXAMIX_KERNEL=escalar), where hay_fusionado holds for
// Q4_K and Q3_K only (src/ops.rs:837-858: Q6_K and Q5_K need AVX2, Q2_K a
// non-scalar copy) and the blocked path falls back to the buffered one
// (src/ops.rs:599-606). So three classes of m give every matrix its order:
//   ROWS_FEW (1..4):  Q4_K, Q3_K fused; Q6_K, Q5_K, Q2_K buffered
//   ROWS_MID (5..23): Q4_K fused; the others buffered (Q3_K's cap is 4)
//   ROWS_MANY (24+):  all buffered (BLOQUES_DESDE = 24, src/ops.rs:1013)
// A step replays one token of such a call with its class's orders; the
// output projection always multiplies one row (src/forward.rs:495-501).
enum RowClass { ROWS_FEW = 0, ROWS_MID = 1, ROWS_MANY = 2 };
int row_class(uint64_t m) { return m >= 24 ? ROWS_MANY : (m >= 5 ? ROWS_MID : ROWS_FEW); }
int order_for(int type, int cls) {
    if (type == Q4K) return cls == ROWS_MANY ? ORD_BUFFERED : ORD_FUSED;
    if (type == Q3K) return cls == ROWS_FEW ? ORD_FUSED : ORD_BUFFERED;  // the same values either way
    return ORD_BUFFERED;  // Q6_K (the same values either way), Q5_K, Q2_K
}

size_t kv_dim(const cxm_model *m) { return (size_t)m->kv_loc * m->cfg.head_dim; }  // this rank's KV heads

int sub_of(int type) { return (type == Q4K || type == Q5K) ? 32 : 16; }

// ── tiles (the layout QMat describes) ──
// Tiled row i is row `row` of the GGUF matrix at `m` (its bytes), or a zero
// row when m is null. The bytes of each block are only moved, never changed.
struct RowSrc {
    const uint8_t *m;
    int row;
    int src_nblk = 0, blk0 = 0;  // a K slice: the source row's blocks, the slice's first (0: the whole row)
};

QMat tiled_desc(int type, int K, int nrows, int lpr) {
    QMat M{};
    M.type = type;
    M.K = K;
    M.nblk = K / 256;
    M.bpb = bytes_per_block(type);
    M.lpr = lpr;
    M.rpt = 32 / lpr;
    M.ngroup = (nrows + M.rpt - 1) / M.rpt;
    M.rows = M.rpt * M.ngroup;
    M.group_stride = (uint32_t)(((size_t)M.rpt * M.nblk * M.bpb + 15) & ~(size_t)15);
    return M;
}

// Lanes per row of a matrix's tiles. A warp works through whole row groups
// (32/lpr rows), so the phase's groups should split evenly over the SMs'
// warps: take the fewest lanes per row (a lane then owns more of a row, and
// the row's chain of additions crosses fewer lanes) for which the busiest
// warp has at most ~12% more groups than the average one; never more lanes
// than the row has super-blocks, and at most 16 so a tile holds both rows of
// an output pair.
int choose_lpr(int phase_rows, int nblk, int sms) {
    const long long warps = (long long)kDW * sms;
    int lpr = 1;
    while (lpr < 16 && lpr < nblk) {
        const long long groups = ((long long)phase_rows * lpr + 31) / 32;
        const long long per_cta = (groups + sms - 1) / sms, busiest = (per_cta + kDW - 1) / kDW;
        if (groups >= warps && busiest * warps <= groups * 9 / 8) break;
        lpr *= 2;
    }
    return lpr;
}

void build_tiles(const QMat &M, const std::vector<RowSrc> &rows, std::vector<uint8_t> &buf) {
    buf.assign((size_t)M.ngroup * M.group_stride, 0);
    const int T = M.type, pa = plane_a_bytes(T), ps = plane_s_bytes(T), pd = plane_d_bytes(T), ach = pa / 16;
    int lo_a = 0, lo_s = pa, lo_d = pa + ps;
    if (T == Q2K) {
        lo_s = 0;
        lo_a = 16;
        lo_d = 80;
    }
    const int ntile = (M.nblk + M.lpr - 1) / M.lpr;
    auto work = [&](int q0, int q1) {
        for (int q = q0; q < q1; q++)
            for (int t = 0; t < ntile; t++) {
                const int nb = tile_nb(M.nblk, M.lpr, t), L = M.rpt * nb;
                uint8_t *tile = buf.data() + tile_offset(M, q, t);
                for (int bl = 0; bl < nb; bl++)
                    for (int sl = 0; sl < M.rpt; sl++) {
                        const size_t ri = (size_t)M.rpt * q + sl;
                        if (ri >= rows.size() || !rows[ri].m) continue;
                        const size_t sn = rows[ri].src_nblk ? (size_t)rows[ri].src_nblk : (size_t)M.nblk;
                        const uint8_t *blk = rows[ri].m + ((size_t)rows[ri].row * sn + (size_t)rows[ri].blk0 +
                                                           (size_t)M.lpr * t + bl) * M.bpb;
                        const int lane = M.rpt * bl + sl;
                        for (int c = 0; c < ach; c++) memcpy(tile + ((size_t)c * L + lane) * 16, blk + lo_a + 16 * c, 16);
                        if (ps) memcpy(tile + (size_t)ach * L * 16 + (size_t)lane * ps, blk + lo_s, ps);
                        if (pd) memcpy(tile + (size_t)ach * L * 16 + (size_t)L * ps + (size_t)lane * pd, blk + lo_d, pd);
                    }
            }
    };
    const int nth = std::max(1, std::min<int>(16, (int)std::thread::hardware_concurrency()));
    if (M.ngroup < 256 || nth == 1) {
        work(0, M.ngroup);
        return;
    }
    std::vector<std::thread> th;
    for (int i = 0; i < nth; i++)
        th.emplace_back(work, (int)((long long)M.ngroup * i / nth), (int)((long long)M.ngroup * (i + 1) / nth));
    for (auto &x : th) x.join();
}

// row orders: PAIR_ADJ (rows in order), PAIR_ROPE (rows i and i + half of a
// head side by side), PAIR_TWO (row u of A, then row u of B)
// (rows from `row0` on: a tensor-parallel rank's share)
std::vector<RowSrc> rows_adj(const uint8_t *a, int n, int row0 = 0) {
    std::vector<RowSrc> r(n);
    for (int i = 0; i < n; i++) r[i] = {a, row0 + i};
    return r;
}
std::vector<RowSrc> rows_rope(const uint8_t *a, int n, int half, int row0 = 0) {
    std::vector<RowSrc> r(n);
    for (int u = 0; u < n / 2; u++) {
        const int h = u / half, i = u % half, r0 = h * 2 * half + i;
        r[2 * u] = {a, row0 + r0};
        r[2 * u + 1] = {a, row0 + r0 + half};
    }
    return r;
}
std::vector<RowSrc> rows_two(const uint8_t *a, const uint8_t *b, int n, int row0 = 0) {
    std::vector<RowSrc> r(2 * (size_t)n);
    for (int u = 0; u < n; u++) {
        r[2 * u] = {a, row0 + u};
        r[2 * u + 1] = {b, row0 + u};
    }
    return r;
}

int check_matrix(const TensorInfo &t) {
    if (t.dims.size() != 2) {
        set_error("%s: expected a matrix", t.name.c_str());
        return -1;
    }
    if (!is_kquant(t.type)) {
        set_error("%s: type %d has no device kernel (k-quants Q2_K..Q6_K only)", t.name.c_str(), t.type);
        return -1;
    }
    if (t.dims[0] % 256) {
        set_error("%s: rows of %llu values are not a multiple of 256", t.name.c_str(),
                  (unsigned long long)t.dims[0]);
        return -1;
    }
    if (t.dims[0] > (uint64_t)kMaxActivation) {
        set_error("%s: rows of %llu values: the decode kernel quantizes activations of at most %d", t.name.c_str(),
                  (unsigned long long)t.dims[0], kMaxActivation);
        return -1;
    }
    return 0;
}

int upload_tiles(cxm_model *m, QMat &M, const std::vector<RowSrc> &rows) {
    std::vector<uint8_t> buf;
    build_tiles(M, rows, buf);
    uint8_t *d = nullptr;
    if (m->alloc(&d, buf.size())) return -1;
    CU(cudaMemcpy(d, buf.data(), buf.size(), cudaMemcpyHostToDevice));
    M.base = d;
    m->slot_bytes = std::max<uint32_t>(m->slot_bytes, (uint32_t)(32 * M.bpb));
    return 0;
}

// one GGUF matrix, rows in order (pairing ADJ) or RoPE order, in tiles of
// `lpr` lanes per row; or its part rows [row0, row0 + nrows) x super-blocks
// [blk0, blk0 + nblk) (a tensor-parallel rank's share; nrows 0: all rows,
// nblk 0: all blocks)
int upload_matrix(cxm_model *m, const Gguf &g, const TensorInfo &t, int pairing, int half, int lpr, QMat *out,
                  int row0 = 0, int nrows = 0, int blk0 = 0, int nblk = 0) {
    if (check_matrix(t)) return -1;
    const int all_blk = (int)(t.dims[0] / 256), all_rows = (int)t.dims[1];
    if (!nrows) nrows = all_rows;
    if (!nblk) nblk = all_blk;
    if (row0 < 0 || row0 + nrows > all_rows || blk0 < 0 || blk0 + nblk > all_blk) {
        set_error("%s: part rows %d+%d, blocks %d+%d outside %dx%d", t.name.c_str(), row0, nrows, blk0, nblk,
                  all_rows, all_blk);
        return -1;
    }
    if (nrows % 2 || (pairing == PAIR_ROPE && (half % 2 || nrows % (2 * half)))) {
        set_error("%s: %d rows do not pair", t.name.c_str(), nrows);
        return -1;
    }
    QMat M = tiled_desc(t.type, nblk * 256, nrows, lpr);
    auto order = pairing == PAIR_ROPE ? rows_rope(g.data(t), nrows, half, row0) : rows_adj(g.data(t), nrows, row0);
    if (nblk != all_blk)
        for (RowSrc &r : order) {
            r.src_nblk = all_blk;
            r.blk0 = blk0;
        }
    if (upload_tiles(m, M, order)) return -1;
    M.rows = nrows;
    *out = M;
    m->weight_bytes += (uint64_t)nrows * nblk * M.bpb;
    return 0;
}

// gate and up as one matrix of PAIR_TWO quads (rows [row0, row0 + n) of
// each; n 0: all)
int upload_pair(cxm_model *m, const Gguf &g, const TensorInfo &a, const TensorInfo &b, int lpr, QMat *out,
                int row0 = 0, int n = 0) {
    if (check_matrix(a) || check_matrix(b)) return -1;
    if (a.type != b.type || a.dims[0] != b.dims[0] || a.dims[1] != b.dims[1] || a.dims[1] % 2) {
        set_error("%s and %s must have the same type and shape", a.name.c_str(), b.name.c_str());
        return -1;
    }
    const int K = (int)a.dims[0];
    if (!n) n = (int)a.dims[1];
    if (row0 < 0 || row0 + n > (int)a.dims[1]) {
        set_error("%s: part rows %d+%d outside %d", a.name.c_str(), row0, n, (int)a.dims[1]);
        return -1;
    }
    QMat M = tiled_desc(a.type, K, 2 * n, lpr);
    if (upload_tiles(m, M, rows_two(g.data(a), g.data(b), n, row0))) return -1;
    M.rows = 2 * n;
    *out = M;
    m->weight_bytes += (uint64_t)2 * n * M.nblk * M.bpb;
    return 0;
}

// a vector of n values (or its part [off, off + len); len 0: all)
int upload_vector(cxm_model *m, const Gguf &g, const TensorInfo &t, size_t n, float **out, size_t off = 0,
                  size_t len = 0) {
    if (t.elements() != n) {
        set_error("%s: %llu values, expected %zu", t.name.c_str(), (unsigned long long)t.elements(), n);
        return -1;
    }
    if (!len) len = n;
    if (off + len > n) {
        set_error("%s: part %zu+%zu outside %zu", t.name.c_str(), off, len, n);
        return -1;
    }
    std::vector<float> h(n);
    const uint8_t *src = g.data(t);
    if (t.type == F32) {
        memcpy(h.data(), src, n * 4);
    } else if (t.type == F16) {
        for (size_t i = 0; i < n; i++) h[i] = f16_to_f32((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8)));
    } else {
        set_error("%s: vectors must be F32 or F16", t.name.c_str());
        return -1;
    }
    if (m->alloc(out, len)) return -1;
    CU(cudaMemcpy(*out, h.data() + off, len * 4, cudaMemcpyHostToDevice));
    m->weight_bytes += (uint64_t)t.nbytes * len / n;
    return 0;
}

// Launch with programmatic dependent launch: the kernel may start while the
// previous one in the stream finishes (each kernel calls griddep_wait()
// before it touches data the previous one produced).
template <typename... Args>
int launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CU(cudaLaunchKernelEx(&cfg, kernel, args...));
    return 0;
}

size_t scores_smem(int hd, int group) {
    return ((size_t)kScoreThreads * kKRow + (size_t)group * hd) * sizeof(float);
}
size_t out_smem(uint32_t max_pos) {
    return (size_t)((max_pos + 3) & ~3u) * sizeof(float);
}

int g_decode_smem_max = 0;  // dynamic shared memory the decode kernel may use
int g_pf_smem_max = 0;      // and the prompt GEMM

int set_kernel_smem_limits() {
    int dev = 0, optin = 0;
    CU(cudaGetDevice(&dev));
    CU(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cudaFuncAttributes fa_{};
    CU(cudaFuncGetAttributes(&fa_, k_decode));
    g_decode_smem_max = optin - (int)fa_.sharedSizeBytes;
    CU(cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, g_decode_smem_max));
    CU(cudaFuncSetAttribute(k_attn_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    CU(cudaFuncSetAttribute(k_attn_out, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    CU(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampSmem));
    CU(cudaFuncGetAttributes(&fa_, k_pf_gemm));
    g_pf_smem_max = optin - (int)fa_.sharedSizeBytes;
    CU(cudaFuncSetAttribute(k_pf_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, g_pf_smem_max));
    return 0;
}

// src/ops.rs:1258-1325 for the token at *d_len (or tokens pos0.. pos0+tokens-1),
// over positions 0..=that one
int launch_attention_on(cudaStream_t st, AttnParams &a, int tokens = 1) {
    const dim3 gs(a.KV, (a.max_pos + kScoreThreads - 1) / kScoreThreads, tokens);
    // the output kernel takes up to kOutTok tokens per CTA (the tokens of one
    // cache: not a batch of conversations), as many as 200 KB of their
    // probabilities allow
    const size_t per_tok = out_smem((uint32_t)a.max_pos);
    a.ntok = tokens;
    a.tpc = (a.kz || tokens == 1) ? 1 : (int)std::max<size_t>(1, std::min<size_t>(kOutTok, (size_t)200 * 1024 / per_tok));
    const dim3 go(a.H, 1, (tokens + a.tpc - 1) / a.tpc);
    if (launch_pdl(k_attn_scores, gs, dim3(kScoreThreads), scores_smem(a.hd, a.H / a.KV), st, a)) return -1;
    return launch_pdl(k_attn_out, go, dim3(kOutThreads), per_tok * a.tpc, st, a);
}

// ── the prompt forward on the tensor cores (prefill.cuh) ──
__global__ void k_set_int(int *p, int v) { *p = v; }
MvSeg mv_seg(const QMat &M, int units, int pairing, int epi, float *out, int cls = ROWS_FEW);
int run_steps(cxm_model *m, cxm_cache *c, int mode, uint64_t rows, uint32_t n);

// i8 quantization (RMSNorm first when norm_w is given) of `t` rows of `in`
// into the prefill scratch's operand tiles
int pf_rows(cxm_model *m, const float *in, int ld, const float *norm_w, float eps, int K, int t, int need16,
            int need32) {
    PfRows P{};
    P.in = in;
    P.ld_in = ld;
    P.norm_w = norm_w;
    P.eps = eps;
    P.K = K;
    P.tokens = t;
    P.need16 = need16;
    P.need32 = need32;
    P.a16 = m->pf.a16;
    P.a32 = m->pf.a32;
    P.e16 = m->pf.e16;
    P.s16 = m->pf.s16;
    P.e32 = m->pf.e32;
    P.s32 = m->pf.s32;
    k_pf_rows<<<t, kDecodeThreads, 0, m->stream>>>(P);
    CU(cudaGetLastError());
    return 0;
}

// rows of several conversations (batched decode): per-row positions and
// cache bases, each row in the order of a forward call of one row (the
// segment's own order: mv_seg with ROWS_FEW)
struct PfRowsDest {
    const int *pos = nullptr;
    float *const *out = nullptr;
    int fused = 0;
};

// measurement: the launch of the prompt GEMM (counted from the arming) whose
// CTA (0, 0) records its roles' steps (cxm_arm_gemm_stamps)
static int g_pf_stamp_target = -1, g_pf_calls = 0;
static unsigned long long *g_pf_stamps = nullptr;

// out = W·x for the t rows quantized last, each output in the buffered
// path's order, then the segment's epilogue (tokens at positions pos0..)
int pf_gemm(cudaStream_t st, const MvSeg &seg, int t, int pos0, int ld_out, const int8_t *a16, const int8_t *a32,
            const float *e16, const float *s16, const float *e32, const float *s32, const float *rc, const float *rs,
            int *err, const PfRowsDest &rd = PfRowsDest{}) {
    const int sub = sub_of(seg.M.type), N = pf_rows_per_tile(sub);
    PfGemm G{};
    G.seg = seg;
    G.tokens = t;
    G.pos0 = pos0;
    G.a = sub == 32 ? a32 : a16;
    G.xe = sub == 32 ? e32 : e16;
    G.xs = sub == 32 ? s32 : s16;
    G.nsub = seg.M.K / sub;
    G.ld_out = ld_out;
    G.rope_cos = rc;
    G.rope_sin = rs;
    G.err = err;
    G.row_pos = rd.pos;
    G.row_out = rd.out;
    // the one-row order is the fused kernel's only where the reference has
    // one for the format (src/ops.rs:837-858); Q5_K and Q2_K stay buffered
    G.fused = rd.fused && seg.ord == ORD_FUSED;
    if (g_pf_stamp_target >= 0 && g_pf_calls++ == g_pf_stamp_target) G.stamps = g_pf_stamps;
    const PfSmem L = pf_smem(seg.M.type, seg.M.K);
    // at least 116 KB, so no two of these CTAs share an SM (each takes all 512 TMEM columns)
    const size_t smem = std::max<size_t>(L.total + 128, 116 * 1024);
    if (N * pf_copy_pieces(seg.M.type) > kPfCopyMax * kPfProducers) {  // every piece of a block has a copier
        set_error("the prompt GEMM's copy plan cannot hold a block of format %d", seg.M.type);
        return -1;
    }
    if (smem > (size_t)g_pf_smem_max) {
        set_error("the prompt GEMM needs %zu bytes of shared memory for K = %d; the device allows %d", smem, seg.M.K,
                  g_pf_smem_max);
        return -1;
    }
    const dim3 grid((seg.M.rows + N - 1) / N, (t + kPfM - 1) / kPfM);
    k_pf_gemm<<<grid, kPfThreads, smem, st>>>(G);
    CU(cudaGetLastError());
    return 0;
}

int pf_reserve(cxm_model *m, int cap) {
    if (m->pf.cap >= cap) return 0;
    for (void *p : {(void *)m->pf.x, (void *)m->pf.q, (void *)m->pf.att, (void *)m->pf.h, (void *)m->pf.scores,
                    (void *)m->pf.a16, (void *)m->pf.a32, (void *)m->pf.e16, (void *)m->pf.s16, (void *)m->pf.e32,
                    (void *)m->pf.s32})
        cudaFree(p);
    m->pf = cxm_model::Prefill{};
    const cxm_config &cfg = m->cfg;
    const int kmax = std::max(std::max(cfg.dim, cfg.ffn), m->h_loc * cfg.head_dim);
    m->pf.score_floats = (size_t)16 << 20;  // 64 MB of attention scores per launch
    CU(cudaMalloc(&m->pf.x, (size_t)cap * cfg.dim * 4));
    CU(cudaMalloc(&m->pf.q, (size_t)cap * m->h_loc * cfg.head_dim * 4));
    CU(cudaMalloc(&m->pf.att, (size_t)cap * m->h_loc * cfg.head_dim * 4));
    CU(cudaMalloc(&m->pf.h, (size_t)cap * cfg.ffn * 4));
    CU(cudaMalloc(&m->pf.scores, m->pf.score_floats * 4));
    CU(cudaMalloc(&m->pf.a16, pfa_bytes(cap, kmax)));
    CU(cudaMalloc(&m->pf.a32, pfa_bytes(cap, kmax)));
    CU(cudaMemset(m->pf.a16, 0, pfa_bytes(cap, kmax)));
    CU(cudaMemset(m->pf.a32, 0, pfa_bytes(cap, kmax)));
    CU(cudaMalloc(&m->pf.e16, pf_es_floats(cap, kmax / 16) * 4));
    CU(cudaMalloc(&m->pf.s16, pf_es_floats(cap, kmax / 16) * 4));
    CU(cudaMalloc(&m->pf.e32, pf_es_floats(cap, kmax / 32) * 4));
    CU(cudaMalloc(&m->pf.s32, pf_es_floats(cap, kmax / 32) * 4));
    m->pf.cap = cap;
    return 0;
}

int pf_seg_gemm(cxm_model *m, const MvSeg &seg, int t, int pos0, int ld_out, const PfRowsDest &rd = PfRowsDest{}) {
    return pf_gemm(m->stream, seg, t, pos0, ld_out, m->pf.a16, m->pf.a32, m->pf.e16, m->pf.s16, m->pf.e32, m->pf.s32,
                   m->rope_cos, m->rope_sin, m->err, rd);
}

// The prompt forward (src/forward.rs:375-492 over several tokens at once)
// of the tokens at positions p0 .. p0+n-1 of cache c (ids in c->toks): their
// K/V rows in every layer, as the reference's forward of a call of 24+
// tokens computes them. The logits are not formed here.
constexpr int kPrefillChunk = 512;
int prefill_tokens(cxm_model *m, cxm_cache *c, uint32_t p0, uint32_t n) {
    const cxm_config &cfg = m->cfg;
    const int D = cfg.dim, hd = cfg.head_dim, H = m->h_loc, KV = m->kv_loc, F = cfg.ffn, dq = H * hd;
    const size_t kvd = kv_dim(m);
    if (pf_reserve(m, kPrefillChunk)) return -1;
    auto need = [](const QMat &M, int s) { return sub_of(M.type) == s ? 1 : 0; };
    for (uint32_t q0 = p0; q0 < p0 + n; q0 += kPrefillChunk) {
        const int t = (int)std::min<uint32_t>(kPrefillChunk, p0 + n - q0);
        {  // embeddings
            const dim3 g((D + 255) / 256, t);
            k_pf_embed<<<g, 256, 0, m->stream>>>(m->embd, m->embd_f32, c->toks + q0, D, m->pf.x);
            CU(cudaGetLastError());
        }
        for (int l = 0; l < cfg.n_layer; l++) {
            const Layer &L = m->layers[l];
            float *kl = c->k + (size_t)l * c->max_tokens * kvd, *vl = c->v + (size_t)l * c->max_tokens * kvd;
            // RMSNorm + quantize; q, k (RoPE, into the cache), v (into the cache)
            if (pf_rows(m, m->pf.x, D, L.attn_norm, cfg.eps, D, t, need(L.q, 16) | need(L.k, 16) | need(L.v, 16),
                        need(L.q, 32) | need(L.k, 32) | need(L.v, 32)))
                return -1;
            MvSeg sq = mv_seg(L.q, dq / 2, PAIR_ROPE, EPI_ROPE, m->pf.q, ROWS_MANY);
            sq.half = hd / 2;
            sq.bias = L.bq;
            MvSeg sk = mv_seg(L.k, (int)kvd / 2, PAIR_ROPE, EPI_ROPE, kl, ROWS_MANY);
            sk.half = hd / 2;
            sk.bias = L.bk;
            sk.at_pos = 1;
            sk.pos_stride = (int)kvd;
            MvSeg sv = mv_seg(L.v, (int)kvd / 2, PAIR_ADJ, EPI_STORE, vl, ROWS_MANY);
            sv.bias = L.bv;
            sv.at_pos = 1;
            sv.pos_stride = (int)kvd;
            if (pf_seg_gemm(m, sq, t, (int)q0, dq) || pf_seg_gemm(m, sk, t, (int)q0, 0) ||
                pf_seg_gemm(m, sv, t, (int)q0, 0))
                return -1;
            // causal attention of the chunk's tokens over the cache
            const int stride = (int)((q0 + t + 3) & ~3u);
            const int tz = (int)std::max<size_t>(1, std::min<size_t>(t, m->pf.score_floats / ((size_t)H * stride)));
            for (int z0 = 0; z0 < t; z0 += tz) {
                AttnParams a{};
                a.q = m->pf.q + (size_t)z0 * dq;
                a.k = kl;
                a.v = vl;
                a.kp = prefix_k(c, l, kvd);
                a.vp = prefix_v(c, l, kvd);
                a.plen = c->prefix ? (int)c->plen : 0;
                a.out = m->pf.att + (size_t)z0 * dq;
                a.scores = m->pf.scores;
                a.d_len = nullptr;
                a.pos0 = (int)q0 + z0;
                a.qs = dq;
                a.os = dq;
                a.H = H;
                a.KV = KV;
                a.hd = hd;
                a.max_pos = (int)c->max_tokens;
                a.score_stride = stride;
                a.scale = 1.0f / sqrtf((float)hd);  // src/ops.rs:1287
                a.err = m->err;
                if (launch_attention_on(m->stream, a, std::min(tz, t - z0))) return -1;
            }
            // o_proj + residual; RMSNorm + gate|up + SwiGLU; down + residual
            if (pf_rows(m, m->pf.att, dq, nullptr, 0.0f, dq, t, need(L.o, 16), need(L.o, 32)) ||
                pf_seg_gemm(m, mv_seg(L.o, D / 2, PAIR_ADJ, EPI_RESID, m->pf.x, ROWS_MANY), t, (int)q0, D))
                return -1;
            if (pf_rows(m, m->pf.x, D, L.ffn_norm, cfg.eps, D, t, need(L.gu, 16), need(L.gu, 32)) ||
                pf_seg_gemm(m, mv_seg(L.gu, F, PAIR_TWO, EPI_SWIGLU, m->pf.h, ROWS_MANY), t, (int)q0, F))
                return -1;
            if (pf_rows(m, m->pf.h, F, nullptr, 0.0f, F, t, need(L.down, 16), need(L.down, 32)) ||
                pf_seg_gemm(m, mv_seg(L.down, D / 2, PAIR_ADJ, EPI_RESID, m->pf.x, ROWS_MANY), t, (int)q0, D))
                return -1;
        }
    }
    return 0;
}

// the prompt tokens before the last of a forward call of n tokens from
// position p0: on the tensor cores when the call takes the buffered path
// (24+ tokens) on a single-GPU model, else replayed step by step
int prompt_prefix(cxm_model *m, cxm_cache *c, uint32_t p0, uint32_t n) {
    if (n < 2) return 0;
    if (m->prefill_tc && m->tp == 1 && row_class(n) == ROWS_MANY) {
        if (prefill_tokens(m, c, p0, n - 1)) return -1;
        k_set_int<<<1, 1, 0, m->stream>>>(c->d_len, (int)(p0 + n - 1));
        CU(cudaGetLastError());
        return 0;
    }
    return run_steps(m, c, STEP_PREFILL, n, n - 1);
}

// ── decode programs ──
MvSeg mv_seg(const QMat &M, int units, int pairing, int epi, float *out, int cls) {
    MvSeg s{};
    s.M = M;
    s.units = units;
    s.pairing = pairing;
    s.epi = epi;
    s.out = out;
    s.ord = order_for(M.type, cls);
    return s;
}

Phase mv_phase(const std::vector<MvSeg> &segs, int K, int prologue, const float *in, const float *norm_w, float eps,
               int barrier) {
    Phase ph{};
    ph.kind = PH_MATVEC;
    ph.barrier = barrier;
    MvPhase &P = ph.mv;
    P.nseg = (int)segs.size();
    for (int i = 0; i < P.nseg; i++) {
        P.seg[i] = segs[i];
        P.ngroup += segs[i].M.ngroup;
        if (sub_of(segs[i].M.type) == 16) P.need16 = 1; else P.need32 = 1;
    }
    P.K = K;
    P.ntile = (K / 256 + segs[0].M.lpr - 1) / segs[0].M.lpr;
    for (int i = 0; i < P.nseg; i++) {  // the offset-term spill of a buffered segment with a minimum
        const QMat &M = segs[i].M;
        if (segs[i].ord == ORD_BUFFERED && has_minimum(M.type))
            P.sv_warp = std::max(P.sv_warp, M.rpt * M.nblk * (sub_of(M.type) == 32 ? 8 : 16));
    }
    P.prologue = prologue;
    P.in = in;
    P.norm_w = norm_w;
    P.eps = eps;
    return ph;
}

// bytes of the region before a matvec phase's offset-term spill
size_t mv_spill_offset(const MvPhase &P) {
    return act_bytes(P.K, P.need16, P.need32) +
           (P.prologue == PRO_QUANT && P.K <= kMaxStaged ? (size_t)P.K * sizeof(float) : 0);
}

size_t phase_region(const Phase &ph, int max_pos) {
    if (ph.kind == PH_MATVEC)  // the quantized activation (+ the staged input of a short quantize-only
                               // prologue, + the warps' offset-term spill)
        return mv_spill_offset(ph.mv) + (size_t)kDW * ph.mv.sv_warp * sizeof(float);
    if (ph.kind == PH_SCORES) return scores_region(ph.at.P, ph.at.H / ph.at.KV, ph.at.hd);
    if (ph.kind == PH_ATTN) return attn_region(max_pos, ph.at.ring);
    return 0;
}

// shared memory an attention phase may take (the rest is the weight ring)
constexpr size_t kAttnBudget = 104 * 1024;

// positions per score item: the G query heads of a kv head share its K rows
int score_positions(int G) { return std::max(1, std::min(64, 256 / std::max(1, G))); }

// V chunks in the attention ring: as many as `budget` bytes hold beside the
// probabilities (at least kAttnMinRing)
int attn_ring(int max_pos, size_t budget) {
    int r = kAttnMinRing;
    while (r < kAttnMaxRing && attn_region(max_pos, r + 1) <= budget) r++;
    return r;
}

// The step for the token at *d_len of cache c (src/forward.rs:375-505):
// embedding (fused into layer 0's first prologue), then per layer q|k|v,
// scores, softmax+output, o, gate|up, down; the output projection unless the
// step only prefills; the commit.
// an exchange phase of a tensor-parallel program
Phase x_phase(int kind, float *dst, int n, size_t src_off, int seq) {
    Phase ph{};
    ph.kind = kind;
    ph.barrier = 1;
    ph.xp.dst = dst;
    ph.xp.n = n;
    ph.xp.src_off = (uint32_t)src_off;
    ph.xp.seq = seq;
    return ph;
}

// One token through the model (src/forward.rs:375-505) as decode-kernel
// phases. With tensor parallelism every rank runs the attention block whole
// (q/k/v, attention, o_proj: replicated) and its rows of the FFN: gate|up
// rows [r·F/N, (r+1)·F/N) and ffn_down rows [r·D/N, (r+1)·D/N) over the whole
// hidden vector; exchange phases gather the hidden vector and the residual
// stream from the ranks' slices, and pick the argmax over their vocabulary
// slices. Every value is computed as on one GPU, in the same order.
std::vector<Phase> step_program(cxm_model *m, cxm_cache *c, int mode, int cls) {
    const cxm_config &cfg = m->cfg;
    const int D = cfg.dim, hd = cfg.head_dim, F = m->f_loc, H = m->h_loc, KV = m->kv_loc, dl = H * hd;
    const size_t kvd = kv_dim(m);
    const bool tp = m->tp > 1;
    const int FF = cfg.ffn, dloc = D / m->tp, r = m->tp_rank;
    float *xo = (float *)(m->xch + xch_xo_off(FF));  // [2][D]: the exported residual slices
    int nx = 0;
    std::vector<Phase> prog;
    for (int l = 0; l < cfg.n_layer; l++) {
        const Layer &L = m->layers[l];
        float *kl = c->k + (size_t)l * c->max_tokens * kvd, *vl = c->v + (size_t)l * c->max_tokens * kvd;
        {  // RMSNorm + quantize, q/k/v with bias, RoPE, KV append
            MvSeg sq = mv_seg(L.q, dl / 2, PAIR_ROPE, EPI_ROPE, m->q, cls);
            sq.half = hd / 2;
            sq.bias = L.bq;
            MvSeg sk = mv_seg(L.k, (int)kvd / 2, PAIR_ROPE, EPI_ROPE, kl, cls);
            sk.half = hd / 2;
            sk.bias = L.bk;
            sk.at_pos = 1;
            sk.pos_stride = (int)kvd;
            MvSeg sv = mv_seg(L.v, (int)kvd / 2, PAIR_ADJ, EPI_STORE, vl, cls);
            sv.bias = L.bv;
            sv.at_pos = 1;
            sv.pos_stride = (int)kvd;
            Phase ph = mv_phase({sq, sk, sv}, D, l == 0 ? PRO_EMBED : PRO_NORM, m->x, L.attn_norm, cfg.eps, l > 0);
            if (l == 0) {
                ph.mv.E = m->embd;
                ph.mv.e32 = m->embd_f32;
                ph.mv.x_out = m->x;
            }
            prog.push_back(ph);
        }
        AtPhase at{};
        at.q = m->q;
        at.k = kl;
        at.v = vl;
        at.kp = prefix_k(c, l, kvd);
        at.vp = prefix_v(c, l, kvd);
        at.plen = c->prefix ? (int)c->plen : 0;
        at.out = m->att;
        at.scores = m->scores;
        at.H = H;
        at.KV = KV;
        at.hd = hd;
        at.score_stride = (cfg.ctx + 3) & ~3;
        at.P = score_positions(H / KV);
        at.ring = attn_ring((int)c->max_tokens, kAttnBudget);
        at.scale = 1.0f / sqrtf((float)hd);  // src/ops.rs:1287
        at.qout = m->attq;
        at.qneed16 = sub_of(L.o.type) == 16;
        at.qneed32 = sub_of(L.o.type) == 32;
        at.qK = dl;
        {
            Phase ph{};
            ph.kind = PH_SCORES;
            ph.barrier = 1;
            ph.at = at;
            prog.push_back(ph);
            ph.kind = PH_ATTN;
            prog.push_back(ph);
        }
        // o_proj + residual; RMSNorm + gate/up + SwiGLU; down + residual
        // o_proj's input arrives quantized by the attention items
        prog.push_back(mv_phase({mv_seg(L.o, D / 2, PAIR_ADJ, EPI_RESID, m->x, cls)}, dl, PRO_COPYQ,
                                (const float *)m->attq, nullptr, 0.0f, 1));
        // one GPU: the gate|up epilogue also quantizes the hidden vector for
        // ffn_down as its sub-blocks complete, and down copies it in
        MvSeg sg = mv_seg(L.gu, F, PAIR_TWO, EPI_SWIGLU, m->h + (size_t)r * F, cls);
        if (!tp) {
            sg.qout = m->hq;
            sg.qcnt = m->hcnt;
            sg.qsub = sub_of(L.down.type);
            sg.qK = FF;
        }
        prog.push_back(mv_phase({sg}, D, PRO_NORM, m->x, L.ffn_norm, cfg.eps, 1));
        if (tp) prog.push_back(x_phase(PH_XGATHER, m->h, FF, 0, ++nx));
        MvSeg sd = mv_seg(L.down, dloc / 2, PAIR_ADJ, EPI_RESID, m->x + (size_t)r * dloc, cls);
        const size_t xo_off = xch_xo_off(FF) + (size_t)(l & 1) * D * sizeof(float);
        if (tp) sd.out2 = xo + (size_t)(l & 1) * D + (size_t)r * dloc;
        if (tp) prog.push_back(mv_phase({sd}, FF, PRO_QUANT, m->h, nullptr, 0.0f, 1));
        else prog.push_back(mv_phase({sd}, FF, PRO_COPYQ, (const float *)m->hq, nullptr, 0.0f, 1));
        if (tp) prog.push_back(x_phase(PH_XGATHER, m->x, D, xo_off, ++nx));
    }
    if (mode != STEP_PREFILL) {  // final RMSNorm, output projection, argmax
        MvSeg so = mv_seg(m->out, m->v_loc / 2, PAIR_ADJ, EPI_LOGITS, m->logits, ROWS_FEW);
        so.idx_off = m->v_off;
        prog.push_back(mv_phase({so}, D, PRO_NORM, m->x, m->out_norm, cfg.eps, 1));
        if (tp) prog.push_back(x_phase(PH_XARGMAX, nullptr, 0, 0, ++nx));
    }
    Phase cm{};
    cm.kind = PH_COMMIT;
    cm.barrier = 1;
    prog.push_back(cm);
    return prog;
}

// one walk-table entry per matvec phase, in program order
std::vector<FeedPhase> feed_table(const std::vector<Phase> &ph) {
    std::vector<FeedPhase> t;
    for (const Phase &x : ph) {
        if (x.kind != PH_MATVEC) continue;
        const MvPhase &P = x.mv;
        FeedPhase f{};
        for (int i = 0; i < P.nseg; i++) {
            f.b[i] = P.seg[i].M.base;
            f.g[i] = P.seg[i].M.group_stride;
            f.p[i] = (uint16_t)P.seg[i].M.bpb;
        }
        f.n0 = P.nseg > 1 ? P.seg[0].M.ngroup : 0x7fffffff;
        f.n1 = P.nseg > 2 ? P.seg[1].M.ngroup : 0x7fffffff;
        f.ngroup = P.ngroup;
        f.ntile = (uint16_t)P.ntile;
        f.nblk = (uint16_t)P.seg[0].M.nblk;
        f.lpr = (uint16_t)P.seg[0].M.lpr;
        f.rpt = (uint16_t)P.seg[0].M.rpt;
        t.push_back(f);
    }
    return t;
}

int upload_program(const std::vector<Phase> &ph, int max_pos, Program *out) {
    Program p;
    p.n = (int)ph.size();
    std::vector<Phase> ph2 = ph;
    for (Phase &x : ph2)
        if (x.kind == PH_MATVEC) x.mv.sv_off = (uint32_t)mv_spill_offset(x.mv);
    for (const Phase &x : ph) p.region = std::max(p.region, phase_region(x, max_pos));
    p.region = (p.region + 127) & ~(size_t)127;
    const std::vector<FeedPhase> ft = feed_table(ph);
    p.nfeed = (int)ft.size();
    for (const Phase &x : ph) p.nx += x.kind == PH_XGATHER || x.kind == PH_XARGMAX;
    const size_t pb = ph.size() * sizeof(Phase), fb = ft.size() * sizeof(FeedPhase);
    CU(cudaMalloc(&p.d, pb + fb));
    CU(cudaMemcpy(p.d, ph2.data(), pb, cudaMemcpyHostToDevice));
    p.feed = (const FeedPhase *)((const char *)p.d + pb);
    if (fb) CU(cudaMemcpy((void *)p.feed, ft.data(), fb, cudaMemcpyHostToDevice));
    *out = p;
    return 0;
}

// Shared memory of a decode launch: per-warp tile rings (as many slots as
// fit, at most kMaxSlots), the activation/attention region, two staged
// phase descriptors, the walk table.
int decode_geometry(uint32_t slot_bytes, const Program &p, DecodeArgs &a, size_t *smem) {
    const size_t fixed = p.region + 2 * sizeof(Phase) + (size_t)p.nfeed * sizeof(FeedPhase) + 128;
    const uint32_t slot = (std::max<uint32_t>(slot_bytes, 16) + 127) & ~127u;
    const long long room = (long long)g_decode_smem_max - (long long)fixed;
    const int ns = (int)std::min<long long>(kMaxSlots, room > 0 ? room / ((long long)kDW * slot) : 0);
    if (ns < 2) {
        set_error("the decode kernel needs %zu bytes of shared memory; the device allows %d", fixed + 2 * kDW * slot,
                  g_decode_smem_max);
        return -1;
    }
    a.ring_slots = ns;
    a.slot_bytes = slot;
    a.region_bytes = (uint32_t)p.region;
    a.prog = p.d;
    a.nphase = p.n;
    a.feed = p.feed;
    a.nfeed = p.nfeed;
    a.nx = p.nx;
    *smem = (size_t)kDW * ns * slot + fixed;
    return 0;
}

// one decode launch: zero the barrier counter, then the cooperative kernel
// (every CTA resident at once: the grid barriers need it)
int launch_decode(int sms, cudaStream_t st, const DecodeArgs &a, size_t smem) {
    CU(cudaMemsetAsync(a.bar, 0, sizeof(unsigned), st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kDecodeThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CU(cudaLaunchKernelEx(&cfg, k_decode, a));
    return 0;
}

DecodeArgs base_args(cxm_model *m) {
    DecodeArgs a{};
    a.tp = m->tp;
    a.tp_rank = m->tp_rank;
    a.xdim = m->cfg.dim;
    a.hdim = m->cfg.ffn;
    for (int p = 0; p < m->tp; p++) a.xch[p] = m->peer[p];
    a.epoch = m->epoch;
    a.bar = m->bar;
    a.err = m->err;
    a.vocab = m->cfg.vocab;
    a.argmax_key = m->argmax_key;
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.qcnt = m->hcnt;
    a.nqcnt = m->cfg.ffn / 16;
    return a;
}

int launch_sample(cxm_model *m, const int *d_len, uint32_t *toks, uint32_t *out, int *d_stop,
                  unsigned long long *stamps = nullptr);

int enqueue_step(cxm_model *m, cxm_cache *c, int mode, int cls) {
    if (!m->connected) {
        set_error("tensor-parallel rank %d of %d: cxm_tp_connect first", m->tp_rank, m->tp);
        return -1;
    }
    if (m->tp > 1 && mode == STEP_SAMPLE) {
        set_error("sampling needs the whole vocabulary on one rank: tensor-parallel models decode greedily");
        return -1;
    }
    if (mode == STEP_SAMPLE)
        return enqueue_step(m, c, STEP_LOGITS, cls) || launch_sample(m, c->d_len, c->toks, nullptr, c->d_stop) ? -1
                                                                                                            : 0;
    Program &p = c->prog[mode][cls];
    if (!p.d && upload_program(step_program(m, c, mode, cls), (int)c->max_tokens, &p)) return -1;
    DecodeArgs a = base_args(m);
    a.prog = p.d;
    a.nphase = p.n;
    a.d_len = c->d_len;
    a.toks = c->toks;
    a.max_pos = (int)c->max_tokens;
    a.write_token = mode == STEP_GREEDY;
    a.commit = 1;
    a.d_stop = c->d_stop;
    a.eos = m->cfg.has_eos ? (int)m->cfg.eos : -1;
    size_t smem = 0;
    if (decode_geometry(m->slot_bytes, p, a, &smem)) return -1;
    return launch_decode(m->sms, m->stream, a, smem);
}

int get_graph(cxm_model *m, cxm_cache *c, int mode, int cls, cudaGraphExec_t *out) {
    if (c->graph[mode][cls]) {
        *out = c->graph[mode][cls];
        return 0;
    }
    const int pm = mode == STEP_SAMPLE ? STEP_LOGITS : mode;
    if (!c->prog[pm][cls].d && upload_program(step_program(m, c, pm, cls), (int)c->max_tokens, &c->prog[pm][cls]))
        return -1;
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, c, mode, cls);
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return -1;
    }
    if (e != cudaSuccess) {
        set_error("graph capture failed: %s", cudaGetErrorString(e));
        return -1;
    }
    e = cudaGraphInstantiate(&c->graph[mode][cls], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        set_error("graph instantiate failed: %s", cudaGetErrorString(e));
        return -1;
    }
    *out = c->graph[mode][cls];
    return 0;
}

// n steps of one mode, replaying the tokens of a forward call of `rows`
// tokens (its row class picks every matrix's float order)
int run_steps(cxm_model *m, cxm_cache *c, int mode, uint64_t rows, uint32_t n) {
    if (n == 0) return 0;
    cudaGraphExec_t g;
    if (get_graph(m, c, mode, row_class(rows), &g)) return -1;
    for (uint32_t i = 0; i < n; i++) CU(cudaGraphLaunch(g, m->stream));
    return 0;
}

// the device Muestreador::elegir on the model's logits, with (1/T, top_p) and
// the RNG state from device memory; the token goes to toks[*d_len] or *out
int launch_sample(cxm_model *m, const int *d_len, uint32_t *toks, uint32_t *out, int *d_stop,
                  unsigned long long *stamps) {
    SampleArgs a{};
    a.stamps = stamps;
    a.logits = m->logits;
    a.n = m->cfg.vocab;
    a.params = m->samp_params;
    a.rng = m->rng;
    a.d_len = d_len;
    a.toks = toks;
    a.out = out;
    a.probs = m->samp_probs;
    a.prefix = m->samp_prefix;
    a.key0 = m->samp_k0;
    a.val0 = m->samp_v0;
    a.key1 = m->samp_k1;
    a.val1 = m->samp_v1;
    a.d_stop = d_stop;
    a.eos = d_stop && m->cfg.has_eos ? (int)m->cfg.eos : -1;
    a.ghist = m->samp_ghist;
    a.gred = m->samp_gred;
    a.bar = m->samp_bar;
    a.err = m->err;
    // about 1024 probabilities per CTA, at most one CTA per SM (all resident)
    const int grid = std::max(1, std::min(m->sms, (a.n + kSampThreads - 1) / kSampThreads));
    CU(cudaMemsetAsync(a.bar, 0, sizeof(unsigned), m->stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSampThreads);
    cfg.dynamicSmemBytes = kSampSmem;
    cfg.stream = m->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CU(cudaLaunchKernelEx(&cfg, k_sample, a));
    return 0;
}

int set_sampler(cxm_model *m, const cxm_sampler *s) {
    const float prm[2] = {1.0f / s->temperature, s->top_p};  // src/sampler.rs:77
    CU(cudaMemcpyAsync(m->samp_params, prm, sizeof(prm), cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(m->rng, &s->state, sizeof(uint64_t), cudaMemcpyHostToDevice, m->stream));
    return 0;
}

// The error word and the argmax key back to the host in one round trip: both
// copies queue behind the steps, then one synchronisation.
int check_err(cxm_model *m) {
    CU(cudaMemcpyAsync(&m->hw->err, m->err, 4, cudaMemcpyDeviceToHost, m->stream));
    CU(cudaMemcpyAsync(&m->hw->key, m->argmax_key, 8, cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    const int e = m->hw->err;
    m->key_valid = e == 0;
    if (e) {
        CU(cudaMemset(m->err, 0, 4));
        set_error("device reported %s", (e & ERR_TOKEN)      ? "a token beyond the vocabulary"
                                        : (e & ERR_POSITION) ? "a position beyond the cache"
                                                             : "a wait that timed out");
        return -1;
    }
    return 0;
}

}  // namespace

// ─────────────────────────────── C ABI ───────────────────────────────

extern "C" const char *cxm_last_error(void) { return last_error(); }

extern "C" int cxm_model_open(const char *path, int device, cxm_model **out) {
    return cxm_model_open_tp(path, device, 0, 1, out);
}

extern "C" int cxm_model_open_tp(const char *path, int device, int tp_rank, int tp_size, cxm_model **out) {
    if (!path || !out) {
        set_error("null argument");
        return -1;
    }
    *out = nullptr;
    if (tp_size < 1 || tp_size > kTpMax || tp_rank < 0 || tp_rank >= tp_size) {
        set_error("tensor-parallel rank %d of %d (1..%d ranks)", tp_rank, tp_size, kTpMax);
        return -1;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        set_error("no CUDA device: this library has no CPU path");
        return -1;
    }
    if (device < 0 || device >= ndev) {
        set_error("device %d out of range (%d devices)", device, ndev);
        return -1;
    }
    CU(cudaSetDevice(device));
    cudaDeviceProp prop;
    CU(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) {
        set_error("device %d is sm_%d%d; this build targets sm_100a", device, prop.major, prop.minor);
        return -1;
    }
    Gguf g;
    if (!g.open(path)) return -1;
    std::unique_ptr<cxm_model> m(new cxm_model);
    m->device = device;
    m->sms = prop.multiProcessorCount;
    m->tp = tp_size;
    m->tp_rank = tp_rank;
    m->connected = tp_size == 1;
    cxm_config &cfg = m->cfg;
    uint64_t v;
    const char *ik[] = {"qwen2.block_count", "qwen2.embedding_length", "qwen2.attention.head_count",
                        "qwen2.attention.head_count_kv", "qwen2.context_length"};
    int32_t *iv[] = {&cfg.n_layer, &cfg.dim, &cfg.n_head, &cfg.n_head_kv, &cfg.ctx};
    for (int i = 0; i < 5; i++) {
        if (!g.meta_int(ik[i], &v)) {
            set_error("missing metadata %s", ik[i]);
            return -1;
        }
        *iv[i] = (int32_t)v;
    }
    double dv;
    cfg.eps = g.meta_float("qwen2.attention.layer_norm_rms_epsilon", &dv) ? (float)dv : 1e-6f;
    cfg.rope_base = g.meta_float("qwen2.rope.freq_base", &dv) ? (float)dv : 10000.0f;
    if (g.meta_int("tokenizer.ggml.eos_token_id", &v)) {
        cfg.has_eos = 1;
        cfg.eos = (uint32_t)v;
    }
    if (cfg.n_head <= 0 || cfg.dim % cfg.n_head || cfg.n_head_kv <= 0 || cfg.n_head % cfg.n_head_kv) {
        set_error("inconsistent head counts");
        return -1;
    }
    cfg.head_dim = cfg.dim / cfg.n_head;
    // this rank's share (src/forward.rs has one rank): the attention block
    // whole (every head, every KV head, o_proj), its rows of the FFN
    // (gate/up rows of its FFN slice, ffn_down rows of its hidden slice, each
    // over the whole input), its vocabulary rows
    const int tp = tp_size, r = tp_rank;
    if (cfg.dim % (4 * tp)) {
        set_error("hidden size %d does not split over %d ranks in groups of 4", cfg.dim, tp);
        return -1;
    }
    m->h_loc = cfg.n_head;
    m->kv_loc = cfg.n_head_kv;
    const int dl = m->h_loc * cfg.head_dim;  // the attention output: o's K
    const TensorInfo *embd = g.tensor("token_embd.weight");
    const TensorInfo *outw = g.tensor("output.weight");
    const TensorInfo *onorm = g.tensor("output_norm.weight");
    if (!embd || !onorm) {
        set_error("missing tensor %s", embd ? "output_norm.weight" : "token_embd.weight");
        return -1;
    }
    cfg.vocab = (int32_t)embd->dims[1];
    cfg.tied = outw == nullptr;
    // output rows: an even share per rank, the last takes the rest
    m->v_loc = tp == 1 ? cfg.vocab : (cfg.vocab / tp) & ~1;
    m->v_off = r * m->v_loc;
    if (r == tp - 1) m->v_loc = cfg.vocab - m->v_off;
    CU(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    CU(cudaHostAlloc((void **)&m->hw, sizeof(cxm_model::HostWords), cudaHostAllocDefault));
    memset(m->hw, 0, sizeof(cxm_model::HostWords));
    if (embd->type == F32) {
        if (upload_vector(m.get(), g, *embd, (size_t)cfg.vocab * cfg.dim, &m->embd_f32)) return -1;
        m->embd.type = 0;
    } else if (upload_matrix(m.get(), g, *embd, PAIR_ADJ, 0,
                             choose_lpr(cfg.vocab, (int)(embd->dims[0] / 256), m->sms), &m->embd)) {
        return -1;
    }
    if (outw) {
        if (check_matrix(*outw) ||
            upload_matrix(m.get(), g, *outw, PAIR_ADJ, 0, choose_lpr(m->v_loc, (int)(outw->dims[0] / 256), m->sms),
                          &m->out, m->v_off, m->v_loc))
            return -1;
    } else {
        if (embd->type == F32) {
            set_error("a tied F32 embedding table has no device output kernel");
            return -1;
        }
        if (tp == 1) {
            m->out = m->embd;
        } else {  // this rank's rows of the tied table, as its own output matrix
            const uint64_t wb = m->weight_bytes;
            if (upload_matrix(m.get(), g, *embd, PAIR_ADJ, 0, choose_lpr(m->v_loc, (int)(embd->dims[0] / 256), m->sms),
                              &m->out, m->v_off, m->v_loc))
                return -1;
            m->weight_bytes = wb;  // the bytes of the table are counted once
        }
    }
    if (upload_vector(m.get(), g, *onorm, (size_t)cfg.dim, &m->out_norm)) return -1;
    const size_t hd = (size_t)cfg.head_dim, kvd = (size_t)cfg.n_head_kv * hd;
    for (int i = 0; i < cfg.n_layer; i++) {
        Layer L{};
        auto T = [&](const char *nm) -> const TensorInfo * {
            std::string n = "blk." + std::to_string(i) + "." + nm;
            const TensorInfo *t = g.tensor(n);
            if (!t) set_error("missing tensor %s", n.c_str());
            return t;
        };
        const TensorInfo *t, *t2;
        const int half = (int)hd / 2, nbd = cfg.dim / 256;
        const TensorInfo *tg = T("ffn_gate.weight"), *td = T("ffn_down.weight");
        if (!tg || !td || check_matrix(*tg) || check_matrix(*td)) return -1;
        const int F = (int)tg->dims[1];
        if (F % (4 * tp)) {
            set_error("FFN of %d rows does not split over %d ranks in groups of 4", F, tp);
            return -1;
        }
        const int fl = F / tp, dloc = cfg.dim / tp, ql = dl, kl = m->kv_loc * (int)hd;  // this rank's rows
        // tile shapes by phase: q|k|v share one; o, gate|up and down their own
        const int lpr_qkv = choose_lpr(ql + 2 * kl, nbd, m->sms), lpr_o = choose_lpr(cfg.dim, dl / 256, m->sms);
        const int lpr_gu = choose_lpr(2 * fl, nbd, m->sms);
        const int lpr_down = choose_lpr(dloc, F / 256, m->sms);
        if (!(t = T("attn_norm.weight")) || upload_vector(m.get(), g, *t, cfg.dim, &L.attn_norm)) return -1;
        if (!(t = T("attn_q.weight")) || upload_matrix(m.get(), g, *t, PAIR_ROPE, half, lpr_qkv, &L.q)) return -1;
        if (!(t = T("attn_q.bias")) || upload_vector(m.get(), g, *t, cfg.dim, &L.bq)) return -1;
        if (!(t = T("attn_k.weight")) || upload_matrix(m.get(), g, *t, PAIR_ROPE, half, lpr_qkv, &L.k)) return -1;
        if (!(t = T("attn_k.bias")) || upload_vector(m.get(), g, *t, kvd, &L.bk)) return -1;
        if (!(t = T("attn_v.weight")) || upload_matrix(m.get(), g, *t, PAIR_ADJ, 0, lpr_qkv, &L.v)) return -1;
        if (!(t = T("attn_v.bias")) || upload_vector(m.get(), g, *t, kvd, &L.bv)) return -1;
        if (!(t = T("attn_output.weight")) || upload_matrix(m.get(), g, *t, PAIR_ADJ, 0, lpr_o, &L.o)) return -1;
        if (!(t = T("ffn_norm.weight")) || upload_vector(m.get(), g, *t, cfg.dim, &L.ffn_norm)) return -1;
        if (!(t2 = T("ffn_up.weight")) || upload_pair(m.get(), g, *tg, *t2, lpr_gu, &L.gu, r * fl, fl)) return -1;
        if (upload_matrix(m.get(), g, *td, PAIR_ADJ, 0, lpr_down, &L.down, r * dloc, dloc)) return -1;
        if (L.q.rows != ql || L.k.rows != kl || L.v.rows != kl || L.o.rows != cfg.dim || L.q.K != cfg.dim ||
            L.k.K != cfg.dim || L.v.K != cfg.dim || L.o.K != dl || L.gu.K != cfg.dim || L.gu.rows != 2 * fl ||
            L.down.K != F || L.down.rows != dloc || (int)td->dims[0] != F) {
            set_error("layer %d: matrix shapes do not match the config", i);
            return -1;
        }
        m->layers.push_back(L);
        cfg.ffn = F;
        m->f_loc = fl;
    }
    if (cfg.dim > kMaxNormed) {
        set_error("hidden size %d: the decode kernel's RMSNorm prologue takes at most %d", cfg.dim, kMaxNormed);
        return -1;
    }
    // RoPE tables exactly as src/ops.rs:1108-1129 (f32 frequency, f64 angle)
    {
        const int half = cfg.head_dim / 2;
        std::vector<float> c((size_t)cfg.ctx * half), s((size_t)cfg.ctx * half);
        for (int j = 0; j < half; j++) {
            volatile float expo = 2.0f * (float)j / (float)cfg.head_dim;
            float freq = 1.0f / powf(cfg.rope_base, expo);
            for (int p = 0; p < cfg.ctx; p++) {
                double ang = (double)p * (double)freq;
                c[(size_t)p * half + j] = (float)cos(ang);
                s[(size_t)p * half + j] = (float)sin(ang);
            }
        }
        if (m->alloc(&m->rope_cos, c.size()) || m->alloc(&m->rope_sin, s.size())) return -1;
        CU(cudaMemcpy(m->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(m->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
    }
    // activations
    if (m->alloc(&m->x, cfg.dim) || m->alloc(&m->q, cfg.dim) || m->alloc(&m->att, cfg.dim) ||
        m->alloc(&m->attq, act_bytes(cfg.n_head * cfg.head_dim, 1, 1)) ||
        m->alloc(&m->hq, act_bytes(cfg.ffn, 1, 1)) || m->alloc(&m->hcnt, (size_t)cfg.ffn / 16) ||
        m->alloc(&m->logits, cfg.vocab) || m->alloc(&m->err, 1) ||
        m->alloc(&m->bar, 1) || m->alloc(&m->argmax_key, 1) || m->alloc(&m->rng, 1) ||
        m->alloc(&m->samp_params, 2) || m->alloc(&m->samp_tok, 1) || m->alloc(&m->samp_probs, cfg.vocab) ||
        m->alloc(&m->samp_prefix, cfg.vocab) || m->alloc(&m->samp_k0, cfg.vocab) ||
        m->alloc(&m->samp_v0, cfg.vocab) || m->alloc(&m->samp_k1, cfg.vocab) || m->alloc(&m->samp_v1, cfg.vocab) ||
        m->alloc(&m->samp_ghist, (size_t)m->sms * 256) || m->alloc(&m->samp_gred, (size_t)m->sms + 1) ||
        m->alloc(&m->samp_bar, 1) ||
        m->alloc(&m->scores, (size_t)cfg.n_head * ((cfg.ctx + 3) & ~3)))
        return -1;
    CU(cudaMemset(m->err, 0, sizeof(int)));
    // the exchange area (it holds the FFN's hidden vector, which peers read
    // under tensor parallelism) and the exchange count
    if (m->alloc(&m->xch, xch_bytes(cfg.ffn, cfg.dim)) || m->alloc(&m->epoch, 1)) return -1;
    CU(cudaMemset(m->xch, 0, xch_bytes(cfg.ffn, cfg.dim)));
    m->h = (float *)m->xch;
    CU(cudaMemset(m->epoch, 0, sizeof(unsigned)));
    m->peer[tp_rank] = m->xch;
    if (set_kernel_smem_limits()) return -1;
    if (out_smem((uint32_t)cfg.ctx) > 200 * 1024 || cfg.head_dim % 32 || cfg.head_dim > kKRow - 4 ||
        cfg.vocab % 2 || cfg.dim % 4) {
        set_error("context %d / head_dim %d / vocab %d are beyond the decode kernels' layouts", cfg.ctx,
                  cfg.head_dim, cfg.vocab);
        return -1;
    }
    int per_sm = 0;
    CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode, kDecodeThreads, (size_t)g_decode_smem_max));
    if (per_sm < 1) {
        set_error("the decode kernel does not fit an SM");
        return -1;
    }
    CU(cudaDeviceSynchronize());
    *out = m.release();
    return 0;
}

extern "C" int cxm_tp_handle(cxm_model *m, uint8_t *handle_out) {
    if (!m || !handle_out) {
        set_error("null argument");
        return -1;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == CXM_TP_HANDLE_BYTES, "IPC handle size");
    CU(cudaSetDevice(m->device));
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, m->xch));
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}

extern "C" int cxm_tp_connect(cxm_model *m, const uint8_t *handles) {
    if (!m || !handles) {
        set_error("null argument");
        return -1;
    }
    if (m->connected) {
        set_error("already connected");
        return -1;
    }
    CU(cudaSetDevice(m->device));
    for (int p = 0; p < m->tp; p++) {
        if (p == m->tp_rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)p * CXM_TP_HANDLE_BYTES, sizeof(h));
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error("rank %d: mapping rank %d's exchange area failed: %s", m->tp_rank, p, cudaGetErrorString(e));
            return -1;
        }
        m->peer[p] = (unsigned char *)ptr;
        m->peer_mapped[p] = true;
    }
    m->connected = true;
    return 0;
}

extern "C" int cxm_model_tp_info(const cxm_model *m, int *tp_rank, int *tp_size, int *vocab_lo, int *vocab_n) {
    if (!m) {
        set_error("null argument");
        return -1;
    }
    if (tp_rank) *tp_rank = m->tp_rank;
    if (tp_size) *tp_size = m->tp;
    if (vocab_lo) *vocab_lo = m->v_off;
    if (vocab_n) *vocab_n = m->v_loc;
    return 0;
}

extern "C" int cxm_model_config(const cxm_model *m, cxm_config *out) {
    if (!m || !out) {
        set_error("null argument");
        return -1;
    }
    *out = m->cfg;
    return 0;
}

extern "C" uint64_t cxm_model_weight_bytes(const cxm_model *m) { return m ? m->weight_bytes : 0; }

extern "C" int cxm_model_set_prefill(cxm_model *m, int tensor_cores) {
    if (!m) {
        set_error("null model");
        return -1;
    }
    m->prefill_tc = tensor_cores != 0;
    return 0;
}

extern "C" void cxm_model_close(cxm_model *m) { delete m; }

extern "C" int cxm_cache_new(cxm_model *m, uint32_t max_tokens, cxm_cache **out) {
    if (!m || !out) {
        set_error("null argument");
        return -1;
    }
    *out = nullptr;
    if (max_tokens == 0 || max_tokens > (uint32_t)m->cfg.ctx) {
        set_error("max_tokens %u must be in 1..=%d (the context)", max_tokens, m->cfg.ctx);
        return -1;
    }
    CU(cudaSetDevice(m->device));
    std::unique_ptr<cxm_cache> c(new cxm_cache);
    c->m = m;
    c->device = m->device;
    c->max_tokens = max_tokens;
    size_t n = (size_t)m->cfg.n_layer * max_tokens * kv_dim(m);
    CU(cudaMalloc(&c->k, n * 4));
    CU(cudaMalloc(&c->v, n * 4));
    CU(cudaMalloc(&c->toks, ((size_t)max_tokens + 2) * 4));
    CU(cudaMalloc(&c->d_len, 4));
    CU(cudaMemset(c->d_len, 0, 4));
    CU(cudaMalloc(&c->d_stop, 4));
    CU(cudaMemset(c->d_stop, 0, 4));
    CU(cudaMemset(c->toks, 0, ((size_t)max_tokens + 2) * 4));
    *out = c.release();
    return 0;
}

extern "C" void cxm_cache_free(cxm_cache *c) {
    if (!c) return;
    release_prefix(c);
    if (c->borrowers > 0) {  // still lent: deleted with its last borrower
        c->orphan = true;
        return;
    }
    delete c;
}
extern "C" uint32_t cxm_cache_len(const cxm_cache *c) { return c ? c->len : 0; }

static int set_len(cxm_cache *c, uint32_t n) {
    cudaSetDevice(c->m->device);
    int v = (int)n;
    CU(cudaMemcpyAsync(c->d_len, &v, 4, cudaMemcpyHostToDevice, c->m->stream));
    CU(cudaStreamSynchronize(c->m->stream));
    c->len = n;
    return 0;
}

extern "C" int cxm_cache_truncate(cxm_cache *c, uint32_t n) {
    if (!c) {
        set_error("null cache");
        return -1;
    }
    if (n >= c->len) return 0;  // Cache::truncar keeps everything when n >= len
    if (n < c->lent) {
        set_error("positions below %u are lent to %d cache(s) as a shared prefix", c->lent, c->borrowers);
        return -1;
    }
    if (n < c->plen) {  // borrows less of its prefix
        c->plen = n;
        c->drop_programs();
    }
    return set_len(c, n);
}

extern "C" int cxm_cache_clear(cxm_cache *c) {
    if (!c) {
        set_error("null cache");
        return -1;
    }
    if (c->lent) {
        set_error("positions below %u are lent to %d cache(s) as a shared prefix", c->lent, c->borrowers);
        return -1;
    }
    release_prefix(c);
    return set_len(c, 0);
}

extern "C" int cxm_cache_copy_prefix(const cxm_cache *src, uint32_t n, cxm_cache *dst) {
    if (!src || !dst || src->m != dst->m) {
        set_error("caches must exist and belong to the same model");
        return -1;
    }
    cxm_model *m = src->m;
    n = std::min(n, src->len);
    if (n > dst->max_tokens) {
        set_error("prefix of %u tokens does not fit a cache of %u", n, dst->max_tokens);
        return -1;
    }
    if (dst == src) {
        set_error("a cache cannot copy its own prefix");
        return -1;
    }
    if (dst->lent) {
        set_error("positions below %u of the destination are lent as a shared prefix", dst->lent);
        return -1;
    }
    CU(cudaSetDevice(m->device));
    const size_t kvd = kv_dim(m);
    release_prefix(dst);  // the copy is the destination's own
    if (n) {
        // rows below the source's borrowed prefix come from the lender
        const uint32_t np = std::min(n, src->plen);
        for (int part = 0; part < 2; part++) {
            const uint32_t r0 = part ? np : 0, r1 = part ? n : np;
            if (r1 <= r0) continue;
            const cxm_cache *from = part ? src : src->prefix;
            const size_t off = (size_t)r0 * kvd;
            CU(cudaMemcpy2DAsync(dst->k + off, dst->max_tokens * kvd * 4, from->k + off, from->max_tokens * kvd * 4,
                                 (r1 - r0) * kvd * 4, m->cfg.n_layer, cudaMemcpyDeviceToDevice, m->stream));
            CU(cudaMemcpy2DAsync(dst->v + off, dst->max_tokens * kvd * 4, from->v + off, from->max_tokens * kvd * 4,
                                 (r1 - r0) * kvd * 4, m->cfg.n_layer, cudaMemcpyDeviceToDevice, m->stream));
        }
        CU(cudaMemcpyAsync(dst->toks, src->toks, (size_t)(n + 1 <= src->max_tokens + 1 ? n + 1 : n) * 4,
                           cudaMemcpyDeviceToDevice, m->stream));
    }
    return set_len(dst, n);
}

extern "C" int cxm_cache_share_prefix(cxm_cache *src, uint32_t n, cxm_cache *dst) {
    if (!src || !dst || src->m != dst->m || src == dst) {
        set_error("two distinct caches of the same model are needed");
        return -1;
    }
    if (src->orphan) {
        set_error("the source cache was freed");
        return -1;
    }
    n = std::min(n, src->len);
    if (n > dst->max_tokens) {
        set_error("prefix of %u tokens does not fit a cache of %u", n, dst->max_tokens);
        return -1;
    }
    if (dst->lent) {
        set_error("positions below %u of the destination are lent as a shared prefix", dst->lent);
        return -1;
    }
    // a prefix of a borrower is a prefix of its lender (one level of lending)
    cxm_cache *lender = src;
    if (src->prefix) {
        if (n > src->plen) {
            set_error("the source borrows its first %u positions: share at most those, or copy", src->plen);
            return -1;
        }
        lender = src->prefix;
    }
    cxm_model *m = src->m;
    CU(cudaSetDevice(m->device));
    release_prefix(dst);
    dst->drop_programs();
    if (n) {
        dst->prefix = lender;
        dst->plen = n;
        lender->borrowers++;
        lender->lent = std::max(lender->lent, n);
        CU(cudaMemcpyAsync(dst->toks, src->toks, (size_t)(n + 1 <= src->max_tokens + 1 ? n + 1 : n) * 4,
                           cudaMemcpyDeviceToDevice, m->stream));
    }
    return set_len(dst, n);
}

extern "C" int cxm_cache_read(const cxm_cache *c, uint32_t layer, int is_v, float *host_out) {
    if (!c || !host_out || layer >= (uint32_t)c->m->cfg.n_layer) {
        set_error("bad cache read");
        return -1;
    }
    cxm_model *m = c->m;
    CU(cudaSetDevice(m->device));
    const size_t kvd = kv_dim(m);
    const float *base = (is_v ? c->v : c->k) + (size_t)layer * c->max_tokens * kvd;
    CU(cudaStreamSynchronize(m->stream));
    const uint32_t np = std::min(c->plen, c->len);
    if (np) {  // the borrowed rows from the lender
        const float *pb = is_v ? prefix_v(c, (int)layer, kvd) : prefix_k(c, (int)layer, kvd);
        CU(cudaMemcpy(host_out, pb, (size_t)np * kvd * 4, cudaMemcpyDeviceToHost));
    }
    CU(cudaMemcpy(host_out + (size_t)np * kvd, base + (size_t)np * kvd, (size_t)(c->len - np) * kvd * 4,
                  cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int cxm_forward(cxm_model *m, cxm_cache *c, const uint32_t *tokens, uint32_t n, float *logits_out) {
    if (!m || !c || c->m != m || (!tokens && n)) {
        set_error("bad arguments");
        return -1;
    }
    if (n == 0) {
        set_error("no tokens to process");  // src/forward.rs:376-378
        return -1;
    }
    if ((uint64_t)c->len + n > (uint64_t)m->cfg.ctx) {
        set_error("%llu tokens exceed the context of %d", (unsigned long long)c->len + n, m->cfg.ctx);
        return -1;
    }
    if ((uint64_t)c->len + n > c->max_tokens) {
        set_error("%llu tokens exceed the cache of %u", (unsigned long long)c->len + n, c->max_tokens);
        return -1;
    }
    for (uint32_t i = 0; i < n; i++)
        if (tokens[i] >= (uint32_t)m->cfg.vocab) {
            set_error("token %u does not fit a vocabulary of %d", tokens[i], m->cfg.vocab);
            return -1;
        }
    CU(cudaSetDevice(m->device));
    CU(cudaMemsetAsync(c->d_stop, 0, 4, m->stream));
    CU(cudaMemcpyAsync(c->toks + c->len, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream));
    if (prompt_prefix(m, c, c->len, n) || run_steps(m, c, STEP_LOGITS, n, 1)) return -1;
    if (logits_out)  // this rank's vocabulary rows (all of them without tensor parallelism)
        CU(cudaMemcpyAsync(logits_out, m->logits, (size_t)m->v_loc * 4, cudaMemcpyDeviceToHost, m->stream));
    if (check_err(m)) return -1;
    c->len += n;
    m->logits_valid = true;
    return 0;
}

extern "C" int cxm_sampler_new(uint64_t seed, float temperature, float top_p, cxm_sampler **out) {
    if (!out) {
        set_error("null argument");
        return -1;
    }
    cxm_sampler *s = new cxm_sampler;
    s->state = seed == 0 ? 0x9E3779B97F4A7C15ull : seed;
    s->temperature = temperature;
    s->top_p = top_p < 0.0f ? 0.0f : (top_p > 1.0f ? 1.0f : top_p);
    *out = s;
    return 0;
}
extern "C" void cxm_sampler_free(cxm_sampler *s) { delete s; }
extern "C" uint64_t cxm_sampler_state(const cxm_sampler *s) { return s ? s->state : 0; }

extern "C" int cxm_sample(cxm_model *m, cxm_sampler *s, uint32_t *token_out) {
    if (!m || !s || !token_out) {
        set_error("null argument");
        return -1;
    }
    if (!m->logits_valid) {
        set_error("no logits: call cxm_forward first");
        return -1;
    }
    CU(cudaSetDevice(m->device));
    if (s->temperature > 0.0f && m->tp > 1) {
        set_error("sampling needs the whole vocabulary on one rank: tensor-parallel models decode greedily");
        return -1;
    }
    if (s->temperature > 0.0f) {  // the device Muestreador::elegir
        if (set_sampler(m, s) || launch_sample(m, nullptr, nullptr, m->samp_tok, nullptr)) return -1;
        uint32_t tok = 0;
        uint64_t st = 0;
        CU(cudaMemcpyAsync(&tok, m->samp_tok, 4, cudaMemcpyDeviceToHost, m->stream));
        CU(cudaMemcpyAsync(&st, m->rng, 8, cudaMemcpyDeviceToHost, m->stream));
        CU(cudaStreamSynchronize(m->stream));
        *token_out = tok;
        s->state = st;
        return 0;
    }
    // greedy: the first maximum (src/sampler.rs:129-137), already read back
    // with the forward's error word
    unsigned long long key = m->hw->key;
    if (!m->key_valid) {
        CU(cudaStreamSynchronize(m->stream));
        CU(cudaMemcpy(&key, m->argmax_key, 8, cudaMemcpyDeviceToHost));
    }
    *token_out = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
    return 0;
}

extern "C" int cxm_generate(cxm_model *m, cxm_cache *c, const uint32_t *prompt, uint32_t n_prompt, uint32_t max_new,
                            cxm_sampler *s, uint32_t *out, uint32_t *n_out) {
    if (!m || !c || !s || !n_out || (max_new && !out) || c->m != m) {
        set_error("bad arguments");
        return -1;
    }
    *n_out = 0;
    if (n_prompt == 0 || !prompt) {
        set_error("no tokens to process");
        return -1;
    }
    const bool sampled = s->temperature > 0.0f;
    const uint64_t after = (uint64_t)c->len + n_prompt;
    const uint64_t limit = std::min<uint64_t>((uint64_t)m->cfg.ctx, c->max_tokens);
    if (after > limit) {
        set_error("%llu tokens exceed the context of %llu", (unsigned long long)after, (unsigned long long)limit);
        return -1;
    }
    for (uint32_t i = 0; i < n_prompt; i++)
        if (prompt[i] >= (uint32_t)m->cfg.vocab) {
            set_error("token %u does not fit a vocabulary of %d", prompt[i], m->cfg.vocab);
            return -1;
        }
    CU(cudaSetDevice(m->device));
    const uint32_t len0 = c->len;
    CU(cudaMemsetAsync(c->d_stop, 0, 4, m->stream));
    CU(cudaMemcpyAsync(c->toks + len0, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    if (prompt_prefix(m, c, len0, n_prompt)) return -1;
    if (max_new == 0) {
        // the prompt is still forwarded (logits of the last token)
        if (run_steps(m, c, STEP_LOGITS, n_prompt, 1) || check_err(m)) return -1;
        c->len = (uint32_t)after;
        m->logits_valid = true;
        return 0;
    }
    // src/forward.rs:544-557: pick, push, stop at the context, forward.
    // Generated tokens: min(max_new, limit - after + 1); each one except a
    // context-limited last one is forwarded.
    const uint64_t gen = std::min<uint64_t>(max_new, limit - after + 1);
    const uint64_t fwd = std::min<uint64_t>(max_new, limit - after);
    // step i (0..gen) forwards toks[after-1+i] and writes token i at toks[after+i]
    const uint64_t state0 = s->state;
    if (sampled && set_sampler(m, s)) return -1;
    // the first pick ends the prompt's forward call (its row class); every
    // later token is a forward call of one row
    const int pick = sampled ? STEP_SAMPLE : STEP_GREEDY;
    if (run_steps(m, c, pick, n_prompt, 1) || run_steps(m, c, pick, 1, (uint32_t)(gen - 1))) return -1;
    if (fwd == gen && run_steps(m, c, STEP_PREFILL, 1, 1)) return -1;
    if (check_err(m)) return -1;
    std::vector<uint32_t> toks(gen);
    CU(cudaMemcpy(toks.data(), c->toks + after, gen * 4, cudaMemcpyDeviceToHost));
    uint64_t n = gen, forwarded = fwd;
    if (m->cfg.has_eos) {
        for (uint64_t i = 0; i < gen; i++)
            if (toks[i] == m->cfg.eos) {
                n = i;
                forwarded = i;
                break;
            }
    }
    for (uint64_t i = 0; i < n; i++) out[i] = toks[i];
    *n_out = (uint32_t)n;
    if (sampled) {  // one draw per pick, the eos pick included (src/forward.rs:544-548)
        const uint64_t draws = n < gen ? n + 1 : gen;
        uint64_t st = state0;
        for (uint64_t i = 0; i < draws; i++) {
            uint64_t x = st;
            x ^= x >> 12;
            x ^= x << 25;
            x ^= x >> 27;
            st = x;
        }
        s->state = st;
    }
    uint32_t final_len = (uint32_t)(after + forwarded);
    if (set_len(c, final_len)) return -1;
    m->logits_valid = false;
    return 0;
}

// ── batched forward of several conversations ──
// Rows of many conversations go through the tensor-core GEMMs together (one
// read of every weight for all of them): the prompts of a batch (every row of
// a prompt in its forward call's order, src/ops.rs:1056-1093 with m = the
// prompt's length), then each greedy step with one row per conversation (the
// order of a forward call of one row). Each row attends over its own
// conversation's cache and borrowed prefix. Every conversation gets, row for
// row, what src/forward.rs:544-557 computes for it alone.

// the step's token and position of each conversation
__global__ void k_batch_gather(uint32_t *const *toks, int *const *len, int n, uint32_t *tok, int *pos) {
    const int z = blockIdx.x * blockDim.x + threadIdx.x;
    if (z < n) {
        const int p = *len[z];
        pos[z] = p;
        tok[z] = toks[z][p];
    }
}

// rows sel[0..c) of x, packed (the rows whose logits are needed)
__global__ void k_batch_rows(const float *x, const int *sel, int D, float *out) {
    const int c = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
        out[(size_t)c * D + i] = x[(size_t)sel[c] * D + i];
}

// For each picked row c (conversation toks[c], len[c], stop[c], at position
// pos[c]): the argmax of its logits (the first maximum, NaNs skipped;
// src/sampler.rs:129-137) appended after the position, the eos flag, and the
// position advanced — unless the conversation met its eos earlier. Without
// `pick` only the position advances (the forward of the last pick).
constexpr int kPickThreads = 512;
__global__ void __launch_bounds__(kPickThreads) k_batch_pick(const float *logits, int V, const int *pos,
                                                             uint32_t *const *toks, int *const *len,
                                                             int *const *stop, int eos, int pick) {
    __shared__ unsigned long long best_s[kPickThreads / 32];
    const int c = blockIdx.x, tid = threadIdx.x;
    if (*(volatile int *)stop[c]) return;  // the whole block
    unsigned long long best = 0ull;
    if (pick) {
        const float *l = logits + (size_t)c * V;
        for (int i = tid; i < V; i += kPickThreads) {
            const float v = l[i];
            const unsigned long long k = v == v ? argmax_key(v, (uint32_t)i) : 0ull;
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if ((tid & 31) == 0) best_s[tid >> 5] = best;
        __syncthreads();
    }
    if (tid == 0) {
        const int p = pos[c];
        if (pick) {
            for (int w = 0; w < kPickThreads / 32; w++) best = best_s[w] > best ? best_s[w] : best;
            const uint32_t t = argmax_index(best);
            toks[c][p + 1] = t;
            if (eos >= 0 && t == (uint32_t)eos) *stop[c] = 1;
        }
        *len[c] = p + 1;
    }
}

// the positions of the picked rows
__global__ void k_batch_sel_pos(const int *pos, const int *sel, int n, int *out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n) out[c] = pos[sel[c]];
}

// A set of rows on the device: row r is conversation cache[r]'s token at
// position pos[r] (decode steps gather both from the caches themselves).
struct BatchRow {
    cxm_cache *c;
    int pos;
    uint32_t tok;
};

static int batch_reserve(cxm_model *m, int rows, int picks) {
    cxm_model::Batch &B = m->bt;
    if (B.cap >= rows && B.pcap >= picks) return 0;
    if (B.graph) cudaGraphExecDestroy(B.graph);
    B.graph = nullptr;
    B.graph_n = 0;
    cudaFree(B.mem);
    const int cap = std::max({rows, B.cap, 8}), pcap = std::max({picks, B.pcap, 8});
    B = cxm_model::Batch{};
    const int L = m->cfg.n_layer;
    const size_t bytes = (size_t)pcap * m->cfg.vocab * 4 + (size_t)pcap * m->cfg.dim * 4 + (size_t)cap * 4 * 3 +
                         (size_t)L * cap * 8 * 4 + (size_t)pcap * (4 * 2 + 8 * 3) + 2048;
    CU(cudaMalloc(&B.mem, bytes));
    char *p = (char *)B.mem;
    auto take = [&](size_t nb) {
        char *r = p;
        p += (nb + 15) & ~(size_t)15;
        return (void *)r;
    };
    B.logits = (float *)take((size_t)pcap * m->cfg.vocab * 4);
    B.xo = (float *)take((size_t)pcap * m->cfg.dim * 4);
    B.tok = (uint32_t *)take((size_t)cap * 4);
    B.pos = (int *)take((size_t)cap * 4);
    B.plenz = (int *)take((size_t)cap * 4);
    B.kz = (float **)take((size_t)L * cap * 8);
    B.vz = (float **)take((size_t)L * cap * 8);
    B.kpz = (const float **)take((size_t)L * cap * 8);
    B.vpz = (const float **)take((size_t)L * cap * 8);
    B.sel = (int *)take((size_t)pcap * 4);
    B.ppos = (int *)take((size_t)pcap * 4);
    B.toks = (uint32_t **)take((size_t)pcap * 8);
    B.len = (int **)take((size_t)pcap * 8);
    B.stop = (int **)take((size_t)pcap * 8);
    B.cap = cap;
    B.pcap = pcap;
    return 0;
}

// upload the views of `rows` (cache layer bases, prefixes, positions,
// tokens) and of the picked rows `picks` (indices into rows)
static int batch_upload(cxm_model *m, const std::vector<BatchRow> &rows, const std::vector<int> &picks) {
    cxm_model::Batch &B = m->bt;
    if (batch_reserve(m, (int)rows.size(), (int)picks.size())) return -1;
    const int L = m->cfg.n_layer, R = (int)rows.size();
    const size_t kvd = kv_dim(m);
    std::vector<const void *> kz((size_t)L * R), vz((size_t)L * R), kpz((size_t)L * R), vpz((size_t)L * R);
    std::vector<int> plen(R), pos(R);
    std::vector<uint32_t> tok(R);
    for (int r = 0; r < R; r++) {
        const cxm_cache *c = rows[r].c;
        for (int l = 0; l < L; l++) {
            kz[(size_t)l * R + r] = c->k + (size_t)l * c->max_tokens * kvd;
            vz[(size_t)l * R + r] = c->v + (size_t)l * c->max_tokens * kvd;
            kpz[(size_t)l * R + r] = prefix_k(c, l, kvd);
            vpz[(size_t)l * R + r] = prefix_v(c, l, kvd);
        }
        plen[r] = c->prefix ? (int)c->plen : 0;
        pos[r] = rows[r].pos;
        tok[r] = rows[r].tok;
    }
    const int P = (int)picks.size();
    std::vector<const void *> tk(P), ln(P), st(P);
    for (int i = 0; i < P; i++) {
        const cxm_cache *c = rows[picks[i]].c;
        tk[i] = c->toks;
        ln[i] = c->d_len;
        st[i] = c->d_stop;
    }
    // layer arrays are [n_layer][R] for this upload
    CU(cudaMemcpyAsync(B.kz, kz.data(), kz.size() * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.vz, vz.data(), vz.size() * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.kpz, kpz.data(), kpz.size() * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.vpz, vpz.data(), vpz.size() * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.plenz, plen.data(), (size_t)R * 4, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.pos, pos.data(), (size_t)R * 4, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.tok, tok.data(), (size_t)R * 4, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.sel, picks.data(), (size_t)P * 4, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.toks, tk.data(), (size_t)P * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.len, ln.data(), (size_t)P * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaMemcpyAsync(B.stop, st.data(), (size_t)P * 8, cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));  // the host vectors go out of scope
    B.rows = R;
    B.picks = P;
    return 0;
}

// The forward of the uploaded rows, in the order of row class `cls`; with
// `gather` the rows' tokens and positions are first read from the picked
// conversations' caches (a decode step: row r is pick r). Then, for the
// picked rows, the output projection and the greedy pick (`pick`), or the
// position advance alone.
static int batch_forward(cxm_model *m, int max_pos, int cls, bool gather, bool pick) {
    const cxm_config &cfg = m->cfg;
    const cxm_model::Batch &B = m->bt;
    const int n = B.rows, D = cfg.dim, hd = cfg.head_dim, H = m->h_loc, F = cfg.ffn, dq = H * hd;
    const size_t kvd = kv_dim(m);
    auto need = [](const QMat &M, int sz) { return sub_of(M.type) == sz ? 1 : 0; };
    if (gather) {
        k_batch_gather<<<(n + 127) / 128, 128, 0, m->stream>>>(B.toks, B.len, n, B.tok, B.pos);
        CU(cudaGetLastError());
    }
    {
        const dim3 g((D + 255) / 256, n);
        k_pf_embed<<<g, 256, 0, m->stream>>>(m->embd, m->embd_f32, B.tok, D, m->pf.x);
        CU(cudaGetLastError());
    }
    PfRowsDest rd;
    rd.pos = B.pos;
    rd.fused = 1;
    for (int l = 0; l < cfg.n_layer; l++) {
        const Layer &L = m->layers[l];
        if (pf_rows(m, m->pf.x, D, L.attn_norm, cfg.eps, D, n, need(L.q, 16) | need(L.k, 16) | need(L.v, 16),
                    need(L.q, 32) | need(L.k, 32) | need(L.v, 32)))
            return -1;
        MvSeg sq = mv_seg(L.q, dq / 2, PAIR_ROPE, EPI_ROPE, m->pf.q, cls);
        sq.half = hd / 2;
        sq.bias = L.bq;
        MvSeg sk = mv_seg(L.k, (int)kvd / 2, PAIR_ROPE, EPI_ROPE, nullptr, cls);
        sk.half = hd / 2;
        sk.bias = L.bk;
        sk.at_pos = 1;
        sk.pos_stride = (int)kvd;
        MvSeg sv = mv_seg(L.v, (int)kvd / 2, PAIR_ADJ, EPI_STORE, nullptr, cls);
        sv.bias = L.bv;
        sv.at_pos = 1;
        sv.pos_stride = (int)kvd;
        PfRowsDest rk = rd, rv = rd;
        rk.out = B.kz + (size_t)l * n;
        rv.out = B.vz + (size_t)l * n;
        if (pf_seg_gemm(m, sq, n, 0, dq, rd) || pf_seg_gemm(m, sk, n, 0, 0, rk) || pf_seg_gemm(m, sv, n, 0, 0, rv))
            return -1;
        AttnParams a{};
        a.scores = m->pf.scores;
        a.qs = dq;
        a.os = dq;
        a.H = H;
        a.KV = m->kv_loc;
        a.hd = hd;
        a.max_pos = max_pos;
        a.score_stride = (max_pos + 3) & ~3;
        a.scale = 1.0f / sqrtf((float)hd);  // src/ops.rs:1287
        a.err = m->err;
        // rows per launch: their score rows fit the scratch
        const int tz = (int)std::max<size_t>(
            1, std::min<size_t>(n, m->pf.score_floats / ((size_t)H * a.score_stride)));
        for (int z0 = 0; z0 < n; z0 += tz) {
            AttnParams az = a;
            az.q = m->pf.q + (size_t)z0 * dq;
            az.out = m->pf.att + (size_t)z0 * dq;
            az.kz = B.kz + (size_t)l * n + z0;
            az.vz = B.vz + (size_t)l * n + z0;
            az.kpz = B.kpz + (size_t)l * n + z0;
            az.vpz = B.vpz + (size_t)l * n + z0;
            az.posz = B.pos + z0;
            az.plenz = B.plenz + z0;
            if (launch_attention_on(m->stream, az, std::min(tz, n - z0))) return -1;
        }
        if (pf_rows(m, m->pf.att, dq, nullptr, 0.0f, dq, n, need(L.o, 16), need(L.o, 32)) ||
            pf_seg_gemm(m, mv_seg(L.o, D / 2, PAIR_ADJ, EPI_RESID, m->pf.x, cls), n, 0, D, rd))
            return -1;
        if (pf_rows(m, m->pf.x, D, L.ffn_norm, cfg.eps, D, n, need(L.gu, 16), need(L.gu, 32)) ||
            pf_seg_gemm(m, mv_seg(L.gu, F, PAIR_TWO, EPI_SWIGLU, m->pf.h, cls), n, 0, F, rd))
            return -1;
        if (pf_rows(m, m->pf.h, F, nullptr, 0.0f, F, n, need(L.down, 16), need(L.down, 32)) ||
            pf_seg_gemm(m, mv_seg(L.down, D / 2, PAIR_ADJ, EPI_RESID, m->pf.x, cls), n, 0, D, rd))
            return -1;
    }
    const int P = B.picks;
    if (P == 0) return 0;
    // the picked rows' positions: row sel[c]'s
    const float *xp = m->pf.x;
    if (pick) {  // final RMSNorm and output projection of the picked rows, one row each (src/forward.rs:495-501)
        if (!gather) {  // prompt rows: the picked (last) rows packed first
            const dim3 g((D + 255) / 256, P);
            k_batch_rows<<<g, 256, 0, m->stream>>>(m->pf.x, B.sel, D, B.xo);
            CU(cudaGetLastError());
            xp = B.xo;
        }
        if (pf_rows(m, xp, D, m->out_norm, cfg.eps, D, P, need(m->out, 16), need(m->out, 32)) ||
            pf_seg_gemm(m, mv_seg(m->out, cfg.vocab / 2, PAIR_ADJ, EPI_STORE, B.logits, ROWS_FEW), P, 0, cfg.vocab,
                        rd))
            return -1;
    }
    // the picked rows' positions (a decode step: the gathered ones, row c = pick c)
    const int *ppos = B.pos;
    if (!gather) {
        k_batch_sel_pos<<<(P + 127) / 128, 128, 0, m->stream>>>(B.pos, B.sel, P, B.ppos);
        CU(cudaGetLastError());
        ppos = B.ppos;
    }
    k_batch_pick<<<P, kPickThreads, 0, m->stream>>>(B.logits, cfg.vocab, ppos, B.toks, B.len, B.stop,
                                                    cfg.has_eos ? (int)cfg.eos : -1, pick ? 1 : 0);
    CU(cudaGetLastError());
    return 0;
}

extern "C" int cxm_generate_batch(cxm_model *m, cxm_cache *const *caches, const uint32_t *const *prompts,
                                  const uint32_t *n_prompt, uint32_t n, uint32_t max_new, uint32_t *out,
                                  uint32_t *n_out) {
    if (!m || !caches || !prompts || !n_prompt || !n_out || (max_new && !out) || n == 0) {
        set_error("bad arguments");
        return -1;
    }
    if (n > (uint32_t)kPrefillChunk) {
        set_error("at most %d conversations per batch", kPrefillChunk);
        return -1;
    }
    if (m->tp > 1) {
        set_error("batched decode runs on a single-GPU model");
        return -1;
    }
    int max_pos = 0;
    for (uint32_t z = 0; z < n; z++) {
        cxm_cache *c = caches[z];
        if (!c || c->m != m || c->orphan || !prompts[z] || n_prompt[z] == 0) {
            set_error("conversation %u: bad cache or empty prompt", z);
            return -1;
        }
        for (uint32_t y = 0; y < z; y++)
            if (caches[y] == c) {
                set_error("conversations %u and %u share a cache", y, z);
                return -1;
            }
        if (c->lent) {
            set_error("conversation %u: its cache is lent as a shared prefix and cannot grow", z);
            return -1;
        }
        const uint64_t need = (uint64_t)c->len + n_prompt[z] + max_new;
        const uint64_t limit = std::min<uint64_t>((uint64_t)m->cfg.ctx, c->max_tokens);
        if (need > limit) {
            set_error("conversation %u: %llu tokens exceed its context of %llu", z, (unsigned long long)need,
                      (unsigned long long)limit);
            return -1;
        }
        for (uint32_t i = 0; i < n_prompt[z]; i++)
            if (prompts[z][i] >= (uint32_t)m->cfg.vocab) {
                set_error("token %u does not fit a vocabulary of %d", prompts[z][i], m->cfg.vocab);
                return -1;
            }
        max_pos = std::max(max_pos, (int)c->max_tokens);
    }
    CU(cudaSetDevice(m->device));
    if (pf_reserve(m, kPrefillChunk)) return -1;
    for (uint32_t z = 0; z < n; z++) n_out[z] = 0;
    std::vector<uint32_t> len0(n), after(n);
    for (uint32_t z = 0; z < n; z++) {
        cxm_cache *c = caches[z];
        len0[z] = c->len;
        after[z] = c->len + n_prompt[z];
        CU(cudaMemsetAsync(c->d_stop, 0, 4, m->stream));
        CU(cudaMemcpyAsync(c->toks + len0[z], prompts[z], (size_t)n_prompt[z] * 4, cudaMemcpyHostToDevice,
                           m->stream));
    }
    // The prompts: each prompt's rows in its forward call's order (its row
    // class), all conversations of a class together, kPrefillChunk rows per
    // pass in position order; each prompt's last row picks its first token
    // (or, with max_new = 0, only advances the position).
    for (int cls = 0; cls < 3; cls++) {
        std::vector<BatchRow> rows;
        std::vector<int> picks;
        auto flush = [&]() -> int {
            if (rows.empty()) return 0;
            if (batch_upload(m, rows, picks) || batch_forward(m, max_pos, cls, false, max_new > 0)) return -1;
            rows.clear();
            picks.clear();
            return 0;
        };
        for (uint32_t z = 0; z < n; z++) {
            if (row_class(n_prompt[z]) != cls) continue;
            for (uint32_t i = 0; i < n_prompt[z]; i++) {
                if (rows.size() == (size_t)kPrefillChunk && flush()) return -1;
                rows.push_back(BatchRow{caches[z], (int)(len0[z] + i), prompts[z][i]});
                if (i + 1 == n_prompt[z]) picks.push_back((int)rows.size() - 1);
            }
        }
        if (flush()) return -1;
    }
    if (max_new) {
        // steps 1 .. max_new-1 pick; the last one forwards the last pick
        std::vector<BatchRow> rows(n);
        std::vector<int> picks(n);
        for (uint32_t z = 0; z < n; z++) {
            rows[z] = BatchRow{caches[z], 0, 0};
            picks[z] = (int)z;
        }
        if (batch_upload(m, rows, picks)) return -1;
        cxm_model::Batch &B = m->bt;
        if (max_new > 1) {
            if (B.graph) cudaGraphExecDestroy(B.graph);
            B.graph = nullptr;
            cudaGraph_t g = nullptr;
            CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
            const int rc = batch_forward(m, max_pos, ROWS_FEW, true, true);
            const cudaError_t ec = cudaStreamEndCapture(m->stream, &g);
            if (rc || ec != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                if (!rc) set_error("capturing the batched step failed: %s", cudaGetErrorString(ec));
                return -1;
            }
            const cudaError_t ei = cudaGraphInstantiate(&B.graph, g, 0);
            cudaGraphDestroy(g);
            if (ei != cudaSuccess) {
                B.graph = nullptr;
                set_error("instantiating the batched step failed: %s", cudaGetErrorString(ei));
                return -1;
            }
            for (uint32_t s = 1; s < max_new; s++) CU(cudaGraphLaunch(B.graph, m->stream));
        }
        if (batch_forward(m, max_pos, ROWS_FEW, true, false)) return -1;
    }
    if (check_err(m)) return -1;
    for (uint32_t z = 0; z < n; z++) {
        cxm_cache *c = caches[z];
        uint32_t gen = 0, fwd = n_prompt[z];
        if (max_new) {
            std::vector<uint32_t> t(max_new);
            CU(cudaMemcpy(t.data(), c->toks + after[z], (size_t)max_new * 4, cudaMemcpyDeviceToHost));
            gen = max_new;
            fwd = n_prompt[z] + max_new;
            if (m->cfg.has_eos)
                for (uint32_t i = 0; i < max_new; i++)
                    if (t[i] == m->cfg.eos) {  // the eos pick ends the generation, unforwarded
                        gen = i;
                        fwd = n_prompt[z] + i;
                        break;
                    }
            for (uint32_t i = 0; i < gen; i++) out[(size_t)z * max_new + i] = t[i];
        }
        n_out[z] = gen;
        if (set_len(c, len0[z] + fwd)) return -1;
    }
    m->logits_valid = false;
    return 0;
}

// ── kernel-level entry points ──

namespace {
struct DevBuf {
    void *p = nullptr;
    ~DevBuf() { cudaFree(p); }
};
// a start/stop pair of CUDA events, destroyed on every return path
struct EventPair {
    cudaEvent_t a = nullptr, b = nullptr;
    ~EventPair() {
        if (a) cudaEventDestroy(a);
        if (b) cudaEventDestroy(b);
    }
};
int dev_matrix_from_host(int type, const uint8_t *w, uint32_t rows, uint32_t k, DevBuf bufs[3], DMat *out) {
    if (!is_kquant(type) || k % 256 || rows == 0) {
        set_error("type %d, k %u: not a k-quant matrix", type, k);
        return -1;
    }
    const int nblk = (int)(k / 256), bb = bytes_per_block(type);
    const int pa = plane_a_bytes(type), ps = plane_s_bytes(type), pd = plane_d_bytes(type);
    DMat d{};
    d.type = type;
    d.rows = (int)rows;
    d.K = (int)k;
    d.nblk = nblk;
    d.a_row = (uint32_t)(nblk * pa);
    d.s_row = pitch16((uint32_t)(nblk * ps));
    d.d_row = pitch16((uint32_t)(nblk * pd));
    std::vector<uint8_t> A((size_t)rows * d.a_row), S((size_t)rows * d.s_row + 16), D((size_t)rows * d.d_row + 16);
    for (uint32_t r = 0; r < rows; r++)
        for (int b = 0; b < nblk; b++) {
            const uint8_t *blk = w + ((size_t)r * nblk + b) * bb;
            uint8_t *a = A.data() + (size_t)r * d.a_row + (size_t)b * pa;
            uint8_t *s = S.data() + (size_t)r * d.s_row + (size_t)b * ps;
            uint8_t *dd = D.data() + (size_t)r * d.d_row + (size_t)b * pd;
            switch (type) {
            case Q4K: case Q5K: memcpy(a, blk, (size_t)bb); break;
            case Q6K: memcpy(a, blk, 192); memcpy(s, blk + 192, 16); memcpy(dd, blk + 208, 2); break;
            case Q3K: memcpy(a, blk, 96); memcpy(s, blk + 96, 12); memcpy(dd, blk + 108, 2); break;
            case Q2K: memcpy(a, blk + 16, 64); memcpy(s, blk, 16); memcpy(dd, blk + 80, 4); break;
            }
        }
    CU(cudaMalloc(&bufs[0].p, A.size()));
    CU(cudaMalloc(&bufs[1].p, S.size()));
    CU(cudaMalloc(&bufs[2].p, D.size()));
    CU(cudaMemcpy(bufs[0].p, A.data(), A.size(), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(bufs[1].p, S.data(), S.size(), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(bufs[2].p, D.data(), D.size(), cudaMemcpyHostToDevice));
    d.a = (const uint8_t *)bufs[0].p;
    d.s = (const uint8_t *)bufs[1].p;
    d.d = (const uint8_t *)bufs[2].p;
    *out = d;
    return 0;
}

int need_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        set_error("no CUDA device: this library has no CPU path");
        return -1;
    }
    return 0;
}
}  // namespace

extern "C" int cxm_debug_subblock_sums(int type, const uint8_t *row, const int8_t *xq, uint32_t nblk, int32_t *out) {
    if (need_device()) return -1;
    if (!row || !xq || !out || nblk == 0) {
        set_error("bad arguments");
        return -1;
    }
    DevBuf b[3], dx, dout;
    DMat W;
    if (dev_matrix_from_host(type, row, 1, nblk * 256, b, &W)) return -1;
    const size_t K = (size_t)nblk * 256, nsub = K / (size_t)sub_of(type);
    CU(cudaMalloc(&dx.p, K));
    CU(cudaMalloc(&dout.p, nsub * 4));
    CU(cudaMemcpy(dx.p, xq, K, cudaMemcpyHostToDevice));
    size_t smem = ((K + 15) & ~(size_t)15) + K / 16 * 8;
    if (smem > 48 * 1024) CU(cudaFuncSetAttribute(k_subblock_sums, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_subblock_sums<<<1, 256, smem>>>(W, (const int8_t *)dx.p, (int32_t *)dout.p);
    CU(cudaGetLastError());
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(out, dout.p, nsub * 4, cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int cxm_debug_matmul(int type, const uint8_t *w, uint32_t rows, uint32_t k, const float *x, uint32_t m,
                                float *y) {
    if (need_device()) return -1;
    if (!w || !x || !y || rows % 2 || rows == 0 || !is_kquant(type) || k == 0 || k % 256 || k > kMaxActivation ||
        m == 0) {
        set_error("bad arguments (k-quant type, k a multiple of 256 up to %d, rows even, m >= 1)", kMaxActivation);
        return -1;
    }
    // 24 rows and more: the prompt forward's tensor-core GEMM (the buffered
    // path's order); fewer: the decode kernel on a one-phase program
    // (quantize x, W·x, store) once per activation row, every row in the
    // order matmul_auto takes for m rows
    int dev = 0, sms = 148;
    CU(cudaGetDevice(&dev));
    CU(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    QMat M = tiled_desc(type, (int)k, (int)rows, choose_lpr((int)rows, (int)(k / 256), sms));
    std::vector<uint8_t> tiles;
    build_tiles(M, rows_adj(w, (int)rows), tiles);
    DevBuf dw, dx, dy, derr, dbar, dprog;
    CU(cudaMalloc(&dw.p, tiles.size()));
    CU(cudaMemcpy(dw.p, tiles.data(), tiles.size(), cudaMemcpyHostToDevice));
    M.base = (const uint8_t *)dw.p;
    M.rows = (int)rows;
    CU(cudaMalloc(&dx.p, (size_t)k * 4));
    CU(cudaMalloc(&dy.p, (size_t)rows * 4));
    CU(cudaMalloc(&derr.p, 4));
    CU(cudaMalloc(&dbar.p, 4));
    CU(cudaMemset(derr.p, 0, 4));
    if (row_class(m) == ROWS_MANY) {
        DevBuf xa, a16, a32, e16, s16, e32, s32, yy, derr2;
        const size_t ab = pfa_bytes((int)m, (int)k);
        CU(cudaMalloc(&xa.p, (size_t)m * k * 4));
        CU(cudaMalloc(&yy.p, (size_t)m * rows * 4));
        CU(cudaMalloc(&a16.p, ab));
        CU(cudaMalloc(&a32.p, ab));
        CU(cudaMemset(a16.p, 0, ab));
        CU(cudaMemset(a32.p, 0, ab));
        CU(cudaMalloc(&e16.p, pf_es_floats((int)m, (int)k / 16) * 4));
        CU(cudaMalloc(&s16.p, pf_es_floats((int)m, (int)k / 16) * 4));
        CU(cudaMalloc(&e32.p, pf_es_floats((int)m, (int)k / 32) * 4));
        CU(cudaMalloc(&s32.p, pf_es_floats((int)m, (int)k / 32) * 4));
        CU(cudaMalloc(&derr2.p, 4));
        CU(cudaMemset(derr2.p, 0, 4));
        CU(cudaMemcpy(xa.p, x, (size_t)m * k * 4, cudaMemcpyHostToDevice));
        if (set_kernel_smem_limits()) return -1;
        PfRows P{};
        P.in = (const float *)xa.p;
        P.ld_in = (int)k;
        P.K = (int)k;
        P.tokens = (int)m;
        P.need16 = sub_of(type) == 16;
        P.need32 = sub_of(type) == 32;
        P.a16 = (int8_t *)a16.p;
        P.a32 = (int8_t *)a32.p;
        P.e16 = (float *)e16.p;
        P.s16 = (float *)s16.p;
        P.e32 = (float *)e32.p;
        P.s32 = (float *)s32.p;
        k_pf_rows<<<m, kDecodeThreads>>>(P);
        CU(cudaGetLastError());
        const MvSeg seg = mv_seg(M, (int)rows / 2, PAIR_ADJ, EPI_STORE, (float *)yy.p, ROWS_MANY);
        if (pf_gemm(0, seg, (int)m, 0, (int)rows, P.a16, P.a32, P.e16, P.s16, P.e32, P.s32, nullptr, nullptr,
                    (int *)derr2.p))
            return -1;
        CU(cudaDeviceSynchronize());
        int e = 0;
        CU(cudaMemcpy(&e, derr2.p, 4, cudaMemcpyDeviceToHost));
        if (e) {
            set_error("prefill GEMM reported error flags %d", e);
            return -1;
        }
        CU(cudaMemcpy(y, yy.p, (size_t)m * rows * 4, cudaMemcpyDeviceToHost));
        return 0;
    }
    Phase ph = mv_phase({mv_seg(M, (int)rows / 2, PAIR_ADJ, EPI_STORE, (float *)dy.p, row_class(m))}, (int)k,
                        PRO_QUANT, (const float *)dx.p, nullptr, 0.0f, 0);
    Program prog;
    if (upload_program({ph}, 0, &prog)) return -1;
    dprog.p = prog.d;
    if (set_kernel_smem_limits()) return -1;
    DecodeArgs a{};
    a.prog = prog.d;
    a.nphase = 1;
    a.bar = (unsigned *)dbar.p;
    a.err = (int *)derr.p;
    size_t smem = 0;
    if (decode_geometry((uint32_t)(32 * M.bpb), prog, a, &smem)) return -1;
    for (uint32_t f = 0; f < m; f++) {
        CU(cudaMemcpy(dx.p, x + (size_t)f * k, (size_t)k * 4, cudaMemcpyHostToDevice));
        if (launch_decode(sms, 0, a, smem)) return -1;
        CU(cudaDeviceSynchronize());
        int e = 0;
        CU(cudaMemcpy(&e, derr.p, 4, cudaMemcpyDeviceToHost));
        if (e) {
            set_error("decode kernel reported error flags %d", e);
            return -1;
        }
        CU(cudaMemcpy(y + (size_t)f * rows, dy.p, (size_t)rows * 4, cudaMemcpyDeviceToHost));
    }
    return 0;
}

extern "C" int cxm_debug_matvec(int type, const uint8_t *w, uint32_t rows, uint32_t k, const float *x, float *y) {
    return cxm_debug_matmul(type, w, rows, k, x, 1, y);
}

extern "C" int cxm_debug_attention(const float *q, const float *k, const float *v, uint32_t total, uint32_t heads,
                                   uint32_t heads_kv, uint32_t hd, float *out) {
    if (need_device()) return -1;
    if (!q || !k || !v || !out || total == 0 || heads_kv == 0 || heads % heads_kv || hd % 16 || hd == 0 ||
        hd > (uint32_t)(kKRow - 4) || out_smem(total) > 200 * 1024) {
        set_error("bad attention arguments");
        return -1;
    }
    const size_t kvd = (size_t)heads_kv * hd;
    DevBuf dq, dk, dv, dout, dlen, derr, dsc;
    CU(cudaMalloc(&dsc.p, (size_t)heads * ((total + 3) & ~3u) * 4));
    CU(cudaMalloc(&dq.p, (size_t)heads * hd * 4));
    CU(cudaMalloc(&dk.p, total * kvd * 4));
    CU(cudaMalloc(&dv.p, total * kvd * 4));
    CU(cudaMalloc(&dout.p, (size_t)heads * hd * 4));
    CU(cudaMalloc(&dlen.p, 4));
    CU(cudaMalloc(&derr.p, 4));
    CU(cudaMemcpy(dq.p, q, (size_t)heads * hd * 4, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dk.p, k, total * kvd * 4, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dv.p, v, total * kvd * 4, cudaMemcpyHostToDevice));
    CU(cudaMemset(derr.p, 0, 4));
    int len = (int)total - 1;
    CU(cudaMemcpy(dlen.p, &len, 4, cudaMemcpyHostToDevice));
    AttnParams a{};
    a.q = (const float *)dq.p;
    a.k = (const float *)dk.p;
    a.v = (const float *)dv.p;
    a.out = (float *)dout.p;
    a.d_len = (const int *)dlen.p;
    a.H = (int)heads;
    a.KV = (int)heads_kv;
    a.hd = (int)hd;
    a.max_pos = (int)total;
    a.score_stride = (int)((total + 3) & ~3u);
    a.scores = (float *)dsc.p;
    a.scale = 1.0f / sqrtf((float)hd);
    a.err = (int *)derr.p;
    if (set_kernel_smem_limits()) return -1;
    if (launch_attention_on(0, a)) return -1;
    CU(cudaDeviceSynchronize());
    int e = 0;
    CU(cudaMemcpy(&e, derr.p, 4, cudaMemcpyDeviceToHost));
    if (e) {
        set_error("attention kernels reported error flags %d", e);
        return -1;
    }
    CU(cudaMemcpy(out, dout.p, (size_t)heads * hd * 4, cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int cxm_debug_expf(const float *x, float *y, uint64_t n) {
    if (need_device()) return -1;
    if (!x || !y || n == 0) {
        set_error("bad arguments");
        return -1;
    }
    DevBuf dx, dy;
    CU(cudaMalloc(&dx.p, n * 4));
    CU(cudaMalloc(&dy.p, n * 4));
    CU(cudaMemcpy(dx.p, x, n * 4, cudaMemcpyHostToDevice));
    k_expf<<<1024, 256>>>((const float *)dx.p, (float *)dy.p, (int)n);
    CU(cudaGetLastError());
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(y, dy.p, n * 4, cudaMemcpyDeviceToHost));
    return 0;
}

// the running sums, then the total again without them (the scan's other
// path: passes without an event skip their walk); *same = 0 when they differ
__global__ void __launch_bounds__(kSampThreads, 1) k_seq_sums(const float *x, float *y, int n, int *same) {
    __shared__ ScanShared sh;
    __shared__ float total;
    exact_scan(x, n, y, SCAN_ALL, 0.0f, sh, nullptr);
    exact_scan(x, n, nullptr, SCAN_ALL, 0.0f, sh, &total);
    if (threadIdx.x == 0) *same = __float_as_uint(total) == __float_as_uint(__ldcg(y + n - 1));
}

extern "C" int cxm_debug_seq_sums(const float *x, float *y, uint64_t n) {
    if (need_device()) return -1;
    if (!x || !y || n == 0 || n > (1ull << 30)) {
        set_error("bad arguments");
        return -1;
    }
    DevBuf dx, dy, ds;
    CU(cudaMalloc(&dx.p, n * 4));
    CU(cudaMalloc(&dy.p, n * 4));
    CU(cudaMalloc(&ds.p, 4));
    CU(cudaMemcpy(dx.p, x, n * 4, cudaMemcpyHostToDevice));
    k_seq_sums<<<1, kSampThreads>>>((const float *)dx.p, (float *)dy.p, (int)n, (int *)ds.p);
    CU(cudaGetLastError());
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(y, dy.p, n * 4, cudaMemcpyDeviceToHost));
    int same = 0;
    CU(cudaMemcpy(&same, ds.p, 4, cudaMemcpyDeviceToHost));
    if (!same) {
        set_error("the total taken without the running sums differs from the last running sum");
        return -1;
    }
    return 0;
}

// ── measurement hooks ──

// the whole step is one launch of the decode kernel
extern "C" int cxm_step_launches(const cxm_model *m) { return m ? 1 : 0; }

extern "C" int cxm_bench_decode(cxm_model *m, cxm_cache *c, uint32_t steps, float *ms_total) {
    return cxm_bench_decode_sampled(m, c, nullptr, steps, ms_total);
}

extern "C" int cxm_bench_decode_sampled(cxm_model *m, cxm_cache *c, cxm_sampler *s, uint32_t steps, float *ms_total) {
    if (!m || !c || !ms_total || c->m != m) {
        set_error("bad arguments");
        return -1;
    }
    const bool sampled = s && s->temperature > 0.0f;
    if (c->len == 0 || (uint64_t)c->len + steps + 1 > std::min<uint64_t>(c->max_tokens, (uint64_t)m->cfg.ctx)) {
        set_error("cache needs a token to start from and room for %u more", steps);
        return -1;
    }
    CU(cudaSetDevice(m->device));
    // the step reads the token at toks[len]; start from the last cached one
    CU(cudaMemsetAsync(c->d_stop, 0, 4, m->stream));
    if (set_len(c, c->len - 1)) return -1;
    if (sampled && set_sampler(m, s)) return -1;
    cudaGraphExec_t g;
    if (get_graph(m, c, sampled ? STEP_SAMPLE : STEP_GREEDY, ROWS_FEW, &g)) return -1;
    EventPair ev;
    CU(cudaEventCreate(&ev.a));
    CU(cudaEventCreate(&ev.b));
    CU(cudaEventRecord(ev.a, m->stream));
    for (uint32_t i = 0; i < steps; i++) CU(cudaGraphLaunch(g, m->stream));
    CU(cudaEventRecord(ev.b, m->stream));
    CU(cudaEventSynchronize(ev.b));
    CU(cudaEventElapsedTime(ms_total, ev.a, ev.b));
    if (check_err(m)) return -1;
    if (sampled) {  // one draw per step
        uint64_t st = s->state;
        for (uint32_t i = 0; i < steps; i++) {
            uint64_t x = st;
            x ^= x >> 12;
            x ^= x << 25;
            x ^= x >> 27;
            st = x;
        }
        s->state = st;
    }
    return set_len(c, c->len + steps);
}

extern "C" int cxm_bench_sample(cxm_model *m, cxm_sampler *s, uint32_t reps, float *ms_total, uint64_t *phase_ns,
                                uint32_t nphase) {
    if (!m || !s || !ms_total || reps == 0 || !(s->temperature > 0.0f) || (phase_ns && nphase > (uint32_t)kSampStamps)) {
        set_error("bad arguments");
        return -1;
    }
    CU(cudaSetDevice(m->device));
    if (set_sampler(m, s)) return -1;
    DevBuf st;
    CU(cudaMalloc(&st.p, kSampStamps * sizeof(unsigned long long)));
    CU(cudaMemsetAsync(st.p, 0, kSampStamps * sizeof(unsigned long long), m->stream));
    EventPair ev;
    CU(cudaEventCreate(&ev.a));
    CU(cudaEventCreate(&ev.b));
    CU(cudaEventRecord(ev.a, m->stream));
    for (uint32_t i = 0; i < reps; i++)
        if (launch_sample(m, nullptr, nullptr, m->samp_tok, nullptr,
                          i + 1 == reps && phase_ns ? (unsigned long long *)st.p : nullptr))
            return -1;
    CU(cudaEventRecord(ev.b, m->stream));
    CU(cudaEventSynchronize(ev.b));
    CU(cudaEventElapsedTime(ms_total, ev.a, ev.b));
    if (check_err(m)) return -1;
    if (phase_ns) {
        unsigned long long h[kSampStamps];
        CU(cudaMemcpy(h, st.p, sizeof(h), cudaMemcpyDeviceToHost));
        for (uint32_t k = 0; k < nphase; k++) phase_ns[k] = (k == 12 || k == 13) ? h[k] : h[k] ? h[k] - h[0] : 0;
    }
    for (uint32_t i = 0; i < reps; i++) {  // one draw per run
        uint64_t x = s->state;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        s->state = x;
    }
    return 0;
}

extern "C" int cxm_arm_gemm_stamps(int launch) {
    if (launch < 0) {
        g_pf_stamp_target = -1;
        return 0;
    }
    if (!g_pf_stamps) CU(cudaMalloc(&g_pf_stamps, kPfStampSlots * sizeof(unsigned long long)));
    CU(cudaMemset(g_pf_stamps, 0, kPfStampSlots * sizeof(unsigned long long)));
    g_pf_stamp_target = launch;
    g_pf_calls = 0;
    return 0;
}

extern "C" int cxm_read_gemm_stamps(uint64_t *out, uint32_t n) {
    if (!out || n > (uint32_t)kPfStampSlots || !g_pf_stamps) {
        set_error("bad arguments (arm first)");
        return -1;
    }
    unsigned long long h[kPfStampSlots];
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(h, g_pf_stamps, sizeof(h), cudaMemcpyDeviceToHost));
    for (uint32_t k = 0; k < n; k++) out[k] = h[k] && h[0] ? h[k] - h[0] : 0;
    g_pf_stamp_target = -1;
    return 0;
}

extern "C" int cxm_bench_matvec(cxm_model *m, uint32_t reps, float *ms_per_launch, uint64_t *bytes_per_launch) {
    if (!m || !ms_per_launch || !bytes_per_launch || reps == 0 || m->layers.empty()) {
        set_error("bad arguments");
        return -1;
    }
    CU(cudaSetDevice(m->device));
    const cxm_config &cfg = m->cfg;
    // `reps` gate|up phases of the decode kernel in one launch, cycling over
    // the layers so every phase streams its own weights from HBM, each
    // behind a grid barrier as in the step
    std::vector<Phase> ph;
    for (uint32_t i = 0; i < reps; i++) {
        const Layer &L = m->layers[i % m->layers.size()];
        ph.push_back(mv_phase({mv_seg(L.gu, cfg.ffn, PAIR_TWO, EPI_SWIGLU, m->h)}, cfg.dim, PRO_NORM, m->x, L.ffn_norm,
                              cfg.eps, i > 0));
    }
    Program prog;
    if (upload_program(ph, 0, &prog)) return -1;
    struct Free {
        Phase *p;
        ~Free() { cudaFree(p); }
    } f{prog.d};
    DecodeArgs a = base_args(m);
    a.prog = prog.d;
    a.nphase = prog.n;
    size_t smem = 0;
    if (decode_geometry(m->slot_bytes, prog, a, &smem)) return -1;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float ms = 0;
    if (launch_decode(m->sms, m->stream, a, smem)) return -1;  // warm-up
    cudaError_t re = cudaEventCreate(&e0);
    if (re == cudaSuccess) re = cudaEventCreate(&e1);
    if (re == cudaSuccess) re = cudaEventRecord(e0, m->stream);
    int rc = re == cudaSuccess ? launch_decode(m->sms, m->stream, a, smem) : 0;
    if (re == cudaSuccess && !rc) re = cudaEventRecord(e1, m->stream);
    if (re == cudaSuccess && !rc) re = cudaEventSynchronize(e1);
    if (re == cudaSuccess && !rc) re = cudaEventElapsedTime(&ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (rc) return -1;
    if (re != cudaSuccess) {
        set_error("matvec timing failed: %s", cudaGetErrorString(re));
        return -1;
    }
    *ms_per_launch = ms / (float)reps;
    const Layer &L = m->layers[0];
    *bytes_per_launch = (uint64_t)L.gu.rows * (uint64_t)L.gu.nblk * (uint64_t)L.gu.bpb;  // 2 x ffn rows
    return check_err(m);
}

// ── attention without allocation ─────────────────────────────────────────
// cxm_attention_noalloc is cxm_debug_attention's kernels on caller-owned
// device buffers, for callers that cannot allocate device memory: a serving
// process that has already given the whole device to weights and KV caches
// (a cudaMalloc there fails), and latency-sensitive callers that cannot take
// the device-wide synchronisation cudaMalloc/cudaFree may imply. It calls no
// cudaMalloc, cudaFree or allocating library routine. Its scratch (the score
// rows, the position word and the error word) is the one file-scope device
// array below, shared by every call on a device: calls whose GPU work
// overlaps (two host threads, or two streams) race on it.
constexpr uint32_t kNoAllocScoreCap = 1u << 16;            // score floats: 256 KiB
constexpr uint32_t kNoAllocFloats = kNoAllocScoreCap + 64;  // + a 256-byte tail: position, error
static __device__ __align__(256) float g_attn_scratch[kNoAllocFloats];

__global__ void k_noalloc_words(int *len, int *err, int value) {
    *len = value;
    *err = 0;
}

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float *g_noalloc_base[kNoAllocMaxDevices];

// Address of the scratch array on the current device, looked up once per
// device with that device current; the same first call sets the attention
// kernels' shared-memory limits on that device.
int noalloc_scratch(float **out) {
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        set_error("device ordinal %d out of range", dev);
        return -1;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
        if (set_kernel_smem_limits()) return -1;
        float *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress((void **)&p, g_attn_scratch);
        if (e != cudaSuccess || !p) {
            set_error("cudaGetSymbolAddress of the attention scratch failed: %s", cudaGetErrorString(e));
            return -1;
        }
        g_noalloc_base[dev] = p;
    }
    *out = g_noalloc_base[dev];
    return 0;
}
}  // namespace

extern "C" int cxm_attention_noalloc(const float *q, const float *k, const float *v, uint32_t total,
                                     uint32_t heads, uint32_t heads_kv, uint32_t hd, float *out, void *stream) {
    if (need_device()) return -1;
    if (!q || !k || !v || !out || total == 0 || heads_kv == 0 || heads % heads_kv || hd % 16 || hd == 0 ||
        hd > (uint32_t)(kKRow - 4) || out_smem(total) > 200 * 1024) {
        set_error("bad attention arguments");
        return -1;
    }
    const uint64_t stride = ((uint64_t)total + 3) & ~(uint64_t)3;
    if ((uint64_t)heads * stride > kNoAllocScoreCap) {
        set_error("attention scratch holds %u scores (heads x positions rounded up to 4); this call needs %llu",
                  kNoAllocScoreCap, (unsigned long long)((uint64_t)heads * stride));
        return -1;
    }
    float *base = nullptr;
    if (noalloc_scratch(&base)) return -1;
    int *len = (int *)(base + kNoAllocScoreCap), *err = len + 1;
    const cudaStream_t st = (cudaStream_t)stream;
    k_noalloc_words<<<1, 1, 0, st>>>(len, err, (int)total - 1);
    CU(cudaGetLastError());
    AttnParams a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.d_len = len;
    a.H = (int)heads;
    a.KV = (int)heads_kv;
    a.hd = (int)hd;
    a.max_pos = (int)total;
    a.score_stride = (int)stride;
    a.scores = base;
    a.scale = 1.0f / sqrtf((float)hd);
    a.err = err;
    if (launch_attention_on(st, a)) return -1;
    int e = 0;
    CU(cudaMemcpyAsync(&e, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (e) {
        set_error("attention kernels reported error flags %d", e);
        return -1;
    }
    return 0;
}
