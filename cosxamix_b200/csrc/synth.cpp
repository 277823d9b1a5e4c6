// Seeded synthetic models: the k-quant writers, the row RNG and a streaming
// GGUF writer.
//
// The Q2_K/Q3_K/Q4_K/Q5_K writers restate the algorithm of
// src/quant_kquants.rs (weighted least-squares search of each sub-block's
// scale and minimum, then 4- or 6-bit block scales). Float expressions keep
// the reference's evaluation order and this file is compiled without FMA
// contraction, so the bytes equal what the reference's writer produces for
// the same input. The reference has no Q6_K writer (src/quant.rs:744-803
// stops at Q5_K); the Q6_K writer here is this library's own, written from
// the layout the reference READS (src/quant.rs:647-679).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "../../include/cxm.h"
#include "cxm_internal.h"

namespace cxm {

static inline int rnd(float x) { return (int)roundf(x); }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
static const float kEps = 1e-15f;  // src/quant_kquants.rs:19

// Signed levels in [-nmax, nmax-1] with the x²-weighted best scale, then
// shifted to [0, 2 nmax). src/quant_kquants.rs:29-84.
static float fit_signed16(const float *x, int nmax, int *l) {
    float mayor = 0.0f, amax = 0.0f;
    for (int i = 0; i < 16; i++)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mayor = x[i];
        }
    if (amax < kEps) {
        for (int i = 0; i < 16; i++) l[i] = 0;
        return 0.0f;
    }
    float iscale = -(float)nmax / mayor;
    float sumlx = 0.0f, suml2 = 0.0f;
    for (int i = 0; i < 16; i++) {
        l[i] = clampi(rnd(iscale * x[i]), -nmax, nmax - 1);
        float w = x[i] * x[i];
        sumlx += w * x[i] * (float)l[i];
        suml2 += w * (float)(l[i] * l[i]);
    }
    for (int it = 0; it < 5; it++) {
        int changes = 0;
        for (int i = 0; i < 16; i++) {
            float w = x[i] * x[i];
            float cur = (float)l[i];
            float slx = sumlx - w * x[i] * cur;
            if (slx > 0.0f) {
                float sl2 = suml2 - w * cur * cur;
                int nw = clampi(rnd(x[i] * sl2 / slx), -nmax, nmax - 1);
                if (nw != l[i]) {
                    slx += w * x[i] * (float)nw;
                    sl2 += w * (float)(nw * nw);
                    if (sl2 > 0.0f && slx * slx * suml2 > sumlx * sumlx * sl2) {
                        l[i] = nw;
                        sumlx = slx;
                        suml2 = sl2;
                        changes++;
                    }
                }
            }
        }
        if (changes == 0) break;
    }
    for (int i = 0; i < 16; i++) l[i] += nmax;
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

struct Search {
    int nmax;
    float from, step;
    int steps;
    bool absolute;
};

// x ≈ scale·l - min with l in [0, nmax]: scan scales around the obvious one,
// least squares for each. Returns (scale, -min). src/quant_kquants.rs:99-157.
static void fit_affine(const float *x, const float *w, int n, int *l, int *aux, const Search &b, float *out_scale,
                       float *out_min) {
    float mn = x[0], mx = x[0], sum_w = w[0], sum_x = w[0] * x[0];
    for (int i = 1; i < n; i++) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
        sum_w += w[i];
        sum_x += w[i] * x[i];
    }
    if (mn > 0.0f) mn = 0.0f;
    if (mn == mx) {
        for (int i = 0; i < n; i++) l[i] = 0;
        *out_scale = 0.0f;
        *out_min = -mn;
        return;
    }
    auto err = [&](float d) { return b.absolute ? fabsf(d) : d * d; };
    float iscale = (float)b.nmax / (mx - mn);
    float scale = 1.0f / iscale;
    float best = 0.0f;
    for (int i = 0; i < n; i++) {
        l[i] = clampi(rnd(iscale * (x[i] - mn)), 0, b.nmax);
        best += w[i] * err(scale * (float)l[i] + mn - x[i]);
    }
    for (int k = 0; k <= b.steps; k++) {
        iscale = (b.from + b.step * (float)k + (float)b.nmax) / (mx - mn);
        float sl = 0.0f, sl2 = 0.0f, sxl = 0.0f;
        for (int i = 0; i < n; i++) {
            aux[i] = clampi(rnd(iscale * (x[i] - mn)), 0, b.nmax);
            float lf = (float)aux[i];
            float wl = w[i] * lf;
            sl += wl;
            sl2 += wl * lf;
            sxl += wl * x[i];
        }
        float d = sum_w * sl2 - sl * sl;
        if (d > 0.0f) {
            float this_scale = (sum_w * sxl - sum_x * sl) / d;
            float this_min = (sl2 * sum_x - sl * sxl) / d;
            if (this_min > 0.0f) {
                this_min = 0.0f;
                this_scale = sxl / sl2;
            }
            float e = 0.0f;
            for (int i = 0; i < n; i++) e += w[i] * err(this_scale * (float)aux[i] + this_min - x[i]);
            if (e < best) {
                for (int i = 0; i < n; i++) l[i] = aux[i];
                best = e;
                scale = this_scale;
                mn = this_min;
            }
        }
    }
    *out_scale = scale;
    *out_min = -mn;
}

static inline void put16(std::vector<uint8_t> &o, uint16_t v) {
    o.push_back((uint8_t)(v & 255));
    o.push_back((uint8_t)(v >> 8));
}

// Q3_K block of 256 values, 110 bytes. src/quant_kquants.rs:160-228.
static void block_q3k(const float *x, std::vector<uint8_t> &out) {
    int l[16][16];
    float sc[16];
    float mayor = 0.0f, amax = 0.0f;
    for (int j = 0; j < 16; j++) {
        sc[j] = fit_signed16(x + 16 * j, 4, l[j]);
        if (fabsf(sc[j]) > amax) {
            amax = fabsf(sc[j]);
            mayor = sc[j];
        }
    }
    uint8_t hmask[32] = {0}, qs[64] = {0}, packed[12] = {0};
    uint16_t dst;
    if (amax < kEps) {
        dst = 0;
        for (auto &row : l)
            for (int &v : row) v = 4;
    } else {
        float iscale = -32.0f / mayor;
        dst = f32_to_f16(1.0f / iscale);
        float d = f16_to_f32(dst);
        for (int j = 0; j < 16; j++) {
            int e = clampi(rnd(iscale * sc[j]), -32, 31);
            float s = d * (float)e;
            if (s != 0.0f) {
                float inv = 1.0f / s;
                for (int i = 0; i < 16; i++) l[j][i] = clampi(rnd(x[16 * j + i] * inv), -4, 3) + 4;
            } else {
                for (int i = 0; i < 16; i++) l[j][i] = 4;
            }
            uint8_t u = (uint8_t)(e + 32);
            if (j < 8)
                packed[j] |= u & 0xF;
            else
                packed[j - 8] |= (uint8_t)((u & 0xF) << 4);
            packed[8 + j % 4] |= (uint8_t)((u >> 4) << (2 * (j / 4)));
        }
    }
    for (int idx = 0; idx < 256; idx++) {
        uint8_t v = (uint8_t)l[idx / 16][idx % 16];
        int half = idx / 128, round_ = (idx % 128) / 32, place = idx % 32;
        qs[half * 32 + place] |= (uint8_t)((v & 3) << (round_ * 2));
        if (v & 4) hmask[place] |= (uint8_t)(1 << (half * 4 + round_));
    }
    out.insert(out.end(), hmask, hmask + 32);
    out.insert(out.end(), qs, qs + 64);
    out.insert(out.end(), packed, packed + 12);
    put16(out, dst);
}

// Q2_K block of 256 values, 84 bytes. src/quant_kquants.rs:231-291.
static void block_q2k(const float *x, std::vector<uint8_t> &out) {
    int l[16][16], aux[16];
    float w[16], sc[16], mins[16], max_sc = 0.0f, max_min = 0.0f;
    const Search b{3, -0.5f, 0.1f, 15, true};
    for (int j = 0; j < 16; j++) {
        for (int i = 0; i < 16; i++) w[i] = fabsf(x[16 * j + i]);
        fit_affine(x + 16 * j, w, 16, l[j], aux, b, &sc[j], &mins[j]);
        max_sc = fmaxf(max_sc, sc[j]);
        max_min = fmaxf(max_min, mins[j]);
    }
    float inv_sc = max_sc > 0.0f ? 15.0f / max_sc : 0.0f;
    float inv_min = max_min > 0.0f ? 15.0f / max_min : 0.0f;
    uint16_t dst = f32_to_f16(max_sc > 0.0f ? 1.0f / inv_sc : 0.0f);
    uint16_t mst = f32_to_f16(max_min > 0.0f ? 1.0f / inv_min : 0.0f);
    float d = f16_to_f32(dst), dm = f16_to_f32(mst);
    uint8_t packed[16];
    for (int j = 0; j < 16; j++) {
        int le = clampi(rnd(inv_sc * sc[j]), 0, 15), lm = clampi(rnd(inv_min * mins[j]), 0, 15);
        packed[j] = (uint8_t)(le | (lm << 4));
        float dl = d * (float)le, ml = dm * (float)lm;
        for (int i = 0; i < 16; i++) l[j][i] = dl > 0.0f ? clampi(rnd((x[16 * j + i] + ml) / dl), 0, 3) : 0;
    }
    uint8_t qs[64] = {0};
    for (int idx = 0; idx < 256; idx++) {
        int half = idx / 128, round_ = (idx % 128) / 32;
        qs[half * 32 + idx % 32] |= (uint8_t)(l[idx / 16][idx % 16] << (round_ * 2));
    }
    out.insert(out.end(), packed, packed + 16);
    out.insert(out.end(), qs, qs + 64);
    put16(out, dst);
    put16(out, mst);
}

// Shared by Q4_K and Q5_K: eight sub-blocks of 32 with 6-bit scale and min.
// src/quant_kquants.rs:295-348.
static void subblocks32(const float *x, const Search &b, uint16_t *dst, uint16_t *mst, uint8_t packed[12],
                        int l[8][32]) {
    int aux[32];
    float w[32], sc[8], mins[8], max_sc = 0.0f, max_min = 0.0f;
    float ss = 0.0f;
    for (int i = 0; i < 256; i++) ss += x[i] * x[i];
    float mean = sqrtf(ss / 256.0f);
    for (int j = 0; j < 8; j++) {
        for (int i = 0; i < 32; i++) w[i] = mean + fabsf(x[32 * j + i]);
        fit_affine(x + 32 * j, w, 32, l[j], aux, b, &sc[j], &mins[j]);
        max_sc = fmaxf(max_sc, sc[j]);
        max_min = fmaxf(max_min, mins[j]);
    }
    float inv_sc = max_sc > 0.0f ? 63.0f / max_sc : 0.0f;
    float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    *dst = f32_to_f16(max_sc > 0.0f ? 1.0f / inv_sc : 0.0f);
    *mst = f32_to_f16(max_min > 0.0f ? 1.0f / inv_min : 0.0f);
    float d = f16_to_f32(*dst), dm = f16_to_f32(*mst);
    memset(packed, 0, 12);
    for (int j = 0; j < 8; j++) {
        uint8_t le = (uint8_t)clampi(rnd(inv_sc * sc[j]), 0, 63), lm = (uint8_t)clampi(rnd(inv_min * mins[j]), 0, 63);
        if (j < 4) {
            packed[j] |= le;
            packed[j + 4] |= lm;
        } else {
            packed[j + 4] = (uint8_t)((le & 0xF) | ((lm & 0xF) << 4));
            packed[j - 4] |= (uint8_t)((le >> 4) << 6);
            packed[j] |= (uint8_t)((lm >> 4) << 6);
        }
        float dl = d * (float)le, ml = dm * (float)lm;
        for (int i = 0; i < 32; i++) l[j][i] = dl > 0.0f ? clampi(rnd((x[32 * j + i] + ml) / dl), 0, b.nmax) : 0;
    }
}

// Q4_K block, 144 bytes. src/quant_kquants.rs:351-369.
static void block_q4k(const float *x, std::vector<uint8_t> &out) {
    int l[8][32];
    uint16_t d, m;
    uint8_t packed[12];
    subblocks32(x, Search{15, -1.0f, 0.1f, 20, false}, &d, &m, packed, l);
    put16(out, d);
    put16(out, m);
    out.insert(out.end(), packed, packed + 12);
    for (int p = 0; p < 4; p++)
        for (int i = 0; i < 32; i++) out.push_back((uint8_t)(l[2 * p][i] | (l[2 * p + 1][i] << 4)));
}

// Q5_K block, 176 bytes. src/quant_kquants.rs:373-399.
static void block_q5k(const float *x, std::vector<uint8_t> &out) {
    int l[8][32];
    uint16_t d, m;
    uint8_t packed[12];
    subblocks32(x, Search{31, -0.5f, 0.1f, 15, false}, &d, &m, packed, l);
    uint8_t qh[32] = {0};
    for (int p = 0; p < 4; p++)
        for (int i = 0; i < 32; i++) {
            qh[i] |= (uint8_t)((l[2 * p][i] >> 4) << (2 * p));
            qh[i] |= (uint8_t)((l[2 * p + 1][i] >> 4) << (2 * p + 1));
        }
    put16(out, d);
    put16(out, m);
    out.insert(out.end(), packed, packed + 12);
    out.insert(out.end(), qh, qh + 32);
    for (int p = 0; p < 4; p++)
        for (int i = 0; i < 32; i++) out.push_back((uint8_t)((l[2 * p][i] & 0xF) | ((l[2 * p + 1][i] & 0xF) << 4)));
}

// Q6_K block, 210 bytes — this library's own writer. Each 16-value
// sub-block gets its x²-weighted best signed 6-bit scale (levels -32..31, the
// same search as the Q3_K writer with nmax = 32); the sixteen scales are then
// stored as int8 under one f16 `d`, and every value is re-quantized against the
// stored scale. Layout (what src/quant.rs:647-679 reads): ql[128] low nibbles,
// qh[64] high 2-bit pairs, int8 scales[16], f16 d.
static void block_q6k(const float *x, std::vector<uint8_t> &out) {
    int l[16][16];
    float sc[16];
    float mayor = 0.0f, amax = 0.0f;
    for (int j = 0; j < 16; j++) {
        sc[j] = fit_signed16(x + 16 * j, 32, l[j]);
        if (fabsf(sc[j]) > amax) {
            amax = fabsf(sc[j]);
            mayor = sc[j];
        }
    }
    int8_t scales[16] = {0};
    uint16_t dst = 0;
    if (amax < kEps) {
        for (auto &row : l)
            for (int &v : row) v = 32;
    } else {
        float iscale = -128.0f / mayor;
        dst = f32_to_f16(1.0f / iscale);
        float d = f16_to_f32(dst);
        for (int j = 0; j < 16; j++) {
            int e = clampi(rnd(iscale * sc[j]), -128, 127);
            scales[j] = (int8_t)e;
            float s = d * (float)e;
            if (s != 0.0f) {
                float inv = 1.0f / s;
                for (int i = 0; i < 16; i++) l[j][i] = clampi(rnd(x[16 * j + i] * inv), -32, 31) + 32;
            } else {
                for (int i = 0; i < 16; i++) l[j][i] = 32;
            }
        }
    }
    uint8_t ql[128] = {0}, qh[64] = {0};
    for (int idx = 0; idx < 256; idx++) {
        int v = l[idx / 16][idx % 16];
        int half = idx / 128, gi = (idx % 128) / 32, i = idx % 32;
        uint8_t &lo = ql[64 * half + 32 * (gi % 2) + i];
        lo |= (uint8_t)(gi < 2 ? (v & 0xF) : ((v & 0xF) << 4));
        qh[32 * half + i] |= (uint8_t)(((v >> 4) & 3) << (2 * gi));
    }
    out.insert(out.end(), ql, ql + 128);
    out.insert(out.end(), qh, qh + 64);
    for (int j = 0; j < 16; j++) out.push_back((uint8_t)scales[j]);
    put16(out, dst);
}

bool quantize_blocks(int type, const float *x, size_t n, std::vector<uint8_t> &out) {
    if (type == F32) {
        const uint8_t *p = (const uint8_t *)x;
        out.insert(out.end(), p, p + 4 * n);
        return true;
    }
    if (type == F16) {
        for (size_t i = 0; i < n; i++) put16(out, f32_to_f16(x[i]));
        return true;
    }
    if (n % 256) return false;
    void (*fn)(const float *, std::vector<uint8_t> &) = nullptr;
    switch (type) {
    case Q2K: fn = block_q2k; break;
    case Q3K: fn = block_q3k; break;
    case Q4K: fn = block_q4k; break;
    case Q5K: fn = block_q5k; break;
    case Q6K: fn = block_q6k; break;
    default: return false;
    }
    for (size_t b = 0; b < n / 256; b++) fn(x + 256 * b, out);
    return true;
}

// Box-Muller pair, src/daiss.rs:350-356.
void Azar::normals(float sigma, float *a, float *b) {
    float u1 = uniform_open0(), u2 = uniform_open0();
    float r = sigma * sqrtf(-2.0f * logf(u1));
    float ang = 6.28318530717958647692f * u2;
    *a = r * cosf(ang);
    *b = r * sinf(ang);
}

// FNV-1a of the tensor name, mixed with the row and the model seed.
// src/daiss.rs:364-379.
uint64_t seed_of(uint64_t model, const std::string &name, uint64_t row) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (unsigned char c : name) {
        h ^= c;
        h *= 0x00000100000001B3ull;
    }
    h ^= row;
    h *= 0x00000100000001B3ull;
    return h ^ ((model << 17) | (model >> 47));
}

// ── streaming GGUF writer (src/gguf_write.rs:121-224) ──

namespace {

struct Decl {
    std::string name;
    std::vector<uint64_t> dims;  // [inputs, outputs]
    int type;
    size_t bytes() const {
        uint64_t e = 1;
        for (auto d : dims) e *= d;
        return (size_t)(e / (uint64_t)values_per_block(type)) * (size_t)bytes_per_block(type);
    }
};

struct Out {
    FILE *f;
    uint64_t written = 0;
    bool ok = true;
    void raw(const void *p, size_t n) {
        if (n && fwrite(p, 1, n, f) != n) ok = false;
        written += n;
    }
    void u32(uint32_t v) { raw(&v, 4); }
    void u64(uint64_t v) { raw(&v, 8); }
    void str(const std::string &s) {
        u64(s.size());
        raw(s.data(), s.size());
    }
    void pad(uint64_t n) {
        static const uint8_t z[64] = {0};
        while (n) {
            size_t c = n > 64 ? 64 : (size_t)n;
            raw(z, c);
            n -= c;
        }
    }
};

enum Init { NORMAL, ONES, ZEROS };

struct RowJob {
    const Decl *d;
    Init init;
    float sigma;
    uint64_t seed;
    size_t first_row, width, row_bytes;
    uint8_t *dst;
    bool failed;
};

void gen_rows(void *c_, size_t b, size_t e) {
    RowJob *c = (RowJob *)c_;
    std::vector<float> row(c->width);
    std::vector<uint8_t> bytes;
    bytes.reserve(c->row_bytes);
    for (size_t r = b; r < e; r++) {
        size_t f = c->first_row + r;
        if (c->init == ONES) {
            std::fill(row.begin(), row.end(), 1.0f);
        } else if (c->init == ZEROS) {
            std::fill(row.begin(), row.end(), 0.0f);
        } else {
            Azar az(seed_of(c->seed, c->d->name, f));
            size_t i = 0;
            for (; i + 1 < c->width; i += 2) az.normals(c->sigma, &row[i], &row[i + 1]);
            if (i < c->width) {
                float a, bb;
                az.normals(c->sigma, &a, &bb);
                row[i] = a;
            }
        }
        bytes.clear();
        if (!quantize_blocks(c->d->type, row.data(), c->width, bytes) || bytes.size() != c->row_bytes) {
            c->failed = true;
            return;
        }
        memcpy(c->dst + r * c->row_bytes, bytes.data(), c->row_bytes);
    }
}

}  // namespace

static int synth_write(const cxm_synth_spec *s, const char *path) {
    if (!s || !path) {
        set_error("null argument");
        return -1;
    }
    if (s->dim <= 0 || s->n_head <= 0 || s->dim % s->n_head || s->n_head_kv <= 0 || s->n_head % s->n_head_kv ||
        s->vocab <= 0 || s->n_layer <= 0 || s->ffn <= 0 || s->ctx <= 0) {
        set_error("invalid synthetic model shape");
        return -1;
    }
    const int hd = s->dim / s->n_head, kv = s->n_head_kv * hd;
    auto mtype = [&](const std::string &what, int layer) -> int {
        if (s->mix == CXM_MIX_UNIFORM) return s->type;
        if (what == "output") return Q6K;
        if (what == "token_embd") return s->tied ? Q6K : Q4K;
        if ((what == "attn_v" || what == "ffn_down") && layer % 2 == 0) return Q6K;
        return Q4K;
    };
    std::vector<Decl> decls;
    const uint64_t D = (uint64_t)s->dim, KV = (uint64_t)kv, F = (uint64_t)s->ffn, V = (uint64_t)s->vocab;
    decls.push_back({"token_embd.weight", {D, V}, mtype("token_embd", 0)});
    for (int i = 0; i < s->n_layer; i++) {
        std::string p = "blk." + std::to_string(i) + ".";
        decls.push_back({p + "attn_norm.weight", {D}, F32});
        decls.push_back({p + "attn_q.weight", {D, D}, mtype("attn_q", i)});
        decls.push_back({p + "attn_q.bias", {D}, F32});
        decls.push_back({p + "attn_k.weight", {D, KV}, mtype("attn_k", i)});
        decls.push_back({p + "attn_k.bias", {KV}, F32});
        decls.push_back({p + "attn_v.weight", {D, KV}, mtype("attn_v", i)});
        decls.push_back({p + "attn_v.bias", {KV}, F32});
        decls.push_back({p + "attn_output.weight", {D, D}, mtype("attn_output", i)});
        decls.push_back({p + "ffn_norm.weight", {D}, F32});
        decls.push_back({p + "ffn_gate.weight", {D, F}, mtype("ffn_gate", i)});
        decls.push_back({p + "ffn_up.weight", {D, F}, mtype("ffn_up", i)});
        decls.push_back({p + "ffn_down.weight", {F, D}, mtype("ffn_down", i)});
    }
    decls.push_back({"output_norm.weight", {D}, F32});
    if (!s->tied) decls.push_back({"output.weight", {D, V}, mtype("output", 0)});
    for (auto &d : decls) {
        int vpb = values_per_block(d.type);
        if (!vpb || d.dims[0] % (uint64_t)vpb) {
            set_error("%s: first dimension %llu is not a multiple of the %d-value block", d.name.c_str(),
                      (unsigned long long)d.dims[0], vpb);
            return -1;
        }
    }

    std::string tmp = std::string(path) + ".partial";
    Out o{fopen(tmp.c_str(), "wb")};
    if (!o.f) {
        set_error("cannot create %s", tmp.c_str());
        return -1;
    }
    setvbuf(o.f, nullptr, _IOFBF, 1 << 22);
    const uint64_t align = 32;
    // header + metadata (src/daiss.rs:428-448; no eos key unless asked, so
    // generation never stops early)
    struct KV_ {
        std::string k;
        int t;  // 4 u32, 6 f32, 8 str, 10 u64
        uint64_t u;
        float f;
        std::string s;
    };
    std::vector<KV_> meta = {
        {"general.alignment", 4, align, 0, ""},
        {"general.architecture", 8, 0, 0, "qwen2"},
        {"general.name", 8, 0, 0, "cxm-synthetic"},
        {"general.file_type", 4, (uint64_t)(s->mix == CXM_MIX_UNIFORM ? s->type : Q4K), 0, ""},
        {"qwen2.block_count", 4, (uint64_t)s->n_layer, 0, ""},
        {"qwen2.context_length", 4, (uint64_t)s->ctx, 0, ""},
        {"qwen2.embedding_length", 4, (uint64_t)s->dim, 0, ""},
        {"qwen2.feed_forward_length", 4, (uint64_t)s->ffn, 0, ""},
        {"qwen2.attention.head_count", 4, (uint64_t)s->n_head, 0, ""},
        {"qwen2.attention.head_count_kv", 4, (uint64_t)s->n_head_kv, 0, ""},
        {"qwen2.attention.layer_norm_rms_epsilon", 6, 0, s->eps, ""},
        {"qwen2.rope.freq_base", 6, 0, s->rope_base, ""},
        {"cosxamix.seed", 10, s->seed, 0, ""},
    };
    if (s->has_eos) meta.push_back({"tokenizer.ggml.eos_token_id", 4, (uint64_t)s->eos, 0, ""});
    o.raw("GGUF", 4);
    o.u32(3);
    o.u64(decls.size());
    o.u64(meta.size());
    for (auto &m : meta) {
        o.str(m.k);
        o.u32((uint32_t)m.t);
        if (m.t == 4) o.u32((uint32_t)m.u);
        if (m.t == 6) o.raw(&m.f, 4);
        if (m.t == 8) o.str(m.s);
        if (m.t == 10) o.u64(m.u);
    }
    uint64_t off = 0;
    for (auto &d : decls) {
        off = (off + align - 1) / align * align;
        o.str(d.name);
        o.u32((uint32_t)d.dims.size());
        for (auto v : d.dims) o.u64(v);
        o.u32((uint32_t)d.type);
        o.u64(off);
        off += d.bytes();
    }
    uint64_t start = (o.written + align - 1) / align * align;
    o.pad(start - o.written);

    const size_t kBatch = 64u << 20;
    std::vector<uint8_t> buf;
    for (auto &d : decls) {
        uint64_t rel = o.written - start;
        o.pad((rel + align - 1) / align * align - rel);
        size_t width = (size_t)d.dims[0];
        size_t rows = (size_t)(d.bytes() / ((width / values_per_block(d.type)) * bytes_per_block(d.type)));
        size_t rb = width / values_per_block(d.type) * bytes_per_block(d.type);
        Init init = NORMAL;
        if (d.name.size() > 5 && d.name.compare(d.name.size() - 5, 5, ".bias") == 0) init = ZEROS;
        if (d.name.size() > 12 && d.name.compare(d.name.size() - 12, 12, "_norm.weight") == 0) init = ONES;
        size_t per = std::max<size_t>(1, kBatch / rb);
        for (size_t r0 = 0; r0 < rows; r0 += per) {
            size_t n = std::min(per, rows - r0);
            buf.resize(n * rb);
            RowJob job{&d, init, s->sigma, s->seed, r0, width, rb, buf.data(), false};
            parallel_for(n, 16, s->threads, gen_rows, &job);
            if (job.failed) {
                fclose(o.f);
                remove(tmp.c_str());
                set_error("%s: cannot quantize to type %d", d.name.c_str(), d.type);
                return -1;
            }
            o.raw(buf.data(), buf.size());
        }
    }
    bool ok = o.ok && fflush(o.f) == 0;
    ok = (fclose(o.f) == 0) && ok;
    if (!ok || rename(tmp.c_str(), path) != 0) {
        remove(tmp.c_str());
        set_error("cannot write %s", path);
        return -1;
    }
    return 0;
}

}  // namespace cxm

extern "C" int cxm_synth_write(const cxm_synth_spec *spec, const char *path) { return cxm::synth_write(spec, path); }

extern "C" int64_t cxm_quantize(int type, const float *x, uint64_t n, uint8_t *out, uint64_t cap) {
    std::vector<uint8_t> v;
    if (!x || !out || !cxm::quantize_blocks(type, x, (size_t)n, v)) {
        cxm::set_error("cannot quantize %llu values to type %d", (unsigned long long)n, type);
        return -1;
    }
    if (v.size() > cap) {
        cxm::set_error("output buffer of %llu bytes is short of %zu", (unsigned long long)cap, v.size());
        return -1;
    }
    memcpy(out, v.data(), v.size());
    return (int64_t)v.size();
}
