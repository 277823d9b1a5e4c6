// GGUF reader (mmap) and the format helpers the rest of the library uses.
// Reader semantics follow src/gguf.rs:274-342 (header) and :413-437 (every
// tensor bounds-checked against the file before it is handed out).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>

#include "cxm_internal.h"

namespace cxm {

static thread_local std::string g_error;

void set_error(const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
}
const char *last_error() { return g_error.c_str(); }

int values_per_block(int t) {
    switch (t) {
    case F32: case F16: return 1;
    case Q4_0: case Q4_1: case Q5_0: case Q5_1: case Q8_0: case Q8_1: return 32;
    case Q2K: case Q3K: case Q4K: case Q5K: case Q6K: case Q8K: return 256;
    default: return 0;
    }
}

int bytes_per_block(int t) {
    switch (t) {
    case F32: return 4;
    case F16: return 2;
    case Q4_0: return 18;
    case Q4_1: return 20;
    case Q5_0: return 22;
    case Q5_1: return 24;
    case Q8_0: return 34;
    case Q8_1: return 36;
    case Q2K: return 84;
    case Q3K: return 110;
    case Q4K: return 144;
    case Q5K: return 176;
    case Q6K: return 210;
    case Q8K: return 292;
    default: return 0;
    }
}

int sub_block(int t) {
    switch (t) {
    case Q8_0: case Q5_0: case Q4K: case Q5K: return 32;
    case Q2K: case Q3K: case Q6K: return 16;
    default: return 0;
    }
}

bool is_kquant(int t) { return t == Q2K || t == Q3K || t == Q4K || t == Q5K || t == Q6K; }

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0 && man == 0) {
        bits = sign;
    } else if (exp == 0) {
        int e = 1;
        while (!(man & 0x400)) {
            man <<= 1;
            e--;
        }
        man &= 0x3FF;
        bits = sign | ((uint32_t)(e - 15 + 127) << 23) | (man << 13);
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t f32_to_f16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    uint32_t mag = bits & 0x7FFFFFFFu;
    if (mag >= 0x7F800000u) return sign | 0x7C00 | ((mag & 0x007FFFFFu) ? 0x0200 : 0);
    int e = (int)(mag >> 23) - 127;
    if (e > 15) return sign | 0x7C00;
    if (e < -14) {
        uint32_t shift = (uint32_t)(-14 - e);
        if (shift > 24) return sign;
        uint32_t m = (mag & 0x007FFFFFu) | 0x00800000u;
        uint32_t val = m >> (shift + 13), rest = m & ((1u << (shift + 13)) - 1), half = 1u << (shift + 12);
        uint32_t up = (rest > half || (rest == half && (val & 1))) ? 1 : 0;
        return sign | (uint16_t)(val + up);
    }
    uint32_t m = mag & 0x007FFFFFu;
    uint32_t val = ((uint32_t)(e + 15) << 10) | (m >> 13), rest = m & 0x1FFF;
    uint32_t up = (rest > 0x1000 || (rest == 0x1000 && (val & 1))) ? 1 : 0;
    return sign | (uint16_t)(val + up);
}

// ── GGUF reader ──

namespace {
struct Reader {
    const uint8_t *p, *end;
    bool bad = false;
    uint64_t n(int bytes) {
        if (p + bytes > end) {
            bad = true;
            return 0;
        }
        uint64_t v = 0;
        for (int i = 0; i < bytes; i++) v |= (uint64_t)p[i] << (8 * i);
        p += bytes;
        return v;
    }
    std::string str() {
        uint64_t len = n(8);
        if (bad || len > (uint64_t)(end - p)) {
            bad = true;
            return {};
        }
        std::string s((const char *)p, (size_t)len);
        p += len;
        return s;
    }
    void value(uint32_t type, MetaValue &m, int depth = 0) {
        switch (type) {
        case 0: m.kind = 1; m.i = n(1); break;
        case 1: m.kind = 1; m.i = (uint64_t)(int64_t)(int8_t)n(1); break;
        case 2: m.kind = 1; m.i = n(2); break;
        case 3: m.kind = 1; m.i = (uint64_t)(int64_t)(int16_t)n(2); break;
        case 4: m.kind = 1; m.i = n(4); break;
        case 5: m.kind = 1; m.i = (uint64_t)(int64_t)(int32_t)n(4); break;
        case 6: {
            uint32_t u = (uint32_t)n(4);
            float f;
            memcpy(&f, &u, 4);
            m.kind = 2;
            m.f = f;
            break;
        }
        case 7: n(1); m.kind = 0; break;
        case 8: m.kind = 3; m.s = str(); break;
        case 9: {
            uint32_t it = (uint32_t)n(4);
            uint64_t cnt = n(8);
            if (depth > 4) {
                bad = true;
                return;
            }
            MetaValue tmp;
            for (uint64_t i = 0; i < cnt && !bad; i++) value(it, tmp, depth + 1);
            m.kind = 0;
            break;
        }
        case 10: m.kind = 1; m.i = n(8); break;
        case 11: m.kind = 1; m.i = n(8); break;
        case 12: {
            uint64_t b = n(8);
            memcpy(&m.f, &b, 8);
            m.kind = 2;
            break;
        }
        default: bad = true;
        }
    }
};
}  // namespace

Gguf::~Gguf() {
    if (map_) munmap(map_, size_);
}

bool Gguf::open(const std::string &path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        set_error("cannot open %s: %s", path.c_str(), strerror(errno));
        return false;
    }
    struct stat st;
    fstat(fd, &st);
    size_ = (size_t)st.st_size;
    void *m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        set_error("cannot map %s", path.c_str());
        return false;
    }
    map_ = (uint8_t *)m;
    Reader r{map_, map_ + size_};
    if (size_ < 4 || memcmp(map_, "GGUF", 4) != 0) {
        set_error("%s does not start with GGUF", path.c_str());
        return false;
    }
    r.p += 4;
    uint32_t version = (uint32_t)r.n(4);
    if (version != 2 && version != 3) {
        set_error("GGUF version %u: only 2 and 3 are read", version);
        return false;
    }
    uint64_t nt = r.n(8), nm = r.n(8);
    if (nt > (1u << 20) || nm > (1u << 20)) {
        set_error("GGUF header counts out of range");
        return false;
    }
    for (uint64_t i = 0; i < nm && !r.bad; i++) {
        std::string key = r.str();
        uint32_t ty = (uint32_t)r.n(4);
        MetaValue v;
        r.value(ty, v);
        meta_.emplace_back(key, v);
    }
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        TensorInfo t;
        t.name = r.str();
        uint32_t nd = (uint32_t)r.n(4);
        if (nd > 4) {
            set_error("%s: %u dimensions, the format allows 4", t.name.c_str(), nd);
            return false;
        }
        for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.n(8));
        t.type = (int)r.n(4);
        t.offset = r.n(8);
        int vpb = values_per_block(t.type);
        if (!vpb) {
            set_error("%s: unknown tensor type %d", t.name.c_str(), t.type);
            return false;
        }
        t.nbytes = (size_t)(t.elements() / (uint64_t)vpb) * (size_t)bytes_per_block(t.type);
        tensors_.push_back(std::move(t));
    }
    if (r.bad) {
        set_error("truncated GGUF header");
        return false;
    }
    uint64_t align = 32, a;
    if (meta_int("general.alignment", &a) && a > 0) align = a;
    uint64_t pos = (uint64_t)(r.p - map_);
    data_start_ = (pos + align - 1) / align * align;
    for (auto &t : tensors_) {
        uint64_t from = data_start_ + t.offset;
        if (from < data_start_ || from + t.nbytes < from || from + t.nbytes > size_) {
            set_error("%s: asks for bytes up to %llu and the file has %zu", t.name.c_str(),
                      (unsigned long long)(from + t.nbytes), size_);
            return false;
        }
    }
    return true;
}

const TensorInfo *Gguf::tensor(const std::string &name) const {
    for (auto &t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

bool Gguf::meta_int(const std::string &key, uint64_t *v) const {
    for (auto &kv : meta_)
        if (kv.first == key && kv.second.kind == 1) {
            *v = kv.second.i;
            return true;
        }
    return false;
}

bool Gguf::meta_float(const std::string &key, double *v) const {
    for (auto &kv : meta_) {
        if (kv.first != key) continue;
        if (kv.second.kind == 2) {
            *v = kv.second.f;
            return true;
        }
        if (kv.second.kind == 1) {
            *v = (double)kv.second.i;
            return true;
        }
    }
    return false;
}

// ── threads ──

int host_threads() {
    unsigned n = std::thread::hardware_concurrency();
    return n ? (int)n : 1;
}

void parallel_for(size_t n, size_t chunk, int threads, void (*fn)(void *, size_t, size_t), void *ctx) {
    if (threads <= 0) threads = host_threads();
    size_t tasks = (n + chunk - 1) / chunk;
    if (threads <= 1 || tasks <= 1) {
        fn(ctx, 0, n);
        return;
    }
    if ((size_t)threads > tasks) threads = (int)tasks;
    std::atomic<size_t> next{0};
    auto work = [&]() {
        for (;;) {
            size_t b = next.fetch_add(chunk);
            if (b >= n) break;
            fn(ctx, b, b + chunk < n ? b + chunk : n);
        }
    };
    std::vector<std::thread> th;
    for (int i = 1; i < threads; i++) th.emplace_back(work);
    work();
    for (auto &t : th) t.join();
}

}  // namespace cxm
