// Internal declarations shared by the host-side C++ and the CUDA sources.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace cxm {

// GGML tensor types (numbers fixed by the file format; src/gguf.rs:39-54).
enum Ggml : int {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
    Q2K = 10, Q3K = 11, Q4K = 12, Q5K = 13, Q6K = 14, Q8K = 15
};

int values_per_block(int type);     // src/gguf.rs:83-90
int bytes_per_block(int type);      // src/gguf.rs:93-111
int sub_block(int type);            // src/quant.rs:213-219 (0 = no i8 path)
bool is_kquant(int type);

float f16_to_f32(uint16_t h);       // src/quant.rs:38-60
uint16_t f32_to_f16(float x);       // src/quant.rs:691-731

void set_error(const char *fmt, ...);
const char *last_error();

// ── GGUF (src/gguf.rs:274-437) ──
struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    int type = 0;
    uint64_t offset = 0;
    size_t nbytes = 0;
    uint64_t elements() const {
        uint64_t e = 1;
        for (auto d : dims) e *= d;
        return e;
    }
};

struct MetaValue {
    int kind = 0;  // 0 other, 1 integer, 2 float, 3 string
    uint64_t i = 0;
    double f = 0;
    std::string s;
};

class Gguf {
  public:
    ~Gguf();
    bool open(const std::string &path);
    const TensorInfo *tensor(const std::string &name) const;
    bool meta_int(const std::string &key, uint64_t *v) const;     // Valor::entero
    bool meta_float(const std::string &key, double *v) const;     // Valor::decimal
    const uint8_t *data(const TensorInfo &t) const { return map_ + data_start_ + t.offset; }
    const std::vector<TensorInfo> &tensors() const { return tensors_; }

  private:
    uint8_t *map_ = nullptr;
    size_t size_ = 0;
    uint64_t data_start_ = 0;
    std::vector<TensorInfo> tensors_;
    std::vector<std::pair<std::string, MetaValue>> meta_;
};

// ── k-quant writers (src/quant_kquants.rs; Q6_K is this library's own) ──
// Appends the blocks of n values (multiple of 256) to out. Returns false for
// unsupported types.
bool quantize_blocks(int type, const float *x, size_t n, std::vector<uint8_t> &out);

// ── seeded RNG (src/daiss.rs:317-379) ──
struct Azar {
    uint64_t state;
    explicit Azar(uint64_t s) : state(s == 0 ? 0x9E3779B97F4A7C15ull : s) {}
    uint64_t next() {
        uint64_t x = state;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        state = x;
        return x * 0x2545F4914F6CDD1Dull;
    }
    float uniform_open0() {  // (0, 1]
        uint64_t bits = next() >> 40;
        return ((float)bits + 1.0f) / 16777216.0f;
    }
    void normals(float sigma, float *a, float *b);
};
uint64_t seed_of(uint64_t model_seed, const std::string &name, uint64_t row);

// parallel for over [0, n) in chunks, on std::threads
void parallel_for(size_t n, size_t chunk, int threads, void (*fn)(void *, size_t, size_t), void *ctx);
int host_threads();

}  // namespace cxm
