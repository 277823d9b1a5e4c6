/*
 * cxm_oracle.c — CPU restatement of Cosxamix's decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * product (cosxamix_b200/) and the timed CPU baseline of bench.py. It is never
 * linked into, or called by, the product library.
 *
 * Compiled with -ffp-contract=off: the reference is Rust, which never fuses
 * a*b+c into an FMA, and several dequantization checks demand bit equality.
 *
 * Citations are file:line inside the Cosxamix project (Rust, v0.10.0).
 * Parity pin: the dot kernels below are checked against the reference's own
 * C and x86 assembly kernels (kernels/q{2,3,5}k_avx2.c, kernels/q{2,3,4,5}k_avx2_sysv.s)
 * built from their sources by oracle/Makefile, and against the known-answer
 * tests of the reference's unit tests (tests/golden/).
 */
#define _GNU_SOURCE
#include "cxm_oracle.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>
#include <immintrin.h>

/* ───────────────────────── errors ───────────────────────── */

static __thread char g_err[512];
static void set_err(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}
const char *orc_last_error(void) { return g_err; }

/* ───────────────────────── threads ───────────────────────── */

static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n; }



/* Kernel backend of orc_forward (cxm_oracle.h). */
static int g_backend = ORC_BACKEND_SCALAR;
static orc_dot_fn g_dot_kernel[16];
static orc_q4k_acc_fn g_q4k_acc;
void orc_set_backend(int b) { g_backend = b == ORC_BACKEND_X86 ? ORC_BACKEND_X86 : ORC_BACKEND_SCALAR; }
int orc_get_backend(void) { return g_backend; }
int orc_set_dot_kernel(int type, orc_dot_fn f) {
    if (type < 0 || type >= 16) return -1;
    g_dot_kernel[type] = f;
    return 0;
}
void orc_set_q4k_acc_kernel(orc_q4k_acc_fn f) { g_q4k_acc = f; }
/* default: one thread per CPU this process may run on (its affinity mask,
 * which a container's cpuset narrows), as rayon's default pool */
int orc_get_threads(void) {
    if (g_threads > 0) return g_threads;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof set, &set) == 0 && CPU_COUNT(&set) > 0) return CPU_COUNT(&set);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*task_fn)(void *ctx, size_t begin, size_t end);

/* A persistent pool, as rayon's: the workers outlive each call, spin for a
 * short while after a job (back-to-back matmuls find them awake) and then
 * sleep on a condition variable. One job at a time; callers on other threads
 * queue on `call_mu`. Chunks are claimed with an atomic counter. */
#define POOL_MAX 256
#define POOL_SPIN_NS 200000L
static struct {
    pthread_mutex_t call_mu, mu;
    pthread_cond_t go, done;
    pthread_t th[POOL_MAX];
    int nworkers, quit;
    unsigned long gen;      /* bumped once per job */
    int pending;            /* workers that have not yet finished the current job */
    task_fn fn;
    void *ctx;
    size_t n, chunk, next;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER,
            PTHREAD_COND_INITIALIZER};

static long now_ns(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1000000000L + ts.tv_nsec;
}

static void pool_run_chunks(void) {
    for (;;) {
        size_t b = __atomic_fetch_add(&g_pool.next, g_pool.chunk, __ATOMIC_RELAXED);
        if (b >= g_pool.n) break;
        size_t e = b + g_pool.chunk < g_pool.n ? b + g_pool.chunk : g_pool.n;
        g_pool.fn(g_pool.ctx, b, e);
    }
}

static void *pool_worker(void *arg) {
    unsigned long seen = (unsigned long)(uintptr_t)arg;
    for (;;) {
        long t0 = now_ns();
        while (__atomic_load_n(&g_pool.gen, __ATOMIC_ACQUIRE) == seen && !__atomic_load_n(&g_pool.quit, __ATOMIC_ACQUIRE) &&
               now_ns() - t0 < POOL_SPIN_NS)
            __builtin_ia32_pause();
        pthread_mutex_lock(&g_pool.mu);
        while (g_pool.gen == seen && !g_pool.quit) pthread_cond_wait(&g_pool.go, &g_pool.mu);
        if (g_pool.quit) {
            pthread_mutex_unlock(&g_pool.mu);
            return NULL;
        }
        seen = g_pool.gen;
        pthread_mutex_unlock(&g_pool.mu);
        pool_run_chunks();
        if (__atomic_sub_fetch(&g_pool.pending, 1, __ATOMIC_ACQ_REL) == 0) {
            pthread_mutex_lock(&g_pool.mu);
            pthread_cond_signal(&g_pool.done);
            pthread_mutex_unlock(&g_pool.mu);
        }
    }
}

static void pool_stop(void) {
    if (g_pool.nworkers == 0) return;
    pthread_mutex_lock(&g_pool.mu);
    __atomic_store_n(&g_pool.quit, 1, __ATOMIC_RELEASE);
    pthread_cond_broadcast(&g_pool.go);
    pthread_mutex_unlock(&g_pool.mu);
    for (int i = 0; i < g_pool.nworkers; i++) pthread_join(g_pool.th[i], NULL);
    g_pool.nworkers = 0;
    g_pool.quit = 0;
}

/* A forked child has only the calling thread: forget the parent's workers. */
static void pool_after_fork(void) {
    pthread_mutex_init(&g_pool.call_mu, NULL);
    pthread_mutex_init(&g_pool.mu, NULL);
    pthread_cond_init(&g_pool.go, NULL);
    pthread_cond_init(&g_pool.done, NULL);
    g_pool.nworkers = 0;
    g_pool.quit = 0;
}

static void pool_register_fork(void) { pthread_atfork(NULL, NULL, pool_after_fork); }

/* (Re)start the pool with `workers` threads besides the caller's. Called with
 * call_mu held. */
static void pool_resize(int workers) {
    static pthread_once_t once = PTHREAD_ONCE_INIT;
    pthread_once(&once, pool_register_fork);
    if (workers == g_pool.nworkers) return;
    pool_stop();
    for (int i = 0; i < workers; i++) {
        if (pthread_create(&g_pool.th[i], NULL, pool_worker, (void *)(uintptr_t)g_pool.gen) != 0) break;
        g_pool.nworkers = i + 1;
    }
}

/* Work split in chunks of `chunk` items, like rayon's par_chunks_mut over
 * 32-row tasks (src/ops.rs:43, :946). */
static void par_for(size_t n, size_t chunk, task_fn fn, void *ctx) {
    int t = orc_get_threads();
    if (t <= 1 || n <= chunk) {
        fn(ctx, 0, n);
        return;
    }
    if (t > POOL_MAX) t = POOL_MAX;
    pthread_mutex_lock(&g_pool.call_mu);
    pool_resize(t - 1);
    if (g_pool.nworkers == 0) {
        pthread_mutex_unlock(&g_pool.call_mu);
        fn(ctx, 0, n);
        return;
    }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = fn;
    g_pool.ctx = ctx;
    g_pool.n = n;
    g_pool.chunk = chunk;
    g_pool.next = 0;
    g_pool.pending = g_pool.nworkers;
    __atomic_store_n(&g_pool.gen, g_pool.gen + 1, __ATOMIC_RELEASE);
    pthread_cond_broadcast(&g_pool.go);
    pthread_mutex_unlock(&g_pool.mu);
    pool_run_chunks();
    long t0 = now_ns();
    while (__atomic_load_n(&g_pool.pending, __ATOMIC_ACQUIRE) != 0 && now_ns() - t0 < POOL_SPIN_NS)
        __builtin_ia32_pause();
    pthread_mutex_lock(&g_pool.mu);
    while (__atomic_load_n(&g_pool.pending, __ATOMIC_ACQUIRE) != 0) pthread_cond_wait(&g_pool.done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
    pthread_mutex_unlock(&g_pool.call_mu);
}

/* ───────────────────────── formats ───────────────────────── */

int orc_values_per_block(int t) {
    switch (t) {
    case ORC_F32: case ORC_F16: return 1;
    case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: case ORC_Q8_1: return 32;
    case ORC_Q2K: case ORC_Q3K: case ORC_Q4K: case ORC_Q5K: case ORC_Q6K: case ORC_Q8K: return 256;
    default: return 0;
    }
}

int orc_bytes_per_block(int t) {
    switch (t) {
    case ORC_F32: return 4;
    case ORC_F16: return 2;
    case ORC_Q4_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q5_1: return 24;
    case ORC_Q8_0: return 34;
    case ORC_Q8_1: return 36;
    case ORC_Q2K: return 84;
    case ORC_Q3K: return 110;
    case ORC_Q4K: return 144;
    case ORC_Q5K: return 176;
    case ORC_Q6K: return 210;
    case ORC_Q8K: return 292;
    default: return 0;
    }
}

int orc_sub_block(int t) {
    switch (t) {
    case ORC_Q8_0: case ORC_Q5_0: case ORC_Q4K: case ORC_Q5K: return 32;
    case ORC_Q2K: case ORC_Q3K: case ORC_Q6K: return 16;
    default: return 0;
    }
}

/* IEEE half -> single, subnormals normalised by shifting (src/quant.rs:38-60). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0 && man == 0) {
        bits = sign;
    } else if (exp == 0) {
        int e = 1;
        while (!(man & 0x400)) { man <<= 1; e--; }
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

/* single -> half, round to nearest even, subnormals, saturation to inf and
 * NaN kept as NaN (src/quant.rs:691-731). */
uint16_t orc_f32_to_f16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    uint32_t mag = bits & 0x7FFFFFFFu;
    if (mag >= 0x7F800000u) {
        int nan = (mag & 0x007FFFFFu) != 0;
        return sign | 0x7C00 | (nan ? 0x0200 : 0);
    }
    int e = (int)(mag >> 23) - 127;
    if (e > 15) return sign | 0x7C00;
    if (e < -14) {
        uint32_t shift = (uint32_t)(-14 - e);
        if (shift > 24) return sign;
        uint32_t m = (mag & 0x007FFFFFu) | 0x00800000u;
        uint32_t val = m >> (shift + 13);
        uint32_t rest = m & ((1u << (shift + 13)) - 1);
        uint32_t half = 1u << (shift + 12);
        uint32_t up = (rest > half || (rest == half && (val & 1))) ? 1 : 0;
        return sign | (uint16_t)(val + up);
    }
    uint32_t m = mag & 0x007FFFFFu;
    uint32_t val = ((uint32_t)(e + 15) << 10) | (m >> 13);
    uint32_t rest = m & 0x1FFF;
    uint32_t up = (rest > 0x1000 || (rest == 0x1000 && (val & 1))) ? 1 : 0;
    return sign | (uint16_t)(val + up);
}

static inline float rd_f16(const uint8_t *b, size_t i) {
    return orc_f16_to_f32((uint16_t)(b[i] | (b[i + 1] << 8)));
}
static inline uint32_t rd_u32(const uint8_t *b, size_t i) {
    return (uint32_t)b[i] | ((uint32_t)b[i + 1] << 8) | ((uint32_t)b[i + 2] << 16) | ((uint32_t)b[i + 3] << 24);
}

/* 6-bit scale and min of sub-block j (0..7) from the 12 packed bytes of a
 * Q4_K/Q5_K block (src/quant.rs:108-117). */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* The sixteen 6-bit Q3_K scales (still biased by +32), from bytes 96..108 of
 * the block at offset o (src/quant.rs:87-106). */
static void scales_q3k(const uint8_t *b, size_t o, int8_t out[16]) {
    const uint32_t m1 = 0x03030303u, m2 = 0x0F0F0F0Fu;
    uint32_t a0 = rd_u32(b, o + 96), a1 = rd_u32(b, o + 100), t = rd_u32(b, o + 104);
    uint32_t w[4];
    w[2] = ((a0 >> 4) & m2) | (((t >> 4) & m1) << 4);
    w[3] = ((a1 >> 4) & m2) | (((t >> 6) & m1) << 4);
    w[0] = (a0 & m2) | ((t & m1) << 4);
    w[1] = (a1 & m2) | (((t >> 2) & m1) << 4);
    for (int j = 0; j < 16; j++) out[j] = (int8_t)(uint8_t)(w[j / 4] >> (8 * (j % 4)));
}

/* per-format readers: src/quant.rs:472-679 */
static void deq_q8_0(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 34;
        float d = rd_f16(b, o);
        for (int j = 0; j < 32; j++) y[i * 32 + j] = (float)(int8_t)b[o + 2 + j] * d;
    }
}
static void deq_q5_0(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 22;
        float d = rd_f16(b, o);
        uint32_t qh = rd_u32(b, o + 2);
        const uint8_t *qs = b + o + 6;
        for (int j = 0; j < 16; j++) {
            uint8_t h0 = (uint8_t)(((qh >> j) << 4) & 0x10);
            uint8_t h1 = (uint8_t)((qh >> (j + 12)) & 0x10);
            y[i * 32 + j] = (float)((int)((qs[j] & 0x0F) | h0) - 16) * d;
            y[i * 32 + 16 + j] = (float)((int)((qs[j] >> 4) | h1) - 16) * d;
        }
    }
}
static void deq_q2k(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 84;
        const uint8_t *sc = b + o, *qs0 = b + o + 16;
        float d = rd_f16(b, o + 80), mn = rd_f16(b, o + 82);
        int is = 0;
        size_t k = i * 256;
        for (int half = 0; half < 2; half++) {
            const uint8_t *qs = qs0 + half * 32;
            int shift = 0;
            for (int r = 0; r < 4; r++) {
                for (int t = 0; t < 2; t++) {
                    uint8_t s = sc[is++];
                    float dl = d * (float)(s & 0xF);
                    float ml = mn * (float)(s >> 4);
                    for (int l = 0; l < 16; l++)
                        y[k + t * 16 + l] = dl * (float)((qs[t * 16 + l] >> shift) & 3) - ml;
                }
                k += 32;
                shift += 2;
            }
        }
    }
}
static void deq_q3k(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 110;
        const uint8_t *hm = b + o, *qs0 = b + o + 32;
        float dall = rd_f16(b, o + 108);
        int8_t sc[16];
        scales_q3k(b, o, sc);
        uint8_t m = 1;
        int is = 0;
        size_t k = i * 256;
        for (int half = 0; half < 2; half++) {
            const uint8_t *qs = qs0 + half * 32;
            int shift = 0;
            for (int r = 0; r < 4; r++) {
                for (int t = 0; t < 2; t++) {
                    float dl = dall * ((float)sc[is++] - 32.0f);
                    for (int l = 0; l < 16; l++) {
                        int idx = t * 16 + l;
                        int8_t hi = (hm[idx] & m) ? 0 : 4;
                        y[k + idx] = dl * (float)((int8_t)((qs[idx] >> shift) & 3) - hi);
                    }
                }
                k += 32;
                shift += 2;
                m <<= 1;
            }
        }
    }
}
static void deq_q4k(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 144;
        float d = rd_f16(b, o), mn = rd_f16(b, o + 2);
        const uint8_t *sc = b + o + 4, *qs = b + o + 16;
        size_t k = i * 256;
        for (int p = 0; p < 4; p++) {
            uint8_t s, m;
            scale_min_k4(2 * p, sc, &s, &m);
            float d1 = d * (float)s, m1 = mn * (float)m;
            scale_min_k4(2 * p + 1, sc, &s, &m);
            float d2 = d * (float)s, m2 = mn * (float)m;
            const uint8_t *q = qs + 32 * p;
            for (int l = 0; l < 32; l++) y[k + l] = d1 * (float)(q[l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) y[k + 32 + l] = d2 * (float)(q[l] >> 4) - m2;
            k += 64;
        }
    }
}
static void deq_q5k(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 176;
        float d = rd_f16(b, o), mn = rd_f16(b, o + 2);
        const uint8_t *sc = b + o + 4, *qh = b + o + 16, *ql = b + o + 48;
        uint8_t u1 = 1, u2 = 2;
        size_t k = i * 256;
        for (int p = 0; p < 4; p++) {
            uint8_t s, m;
            scale_min_k4(2 * p, sc, &s, &m);
            float d1 = d * (float)s, m1 = mn * (float)m;
            scale_min_k4(2 * p + 1, sc, &s, &m);
            float d2 = d * (float)s, m2 = mn * (float)m;
            const uint8_t *q = ql + 32 * p;
            for (int l = 0; l < 32; l++)
                y[k + l] = d1 * ((float)(q[l] & 0xF) + ((qh[l] & u1) ? 16.0f : 0.0f)) - m1;
            for (int l = 0; l < 32; l++)
                y[k + 32 + l] = d2 * ((float)(q[l] >> 4) + ((qh[l] & u2) ? 16.0f : 0.0f)) - m2;
            k += 64;
            u1 <<= 2;
            u2 <<= 2;
        }
    }
}
static void deq_q6k(const uint8_t *b, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        size_t o = i * 210;
        const uint8_t *ql0 = b + o, *qh0 = b + o + 128, *sc0 = b + o + 192;
        float d = rd_f16(b, o + 208);
        for (int half = 0; half < 2; half++) {
            size_t base = i * 256 + half * 128;
            const uint8_t *ql = ql0 + 64 * half, *qh = qh0 + 32 * half, *sc = sc0 + 8 * half;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int8_t q1 = (int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[base + l] = d * (float)(int8_t)sc[is] * (float)q1;
                y[base + 32 + l] = d * (float)(int8_t)sc[is + 2] * (float)q2;
                y[base + 64 + l] = d * (float)(int8_t)sc[is + 4] * (float)q3;
                y[base + 96 + l] = d * (float)(int8_t)sc[is + 6] * (float)q4;
            }
        }
    }
}

int orc_dequantize(int type, const uint8_t *b, size_t nbytes, size_t n, float *y) {
    int vpb = orc_values_per_block(type);
    if (vpb == 0) { set_err("type %d: unknown", type); return -1; }
    if (n % (size_t)vpb) { set_err("type %d: %zu values, block is %d", type, n, vpb); return -1; }
    size_t nb = n / (size_t)vpb;
    if (nbytes < nb * (size_t)orc_bytes_per_block(type)) { set_err("type %d: missing bytes", type); return -1; }
    switch (type) {
    case ORC_F32: for (size_t i = 0; i < n; i++) { uint32_t u = rd_u32(b, 4 * i); memcpy(&y[i], &u, 4); } break;
    case ORC_F16: for (size_t i = 0; i < n; i++) y[i] = rd_f16(b, 2 * i); break;
    case ORC_Q8_0: deq_q8_0(b, y, nb); break;
    case ORC_Q5_0: deq_q5_0(b, y, nb); break;
    case ORC_Q2K: deq_q2k(b, y, nb); break;
    case ORC_Q3K: deq_q3k(b, y, nb); break;
    case ORC_Q4K: deq_q4k(b, y, nb); break;
    case ORC_Q5K: deq_q5k(b, y, nb); break;
    case ORC_Q6K: deq_q6k(b, y, nb); break;
    default: set_err("type %d: not implemented", type); return -1;
    }
    return 0;
}

/* Unpack straight to i8 + scale + offset per sub-block (src/quant.rs:238-468). */
int orc_unpack_i8(int type, const uint8_t *b, size_t nbytes, size_t n, int8_t *q, float *esc, float *des) {
    int vpb = orc_values_per_block(type), sub = orc_sub_block(type);
    if (!vpb || !sub) { set_err("type %d: no direct i8 unpack", type); return -1; }
    if (n % (size_t)vpb) { set_err("values not a multiple of the block"); return -1; }
    size_t nb = n / (size_t)vpb;
    if (nbytes < nb * (size_t)orc_bytes_per_block(type)) { set_err("missing bytes"); return -1; }
    size_t nsub = n / (size_t)sub;
    for (size_t i = 0; i < nsub; i++) des[i] = 0.0f;
    switch (type) {
    case ORC_Q8_0:
        for (size_t i = 0; i < nb; i++) {
            esc[i] = rd_f16(b, i * 34);
            for (int j = 0; j < 32; j++) q[i * 32 + j] = (int8_t)b[i * 34 + 2 + j];
        }
        break;
    case ORC_Q5_0:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 22;
            esc[i] = rd_f16(b, o);
            uint32_t qh = rd_u32(b, o + 2);
            const uint8_t *qs = b + o + 6;
            for (int j = 0; j < 16; j++) {
                uint8_t h0 = (uint8_t)(((qh >> j) << 4) & 0x10), h1 = (uint8_t)((qh >> (j + 12)) & 0x10);
                q[i * 32 + j] = (int8_t)((qs[j] & 0x0F) | h0) - 16;
                q[i * 32 + 16 + j] = (int8_t)((qs[j] >> 4) | h1) - 16;
            }
        }
        break;
    case ORC_Q4K:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 144;
            float d = rd_f16(b, o), mn = rd_f16(b, o + 2);
            const uint8_t *sc = b + o + 4, *qs = b + o + 16;
            for (int p = 0; p < 4; p++) {
                uint8_t s, m, s2, m2;
                scale_min_k4(2 * p, sc, &s, &m);
                scale_min_k4(2 * p + 1, sc, &s2, &m2);
                size_t s0 = i * 8 + 2 * p;
                esc[s0] = d * (float)s;
                des[s0] = -(mn * (float)m);
                esc[s0 + 1] = d * (float)s2;
                des[s0 + 1] = -(mn * (float)m2);
                size_t from = i * 256 + p * 64;
                for (int l = 0; l < 32; l++) {
                    q[from + l] = (int8_t)(qs[32 * p + l] & 0xF);
                    q[from + 32 + l] = (int8_t)(qs[32 * p + l] >> 4);
                }
            }
        }
        break;
    case ORC_Q5K:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 176;
            float d = rd_f16(b, o), mn = rd_f16(b, o + 2);
            const uint8_t *sc = b + o + 4, *qh = b + o + 16, *ql = b + o + 48;
            uint8_t u1 = 1, u2 = 2;
            for (int p = 0; p < 4; p++) {
                uint8_t s, m, s2, m2;
                scale_min_k4(2 * p, sc, &s, &m);
                scale_min_k4(2 * p + 1, sc, &s2, &m2);
                esc[i * 8 + 2 * p] = d * (float)s;
                des[i * 8 + 2 * p] = -(mn * (float)m);
                esc[i * 8 + 2 * p + 1] = d * (float)s2;
                des[i * 8 + 2 * p + 1] = -(mn * (float)m2);
                size_t k = i * 256 + p * 64;
                for (int l = 0; l < 32; l++) {
                    uint8_t v = ql[32 * p + l];
                    q[k + l] = (int8_t)((v & 0xF) + ((qh[l] & u1) ? 16 : 0));
                    q[k + 32 + l] = (int8_t)((v >> 4) + ((qh[l] & u2) ? 16 : 0));
                }
                u1 <<= 2;
                u2 <<= 2;
            }
        }
        break;
    case ORC_Q2K:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 84;
            const uint8_t *sc = b + o, *qs0 = b + o + 16;
            float d = rd_f16(b, o + 80), mn = rd_f16(b, o + 82);
            int is = 0;
            size_t k = i * 256;
            for (int half = 0; half < 2; half++) {
                const uint8_t *qs = qs0 + half * 32;
                int shift = 0;
                for (int r = 0; r < 4; r++) {
                    for (int t = 0; t < 2; t++) {
                        uint8_t s = sc[is + t];
                        esc[i * 16 + is + t] = d * (float)(s & 0xF);
                        des[i * 16 + is + t] = -(mn * (float)(s >> 4));
                    }
                    is += 2;
                    for (int l = 0; l < 32; l++) q[k + l] = (int8_t)((qs[l] >> shift) & 3);
                    k += 32;
                    shift += 2;
                }
            }
        }
        break;
    case ORC_Q3K:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 110;
            const uint8_t *hm = b + o, *qs0 = b + o + 32;
            float dall = rd_f16(b, o + 108);
            int8_t sc[16];
            scales_q3k(b, o, sc);
            uint8_t m = 1;
            int is = 0;
            size_t k = i * 256;
            for (int half = 0; half < 2; half++) {
                const uint8_t *qs = qs0 + half * 32;
                int shift = 0;
                for (int r = 0; r < 4; r++) {
                    for (int t = 0; t < 2; t++) esc[i * 16 + is + t] = dall * ((float)sc[is + t] - 32.0f);
                    is += 2;
                    for (int l = 0; l < 32; l++) {
                        int8_t hi = (hm[l] & m) ? 0 : 4;
                        q[k + l] = (int8_t)((int8_t)((qs[l] >> shift) & 3) - hi);
                    }
                    k += 32;
                    shift += 2;
                    m <<= 1;
                }
            }
        }
        break;
    case ORC_Q6K:
        for (size_t i = 0; i < nb; i++) {
            size_t o = i * 210;
            const uint8_t *ql0 = b + o, *qh0 = b + o + 128, *sc0 = b + o + 192;
            float d = rd_f16(b, o + 208);
            for (int half = 0; half < 2; half++) {
                size_t base = i * 256 + half * 128;
                const uint8_t *ql = ql0 + 64 * half, *qh = qh0 + 32 * half, *sc = sc0 + 8 * half;
                for (int p = 0; p < 8; p++) esc[i * 16 + half * 8 + p] = d * (float)(int8_t)sc[p];
                for (int l = 0; l < 32; l++) {
                    uint8_t h = qh[l];
                    q[base + l] = (int8_t)((ql[l] & 0xF) | ((h & 3) << 4)) - 32;
                    q[base + 32 + l] = (int8_t)((ql[32 + l] & 0xF) | (((h >> 2) & 3) << 4)) - 32;
                    q[base + 64 + l] = (int8_t)((ql[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
                    q[base + 96 + l] = (int8_t)((ql[32 + l] >> 4) | (((h >> 6) & 3) << 4)) - 32;
                }
            }
        }
        break;
    default:
        set_err("type %d: no direct i8 unpack", type);
        return -1;
    }
    return sub;
}

/* ───────────────────────── activation quantization ───────────────────────── */

/* src/ops.rs:178-198: per block, amax; inv = 127/amax (0 for amax = 0);
 * q = round-half-away(x*inv); scale = amax/127. Sums: src/ops.rs:873-876. */
void orc_quantize_i8(const float *x, size_t n, int sub, int8_t *q, float *scales, float *sums) {
    size_t nb = (n + (size_t)sub - 1) / (size_t)sub;
    for (size_t b = 0; b < nb; b++) {
        size_t from = b * (size_t)sub, to = from + (size_t)sub < n ? from + (size_t)sub : n;
        float amax = 0.0f;
        for (size_t i = from; i < to; i++) amax = fmaxf(amax, fabsf(x[i]));
        float d = 0.0f, inv = 0.0f;
        if (amax > 0.0f) {
            d = amax / 127.0f;
            inv = 127.0f / amax;
        }
        scales[b] = d;
        int32_t s = 0;
        for (size_t i = from; i < to; i++) {
            float r = roundf(x[i] * inv);
            int32_t v = isnan(r) ? 0 : (r >= 2147483647.0f ? 2147483647 : (r <= -2147483648.0f ? (int32_t)0x80000000 : (int32_t)r));
            q[i] = (int8_t)v;
            s += q[i];
        }
        if (sums) sums[b] = (float)s;
    }
}

/* ───────────────────────── dots ───────────────────────── */

int32_t orc_dot_i8(const int8_t *a, const int8_t *b, size_t n) {
    int32_t s = 0;
    for (size_t i = 0; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

float orc_dot_i8_scaled(const int8_t *a, const int8_t *b, const float *ea, const float *eb, size_t n, int block) {
    float total = 0.0f;
    size_t nb = (n + (size_t)block - 1) / (size_t)block;
    for (size_t i = 0; i < nb; i++) {
        size_t r = i * (size_t)block, to = r + (size_t)block < n ? r + (size_t)block : n;
        int32_t p = 0;
        for (size_t j = r; j < to; j++) p += (int32_t)a[j] * (int32_t)b[j];
        total += ea[i] * eb[i] * (float)p;
    }
    return total;
}

float orc_dot_f32(const float *a, const float *b, size_t n) {
    float s = 0.0f;
    for (size_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* Integer sub-block sums of one row. These are the `entero` values the
 * scalar kernels build; see the per-format dots below for the citations. */
int orc_subblock_sums(int type, const uint8_t *row, const int8_t *xq, size_t nblk, int32_t *out) {
    for (size_t bl = 0; bl < nblk; bl++) {
        const int8_t *xb = xq + bl * 256;
        if (type == ORC_Q4K || type == ORC_Q5K) {
            const uint8_t *blk = row + bl * (type == ORC_Q4K ? 144 : 176);
            const uint8_t *qs = blk + (type == ORC_Q4K ? 16 : 48), *qh = blk + 16;
            for (int j = 0; j < 8; j++) {
                int p = j / 2, half = j % 2;
                const int8_t *x = xb + p * 64 + half * 32;
                int32_t e = 0;
                for (int i = 0; i < 32; i++) {
                    int v = half == 0 ? (qs[32 * p + i] & 0x0F) : (qs[32 * p + i] >> 4);
                    if (type == ORC_Q5K && (qh[i] & (1 << j))) v += 16;
                    e += (int32_t)x[i] * v;
                }
                out[bl * 8 + j] = e;
            }
        } else if (type == ORC_Q3K) {
            const uint8_t *blk = row + bl * 110, *hm = blk, *qs = blk + 32;
            for (int g = 0; g < 8; g++) {
                const uint8_t *qsg = qs + (g / 4) * 32;
                int sh = 2 * (g % 4);
                const int8_t *x = xb + g * 32;
                for (int md = 0; md < 2; md++) {
                    int32_t e = 0;
                    for (int l = 0; l < 16; l++) {
                        int idx = md * 16 + l;
                        int v = ((qsg[idx] >> sh) & 3) + ((hm[idx] & (1 << g)) ? 4 : 0);
                        e += (int32_t)x[idx] * v;
                    }
                    out[bl * 16 + g * 2 + md] = e;
                }
            }
        } else if (type == ORC_Q6K) {
            const uint8_t *blk = row + bl * 210;
            for (int g = 0; g < 8; g++) {
                int half = g / 4, gi = g % 4;
                const uint8_t *ql = blk + 64 * half + 32 * (gi % 2), *qh = blk + 128 + 32 * half;
                const int8_t *x = xb + g * 32;
                for (int md = 0; md < 2; md++) {
                    int32_t e = 0;
                    for (int l = 0; l < 16; l++) {
                        int i = md * 16 + l;
                        int nib = gi < 2 ? (ql[i] & 0x0F) : (ql[i] >> 4);
                        int v = nib | (((qh[i] >> (2 * gi)) & 3) << 4);
                        e += (int32_t)x[i] * v;
                    }
                    out[bl * 16 + g * 2 + md] = e;
                }
            }
        } else if (type == ORC_Q2K) {
            const uint8_t *blk = row + bl * 84, *qs = blk + 16;
            for (int g = 0; g < 8; g++) {
                const uint8_t *qsg = qs + (g / 4) * 32;
                int sh = 2 * (g % 4);
                const int8_t *x = xb + g * 32;
                for (int md = 0; md < 2; md++) {
                    int32_t e = 0;
                    for (int l = 0; l < 16; l++) {
                        int idx = md * 16 + l;
                        e += (int32_t)x[idx] * (int32_t)((qsg[idx] >> sh) & 3);
                    }
                    out[bl * 16 + g * 2 + md] = e;
                }
            }
        } else {
            set_err("type %d: no fused kernel", type);
            return -1;
        }
    }
    return 0;
}

/* src/kernels/scalar.rs:132-170 */
float orc_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    float total = 0.0f;
    for (size_t bl = 0; bl < nblk; bl++) {
        const uint8_t *blk = row + bl * 144;
        float d = rd_f16(blk, 0), dmin = rd_f16(blk, 2);
        const uint8_t *sc = blk + 4, *qs = blk + 16;
        for (int p = 0; p < 4; p++) {
            for (int half = 0; half < 2; half++) {
                int j = p * 2 + half;
                uint8_t s, m;
                scale_min_k4(j, sc, &s, &m);
                size_t sub = bl * 8 + (size_t)j;
                const int8_t *x = xq + bl * 256 + p * 64 + half * 32;
                int32_t e = 0;
                for (int i = 0; i < 32; i++) {
                    int v = half == 0 ? (qs[32 * p + i] & 0x0F) : (qs[32 * p + i] >> 4);
                    e += (int32_t)x[i] * v;
                }
                total += xe[sub] * (d * (float)s * (float)e - dmin * (float)m * xs[sub]);
            }
        }
    }
    return total;
}

/* src/kernels/scalar.rs:179-217 */
float orc_dot_q5k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    float total = 0.0f;
    for (size_t bl = 0; bl < nblk; bl++) {
        const uint8_t *blk = row + bl * 176;
        float d = rd_f16(blk, 0), dmin = rd_f16(blk, 2);
        const uint8_t *sc = blk + 4, *qh = blk + 16, *qs = blk + 48;
        for (int p = 0; p < 4; p++) {
            for (int half = 0; half < 2; half++) {
                int j = p * 2 + half;
                uint8_t s, m;
                scale_min_k4(j, sc, &s, &m);
                size_t sub = bl * 8 + (size_t)j;
                const int8_t *x = xq + bl * 256 + p * 64 + half * 32;
                int32_t e = 0;
                for (int i = 0; i < 32; i++) {
                    int v = half == 0 ? (qs[32 * p + i] & 0x0F) : (qs[32 * p + i] >> 4);
                    int hi = (qh[i] & (1 << j)) ? 16 : 0;
                    e += (int32_t)x[i] * (v + hi);
                }
                total += xe[sub] * (d * (float)s * (float)e - dmin * (float)m * xs[sub]);
            }
        }
    }
    return total;
}

/* src/kernels/scalar.rs:236-275 */
float orc_dot_q3k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    float total = 0.0f;
    for (size_t bl = 0; bl < nblk; bl++) {
        size_t o = bl * 110;
        const uint8_t *hm = row + o, *qs = row + o + 32;
        float d = rd_f16(row, o + 108);
        int8_t esc[16];
        scales_q3k(row, o, esc);
        for (int g = 0; g < 8; g++) {
            const uint8_t *qsg = qs + (g / 4) * 32;
            int sh = 2 * (g % 4);
            uint8_t m = (uint8_t)(1u << g);
            const int8_t *x = xq + bl * 256 + g * 32;
            for (int md = 0; md < 2; md++) {
                size_t sub = bl * 16 + (size_t)(g * 2 + md);
                float scale = d * ((float)esc[g * 2 + md] - 32.0f);
                int32_t e = 0;
                for (int l = 0; l < 16; l++) {
                    int idx = md * 16 + l;
                    int extra = (hm[idx] & m) ? 4 : 0;
                    int v = ((qsg[idx] >> sh) & 3) + extra;
                    e += (int32_t)x[idx] * v;
                }
                total += xe[sub] * scale * ((float)e - 4.0f * xs[sub]);
            }
        }
    }
    return total;
}

/* src/kernels/scalar.rs:294-324 */
float orc_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    float total = 0.0f;
    for (size_t bl = 0; bl < nblk; bl++) {
        size_t o = bl * 210;
        const uint8_t *esc = row + o + 192;
        float d = rd_f16(row, o + 208);
        for (int g = 0; g < 8; g++) {
            int half = g / 4, gi = g % 4;
            const uint8_t *ql = row + o + 64 * half + 32 * (gi % 2), *qh = row + o + 128 + 32 * half;
            const int8_t *x = xq + bl * 256 + g * 32;
            for (int md = 0; md < 2; md++) {
                size_t sub = bl * 16 + (size_t)(g * 2 + md);
                float scale = d * (float)(int8_t)esc[g * 2 + md];
                int32_t e = 0;
                for (int l = 0; l < 16; l++) {
                    int i = md * 16 + l;
                    int nib = gi < 2 ? (ql[i] & 0x0F) : (ql[i] >> 4);
                    int v = nib | (((qh[i] >> (2 * gi)) & 3) << 4);
                    e += (int32_t)x[i] * v;
                }
                total += xe[sub] * scale * ((float)e - 32.0f * xs[sub]);
            }
        }
    }
    return total;
}

/* src/kernels/q2k.rs:41-69 */
float orc_dot_q2k(const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    float total = 0.0f;
    for (size_t bl = 0; bl < nblk; bl++) {
        size_t o = bl * 84;
        const uint8_t *esc = row + o, *qs = row + o + 16;
        float d = rd_f16(row, o + 80), dm = rd_f16(row, o + 82);
        for (int g = 0; g < 8; g++) {
            const uint8_t *qsg = qs + (g / 4) * 32;
            int sh = 2 * (g % 4);
            const int8_t *x = xq + bl * 256 + g * 32;
            for (int md = 0; md < 2; md++) {
                int s = g * 2 + md;
                size_t sub = bl * 16 + (size_t)s;
                int32_t e = 0;
                for (int l = 0; l < 16; l++) {
                    int idx = md * 16 + l;
                    e += (int32_t)x[idx] * (int32_t)((qsg[idx] >> sh) & 3);
                }
                float ev = d * (float)(esc[s] & 0xF);
                float mv = dm * (float)(esc[s] >> 4);
                total += xe[sub] * (ev * (float)e - mv * xs[sub]);
            }
        }
    }
    return total;
}

float orc_dot_row(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    switch (type) {
    case ORC_Q4K: return orc_dot_q4k(row, xq, xe, xs, nblk);
    case ORC_Q5K: return orc_dot_q5k(row, xq, xe, xs, nblk);
    case ORC_Q6K: return orc_dot_q6k(row, xq, xe, xs, nblk);
    case ORC_Q3K: return orc_dot_q3k(row, xq, xe, xs, nblk);
    case ORC_Q2K: return orc_dot_q2k(row, xq, xe, xs, nblk);
    default: return NAN;
    }
}

/* What the reference's dispatch (src/kernels/mod.rs:347-509) runs on an AVX2
 * host: a registered kernel of the reference's own where one was given, else
 * the AVX2 restatement (Q4_K, Q6_K), else the scalar restatement. */
float orc_x86_dot_row(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs, size_t nblk) {
    if (type >= 0 && type < 16 && g_dot_kernel[type]) return g_dot_kernel[type](row, xq, xe, xs, nblk);
    switch (type) {
    case ORC_Q4K:
        if (g_q4k_acc) {
            /* the kernel adds into the accumulators; its caller zeroes them */
            float acc[16] = {0};
            g_q4k_acc(row, xq, xe, xs, nblk, acc);
            return orc_x86_reduce_q4k_acc(acc);
        }
        return orc_x86_dot_q4k(row, xq, xe, xs, nblk);
    case ORC_Q6K: return orc_x86_dot_q6k(row, xq, xe, xs, nblk);
    default: return orc_dot_row(type, row, xq, xe, xs, nblk);
    }
}

/* ───────────────────────── elementwise ops ───────────────────────── */

/* src/kernels/scalar.rs:36-54 — the sum of squares in f64 */
void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps) {
    if (n == 0) return;
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) sum += (double)in[i] * (double)in[i];
    double scale = 1.0 / sqrt((sum / (double)n) + (double)eps);
    for (size_t i = 0; i < n; i++) out[i] = (float)((double)in[i] * scale) * w[i];
}

/* src/kernels/scalar.rs:63-67 */
void orc_silu(float *out, const float *in, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = in[i] / (1.0f + expf(-in[i]));
}

/* src/ops.rs:1108-1129: f32 frequency, f64 angle, f64 cos/sin stored as f32 */
void orc_rope_tables(int hd, float base, int ctx, float *cos_t, float *sin_t) {
    int half = hd / 2;
    for (int j = 0; j < half; j++) {
        float freq = 1.0f / powf(base, 2.0f * (float)j / (float)hd);
        for (int p = 0; p < ctx; p++) {
            double ang = (double)p * (double)freq;
            cos_t[(size_t)p * half + j] = (float)cos(ang);
            sin_t[(size_t)p * half + j] = (float)sin(ang);
        }
    }
}

/* src/ops.rs:1150-1193: split-half (NEOX) rotation at absolute positions */
int orc_rope(float *x, int tokens, int heads, int hd, const float *cos_t, const float *sin_t, int ctx, int pos) {
    if (hd % 2) { set_err("head_dim %d must be even", hd); return -1; }
    if (pos + tokens > ctx) { set_err("positions %d..%d beyond table %d", pos, pos + tokens, ctx); return -1; }
    int half = hd / 2, width = heads * hd;
    for (int t = 0; t < tokens; t++) {
        const float *c = cos_t + (size_t)(pos + t) * half, *s = sin_t + (size_t)(pos + t) * half;
        for (int h = 0; h < heads; h++) {
            float *head = x + (size_t)t * width + (size_t)h * hd;
            for (int i = 0; i < half; i++) {
                float x0 = head[i], x1 = head[i + half];
                head[i] = x0 * c[i] - x1 * s[i];
                head[i + half] = x0 * s[i] + x1 * c[i];
            }
        }
    }
    return 0;
}

/* src/ops.rs:1206-1230 */
int orc_softmax(float *x, size_t n, size_t width) {
    if (width == 0 || n % width) { set_err("%zu values not a multiple of %zu", n, width); return -1; }
    for (size_t r = 0; r < n / width; r++) {
        float *row = x + r * width;
        float mx = -INFINITY;
        for (size_t i = 0; i < width; i++) mx = fmaxf(mx, row[i]);
        if (!isfinite(mx)) {
            float p = 1.0f / (float)width;
            for (size_t i = 0; i < width; i++) row[i] = p;
            continue;
        }
        float total = 0.0f;
        for (size_t i = 0; i < width; i++) {
            row[i] = expf(row[i] - mx);
            total += row[i];
        }
        float inv = 1.0f / total;
        for (size_t i = 0; i < width; i++) row[i] *= inv;
    }
    return 0;
}

/* src/ops.rs:1258-1325: causal GQA; head h reads kv head h / (H/KV) */
int orc_attention(const float *q, const float *k, const float *v, int tokens, int total, int heads,
                  int heads_kv, int hd, float *out) {
    if (heads_kv == 0 || heads % heads_kv) { set_err("%d heads not divisible in %d groups", heads, heads_kv); return -1; }
    if (tokens > total) { set_err("%d new tokens and only %d total", tokens, total); return -1; }
    int wq = heads * hd, wkv = heads_kv * hd, per = heads / heads_kv;
    float scale = 1.0f / sqrtf((float)hd);
    int offset = total - tokens;
    float *pts = (float *)malloc(sizeof(float) * (size_t)(total > 0 ? total : 1));
    /* kernels::dot is the AVX2 one on an AVX2 host (src/kernels/mod.rs:240-262) */
    float (*dotf)(const float *, const float *, size_t) = g_backend == ORC_BACKEND_X86 ? orc_x86_dot_f32 : orc_dot_f32;
    for (int t = 0; t < tokens; t++) {
        int vis = offset + t + 1;
        for (int h = 0; h < heads; h++) {
            const float *qh = q + (size_t)t * wq + (size_t)h * hd;
            int base = (h / per) * hd;
            for (int p = 0; p < vis; p++) pts[p] = dotf(qh, k + (size_t)p * wkv + base, (size_t)hd) * scale;
            orc_softmax(pts, (size_t)vis, (size_t)vis);
            float *dst = out + (size_t)t * wq + (size_t)h * hd;
            for (int d = 0; d < hd; d++) dst[d] = 0.0f;
            for (int p = 0; p < vis; p++) {
                const float *vh = v + (size_t)p * wkv + base;
                for (int d = 0; d < hd; d++) dst[d] += pts[p] * vh[d];
            }
        }
    }
    free(pts);
    return 0;
}

/* ───────────────────────── matmul dispatch ───────────────────────── */

/* src/ops.rs:837-858 `hay_fusionado`: the formats whose per-row fused kernel
 * the reference uses. Q4_K and Q3_K always; Q6_K and Q5_K only when the AVX2
 * kernels are in use (usar_avx2(), src/kernels/mod.rs:184-190); Q2_K only when
 * its chosen copy is not the scalar one (src/kernels/q2k.rs:210-238), which
 * under COSXAMIX_KERNEL=escalar it is. So on the scalar backend only Q4_K and
 * Q3_K are fused; Q6_K, Q5_K and Q2_K take the buffered path even for one
 * activation row. */
static int fused_available(int type, int k) {
    if (k % 256) return 0;
    if (type == ORC_Q4K || type == ORC_Q3K) return 1;
    if (type == ORC_Q6K || type == ORC_Q5K || type == ORC_Q2K) return g_backend == ORC_BACKEND_X86;
    return 0;
}

int orc_matmul_path(int m, int k, int type) {
    if (orc_sub_block(type) == 0) return ORC_PATH_F32;              /* ops.rs:1062-1068 */
    if (m >= ORC_BLOCKED_FROM)                                      /* ops.rs:1073-1079 */
        return g_backend == ORC_BACKEND_X86 && k % 32 == 0 ? ORC_PATH_BLOCKED : ORC_PATH_BUFFERED;  /* :599-606 */
    const int cap = type == ORC_Q4K ? 0x7fffffff : 4;               /* ops.rs:1081-1085 */
    if (fused_available(type, k) && m <= cap) return ORC_PATH_FUSED;
    return ORC_PATH_BUFFERED;                                       /* ops.rs:1090-1092 */
}

typedef struct {
    int m, k, n, sub, type, path;
    size_t row_bytes, nblk;
    const uint8_t *w;
    const int8_t *xq;
    const float *xe, *xs;
    float *dst;
} mm_ctx;

/* kernels::dot_i8_escalado (src/kernels/mod.rs:303-339): the AVX2 kernel on
 * the x86 backend for the sub-block sizes and lengths it accepts, else the
 * scalar one (scalar.rs:95-109: total += ea * eb * parcial, block by block) */
static float dot_i8_scaled_dispatch(const int8_t *a, const int8_t *b, const float *ea, const float *eb, size_t n,
                                    int block) {
    const size_t wide = block > 32 ? (size_t)block : 32;
    if (g_backend == ORC_BACKEND_X86 && (block == 16 || block % 32 == 0) && n % wide == 0)
        return orc_x86_dot_i8_scaled(a, b, ea, eb, n, block);
    return orc_dot_i8_scaled(a, b, ea, eb, n, block);
}

/* One output of the buffered path for an unpacked column (q, esc, des of its
 * sub-blocks): src/ops.rs:383-405 (matmul_i8_directo) and :986-1006
 * (matmul_varias_una_fila's buffered path), which compute the same thing:
 * dot_i8_escalado over the whole row, then, when any shift of the column is
 * nonzero, total += des[b] * xe[b] * xs[b] sub-block by sub-block. */
static float buffered_out(const int8_t *colq, const float *esc, const float *des, int shifted, const int8_t *xq,
                          const float *xe, const float *xs, size_t k, int sub) {
    float total = dot_i8_scaled_dispatch(colq, xq, esc, xe, k, sub);
    if (shifted) {
        const size_t nsub = k / (size_t)sub;
        for (size_t b = 0; b < nsub; b++) total += des[b] * xe[b] * xs[b];
    }
    return total;
}

static int any_nonzero(const float *v, size_t n) {
    for (size_t i = 0; i < n; i++)
        if (v[i] != 0.0f) return 1;
    return 0;
}

float orc_dot_row_buffered(int type, const uint8_t *row, const int8_t *xq, const float *xe, const float *xs,
                           size_t nblk) {
    const int sub = orc_sub_block(type);
    const size_t k = nblk * 256, nsub = k / (size_t)sub;
    int8_t *q = (int8_t *)malloc(k);
    float *esc = (float *)malloc(sizeof(float) * nsub), *des = (float *)malloc(sizeof(float) * nsub);
    float r = NAN;
    if (orc_unpack_i8(type, row, nblk * (size_t)orc_bytes_per_block(type), k, q, esc, des) > 0)
        r = buffered_out(q, esc, des, any_nonzero(des, nsub), xq, xe, xs, k, sub);
    free(q);
    free(esc);
    free(des);
    return r;
}

static void mm_task(void *c_, size_t b, size_t e) {
    mm_ctx *c = (mm_ctx *)c_;
    size_t nsub = (size_t)c->k / (size_t)c->sub;
    if (c->path == ORC_PATH_BUFFERED) {
        /* src/ops.rs:372-405: each column unpacked once (desempaquetar_i8),
         * then one output per activation row */
        int8_t *q = (int8_t *)malloc((size_t)c->k);
        float *esc = (float *)malloc(sizeof(float) * nsub), *des = (float *)malloc(sizeof(float) * nsub);
        for (size_t col = b; col < e; col++) {
            if (orc_unpack_i8(c->type, c->w + col * c->row_bytes, c->row_bytes, (size_t)c->k, q, esc, des) < 0) continue;
            const int shifted = any_nonzero(des, nsub);
            for (int f = 0; f < c->m; f++)
                c->dst[(size_t)f * c->n + col] = buffered_out(q, esc, des, shifted, c->xq + (size_t)f * c->k,
                                                              c->xe + f * nsub, c->xs + f * nsub, (size_t)c->k, c->sub);
        }
        free(q);
        free(esc);
        free(des);
        return;
    }
    if (g_backend == ORC_BACKEND_X86) {
        /* src/ops.rs:486-506: the row two ahead is prefetched line by line
         * (:45-80) while this one is computed */
        for (size_t col = b; col < e; col++) {
            const uint8_t *row = c->w + col * c->row_bytes;
            if (col + 2 < e)
                for (size_t o = 0; o < c->row_bytes; o += 64) _mm_prefetch((const char *)(row + 2 * c->row_bytes + o), _MM_HINT_T0);
            for (int f = 0; f < c->m; f++)
                c->dst[(size_t)f * c->n + col] = orc_x86_dot_row(c->type, row, c->xq + (size_t)f * c->k,
                                                                 c->xe + f * nsub, c->xs + f * nsub, c->nblk);
        }
        return;
    }
    for (size_t col = b; col < e; col++) {
        const uint8_t *row = c->w + col * c->row_bytes;
        for (int f = 0; f < c->m; f++)
            c->dst[(size_t)f * c->n + col] = orc_dot_row(c->type, row, c->xq + (size_t)f * c->k,
                                                         c->xe + f * nsub, c->xs + f * nsub, c->nblk);
    }
}

/* ── the blocked prefill path of the x86 backend (src/ops.rs:633-829) ── */

/* src/ops.rs:565-580 `expandir_escalas`: one scale per 32-bit lane of each
 * 32-value chunk (lanes 0-3 / 4-7 of a chunk take sub-blocks 2t / 2t+1 when
 * sub-blocks hold 16 values; all eight take sub-block t when they hold 32) */
static void expand_scales(const float *esc, int sub, size_t chunks, float *out) {
    for (size_t t = 0; t < chunks; t++)
        for (int l = 0; l < 8; l++) out[t * 8 + l] = sub == 16 ? esc[2 * t + (l >= 4)] : esc[t];
}

typedef struct {
    int m, k, n, sub, type;
    size_t row_bytes, nsub, chunks;
    const uint8_t *w;
    const int8_t *xq;     /* [m][k] */
    const float *xe8;     /* [m][chunks*8] expanded activation scales */
    const float *xes;     /* [m][nsub] scale x sum (src/ops.rs:671-675) */
    float *dst;           /* [m][n] */
} blk_ctx;

/* One task = one tramo of COLUMNAS_MINIMAS (32) columns, as the
 * reference's par_chunks_mut over salida_t (src/ops.rs:683-687). The tile
 * walk of :758-820 (4x2 register tiles over row strips) only changes which
 * outputs are computed together; each output's arithmetic is the tile
 * kernel's for one (row, column), so it is computed here one by one. */
static void blk_task(void *c_, size_t b, size_t e) {
    blk_ctx *c = (blk_ctx *)c_;
    const size_t ncols = e - b, k = (size_t)c->k, nsub = c->nsub, ch8 = c->chunks * 8;
    int8_t *q = (int8_t *)malloc(ncols * k);
    float *e8 = (float *)malloc(sizeof(float) * ncols * ch8), *des = (float *)malloc(sizeof(float) * ncols * nsub);
    float *esc = (float *)malloc(sizeof(float) * nsub);
    char *ok = (char *)calloc(ncols, 1), *has = (char *)calloc(ncols, 1);
    /* :693-710 the tramo unpacked once */
    for (size_t j = 0; j < ncols; j++) {
        if (orc_unpack_i8(c->type, c->w + (b + j) * c->row_bytes, c->row_bytes, k, q + j * k, esc, des + j * nsub) < 0) {
            memset(q + j * k, 0, k);
            memset(e8 + j * ch8, 0, sizeof(float) * ch8);
            continue;
        }
        ok[j] = 1;
        expand_scales(esc, c->sub, c->chunks, e8 + j * ch8);
    }
    /* :712-736 unsigned weights when the tramo's range allows: every value
     * shifted by -min, the shift taken out of the offset term */
    int mn = 127, mx = -128;
    for (size_t i = 0; i < ncols * k; i++) {
        if (q[i] < mn) mn = q[i];
        if (q[i] > mx) mx = q[i];
    }
    const int corr = -mn, unsig = mx + corr <= 129;
    if (unsig && corr != 0)
        for (size_t i = 0; i < ncols * k; i++) q[i] = (int8_t)(uint8_t)((int)q[i] + corr);
    for (size_t j = 0; j < ncols; j++) {
        float *d = des + j * nsub;
        if (unsig && corr != 0)
            for (size_t s = 0; s < nsub; s++) d[s] -= (float)corr * e8[j * ch8 + s * (size_t)c->sub / 4];
        has[j] = (char)any_nonzero(d, nsub);
    }
    /* :758-820 the tile kernel, one output at a time (same arithmetic) */
    for (size_t j = 0; j < ncols; j++)
        for (int f = 0; f < c->m; f++) {
            const int8_t *x = c->xq + (size_t)f * k;
            const float *ef = c->xe8 + (size_t)f * ch8;
            c->dst[(size_t)f * c->n + b + j] = orc_x86_tile_out(x, ef, q + j * k, e8 + j * ch8, c->chunks, unsig);
        }
    /* :822-831 the offset term, in the formats that have one */
    for (size_t j = 0; j < ncols; j++) {
        if (!has[j]) continue;
        for (int f = 0; f < c->m; f++)
            c->dst[(size_t)f * c->n + b + j] += orc_x86_dot_f32(des + j * nsub, c->xes + (size_t)f * nsub, nsub);
    }
    (void)ok;
    free(q);
    free(e8);
    free(des);
    free(esc);
    free(ok);
    free(has);
}

static int matmul_blocked_x86(int m, int k, int n, const float *lhs, const uint8_t *w, int type, float *dst) {
    const int sub = orc_sub_block(type);
    const size_t nsub = (size_t)k / sub, chunks = (size_t)k / 32;
    int8_t *xq = (int8_t *)malloc((size_t)m * k);
    float *xe = (float *)malloc(sizeof(float) * (size_t)m * nsub), *xs = (float *)malloc(sizeof(float) * (size_t)m * nsub);
    float *xe8 = (float *)malloc(sizeof(float) * (size_t)m * chunks * 8), *xes = (float *)malloc(sizeof(float) * (size_t)m * nsub);
    /* :662-677 the input quantized row by row, scales expanded, scale x sum */
    for (int f = 0; f < m; f++) {
        orc_quantize_i8(lhs + (size_t)f * k, (size_t)k, sub, xq + (size_t)f * k, xe + f * nsub, xs + f * nsub);
        expand_scales(xe + f * nsub, sub, chunks, xe8 + (size_t)f * chunks * 8);
        for (size_t s = 0; s < nsub; s++) xes[f * nsub + s] = xe[f * nsub + s] * xs[f * nsub + s];
    }
    blk_ctx c = {m, k, n, sub, type, (size_t)k / orc_values_per_block(type) * (size_t)orc_bytes_per_block(type),
                 nsub, chunks, w, xq, xe8, xes, dst};
    par_for((size_t)n, 32, blk_task, &c);
    free(xq);
    free(xe);
    free(xs);
    free(xe8);
    free(xes);
    return 0;
}

/* ops::matmul_auto (src/ops.rs:1056-1093) on this oracle's backend:
 * dst[m][n] = lhs[m][k] · W[n][k]ᵀ by the path orc_matmul_path names. */
int orc_matmul_auto(int m, int k, int n, const float *lhs, const uint8_t *w, size_t wbytes, int type, float *dst) {
    return orc_matmul_by_path(orc_matmul_path(m, k, type), m, k, n, lhs, w, wbytes, type, dst);
}

/* One path forced (test access: the reference's own tests call
 * matmul_i8_directo and matmul_i8_bloques directly, src/ops.rs:1517-1561). */
int orc_matmul_by_path(int path, int m, int k, int n, const float *lhs, const uint8_t *w, size_t wbytes, int type,
                       float *dst) {
    if (path == ORC_PATH_BLOCKED && (g_backend != ORC_BACKEND_X86 || k % 32)) path = ORC_PATH_BUFFERED;  /* :599-606 */
    if (path == ORC_PATH_FUSED && !(type == ORC_Q2K || type == ORC_Q3K || type == ORC_Q4K || type == ORC_Q5K ||
                                    type == ORC_Q6K) ) path = ORC_PATH_BUFFERED;  /* :443-452 */
    if (path == ORC_PATH_FUSED && k % 256) path = ORC_PATH_BUFFERED;              /* :453-455 */
    if (orc_sub_block(type) == 0) path = ORC_PATH_F32;
    if (path == ORC_PATH_F32) {
        /* F32/F16: ops::matmul (src/ops.rs:88-156): dequantize a row, f32 dot */
        int vpb = orc_values_per_block(type);
        if (!vpb || k % vpb) { set_err("type %d unsupported for matmul", type); return -1; }
        size_t rb = (size_t)k / (size_t)vpb * (size_t)orc_bytes_per_block(type);
        if (wbytes < (size_t)n * rb) { set_err("missing weight bytes"); return -1; }
        float *col = (float *)malloc(sizeof(float) * (size_t)k);
        for (int c = 0; c < n; c++) {
            if (orc_dequantize(type, w + (size_t)c * rb, rb, (size_t)k, col)) { free(col); return -1; }
            for (int f = 0; f < m; f++) dst[(size_t)f * n + c] = orc_dot_f32(lhs + (size_t)f * k, col, (size_t)k);
        }
        free(col);
        return 0;
    }
    const int sub = orc_sub_block(type), vpb = orc_values_per_block(type);
    if (k % vpb || k % sub) { set_err("row of %d is not a multiple of the blocks", k); return -1; }
    size_t rb = (size_t)k / (size_t)vpb * (size_t)orc_bytes_per_block(type);
    if (wbytes < (size_t)n * rb) { set_err("missing weight bytes"); return -1; }
    if (path == ORC_PATH_BLOCKED) return matmul_blocked_x86(m, k, n, lhs, w, type, dst);
    size_t nsub = (size_t)k / (size_t)sub;
    int8_t *xq = (int8_t *)malloc((size_t)m * k);
    float *xe = (float *)malloc(sizeof(float) * (size_t)m * nsub);
    float *xs = (float *)malloc(sizeof(float) * (size_t)m * nsub);
    for (int f = 0; f < m; f++)
        orc_quantize_i8(lhs + (size_t)f * k, (size_t)k, sub, xq + (size_t)f * k, xe + f * nsub, xs + f * nsub);
    mm_ctx c = {m, k, n, sub, type, path, rb, (size_t)k / 256, w, xq, xe, xs, dst};
    par_for((size_t)n, 32, mm_task, &c);
    free(xq);
    free(xe);
    free(xs);
    return 0;
}

/* ───────────────────────── RNG ───────────────────────── */

uint64_t orc_azar_seed(uint64_t s) { return s == 0 ? 0x9E3779B97F4A7C15ull : s; }

uint64_t orc_azar_next(uint64_t *st) {
    uint64_t x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return x * 0x2545F4914F6CDD1Dull;
}

static float azar_uniform(uint64_t *st) {
    uint64_t bits = orc_azar_next(st) >> 40;
    return ((float)bits + 1.0f) / 16777216.0f;
}

/* Box-Muller pair, src/daiss.rs:350-356 */
void orc_azar_normals(uint64_t *st, float sigma, float *a, float *b) {
    float u1 = azar_uniform(st), u2 = azar_uniform(st);
    float r = sigma * sqrtf(-2.0f * logf(u1));
    float ang = 6.28318530717958647692f * u2;
    *a = r * cosf(ang);
    *b = r * sinf(ang);
}

/* ───────────────────────── sampler ───────────────────────── */

struct orc_sampler {
    uint64_t state;
    float temperature, top_p;
};

orc_sampler *orc_sampler_new(uint64_t seed, float temperature, float top_p) {
    orc_sampler *s = (orc_sampler *)calloc(1, sizeof *s);
    s->state = orc_azar_seed(seed);
    s->temperature = temperature;
    s->top_p = top_p < 0.0f ? 0.0f : (top_p > 1.0f ? 1.0f : top_p);
    return s;
}
void orc_sampler_free(orc_sampler *s) { free(s); }
uint64_t orc_sampler_state(const orc_sampler *s) { return s->state; }

/* first max wins ties (src/sampler.rs:129-137) */
uint32_t orc_argmax(const float *v, size_t n) {
    size_t best = 0;
    for (size_t i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return (uint32_t)best;
}

static const float *g_sort_probs;
/* descending probability; ties by index so the order is deterministic (the
 * reference's unstable sort leaves tie order unspecified) */
static int cmp_desc(const void *a, const void *b) {
    uint32_t i = *(const uint32_t *)a, j = *(const uint32_t *)b;
    float pi = g_sort_probs[i], pj = g_sort_probs[j];
    if (pi > pj) return -1;
    if (pi < pj) return 1;
    return i < j ? -1 : (i > j ? 1 : 0);
}

static uint32_t sample_walk(const float *probs, const uint32_t *idx, size_t n, float u) {
    float acc = 0.0f;
    uint32_t last = 0;
    for (size_t i = 0; i < n; i++) {
        acc += probs[idx[i]];
        last = idx[i];
        if (acc > u) return idx[i];
    }
    return last;
}

/* src/sampler.rs:61-126 */
uint32_t orc_sampler_pick(orc_sampler *s, const float *logits, size_t n) {
    if (n == 0) return 0;
    if (s->temperature <= 0.0f) return orc_argmax(logits, n);
    float u = (float)(orc_azar_next(&s->state) >> 40) / 16777216.0f;
    float *probs = (float *)malloc(sizeof(float) * n);
    float inv = 1.0f / s->temperature;
    for (size_t i = 0; i < n; i++) probs[i] = logits[i] * inv;
    orc_softmax(probs, n, n);
    uint32_t *order = (uint32_t *)malloc(sizeof(uint32_t) * n);
    for (size_t i = 0; i < n; i++) order[i] = (uint32_t)i;
    uint32_t r;
    if (s->top_p >= 1.0f) {
        r = sample_walk(probs, order, n, u);
    } else {
        size_t k = n < 1024 ? n : 1024;
        g_sort_probs = probs;
        /* the k most probable, sorted (select_nth_unstable + sort) */
        qsort(order, n, sizeof(uint32_t), cmp_desc);
        float mass = 0.0f;
        for (size_t i = 0; i < k; i++) mass += probs[order[i]];
        size_t len = k;
        if (mass < s->top_p && k < n) len = n; /* flat: the full order */
        float acc = 0.0f;
        size_t cut = len;
        for (size_t i = 0; i < len; i++) {
            acc += probs[order[i]];
            if (acc >= s->top_p) { cut = i + 1; break; }
        }
        float total = 0.0f;
        for (size_t i = 0; i < cut; i++) total += probs[order[i]];
        r = sample_walk(probs, order, cut, u * total);
    }
    free(order);
    free(probs);
    return r;
}

/* ───────────────────────── GGUF ───────────────────────── */

typedef struct {
    char name[96];
    uint64_t dims[4];
    int nd, type;
    uint64_t offset;
    size_t nbytes;
} orc_tensor;

typedef struct {
    char key[96];
    int kind; /* 0 none, 1 int, 2 float */
    uint64_t i;
    double f;
} orc_meta;

typedef struct {
    uint8_t *map;
    size_t size;
    uint64_t data_start;
    orc_tensor *t;
    int nt;
    orc_meta *meta;
    int nmeta;
} orc_gguf;

typedef struct {
    const uint8_t *p, *end;
    int bad;
} rd_t;

static uint64_t rd_n(rd_t *r, int n) {
    if (r->p + n > r->end) { r->bad = 1; return 0; }
    uint64_t v = 0;
    for (int i = 0; i < n; i++) v |= (uint64_t)r->p[i] << (8 * i);
    r->p += n;
    return v;
}

static void rd_str(rd_t *r, char *dst, size_t cap) {
    uint64_t len = rd_n(r, 8);
    if (r->bad || r->p + len > r->end) { r->bad = 1; return; }
    if (dst) {
        size_t c = len < cap - 1 ? (size_t)len : cap - 1;
        memcpy(dst, r->p, c);
        dst[c] = 0;
    }
    r->p += len;
}

static void rd_value(rd_t *r, uint32_t type, orc_meta *m) {
    uint64_t bits;
    switch (type) {
    case 0: m->kind = 1; m->i = rd_n(r, 1); break;
    case 1: m->kind = 1; m->i = (uint64_t)(int64_t)(int8_t)rd_n(r, 1); break;
    case 2: m->kind = 1; m->i = rd_n(r, 2); break;
    case 3: m->kind = 1; m->i = (uint64_t)(int64_t)(int16_t)rd_n(r, 2); break;
    case 4: m->kind = 1; m->i = rd_n(r, 4); break;
    case 5: m->kind = 1; m->i = (uint64_t)(int64_t)(int32_t)rd_n(r, 4); break;
    case 6: { uint32_t u = (uint32_t)rd_n(r, 4); float f; memcpy(&f, &u, 4); m->kind = 2; m->f = f; break; }
    case 7: rd_n(r, 1); m->kind = 0; break;
    case 8: rd_str(r, NULL, 0); m->kind = 0; break;
    case 9: {
        uint32_t it = (uint32_t)rd_n(r, 4);
        uint64_t cnt = rd_n(r, 8);
        orc_meta tmp;
        for (uint64_t i = 0; i < cnt && !r->bad; i++) rd_value(r, it, &tmp);
        m->kind = 0;
        break;
    }
    case 10: m->kind = 1; m->i = rd_n(r, 8); break;
    case 11: m->kind = 1; m->i = rd_n(r, 8); break;
    case 12: bits = rd_n(r, 8); memcpy(&m->f, &bits, 8); m->kind = 2; break;
    default: r->bad = 1;
    }
}

static void gguf_close(orc_gguf *g) {
    if (g->map) munmap(g->map, g->size);
    free(g->t);
    free(g->meta);
    memset(g, 0, sizeof *g);
}

/* src/gguf.rs:274-342 (header) and :413-437 (bounds-checked tensor bytes) */
static int gguf_open(const char *path, orc_gguf *g) {
    memset(g, 0, sizeof *g);
    int fd = open(path, O_RDONLY);
    if (fd < 0) { set_err("cannot open %s: %s", path, strerror(errno)); return -1; }
    struct stat st;
    fstat(fd, &st);
    g->size = (size_t)st.st_size;
    g->map = (uint8_t *)mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (g->map == MAP_FAILED) { g->map = NULL; set_err("mmap failed"); return -1; }
    rd_t r = {g->map, g->map + g->size, 0};
    if (g->size < 4 || memcmp(g->map, "GGUF", 4)) { set_err("not a GGUF file"); gguf_close(g); return -1; }
    r.p += 4;
    uint32_t ver = (uint32_t)rd_n(&r, 4);
    if (ver != 2 && ver != 3) { set_err("GGUF version %u", ver); gguf_close(g); return -1; }
    uint64_t nt = rd_n(&r, 8), nm = rd_n(&r, 8);
    if (nt > 100000 || nm > 100000) { set_err("absurd counts"); gguf_close(g); return -1; }
    g->meta = (orc_meta *)calloc(nm + 1, sizeof(orc_meta));
    g->t = (orc_tensor *)calloc(nt + 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < nm && !r.bad; i++) {
        rd_str(&r, g->meta[i].key, sizeof g->meta[i].key);
        uint32_t ty = (uint32_t)rd_n(&r, 4);
        rd_value(&r, ty, &g->meta[i]);
    }
    g->nmeta = (int)nm;
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        orc_tensor *t = &g->t[i];
        rd_str(&r, t->name, sizeof t->name);
        t->nd = (int)rd_n(&r, 4);
        if (t->nd > 4) { set_err("%s: %d dims", t->name, t->nd); gguf_close(g); return -1; }
        uint64_t elems = 1;
        for (int d = 0; d < t->nd; d++) { t->dims[d] = rd_n(&r, 8); elems *= t->dims[d]; }
        t->type = (int)rd_n(&r, 4);
        t->offset = rd_n(&r, 8);
        int vpb = orc_values_per_block(t->type);
        if (!vpb) { set_err("%s: unknown type %d", t->name, t->type); gguf_close(g); return -1; }
        t->nbytes = (size_t)(elems / (uint64_t)vpb) * (size_t)orc_bytes_per_block(t->type);
    }
    g->nt = (int)nt;
    if (r.bad) { set_err("truncated header"); gguf_close(g); return -1; }
    uint64_t align = 32;
    for (int i = 0; i < g->nmeta; i++)
        if (!strcmp(g->meta[i].key, "general.alignment") && g->meta[i].kind == 1 && g->meta[i].i > 0) align = g->meta[i].i;
    uint64_t pos = (uint64_t)(r.p - g->map);
    g->data_start = (pos + align - 1) / align * align;
    for (int i = 0; i < g->nt; i++) {
        if (g->data_start + g->t[i].offset + g->t[i].nbytes > g->size) {
            set_err("%s: data beyond the end of the file", g->t[i].name);
            gguf_close(g);
            return -1;
        }
    }
    return 0;
}

static const orc_meta *gguf_meta(const orc_gguf *g, const char *key) {
    for (int i = 0; i < g->nmeta; i++)
        if (!strcmp(g->meta[i].key, key)) return &g->meta[i];
    return NULL;
}
static const orc_tensor *gguf_tensor(const orc_gguf *g, const char *name) {
    for (int i = 0; i < g->nt; i++)
        if (!strcmp(g->t[i].name, name)) return &g->t[i];
    return NULL;
}
static const uint8_t *gguf_data(const orc_gguf *g, const orc_tensor *t) { return g->map + g->data_start + t->offset; }

/* ───────────────────────── model ───────────────────────── */

typedef struct {
    const orc_tensor *attn_norm, *q, *qb, *k, *kb, *v, *vb, *o, *ffn_norm, *gate, *up, *down;
} orc_layer;

struct orc_model {
    orc_gguf g;
    orc_config cfg;
    orc_layer *layers;
    const orc_tensor *embd, *out, *out_norm;
    float *cos_t, *sin_t;
    int has_eos;
    uint32_t eos;
};

struct orc_cache {
    int n_layer, kv_dim, len, cap;
    float **k, **v;
};

void orc_model_close(orc_model *m) {
    if (!m) return;
    gguf_close(&m->g);
    free(m->layers);
    free(m->cos_t);
    free(m->sin_t);
    free(m);
}

/* src/forward.rs:187-266: qwen2.* keys; Q/K/V biases required; output tied
 * to token_embd when output.weight is absent. */
orc_model *orc_model_open(const char *path) {
    orc_model *m = (orc_model *)calloc(1, sizeof *m);
    if (gguf_open(path, &m->g)) { free(m); return NULL; }
    const char *ik[] = {"qwen2.block_count", "qwen2.embedding_length", "qwen2.attention.head_count",
                        "qwen2.attention.head_count_kv", "qwen2.context_length"};
    uint64_t iv[5];
    for (int i = 0; i < 5; i++) {
        const orc_meta *me = gguf_meta(&m->g, ik[i]);
        if (!me || me->kind != 1) { set_err("missing metadata %s", ik[i]); orc_model_close(m); return NULL; }
        iv[i] = me->i;
    }
    m->cfg.n_layer = (int)iv[0];
    m->cfg.dim = (int)iv[1];
    m->cfg.n_head = (int)iv[2];
    m->cfg.n_head_kv = (int)iv[3];
    m->cfg.ctx = (int)iv[4];
    const orc_meta *me = gguf_meta(&m->g, "qwen2.attention.layer_norm_rms_epsilon");
    m->cfg.eps = me ? (float)(me->kind == 2 ? me->f : (double)me->i) : 1e-6f;
    me = gguf_meta(&m->g, "qwen2.rope.freq_base");
    m->cfg.rope_base = me ? (float)(me->kind == 2 ? me->f : (double)me->i) : 10000.0f;
    me = gguf_meta(&m->g, "tokenizer.ggml.eos_token_id");
    if (me && me->kind == 1) { m->has_eos = 1; m->eos = (uint32_t)me->i; }
    if (m->cfg.n_head <= 0 || m->cfg.dim % m->cfg.n_head) { set_err("bad head count"); orc_model_close(m); return NULL; }
    m->cfg.head_dim = m->cfg.dim / m->cfg.n_head;
    m->embd = gguf_tensor(&m->g, "token_embd.weight");
    if (!m->embd) { set_err("missing tensor token_embd.weight"); orc_model_close(m); return NULL; }
    m->cfg.vocab = (int)m->embd->dims[1];
    m->out = gguf_tensor(&m->g, "output.weight");
    m->cfg.tied = m->out == NULL;
    if (!m->out) m->out = m->embd;
    m->out_norm = gguf_tensor(&m->g, "output_norm.weight");
    if (!m->out_norm) { set_err("missing tensor output_norm.weight"); orc_model_close(m); return NULL; }
    m->layers = (orc_layer *)calloc((size_t)m->cfg.n_layer, sizeof(orc_layer));
    for (int i = 0; i < m->cfg.n_layer; i++) {
        const char *names[12] = {"attn_norm.weight", "attn_q.weight", "attn_q.bias", "attn_k.weight", "attn_k.bias",
                                 "attn_v.weight", "attn_v.bias", "attn_output.weight", "ffn_norm.weight",
                                 "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
        const orc_tensor **slots[12] = {&m->layers[i].attn_norm, &m->layers[i].q, &m->layers[i].qb, &m->layers[i].k,
                                        &m->layers[i].kb, &m->layers[i].v, &m->layers[i].vb, &m->layers[i].o,
                                        &m->layers[i].ffn_norm, &m->layers[i].gate, &m->layers[i].up, &m->layers[i].down};
        for (int j = 0; j < 12; j++) {
            char nm[96];
            snprintf(nm, sizeof nm, "blk.%d.%s", i, names[j]);
            *slots[j] = gguf_tensor(&m->g, nm);
            if (!*slots[j]) { set_err("missing tensor %s", nm); orc_model_close(m); return NULL; }
        }
    }
    m->cfg.ffn = (int)m->layers[0].gate->dims[1];
    int half = m->cfg.head_dim / 2;
    m->cos_t = (float *)malloc(sizeof(float) * (size_t)m->cfg.ctx * half);
    m->sin_t = (float *)malloc(sizeof(float) * (size_t)m->cfg.ctx * half);
    orc_rope_tables(m->cfg.head_dim, m->cfg.rope_base, m->cfg.ctx, m->cos_t, m->sin_t);
    return m;
}

void orc_model_config(const orc_model *m, orc_config *out) { *out = m->cfg; }

orc_cache *orc_cache_new(const orc_model *m) {
    orc_cache *c = (orc_cache *)calloc(1, sizeof *c);
    c->n_layer = m->cfg.n_layer;
    c->kv_dim = m->cfg.n_head_kv * m->cfg.head_dim;
    c->k = (float **)calloc((size_t)c->n_layer, sizeof(float *));
    c->v = (float **)calloc((size_t)c->n_layer, sizeof(float *));
    return c;
}
void orc_cache_free(orc_cache *c) {
    if (!c) return;
    for (int i = 0; i < c->n_layer; i++) { free(c->k[i]); free(c->v[i]); }
    free(c->k);
    free(c->v);
    free(c);
}
int orc_cache_len(const orc_cache *c) { return c->len; }
void orc_cache_truncate(orc_cache *c, int n) {
    if (n < c->len) c->len = n < 0 ? 0 : n;
}
void orc_cache_clear(orc_cache *c) { c->len = 0; }
const float *orc_cache_layer(const orc_cache *c, int layer, int is_v) { return is_v ? c->v[layer] : c->k[layer]; }

static void cache_reserve(orc_cache *c, int need) {
    if (need <= c->cap) return;
    int cap = c->cap ? c->cap : 16;
    while (cap < need) cap *= 2;
    for (int i = 0; i < c->n_layer; i++) {
        c->k[i] = (float *)realloc(c->k[i], sizeof(float) * (size_t)cap * c->kv_dim);
        c->v[i] = (float *)realloc(c->v[i], sizeof(float) * (size_t)cap * c->kv_dim);
    }
    c->cap = cap;
}

orc_cache *orc_cache_prefix(const orc_cache *c, int n) {
    orc_cache *p = (orc_cache *)calloc(1, sizeof *p);
    p->n_layer = c->n_layer;
    p->kv_dim = c->kv_dim;
    p->k = (float **)calloc((size_t)p->n_layer, sizeof(float *));
    p->v = (float **)calloc((size_t)p->n_layer, sizeof(float *));
    if (n > c->len) n = c->len;
    if (n < 0) n = 0;
    cache_reserve(p, n > 0 ? n : 1);
    for (int i = 0; i < p->n_layer; i++) {
        if (n > 0) {
            memcpy(p->k[i], c->k[i], sizeof(float) * (size_t)n * c->kv_dim);
            memcpy(p->v[i], c->v[i], sizeof(float) * (size_t)n * c->kv_dim);
        }
    }
    p->len = n;
    return p;
}

static int project(orc_model *m, const float *x, int t, const orc_tensor *w, const orc_tensor *bias, float *dst) {
    int k = (int)w->dims[0], n = (int)w->dims[1];
    if (orc_matmul_auto(t, k, n, x, gguf_data(&m->g, w), w->nbytes, w->type, dst)) return -1;
    if (bias) {
        const float *b = (const float *)gguf_data(&m->g, bias); /* f32, forward.rs:316-322 */
        for (int f = 0; f < t; f++)
            for (int j = 0; j < n; j++) dst[(size_t)f * n + j] += b[j];
    }
    return 0;
}

/* Several projections of one token's x (q, k, v; gate, up) as ONE parallel
 * region over all their 32-row tasks, x quantized once per sub-block size
 * (src/forward.rs:333-368, src/ops.rs:895-1009). Each matrix takes the fused
 * kernel when hay_fusionado allows it and the buffered path otherwise
 * (src/ops.rs:956-1006); the values are those of separate project() calls,
 * bit for bit (the reference's own check, src/ops.rs:1613-1670). */
#define MANY_MAX 3
typedef struct {
    int nw;
    mm_ctx mm[MANY_MAX];
    size_t first_task[MANY_MAX + 1];
} many_ctx;

static void many_task(void *c_, size_t b, size_t e) {
    many_ctx *c = (many_ctx *)c_;
    for (size_t task = b; task < e; task++) {
        int i = 0;
        while (task >= c->first_task[i + 1]) i++;
        const size_t r0 = (task - c->first_task[i]) * 32, n = (size_t)c->mm[i].n;
        mm_task(&c->mm[i], r0, r0 + 32 < n ? r0 + 32 : n);
    }
}

/* 0: one call per matrix, as the reference's COSXAMIX_SIN_VARIAS (src/forward.rs:340-342) */
static int g_varias = 1;
void orc_set_varias(int on) { g_varias = on != 0; }

static int project_many(orc_model *m, const float *x, int t, const orc_tensor *const *ws,
                        const orc_tensor *const *bs, float *const *dsts, int nw) {
    int k = (int)ws[0]->dims[0], many = g_varias && t == 1 && nw <= MANY_MAX;
    for (int i = 0; i < nw && many; i++) {
        const int ty = ws[i]->type, sub = orc_sub_block(ty), vpb = orc_values_per_block(ty);
        many = (int)ws[i]->dims[0] == k && sub != 0 && k % vpb == 0 && k % sub == 0 &&
               ws[i]->nbytes >= (size_t)ws[i]->dims[1] * (size_t)(k / vpb) * (size_t)orc_bytes_per_block(ty);
    }
    if (!many) {
        for (int i = 0; i < nw; i++)
            if (project(m, x, t, ws[i], bs[i], dsts[i])) return -1;
        return 0;
    }
    int8_t q16[k], q32[k];
    float e16[k / 16], s16[k / 16], e32[k / 32], s32[k / 32];
    int need16 = 0, need32 = 0;
    for (int i = 0; i < nw; i++) {
        if (orc_sub_block(ws[i]->type) == 16) need16 = 1;
        else need32 = 1;
    }
    if (need16) orc_quantize_i8(x, (size_t)k, 16, q16, e16, s16);
    if (need32) orc_quantize_i8(x, (size_t)k, 32, q32, e32, s32);
    many_ctx c;
    c.nw = nw;
    c.first_task[0] = 0;
    for (int i = 0; i < nw; i++) {
        const int ty = ws[i]->type, sub = orc_sub_block(ty), n = (int)ws[i]->dims[1];
        const int s16b = sub == 16;
        const size_t rb = (size_t)(k / orc_values_per_block(ty)) * (size_t)orc_bytes_per_block(ty);
        c.mm[i] = (mm_ctx){1, k, n, sub, ty, fused_available(ty, k) ? ORC_PATH_FUSED : ORC_PATH_BUFFERED, rb,
                           (size_t)(k / 256), gguf_data(&m->g, ws[i]), s16b ? q16 : q32, s16b ? e16 : e32,
                           s16b ? s16 : s32, dsts[i]};
        c.first_task[i + 1] = c.first_task[i] + ((size_t)n + 31) / 32;
    }
    par_for(c.first_task[nw], 1, many_task, &c);
    for (int i = 0; i < nw; i++)
        if (bs[i]) {
            const float *b = (const float *)gguf_data(&m->g, bs[i]);
            for (int j = 0; j < (int)ws[i]->dims[1]; j++) dsts[i][j] += b[j];
        }
    return 0;
}

static int read_vec(orc_model *m, const orc_tensor *t, float *dst, size_t n) {
    return orc_dequantize(t->type, gguf_data(&m->g, t), t->nbytes, n, dst);
}

/* src/forward.rs:375-505 */
int orc_forward(orc_model *m, orc_cache *c, const uint32_t *tokens, int t, float *logits) {
    const orc_config *cfg = &m->cfg;
    if (t <= 0) { set_err("no tokens to process"); return -1; }
    /* kernels::rmsnorm is the f32 AVX2 one on an AVX2 host (src/kernels/mod.rs:511) */
    void (*norm)(float *, const float *, const float *, size_t, float) =
        g_backend == ORC_BACKEND_X86 ? orc_x86_rmsnorm : orc_rmsnorm;
    int total = c->len + t;
    if (total > cfg->ctx) { set_err("%d tokens exceed the context of %d", total, cfg->ctx); return -1; }
    int D = cfg->dim, hd = cfg->head_dim, H = cfg->n_head, KV = cfg->n_head_kv, F = cfg->ffn;
    int kvd = KV * hd;
    size_t T = (size_t)t;
    float *x = (float *)calloc(T * D, sizeof(float));
    float *xn = (float *)calloc(T * D, sizeof(float));
    float *w = (float *)calloc((size_t)(D > F ? D : F), sizeof(float));
    float *q = (float *)calloc(T * D, sizeof(float));
    float *kk = (float *)calloc(T * kvd, sizeof(float));
    float *vv = (float *)calloc(T * kvd, sizeof(float));
    float *att = (float *)calloc(T * D, sizeof(float));
    float *proj = (float *)calloc(T * D, sizeof(float));
    float *gate = (float *)calloc(T * F, sizeof(float));
    float *up = (float *)calloc(T * F, sizeof(float));
    float *act = (float *)calloc(T * F, sizeof(float));
    int rc = -1;

    /* embeddings: one dequantized row per token (forward.rs:389-405) */
    int vpb = orc_values_per_block(m->embd->type);
    size_t row_bytes = (size_t)D / (size_t)vpb * (size_t)orc_bytes_per_block(m->embd->type);
    for (int i = 0; i < t; i++) {
        if ((int)tokens[i] >= cfg->vocab) { set_err("token %u beyond vocab %d", tokens[i], cfg->vocab); goto done; }
        if (orc_dequantize(m->embd->type, gguf_data(&m->g, m->embd) + tokens[i] * row_bytes, row_bytes, (size_t)D, x + (size_t)i * D)) goto done;
    }
    cache_reserve(c, total);
    for (int l = 0; l < cfg->n_layer; l++) {
        const orc_layer *L = &m->layers[l];
        read_vec(m, L->attn_norm, w, (size_t)D);
        for (int i = 0; i < t; i++) norm(xn + (size_t)i * D, x + (size_t)i * D, w, (size_t)D, cfg->eps);
        {
            const orc_tensor *ws[3] = {L->q, L->k, L->v}, *bs[3] = {L->qb, L->kb, L->vb};
            float *ds[3] = {q, kk, vv};
            if (project_many(m, xn, t, ws, bs, ds, 3)) goto done;
        }
        orc_rope(q, t, H, hd, m->cos_t, m->sin_t, cfg->ctx, c->len);
        orc_rope(kk, t, KV, hd, m->cos_t, m->sin_t, cfg->ctx, c->len);
        memcpy(c->k[l] + (size_t)c->len * kvd, kk, sizeof(float) * T * kvd);
        memcpy(c->v[l] + (size_t)c->len * kvd, vv, sizeof(float) * T * kvd);
        if (orc_attention(q, c->k[l], c->v[l], t, total, H, KV, hd, att)) goto done;
        if (project(m, att, t, L->o, NULL, proj)) goto done;
        for (size_t i = 0; i < T * D; i++) x[i] += proj[i];
        read_vec(m, L->ffn_norm, w, (size_t)D);
        for (int i = 0; i < t; i++) norm(xn + (size_t)i * D, x + (size_t)i * D, w, (size_t)D, cfg->eps);
        {
            const orc_tensor *ws[2] = {L->gate, L->up}, *bs[2] = {NULL, NULL};
            float *ds[2] = {gate, up};
            if (project_many(m, xn, t, ws, bs, ds, 2)) goto done;
        }
        orc_silu(act, gate, T * F);
        for (size_t i = 0; i < T * F; i++) act[i] *= up[i];
        if (project(m, act, t, L->down, NULL, proj)) goto done;
        for (size_t i = 0; i < T * D; i++) x[i] += proj[i];
    }
    read_vec(m, m->out_norm, w, (size_t)D);
    norm(xn, x + (size_t)(t - 1) * D, w, (size_t)D, cfg->eps);
    if (project(m, xn, 1, m->out, NULL, logits)) goto done;
    c->len = total;
    rc = 0;
done:
    free(x); free(xn); free(w); free(q); free(kk); free(vv); free(att); free(proj); free(gate); free(up); free(act);
    return rc;
}

/* src/forward.rs:533-559 */
int orc_generate(orc_model *m, orc_cache *c, const uint32_t *prompt, int n_prompt, int max_new, orc_sampler *s,
                 uint32_t *out, int *n_out) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)m->cfg.vocab);
    int n = 0, rc = orc_forward(m, c, prompt, n_prompt, logits);
    for (int i = 0; rc == 0 && i < max_new; i++) {
        uint32_t t = orc_sampler_pick(s, logits, (size_t)m->cfg.vocab);
        if (m->has_eos && t == m->eos) break;
        out[n++] = t;
        if (c->len >= m->cfg.ctx) break;
        rc = orc_forward(m, c, &t, 1, logits);
    }
    free(logits);
    *n_out = n;
    return rc;
}

/* Test infrastructure for the timed CPU baseline: fill positions [len, n) of
 * every layer with seeded values in [-1, 1) so a decode step sees a context
 * of n positions without paying for an n-token CPU prefill. The values only
 * shape the attention's cost, never a parity check. */
void orc_cache_fill(orc_cache *c, int n, uint64_t seed) {
    if (n <= c->len) return;
    cache_reserve(c, n);
    uint64_t st = orc_azar_seed(seed);
    for (int l = 0; l < c->n_layer; l++)
        for (size_t i = (size_t)c->len * c->kv_dim; i < (size_t)n * c->kv_dim; i++) {
            c->k[l][i] = (float)(orc_azar_next(&st) >> 40) / 8388608.0f - 1.0f;
            c->v[l][i] = (float)(orc_azar_next(&st) >> 40) / 8388608.0f - 1.0f;
        }
    c->len = n;
}

/* the host C library's expf over an array (the function the reference's
 * f32::exp calls); used to check the device exp */
void orc_expf(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = expf(x[i]);
}
