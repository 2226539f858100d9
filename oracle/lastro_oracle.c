/*
 * lastro_oracle.c -- TEST INFRASTRUCTURE ONLY (checker + timed CPU baseline).
 *
 * A C restatement of the reference's CPU decode path.  Every function names the
 * reference file:line it follows (paths inside brenoperucchi/lastro-rust).  The
 * product library never links this file; tests, the smoke check and bench.py's
 * cpu_baseline leg load it through oracle/oracle.py.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off; the AVX2 dot is compiled
 * with a target attribute and chosen at run time, like cpu.rs:54-62).
 */
#define _GNU_SOURCE
#include "lastro_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------------- */
/* bf16 <-> f32                                                                */
/* ------------------------------------------------------------------------- */

/* cpu.rs:12-15: bf16 -> f32 is a 16-bit shift */
static inline float bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float lo_bf16_to_f32(uint16_t b) { return bf2f(b); }

/* round-to-nearest-even, as half::bf16::from_f32 (finite inputs) */
uint16_t lo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ------------------------------------------------------------------------- */
/* synthetic generator: identical formula in lastro-rust_b200/csrc/synth.cu    */
/* ------------------------------------------------------------------------- */
#define LO_GOLDEN 0x9E3779B97F4A7C15ull

uint64_t lo_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t lo_tensor_seed(uint64_t base, int32_t layer, int32_t kind) {
    return lo_mix64(base * LO_GOLDEN + ((uint64_t)(uint32_t)(layer + 1) << 8) + (uint64_t)kind + 1u);
}

float lo_synth_scale(float stddev) { return stddev / 37837.2265f; }

float lo_synth_value(uint64_t seed, uint64_t idx, float scale) {
    uint64_t h = lo_mix64(seed + (idx + 1u) * LO_GOLDEN);
    int32_t s = (int32_t)(h & 0xffffu) + (int32_t)((h >> 16) & 0xffffu) + (int32_t)((h >> 32) & 0xffffu) +
                (int32_t)(h >> 48);
    return (float)(s - 131070) * scale;
}

typedef struct {
    void *out;
    size_t n;
    uint64_t seed;
    float scale, mean;
    int bf16;
    int part, parts;
} synth_job;

static void *synth_thread(void *arg) {
    synth_job *j = (synth_job *)arg;
    size_t per = (j->n + (size_t)j->parts - 1) / (size_t)j->parts;
    size_t i0 = per * (size_t)j->part, i1 = i0 + per < j->n ? i0 + per : j->n;
    for (size_t i = i0; i < i1; ++i) {
        float v = lo_synth_value(j->seed, i, j->scale);
        if (j->mean != 0.0f) v = v + j->mean;
        if (j->bf16)
            ((uint16_t *)j->out)[i] = lo_f32_to_bf16(v);
        else
            ((float *)j->out)[i] = v;
    }
    return NULL;
}

static void synth_run(void *out, size_t n, uint64_t seed, float stddev, float mean, int bf16, int threads) {
    if (threads < 1) threads = 1;
    if (n < (size_t)1 << 16) threads = 1;
    if (threads > 64) threads = 64;
    synth_job jobs[64];
    pthread_t th[64];
    float scale = lo_synth_scale(stddev);
    for (int t = 0; t < threads; ++t) {
        synth_job j = {out, n, seed, scale, mean, bf16, t, threads};
        jobs[t] = j;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&th[t], NULL, synth_thread, &jobs[t]);
    synth_thread(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(th[t], NULL);
}

void lo_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float stddev, float mean, int threads) {
    synth_run(out, n, seed, stddev, mean, 1, threads);
}

void lo_synth_f32(float *out, size_t n, uint64_t seed, float stddev, float mean, int threads) {
    synth_run(out, n, seed, stddev, mean, 0, threads);
}

void lo_synth_tokens(int32_t *out, size_t n, uint64_t seed, int32_t vocab) {
    for (size_t i = 0; i < n; ++i) out[i] = (int32_t)(lo_mix64(seed + (i + 1u) * LO_GOLDEN) % (uint64_t)vocab);
}

/* tests/common/mod.rs:28-38 of the reference: xorshift values in [-1, 1), the
 * deterministic data of the reference's own tests */
void lo_ref_values(float *out, size_t n, uint64_t seed) {
    uint64_t s = seed | 1u;
    for (size_t i = 0; i < n; ++i) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        out[i] = ((float)(s >> 40) / (float)(1u << 23)) * 2.0f - 1.0f;
    }
}

/* ------------------------------------------------------------------------- */
/* thread pool -- pool.rs:1-120: fixed workers that spin briefly then sleep,    */
/* tasks claimed through an atomic counter, the caller takes part.             */
/* ------------------------------------------------------------------------- */
typedef void (*lo_task_fn)(void *ctx, size_t task);

struct lo_pool {
    int n; /* participants including the caller */
    pthread_t *th;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    _Atomic uint64_t gen;
    _Atomic int stop;
    lo_task_fn fn;
    void *ctx;
    size_t tasks;
    _Atomic size_t next;
    _Atomic int finished;
};

static inline void cpu_relax(void) {
#if defined(__x86_64__)
    _mm_pause();
#endif
}

static void pool_take(lo_pool *p) {
    for (;;) {
        size_t t = atomic_fetch_add_explicit(&p->next, 1, memory_order_relaxed);
        if (t >= p->tasks) return;
        p->fn(p->ctx, t);
    }
}

static void *pool_worker(void *arg) {
    lo_pool *p = (lo_pool *)arg;
    uint64_t seen = 0;
    for (;;) {
        uint64_t g;
        int spins = 0;
        while ((g = atomic_load_explicit(&p->gen, memory_order_acquire)) == seen) {
            if (atomic_load_explicit(&p->stop, memory_order_acquire)) return NULL;
            if (++spins < (1 << 16)) {
                cpu_relax();
                continue;
            }
            pthread_mutex_lock(&p->mu);
            while (atomic_load_explicit(&p->gen, memory_order_acquire) == seen &&
                   !atomic_load_explicit(&p->stop, memory_order_acquire))
                pthread_cond_wait(&p->cv, &p->mu);
            pthread_mutex_unlock(&p->mu);
            spins = 0;
        }
        if (atomic_load_explicit(&p->stop, memory_order_acquire)) return NULL;
        seen = g;
        pool_take(p);
        atomic_fetch_add_explicit(&p->finished, 1, memory_order_release);
    }
}

lo_pool *lo_pool_create(int threads) {
    lo_pool *p = (lo_pool *)calloc(1, sizeof(lo_pool));
    if (!p) return NULL;
    p->n = threads < 1 ? 1 : threads;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv, NULL);
    atomic_init(&p->gen, 0);
    atomic_init(&p->stop, 0);
    atomic_init(&p->next, 0);
    atomic_init(&p->finished, 0);
    p->th = (pthread_t *)calloc((size_t)p->n, sizeof(pthread_t));
    for (int i = 1; i < p->n; ++i) pthread_create(&p->th[i], NULL, pool_worker, p);
    return p;
}

void lo_pool_destroy(lo_pool *p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    atomic_store_explicit(&p->stop, 1, memory_order_release);
    pthread_cond_broadcast(&p->cv);
    pthread_mutex_unlock(&p->mu);
    for (int i = 1; i < p->n; ++i) pthread_join(p->th[i], NULL);
    pthread_cond_destroy(&p->cv);
    pthread_mutex_destroy(&p->mu);
    free(p->th);
    free(p);
}

int lo_pool_threads(const lo_pool *p) { return p ? p->n : 1; }

/* pool.rs Pool::run: returns when every task has run */
static void pool_run(lo_pool *p, size_t tasks, lo_task_fn fn, void *ctx) {
    if (!p || p->n == 1 || tasks <= 1) {
        for (size_t t = 0; t < tasks; ++t) fn(ctx, t);
        return;
    }
    p->fn = fn;
    p->ctx = ctx;
    p->tasks = tasks;
    atomic_store_explicit(&p->next, 0, memory_order_relaxed);
    atomic_store_explicit(&p->finished, 0, memory_order_relaxed);
    pthread_mutex_lock(&p->mu);
    atomic_fetch_add_explicit(&p->gen, 1, memory_order_release);
    pthread_cond_broadcast(&p->cv);
    pthread_mutex_unlock(&p->mu);
    pool_take(p);
    while (atomic_load_explicit(&p->finished, memory_order_acquire) < p->n - 1) cpu_relax();
}

/* ------------------------------------------------------------------------- */
/* Q8_0 (no reference implementation): blocks of 32 int8    */
/* values with one fp16 scale, stored as 34 bytes (the scale, then the values);  */
/* a weight is scale * value, exact in f32.                                      */
/* ------------------------------------------------------------------------- */

/* f32 -> IEEE fp16, round to nearest even (finite inputs; overflow gives inf) */
uint16_t lo_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a >= 0x47800000u) return (uint16_t)(sign | 0x7c00u); /* |f| >= 65536: inf */
    if (a < 0x38800000u) {                                 /* below the smallest normal fp16: subnormal */
        if (a < 0x33000000u) return (uint16_t)sign;          /* rounds to zero */
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        int e = (int)(a >> 23);                               /* 103 .. 112 */
        int sh = 126 - e;                                     /* m >> sh is the subnormal mantissa, 14..23 */
        uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t r = a - 0x38000000u; /* rebias the exponent by 127 - 15 */
    uint32_t q = r >> 13, rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

float lo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, u;
    if (e == 0) {
        if (m == 0) {
            u = sign;
        } else { /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) {
                m <<= 1;
                ++sh;
            }
            u = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* synthetic Q8_0: element idx of the row-major matrix -> int8 uniform in [-127, 127];
 * block b (row-major over rows x cols/32) -> fp16 scale 1e-4 + u * 3.9e-3, u uniform in [0, 1) from 24 hash bits */
int8_t lo_synth_q8_value(uint64_t seed, uint64_t idx) {
    return (int8_t)((int32_t)(lo_mix64(seed + (idx + 1u) * LO_GOLDEN) % 255u) - 127);
}

uint16_t lo_synth_q8_scale(uint64_t seed, uint64_t block) {
    uint64_t h = lo_mix64((seed ^ 0xA5A5A5A5A5A5A5A5ull) + (block + 1u) * LO_GOLDEN);
    float u = (float)(h >> 40) * (1.0f / 16777216.0f);
    return lo_f32_to_f16(1e-4f + u * 3.9e-3f);
}

size_t lo_row_bytes(int32_t dtype, size_t cols) { return dtype == LO_W_Q8_0 ? cols / 32 * 34 : cols * 2; }

typedef struct {
    uint8_t *out;
    size_t rows, cols;
    uint64_t seed;
    int part, parts;
} q8_job;

static void *q8_thread(void *arg) {
    q8_job *j = (q8_job *)arg;
    size_t per = (j->rows + (size_t)j->parts - 1) / (size_t)j->parts;
    size_t r0 = per * (size_t)j->part, r1 = r0 + per < j->rows ? r0 + per : j->rows;
    size_t nb = j->cols / 32;
    for (size_t r = r0; r < r1; ++r)
        for (size_t b = 0; b < nb; ++b) {
            uint8_t *blk = j->out + (r * nb + b) * 34;
            uint16_t d = lo_synth_q8_scale(j->seed, r * nb + b);
            memcpy(blk, &d, 2);
            for (size_t i = 0; i < 32; ++i) blk[2 + i] = (uint8_t)lo_synth_q8_value(j->seed, r * j->cols + b * 32 + i);
        }
    return NULL;
}

void lo_synth_q8_0(uint8_t *out, size_t rows, size_t cols, uint64_t seed, int threads) {
    if (threads < 1) threads = 1;
    if (rows * cols < (size_t)1 << 16) threads = 1;
    if (threads > 64) threads = 64;
    q8_job jobs[64];
    pthread_t th[64];
    for (int t = 0; t < threads; ++t) {
        q8_job j = {out, rows, cols, seed, t, threads};
        jobs[t] = j;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&th[t], NULL, q8_thread, &jobs[t]);
    q8_thread(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* dot product -- cpu.rs:12-62                                               */
/* ------------------------------------------------------------------------- */

/* cpu.rs:17-26 dot_scalar: 4 accumulators over chunks of 4, then the tail */
static float dot_scalar(const uint16_t *w, const float *x, size_t n) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    size_t c = n & ~(size_t)3;
    for (size_t i = 0; i < c; i += 4)
        for (int j = 0; j < 4; ++j) acc[j] += bf2f(w[i + j]) * x[i + j];
    float tail = 0.0f;
    for (size_t i = c; i < n; ++i) tail += bf2f(w[i]) * x[i];
    return acc[0] + acc[1] + acc[2] + acc[3] + tail;
}

/* cpu.rs:28-53 dot_avx2, lane by lane: 4 vectors of 8 FMA accumulators over
 * blocks of 32, the same horizontal reduction, then dot_scalar on the rest. */
float lo_dot_portable(const uint16_t *w, const float *x, size_t n) {
    float acc[4][8];
    memset(acc, 0, sizeof(acc));
    size_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 8; ++l) acc[j][l] = fmaf(bf2f(w[i + 8 * j + l]), x[i + 8 * j + l], acc[j][l]);
    float s[8], s4[4];
    for (int l = 0; l < 8; ++l) s[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
    for (int l = 0; l < 4; ++l) s4[l] = s[l] + s[l + 4];
    float r = (s4[0] + s4[2]) + (s4[1] + s4[3]);
    return r + dot_scalar(w + i, x + i, n - i);
}

#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) static float dot_avx2(const uint16_t *w, const float *x, size_t n) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    size_t i = 0;
    for (; i + 32 <= n; i += 32) {
        for (int j = 0; j < 4; ++j) {
            __m128i raw = _mm_loadu_si128((const __m128i *)(w + i + 8 * j));
            __m256 wf = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(raw), 16));
            acc[j] = _mm256_fmadd_ps(wf, _mm256_loadu_ps(x + i + 8 * j), acc[j]);
        }
    }
    __m256 s = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 1));
    return _mm_cvtss_f32(h) + dot_scalar(w + i, x + i, n - i);
}

static int have_avx2(void) {
    static int v = -1;
    if (v < 0) {
        __builtin_cpu_init();
        v = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
    return v;
}
#endif

/* cpu.rs:54-62 */
float lo_dot(const uint16_t *w, const float *x, size_t n) {
#if defined(__x86_64__)
    if (have_avx2()) return dot_avx2(w, x, n);
#endif
    return lo_dot_portable(w, x, n);
}

/* The dequantised path (a Q8_0 row, n a multiple of 32): each weight is dequantised exactly (fp16 scale x int8) and
 * enters the same 4 x 8-lane FMA accumulators and horizontal reduction as lo_dot -- a block of 32 is one step. */
float lo_dot_q8_portable(const uint8_t *row, const float *x, size_t n) {
    float acc[4][8];
    memset(acc, 0, sizeof(acc));
    for (size_t b = 0; b * 32 < n; ++b) {
        const uint8_t *blk = row + b * 34;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        float d = lo_f16_to_f32(dh);
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 8; ++l) {
                float w = d * (float)(int8_t)blk[2 + 8 * j + l];
                acc[j][l] = fmaf(w, x[b * 32 + 8 * j + l], acc[j][l]);
            }
    }
    float s[8], s4[4];
    for (int l = 0; l < 8; ++l) s[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
    for (int l = 0; l < 4; ++l) s4[l] = s[l] + s[l + 4];
    return (s4[0] + s4[2]) + (s4[1] + s4[3]);
}

#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) static float dot_q8_avx2(const uint8_t *row, const float *x, size_t n) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (size_t b = 0; b * 32 < n; ++b) {
        const uint8_t *blk = row + b * 34;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        __m256 d = _mm256_set1_ps(lo_f16_to_f32(dh));
        for (int j = 0; j < 4; ++j) {
            __m128i raw = _mm_loadl_epi64((const __m128i *)(blk + 2 + 8 * j));
            __m256 w = _mm256_mul_ps(d, _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(raw)));
            acc[j] = _mm256_fmadd_ps(w, _mm256_loadu_ps(x + b * 32 + 8 * j), acc[j]);
        }
    }
    __m256 s = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 1));
    return _mm_cvtss_f32(h);
}
#endif

float lo_dot_q8(const uint8_t *row, const float *x, size_t n) {
#if defined(__x86_64__)
    if (have_avx2()) return dot_q8_avx2(row, x, n);
#endif
    return lo_dot_q8_portable(row, x, n);
}

/* a row of either weight type */
static inline float dot_w(int32_t dtype, const void *row, const float *x, size_t n) {
    return dtype == LO_W_Q8_0 ? lo_dot_q8((const uint8_t *)row, x, n) : lo_dot((const uint16_t *)row, x, n);
}

/* ------------------------------------------------------------------------- */
/* GEMV, SwiGLU, experts -- cpu.rs:64-150                                     */
/* ------------------------------------------------------------------------- */
#define ROWS_PER_TASK 16 /* cpu.rs:9-10 */

typedef struct {
    const void *w;
    int32_t dtype;
    int32_t rows, cols;
    const float *x;
    float *y;
} gemv_ctx;

static void gemv_task(void *c, size_t t) {
    gemv_ctx *g = (gemv_ctx *)c;
    size_t r0 = t * ROWS_PER_TASK, r1 = r0 + ROWS_PER_TASK;
    if (r1 > (size_t)g->rows) r1 = (size_t)g->rows;
    size_t rb = lo_row_bytes(g->dtype, (size_t)g->cols);
    for (size_t r = r0; r < r1; ++r) g->y[r] = dot_w(g->dtype, (const uint8_t *)g->w + r * rb, g->x, (size_t)g->cols);
}

/* cpu.rs:107-113 Cpu::gemv (rows in tasks of 16 over the pool, cpu.rs:95-106), either weight type */
void lo_gemv_w(lo_pool *p, int32_t dtype, const void *w, int32_t rows, int32_t cols, const float *x, float *y) {
    gemv_ctx g = {w, dtype, rows, cols, x, y};
    pool_run(p, ((size_t)rows + ROWS_PER_TASK - 1) / ROWS_PER_TASK, gemv_task, &g);
}

void lo_gemv(lo_pool *p, const uint16_t *w, int32_t rows, int32_t cols, const float *x, float *y) {
    lo_gemv_w(p, LO_W_BF16, w, rows, cols, x, y);
}

/* cpu.rs:64-68: a[j] = h[j] / (1 + exp(-h[j])) * h[I + j] */
void lo_swiglu(const float *h, int32_t inter, float *a) {
    for (int32_t j = 0; j < inter; ++j) a[j] = h[j] / (1.0f + expf(-h[j])) * h[inter + j];
}

typedef struct {
    const float *x;
    int32_t k, hidden, inter, dtype;
    const void *const *gate_up;
    const void *const *down;
    const float *weights;
    float *h; /* [k, 2I] */
    float *a; /* [k, I] */
    float *y; /* [H] */
    size_t per;
} experts_ctx;

static void experts_gu_task(void *c, size_t t) {
    experts_ctx *e = (experts_ctx *)c;
    size_t ex = t / e->per, ch = t % e->per;
    size_t rows = 2 * (size_t)e->inter;
    size_t r0 = ch * ROWS_PER_TASK, r1 = r0 + ROWS_PER_TASK;
    if (r1 > rows) r1 = rows;
    const uint8_t *w = (const uint8_t *)e->gate_up[ex];
    size_t rb = lo_row_bytes(e->dtype, (size_t)e->hidden);
    for (size_t r = r0; r < r1; ++r) e->h[ex * rows + r] = dot_w(e->dtype, w + r * rb, e->x, (size_t)e->hidden);
}

static void experts_down_task(void *c, size_t t) {
    experts_ctx *e = (experts_ctx *)c;
    size_t r0 = t * ROWS_PER_TASK, r1 = r0 + ROWS_PER_TASK;
    if (r1 > (size_t)e->hidden) r1 = (size_t)e->hidden;
    size_t rb = lo_row_bytes(e->dtype, (size_t)e->inter);
    for (size_t r = r0; r < r1; ++r) {
        float acc = 0.0f;
        for (int32_t j = 0; j < e->k; ++j)
            acc += e->weights[j] * dot_w(e->dtype, (const uint8_t *)e->down[j] + r * rb, e->a + (size_t)j * e->inter,
                                         (size_t)e->inter);
        e->y[r] = acc;
    }
}

/* cpu.rs:115-150 Cpu::experts: dispatch 1 = the 2I gate_up rows of every chosen
 * expert, SwiGLU per expert, dispatch 2 = each row of y summed over the experts
 * in routing order. */
void lo_experts_w(lo_pool *p, int32_t dtype, const float *x, int32_t k, const void *const *gate_up,
                  const void *const *down, const float *weights, int32_t hidden, int32_t inter, float *y) {
    memset(y, 0, sizeof(float) * (size_t)hidden);
    if (k == 0) return;
    float *h = (float *)malloc(sizeof(float) * (size_t)k * 2 * (size_t)inter);
    float *a = (float *)malloc(sizeof(float) * (size_t)k * (size_t)inter);
    experts_ctx e = {x, k, hidden, inter, dtype, gate_up, down, weights, h, a, y,
                     ((size_t)2 * inter + ROWS_PER_TASK - 1) / ROWS_PER_TASK};
    pool_run(p, (size_t)k * e.per, experts_gu_task, &e);
    for (int32_t j = 0; j < k; ++j) lo_swiglu(h + (size_t)j * 2 * inter, inter, a + (size_t)j * inter);
    pool_run(p, ((size_t)hidden + ROWS_PER_TASK - 1) / ROWS_PER_TASK, experts_down_task, &e);
    free(h);
    free(a);
}

void lo_experts(lo_pool *p, const float *x, int32_t k, const uint16_t *const *gate_up,
                const uint16_t *const *down, const float *weights, int32_t hidden, int32_t inter,
                float *y) {
    lo_experts_w(p, LO_W_BF16, x, k, (const void *const *)gate_up, (const void *const *)down, weights, hidden, inter, y);
}

/* ------------------------------------------------------------------------- */
/* routing -- block.rs:79-89                                                   */
/* ------------------------------------------------------------------------- */

/* f32::total_cmp: -1, 0, 1 */
int lo_total_cmp(float a, float b) {
    int32_t x, y;
    memcpy(&x, &a, 4);
    memcpy(&y, &b, 4);
    x ^= (int32_t)(((uint32_t)(x >> 31)) >> 1);
    y ^= (int32_t)(((uint32_t)(y >> 31)) >> 1);
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* block.rs:81-89: order by logit descending (total_cmp), ties by lower index,
 * keep k, softmax over the k with the first (largest) subtracted. */
void lo_routing(const float *logits, int32_t e, int32_t k, int32_t *ids, float *weights) {
    int32_t *order = (int32_t *)malloc(sizeof(int32_t) * (size_t)e);
    for (int32_t i = 0; i < e; ++i) order[i] = i;
    /* insertion sort with the comparator of block.rs:83 (stable, E is small) */
    for (int32_t i = 1; i < e; ++i) {
        int32_t v = order[i], j = i - 1;
        while (j >= 0) {
            int c = lo_total_cmp(logits[v], logits[order[j]]);
            if (c > 0 || (c == 0 && v < order[j])) {
                order[j + 1] = order[j];
                --j;
            } else
                break;
        }
        order[j + 1] = v;
    }
    float top = logits[order[0]];
    float *ex = (float *)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
    float sum = 0.0f;
    for (int32_t j = 0; j < k; ++j) {
        ex[j] = expf(logits[order[j]] - top);
    }
    for (int32_t j = 0; j < k; ++j) sum += ex[j];
    for (int32_t j = 0; j < k; ++j) {
        ids[j] = order[j];
        weights[j] = ex[j] / sum;
    }
    free(ex);
    free(order);
}

/* block.rs:56-62 HostLayer::forward_cpu, either weight type; `bias` (or NULL) is added to the router logits before
 * the routing (a workload knob of the batched benchmark, not part of Granite) */
static void block_forward_impl(lo_pool *p, int32_t dtype, const void *router, const void *gate_up, const void *down,
                               int32_t experts, int32_t hidden, int32_t inter, int32_t k, const float *x, float *y,
                               int32_t *ids, float *weights, float *logits_or_null, const float *bias) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)experts);
    lo_gemv_w(p, dtype, router, experts, hidden, x, logits);
    if (bias)
        for (int32_t e = 0; e < experts; ++e) logits[e] += bias[e];
    lo_routing(logits, experts, k, ids, weights);
    const void **gu = (const void **)malloc(sizeof(void *) * (size_t)k);
    const void **dn = (const void **)malloc(sizeof(void *) * (size_t)k);
    size_t gu_bytes = 2 * (size_t)inter * lo_row_bytes(dtype, (size_t)hidden);
    size_t dn_bytes = (size_t)hidden * lo_row_bytes(dtype, (size_t)inter);
    for (int32_t j = 0; j < k; ++j) {
        gu[j] = (const uint8_t *)gate_up + (size_t)ids[j] * gu_bytes;
        dn[j] = (const uint8_t *)down + (size_t)ids[j] * dn_bytes;
    }
    lo_experts_w(p, dtype, x, k, gu, dn, weights, hidden, inter, y);
    if (logits_or_null) memcpy(logits_or_null, logits, sizeof(float) * (size_t)experts);
    free(gu);
    free(dn);
    free(logits);
}

void lo_block_forward_w(lo_pool *p, int32_t dtype, const void *router, const void *gate_up, const void *down,
                        int32_t experts, int32_t hidden, int32_t inter, int32_t k, const float *x, float *y,
                        int32_t *ids, float *weights, float *logits_or_null) {
    block_forward_impl(p, dtype, router, gate_up, down, experts, hidden, inter, k, x, y, ids, weights, logits_or_null,
                       NULL);
}

void lo_block_forward(lo_pool *p, const uint16_t *router, const uint16_t *gate_up, const uint16_t *down,
                      int32_t experts, int32_t hidden, int32_t inter, int32_t k, const float *x, float *y,
                      int32_t *ids, float *weights, float *logits_or_null) {
    lo_block_forward_w(p, LO_W_BF16, router, gate_up, down, experts, hidden, inter, k, x, y, ids, weights,
                       logits_or_null);
}

/* ------------------------------------------------------------------------- */
/* norm, RoPE, argmax -- model.rs:63-73, 141-158; bin/m1b-gulosa.rs:22-24      */
/* ------------------------------------------------------------------------- */

/* model.rs:141-145 */
void lo_rmsnorm(const float *x, const float *w, int32_t n, float eps, float *out) {
    float ss = 0.0f;
    for (int32_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float ms = ss / (float)n;
    float r = 1.0f / sqrtf(ms + eps);
    for (int32_t i = 0; i < n; ++i) out[i] = w[i] * (x[i] * r);
}

/* model.rs:63-73: inv_freq[j] = 1/theta^(2j/d) in f32; cs = [cos; sin] */
void lo_rope_cos_sin(float theta, int32_t head_dim, int32_t pos, float *cs) {
    int32_t half = head_dim / 2;
    float d = (float)head_dim;
    for (int32_t j = 0; j < half; ++j) {
        float inv = 1.0f / powf(theta, (float)(2 * j) / d);
        float f = (float)pos * inv;
        cs[j] = cosf(f);
        cs[half + j] = sinf(f);
    }
}

/* model.rs:147-158 rotate_half RoPE on every head of d elements */
void lo_rope(float *x, int32_t n, int32_t d, const float *cs) {
    int32_t half = d / 2;
    const float *c = cs, *s = cs + half;
    for (int32_t h0 = 0; h0 + d <= n; h0 += d) {
        float *head = x + h0;
        for (int32_t j = 0; j < half; ++j) {
            float x1 = head[j], x2 = head[j + half];
            head[j] = x1 * c[j] - x2 * s[j];
            head[j + half] = x2 * c[j] + x1 * s[j];
        }
    }
}

/* bin/m1b-gulosa.rs:22-24, e4b_regra.rs:187-189: max_by(total_cmp) keeps the last maximum */
int32_t lo_argmax_last(const float *v, int32_t n) {
    int32_t best = 0;
    for (int32_t i = 1; i < n; ++i)
        if (lo_total_cmp(v[i], v[best]) >= 0) best = i;
    return best;
}

/* ------------------------------------------------------------------------- */
/* whole model -- model.rs:76-243                                              */
/* ------------------------------------------------------------------------- */
struct lo_model {
    lo_config cfg;
    const uint16_t *embed;
    const float *norm;
    lo_layer_weights *layers;
    float *router_bias; /* [layers, experts] or NULL */
    /* owned storage (synthetic models) */
    void **owned;
    int n_owned;
};

lo_model *lo_model_create(const lo_config *cfg, const uint16_t *embed, const float *norm,
                          const lo_layer_weights *layers) {
    lo_model *m = (lo_model *)calloc(1, sizeof(lo_model));
    m->cfg = *cfg;
    m->embed = embed;
    m->norm = norm;
    m->layers = (lo_layer_weights *)malloc(sizeof(lo_layer_weights) * (size_t)cfg->layers);
    memcpy(m->layers, layers, sizeof(lo_layer_weights) * (size_t)cfg->layers);
    return m;
}

static void *own(lo_model *m, size_t bytes) {
    void *p = malloc(bytes);
    m->owned = (void **)realloc(m->owned, sizeof(void *) * (size_t)(m->n_owned + 1));
    m->owned[m->n_owned++] = p;
    return p;
}

static uint16_t *synth_bf16_owned(lo_model *m, size_t n, uint64_t seed, float sd, float mean, int threads) {
    uint16_t *p = (uint16_t *)own(m, n * 2);
    lo_synth_bf16(p, n, seed, sd, mean, threads);
    return p;
}

static uint8_t *synth_q8_owned(lo_model *m, size_t rows, size_t cols, uint64_t seed, int threads) {
    uint8_t *p = (uint8_t *)own(m, rows * lo_row_bytes(LO_W_Q8_0, cols));
    lo_synth_q8_0(p, rows, cols, seed, threads);
    return p;
}

/* a linear weight [rows, cols] of the model's weight type */
static const void *synth_linear_owned(lo_model *m, size_t rows, size_t cols, uint64_t seed, float sd, int threads) {
    if (m->cfg.weight_dtype == LO_W_Q8_0) return synth_q8_owned(m, rows, cols, seed, threads);
    return synth_bf16_owned(m, rows * cols, seed, sd, 0.0f, threads);
}

static float *synth_norm_owned(lo_model *m, size_t n, uint64_t seed, float sd, int threads) {
    /* norms live as bf16 in checkpoints and are widened to f32 (model.rs:95-97, 117-118) */
    uint16_t *b = (uint16_t *)malloc(n * 2);
    lo_synth_bf16(b, n, seed, sd, 1.0f, threads);
    float *p = (float *)own(m, n * 4);
    for (size_t i = 0; i < n; ++i) p[i] = bf2f(b[i]);
    free(b);
    return p;
}

lo_model *lo_model_create_synthetic(const lo_config *cfg, uint64_t seed, float sd, float norm_sd, int threads) {
    lo_model *m = (lo_model *)calloc(1, sizeof(lo_model));
    m->cfg = *cfg;
    size_t H = (size_t)cfg->hidden, I = (size_t)cfg->inter, E = (size_t)cfg->experts;
    size_t qd = (size_t)cfg->heads * cfg->head_dim, kvd = (size_t)cfg->kv_heads * cfg->head_dim;
    m->embed = synth_bf16_owned(m, (size_t)cfg->vocab * H, lo_tensor_seed(seed, -1, LO_T_EMBED), sd, 0.0f, threads);
    m->norm = synth_norm_owned(m, H, lo_tensor_seed(seed, -1, LO_T_NORM), norm_sd, threads);
    m->layers = (lo_layer_weights *)calloc((size_t)cfg->layers, sizeof(lo_layer_weights));
    for (int32_t l = 0; l < cfg->layers; ++l) {
        lo_layer_weights *w = &m->layers[l];
        w->ln_attn = synth_norm_owned(m, H, lo_tensor_seed(seed, l, LO_T_LN_ATTN), norm_sd, threads);
        w->ln_moe = synth_norm_owned(m, H, lo_tensor_seed(seed, l, LO_T_LN_MOE), norm_sd, threads);
        w->q = synth_linear_owned(m, qd, H, lo_tensor_seed(seed, l, LO_T_Q), sd, threads);
        w->k = synth_linear_owned(m, kvd, H, lo_tensor_seed(seed, l, LO_T_K), sd, threads);
        w->v = synth_linear_owned(m, kvd, H, lo_tensor_seed(seed, l, LO_T_V), sd, threads);
        w->o = synth_linear_owned(m, H, qd, lo_tensor_seed(seed, l, LO_T_O), sd, threads);
        w->router = synth_linear_owned(m, E, H, lo_tensor_seed(seed, l, LO_T_ROUTER), sd, threads);
        w->gate_up = synth_linear_owned(m, E * 2 * I, H, lo_tensor_seed(seed, l, LO_T_GATE_UP), sd, threads);
        w->down = synth_linear_owned(m, E * H, I, lo_tensor_seed(seed, l, LO_T_DOWN), sd, threads);
    }
    return m;
}

void lo_model_destroy(lo_model *m) {
    if (!m) return;
    for (int i = 0; i < m->n_owned; ++i) free(m->owned[i]);
    free(m->owned);
    free(m->layers);
    free(m->router_bias);
    free(m);
}

void lo_model_set_router_bias(lo_model *m, const float *bias) {
    free(m->router_bias);
    m->router_bias = NULL;
    if (!bias) return;
    size_t n = (size_t)m->cfg.layers * m->cfg.experts;
    m->router_bias = (float *)malloc(sizeof(float) * n);
    memcpy(m->router_bias, bias, sizeof(float) * n);
}

const lo_config *lo_model_config(const lo_model *m) { return &m->cfg; }

const void *lo_model_tensor(const lo_model *m, int32_t layer, int32_t kind) {
    if (kind == LO_T_EMBED) return m->embed;
    if (kind == LO_T_NORM) return m->norm;
    if (layer < 0 || layer >= m->cfg.layers) return NULL;
    const lo_layer_weights *w = &m->layers[layer];
    switch (kind) {
    case LO_T_LN_ATTN: return w->ln_attn;
    case LO_T_LN_MOE: return w->ln_moe;
    case LO_T_Q: return w->q;
    case LO_T_K: return w->k;
    case LO_T_V: return w->v;
    case LO_T_O: return w->o;
    case LO_T_ROUTER: return w->router;
    case LO_T_GATE_UP: return w->gate_up;
    case LO_T_DOWN: return w->down;
    default: return NULL;
    }
}

struct lo_session {
    const lo_model *m;
    lo_pool *pool;
    int32_t max_len, pos;
    int32_t layers; /* own copy: the session may be destroyed after its model */
    int32_t kv_bf16; /* store K/V rows rounded to bf16 (RNE), as a paged bf16 KV cache holds them */
    float **k_cache, **v_cache; /* per layer [max_len, kvd] */
    float *router_logits;       /* [layers, experts] of the last step (bias included) */
    struct lo_step *st;         /* buffers of the step in progress (lo_session_step_begin .. _end) */
};

lo_session *lo_session_create(const lo_model *m, lo_pool *p, int32_t max_len) {
    lo_session *s = (lo_session *)calloc(1, sizeof(lo_session));
    s->m = m;
    s->pool = p;
    s->max_len = max_len;
    s->layers = m->cfg.layers;
    size_t kvd = (size_t)m->cfg.kv_heads * m->cfg.head_dim;
    s->router_logits = (float *)calloc((size_t)m->cfg.layers * m->cfg.experts, sizeof(float));
    s->k_cache = (float **)calloc((size_t)m->cfg.layers, sizeof(float *));
    s->v_cache = (float **)calloc((size_t)m->cfg.layers, sizeof(float *));
    for (int32_t l = 0; l < m->cfg.layers; ++l) {
        s->k_cache[l] = (float *)calloc((size_t)max_len * kvd, sizeof(float));
        s->v_cache[l] = (float *)calloc((size_t)max_len * kvd, sizeof(float));
    }
    return s;
}

static void step_free(lo_session *s);

void lo_session_destroy(lo_session *s) {
    if (!s) return;
    step_free(s);
    for (int32_t l = 0; l < s->layers; ++l) {
        free(s->k_cache[l]);
        free(s->v_cache[l]);
    }
    free(s->k_cache);
    free(s->v_cache);
    free(s->router_logits);
    free(s);
}

void lo_session_reset(lo_session *s) { s->pos = 0; }
void lo_session_set_kv_bf16(lo_session *s, int32_t on) { s->kv_bf16 = on != 0; }
const float *lo_session_router_logits(const lo_session *s) { return s->router_logits; }

static void round_bf16(float *v, size_t n) {
    for (size_t i = 0; i < n; ++i) v[i] = bf2f(lo_f32_to_bf16(v[i]));
}
int32_t lo_session_pos(const lo_session *s) { return s->pos; }
const float *lo_session_k(const lo_session *s, int32_t layer) { return s->k_cache[layer]; }
const float *lo_session_v(const lo_session *s, int32_t layer) { return s->v_cache[layer]; }

int lo_session_fill_kv(lo_session *s, int32_t n, uint64_t seed, float sd) {
    if (s->pos + n > s->max_len) return -1;
    size_t kvd = (size_t)s->m->cfg.kv_heads * s->m->cfg.head_dim;
    for (int32_t l = 0; l < s->m->cfg.layers; ++l) {
        lo_synth_f32(s->k_cache[l] + (size_t)s->pos * kvd, (size_t)n * kvd, lo_mix64(seed + 2 * (uint64_t)l), sd, 0.0f, 1);
        lo_synth_f32(s->v_cache[l] + (size_t)s->pos * kvd, (size_t)n * kvd, lo_mix64(seed + 2 * (uint64_t)l + 1), sd, 0.0f, 1);
        if (s->kv_bf16) {
            round_bf16(s->k_cache[l] + (size_t)s->pos * kvd, (size_t)n * kvd);
            round_bf16(s->v_cache[l] + (size_t)s->pos * kvd, (size_t)n * kvd);
        }
    }
    s->pos += n;
    return 0;
}

typedef struct {
    const lo_config *c;
    const float *q;
    const float *kc, *vc;
    int32_t len;
    float *att;
} attn_ctx;

/* model.rs:203-222, one query head per task (heads are independent) */
static void attn_task(void *cx, size_t hq) {
    attn_ctx *a = (attn_ctx *)cx;
    const lo_config *c = a->c;
    int32_t d = c->head_dim, kvd = c->kv_heads * d, group = c->heads / c->kv_heads;
    int32_t kvh = (int32_t)hq / group;
    const float *qh = a->q + hq * (size_t)d;
    float *scores = (float *)malloc(sizeof(float) * (size_t)a->len);
    for (int32_t p = 0; p < a->len; ++p) {
        const float *kr = a->kc + (size_t)p * kvd + (size_t)kvh * d;
        float dot = 0.0f;
        for (int32_t i = 0; i < d; ++i) dot += qh[i] * kr[i];
        scores[p] = dot * c->attention_multiplier;
    }
    float mx = -INFINITY;
    for (int32_t p = 0; p < a->len; ++p) mx = fmaxf(mx, scores[p]);
    float sum = 0.0f;
    for (int32_t p = 0; p < a->len; ++p) {
        scores[p] = expf(scores[p] - mx);
    }
    for (int32_t p = 0; p < a->len; ++p) sum += scores[p];
    float *out = a->att + hq * (size_t)d;
    for (int32_t p = 0; p < a->len; ++p) {
        const float *vr = a->vc + (size_t)p * kvd + (size_t)kvh * d;
        for (int32_t i = 0; i < d; ++i) out[i] += scores[p] / sum * vr[i];
    }
    free(scores);
}

/* model.rs:181-243 CpuSession::step, in phases: the decoder layer's attention half (lo_session_layer_attention), its
 * MoE half (the block, or lo_session_layer_moe with a result computed elsewhere), then the head.  A step that runs
 * the phases in order is the same arithmetic as lo_session_step, which is written with them. */
struct lo_step {
    float *cs, *x, *xn, *q, *att, *o, *y, *rw;
    int32_t *ri;
};

static void step_free(lo_session *s) {
    struct lo_step *t = s->st;
    if (!t) return;
    free(t->cs);
    free(t->x);
    free(t->xn);
    free(t->q);
    free(t->att);
    free(t->o);
    free(t->y);
    free(t->rw);
    free(t->ri);
    free(t);
    s->st = NULL;
}

int lo_session_step_begin(lo_session *s, int32_t token) {
    const lo_model *m = s->m;
    const lo_config *c = &m->cfg;
    if (s->pos >= s->max_len || token < 0 || token >= c->vocab) return -1;
    step_free(s);
    struct lo_step *t = (struct lo_step *)calloc(1, sizeof(struct lo_step));
    int32_t h = c->hidden, d = c->head_dim, qd = c->heads * d;
    t->cs = (float *)malloc(sizeof(float) * (size_t)d);
    lo_rope_cos_sin(c->rope_theta, d, s->pos, t->cs);
    t->x = (float *)malloc(sizeof(float) * (size_t)h);
    t->xn = (float *)malloc(sizeof(float) * (size_t)h);
    t->q = (float *)malloc(sizeof(float) * (size_t)qd);
    t->att = (float *)malloc(sizeof(float) * (size_t)qd);
    t->o = (float *)malloc(sizeof(float) * (size_t)h);
    t->y = (float *)malloc(sizeof(float) * (size_t)h);
    t->rw = (float *)malloc(sizeof(float) * (size_t)c->k);
    t->ri = (int32_t *)malloc(sizeof(int32_t) * (size_t)c->k);
    s->st = t;
    /* model.rs:134-138 embedding x embedding_multiplier */
    for (int32_t i = 0; i < h; ++i) t->x[i] = bf2f(m->embed[(size_t)token * h + i]) * c->embedding_multiplier;
    return 0;
}

/* layer l up to the MoE input: xn_out = RMSNorm(x + resid * attention, ln_moe) [H] */
void lo_session_layer_attention(lo_session *s, int32_t l, float *xn_out) {
    const lo_model *m = s->m;
    const lo_config *c = &m->cfg;
    struct lo_step *t = s->st;
    int32_t h = c->hidden, d = c->head_dim, qd = c->heads * d, kvd = c->kv_heads * d;
    const lo_layer_weights *w = &m->layers[l];
    lo_rmsnorm(t->x, w->ln_attn, h, c->eps, t->xn);
    float *kr = s->k_cache[l] + (size_t)s->pos * kvd;
    float *vr = s->v_cache[l] + (size_t)s->pos * kvd;
    lo_gemv_w(s->pool, c->weight_dtype, w->q, qd, h, t->xn, t->q);
    lo_gemv_w(s->pool, c->weight_dtype, w->k, kvd, h, t->xn, kr);
    lo_gemv_w(s->pool, c->weight_dtype, w->v, kvd, h, t->xn, vr);
    lo_rope(t->q, qd, d, t->cs);
    lo_rope(kr, kvd, d, t->cs);
    if (s->kv_bf16) {
        round_bf16(kr, (size_t)kvd);
        round_bf16(vr, (size_t)kvd);
    }
    memset(t->att, 0, sizeof(float) * (size_t)qd);
    attn_ctx ac = {c, t->q, s->k_cache[l], s->v_cache[l], s->pos + 1, t->att};
    pool_run(s->pool, (size_t)c->heads, attn_task, &ac);
    lo_gemv_w(s->pool, c->weight_dtype, w->o, h, qd, t->att, t->o);
    for (int32_t i = 0; i < h; ++i) t->x[i] += c->residual_multiplier * t->o[i];
    lo_rmsnorm(t->x, w->ln_moe, h, c->eps, t->xn);
    if (xn_out) memcpy(xn_out, t->xn, sizeof(float) * (size_t)h);
}

/* the residual stream of the step in progress [H] (before the next lo_session_layer_attention: that layer's input) */
void lo_session_residual(const lo_session *s, float *out) {
    memcpy(out, s->st->x, sizeof(float) * (size_t)s->m->cfg.hidden);
}

/* layer l's MoE half from a block output y computed elsewhere: x += resid * y */
void lo_session_layer_moe(lo_session *s, int32_t l, const float *y) {
    const lo_config *c = &s->m->cfg;
    (void)l;
    for (int32_t i = 0; i < c->hidden; ++i) s->st->x[i] += c->residual_multiplier * y[i];
}

/* final norm, tied lm_head, / logits_scaling (gpu_model.rs:436-439); the position advances */
void lo_session_step_end(lo_session *s, float *logits) {
    const lo_model *m = s->m;
    const lo_config *c = &m->cfg;
    struct lo_step *t = s->st;
    lo_rmsnorm(t->x, m->norm, c->hidden, c->eps, t->xn);
    lo_gemv(s->pool, m->embed, c->vocab, c->hidden, t->xn, logits);
    for (int32_t v = 0; v < c->vocab; ++v) logits[v] /= c->logits_scaling;
    s->pos += 1;
    step_free(s);
}

int lo_session_step(lo_session *s, int32_t token, float *logits, int32_t *ids, float *weights) {
    const lo_model *m = s->m;
    const lo_config *c = &m->cfg;
    if (lo_session_step_begin(s, token)) return -1;
    struct lo_step *t = s->st;
    int32_t h = c->hidden;
    for (int32_t l = 0; l < c->layers; ++l) {
        const lo_layer_weights *w = &m->layers[l];
        lo_session_layer_attention(s, l, NULL);
        block_forward_impl(s->pool, c->weight_dtype, w->router, w->gate_up, w->down, c->experts, h, c->inter, c->k,
                           t->xn, t->y, t->ri, t->rw, s->router_logits + (size_t)l * c->experts,
                           m->router_bias ? m->router_bias + (size_t)l * c->experts : NULL);
        lo_session_layer_moe(s, l, t->y);
        if (ids) memcpy(ids + (size_t)l * c->k, t->ri, sizeof(int32_t) * (size_t)c->k);
        if (weights) memcpy(weights + (size_t)l * c->k, t->rw, sizeof(float) * (size_t)c->k);
    }
    lo_session_step_end(s, logits);
    return 0;
}
