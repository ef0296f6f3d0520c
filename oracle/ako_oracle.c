/*
 * CPU oracle for the hot path, in C — TEST INFRASTRUCTURE ONLY.
 *
 * A restatement of AKO's unfused PyTorch references (ako/ops/rmsnorm_ref.py,
 * rope_ref.py, swiglu_ref.py) on raw buffers, parallel over rows with
 * pthreads. Used by tests/ to check the CUDA path at sizes numpy is slow on
 * and by bench.py as the timed CPU baseline. The product library never links
 * or calls it. Compiled by oracle/Makefile with -ffp-contract=off so every
 * fp32 multiply and add rounds separately, as the reference's tensor ops do.
 *
 * Storage dtypes: 0 = float32, 1 = float16 (_Float16), 2 = bfloat16 (bits).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define F32 0
#define F16 1
#define BF16 2

static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float load(const void* p, int64_t i, int dtype) {
    switch (dtype) {
        case F16: return (float)((const _Float16*)p)[i];
        case BF16: return bf16_to_f32(((const uint16_t*)p)[i]);
        default: return ((const float*)p)[i];
    }
}

static inline void store(void* p, int64_t i, float v, int dtype) {
    switch (dtype) {
        case F16: ((_Float16*)p)[i] = (_Float16)v; break;
        case BF16: ((uint16_t*)p)[i] = f32_to_bf16(v); break;
        default: ((float*)p)[i] = v; break;
    }
}

/* ------------------------------------------------------------ row threads */
typedef void (*row_fn)(const void* ctx, int64_t begin, int64_t end);

typedef struct {
    row_fn fn;
    const void* ctx;
    int64_t begin, end;
} job_t;

static void* run_job(void* arg) {
    job_t* j = (job_t*)arg;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static void parallel_rows(row_fn fn, const void* ctx, int64_t rows, int threads) {
    if (threads > 256) threads = 256;
    if (threads < 1 || rows < 2 * (int64_t)threads) threads = rows > 0 ? 1 : 0;
    if (threads <= 1) {
        if (rows > 0) fn(ctx, 0, rows);
        return;
    }
    pthread_t tid[256];
    job_t jobs[256];
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].begin = rows * t / threads;
        jobs[t].end = rows * (t + 1) / threads;
        if (pthread_create(&tid[t], NULL, run_job, &jobs[t]) == 0) {
            ++started;
        } else {
            run_job(&jobs[t]);
            tid[t] = 0;
        }
    }
    for (int t = 0; t < threads; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
    (void)started;
}

/* ---------------------------------------------------------------- rmsnorm */
typedef struct {
    const void *x, *r, *w;
    void *y, *ro;
    int64_t h;
    float eps;
    int dtype, wdtype;
    int fixed_order; /* 1: the CUDA kernels' summation order (fixed_order_sum) */
} rms_ctx;

/* Pairwise sum of n floats (blocks of 8 summed in order). torch's CPU
 * reduction is a cascade of the same kind; a running sum would drift several
 * fp32 ulp from it on rows of thousands of elements. */
static float pairwise_sum(const float* v, int64_t n) {
    if (n <= 8) {
        float s = 0.0f;
        for (int64_t i = 0; i < n; ++i) s = s + v[i];
        return s;
    }
    const int64_t m = ((n / 2) + 7) & ~(int64_t)7;
    return pairwise_sum(v, m) + pairwise_sum(v + m, n - m);
}

/* Fold of n = 2^k values in place: v[i] += v[i + n/2], then n/4, ... 1. */
static float fold(float* v, int64_t n) {
    for (int64_t off = n / 2; off >= 1; off /= 2)
        for (int64_t i = 0; i < off; ++i) v[i] = v[i] + v[i + off];
    return v[0];
}

/* The summation order of the CUDA RMSNorm kernels on rows of 16-byte
 * vectors (`vec` elements each; ako_b200/csrc/rmsnorm.cuh, "Fixed summation
 * order"). It is a model of the kernels, not of the reference, and depends
 * on the row width only:
 *   1. each vector's squares pairwise (pairs 1, 2, 4 apart);
 *   2. each group of 32 consecutive vectors by a fold (pairs 16, 8, 4, 2, 1
 *      apart), zeros past the row's end;
 *   3. the groups by the same fold over group indices, zero-padded to a
 *      power of two.
 * Adding a zero to a sum of squares is exact, so any padding gives the same
 * bits. */
static float fixed_order_sum(const float* sq, int64_t h, int vec) {
    const int64_t nvec = h / vec;
    const int64_t groups = (nvec + 31) / 32;
    int64_t padded = 1;
    while (padded < groups) padded *= 2;
    float* g = (float*)calloc((size_t)padded, sizeof(float));
    if (!g) return NAN;
    for (int64_t k = 0; k < groups; ++k) {
        float lanes[32];
        for (int l = 0; l < 32; ++l) {
            const int64_t v = k * 32 + l;
            lanes[l] = 0.0f;
            if (v < nvec) {
                float e[8];
                for (int i = 0; i < vec; ++i) e[i] = sq[v * vec + i];
                for (int st = 1; st < vec; st *= 2)
                    for (int i = 0; i + st < vec; i += 2 * st) e[i] = e[i] + e[i + st];
                lanes[l] = e[0];
            }
        }
        g[k] = fold(lanes, 32);
    }
    const float total = fold(g, padded);
    free(g);
    return total;
}

/* ako/ops/rmsnorm_ref.py:8-23 and :26-50 */
static void rms_rows(const void* vctx, int64_t begin, int64_t end) {
    const rms_ctx* c = (const rms_ctx*)vctx;
    const int64_t h = c->h;
    float* sq = (float*)malloc((size_t)h * sizeof(float));
    if (!sq) return;
    for (int64_t row = begin; row < end; ++row) {
        const int64_t base = row * h;
        for (int64_t i = 0; i < h; ++i) {
            float v = load(c->x, base + i, c->dtype);
            if (c->r) {
                store(c->ro, base + i, v + load(c->r, base + i, c->dtype), c->dtype);
                v = load(c->ro, base + i, c->dtype);
            }
            sq[i] = v * v; /* x.pow(2), rounded per element */
        }
        const int es = c->dtype == F32 ? 4 : 2;
        const float total = c->fixed_order ? fixed_order_sum(sq, h, 16 / es) : pairwise_sum(sq, h);
        const float mean = total / (float)h;
        const float inv = 1.0f / sqrtf(mean + c->eps);
        for (int64_t i = 0; i < h; ++i) {
            const float v = load(c->r ? c->ro : c->x, base + i, c->dtype);
            const float normed = v * inv;
            store(c->y, base + i, normed * load(c->w, i, c->wdtype), c->dtype);
        }
    }
    free(sq);
}

int ako_oracle_rmsnorm(const void* x, const void* w, int wdtype, void* y, int64_t rows, int64_t h, float eps,
                       int dtype, int threads) {
    rms_ctx c = {x, NULL, w, y, NULL, h, eps, dtype, wdtype, 0};
    parallel_rows(rms_rows, &c, rows, threads);
    return 0;
}

int ako_oracle_rmsnorm_residual(const void* x, const void* r, const void* w, int wdtype, void* y, void* ro,
                                int64_t rows, int64_t h, float eps, int dtype, int threads) {
    rms_ctx c = {x, r, w, y, ro, h, eps, dtype, wdtype, 0};
    parallel_rows(rms_rows, &c, rows, threads);
    return 0;
}

/* Both forms with the kernels' summation order (fixed_order_sum); `r` may be
 * NULL for plain RMSNorm. h * element size must be a multiple of 16. */
int ako_oracle_rmsnorm_fixed_order(const void* x, const void* r, const void* w, int wdtype, void* y, void* ro,
                                   int64_t rows, int64_t h, float eps, int dtype, int threads) {
    const int es = dtype == F32 ? 4 : 2;
    if ((h * es) % 16 != 0) return 1;
    rms_ctx c = {x, r, w, y, r ? ro : NULL, h, eps, dtype, wdtype, 1};
    parallel_rows(rms_rows, &c, rows, threads);
    return 0;
}

/* ------------------------------------------------------------------- rope */
typedef struct {
    const void* x;
    const float *cos, *sin;
    void* y;
    int64_t seq, heads, d;
    int style, dtype;
} rope_ctx;

/* ako/ops/rope_ref.py:73-107; x and y are contiguous (batch, seq, heads, d). */
static void rope_rows(const void* vctx, int64_t begin, int64_t end) {
    const rope_ctx* c = (const rope_ctx*)vctx;
    const int64_t half = c->d / 2;
    for (int64_t pos = begin; pos < end; ++pos) {
        const int64_t s = pos % c->seq;
        const float* cr = c->cos + s * half;
        const float* sr = c->sin + s * half;
        for (int64_t hd = 0; hd < c->heads; ++hd) {
            const int64_t base = (pos * c->heads + hd) * c->d;
            for (int64_t i = 0; i < half; ++i) {
                const int64_t lo = c->style ? base + 2 * i : base + i;
                const int64_t hi = c->style ? base + 2 * i + 1 : base + half + i;
                const float x0 = load(c->x, lo, c->dtype), x1 = load(c->x, hi, c->dtype);
                const float a = x0 * cr[i], b = x1 * sr[i];
                const float p = x0 * sr[i], q = x1 * cr[i];
                store(c->y, lo, a - b, c->dtype);
                store(c->y, hi, p + q, c->dtype);
            }
        }
    }
}

int ako_oracle_rope(const void* x, const float* cos, const float* sin, void* y, int64_t batch, int64_t seq,
                    int64_t heads, int64_t head_dim, int style, int dtype, int threads) {
    rope_ctx c = {x, cos, sin, y, seq, heads, head_dim, style, dtype};
    parallel_rows(rope_rows, &c, batch * seq, threads);
    return 0;
}

/* ----------------------------------------------------------------- swiglu */
typedef struct {
    const void *g, *u;
    void* y;
    int64_t h;
    int dtype;
} swiglu_ctx;

/* ako/ops/swiglu_ref.py:16-32: silu(g) = g / (1 + exp(-g)), times up. */
static void swiglu_rows(const void* vctx, int64_t begin, int64_t end) {
    const swiglu_ctx* c = (const swiglu_ctx*)vctx;
    for (int64_t i = begin * c->h; i < end * c->h; ++i) {
        const float g = load(c->g, i, c->dtype);
        const float e = expf(-g);
        const float den = 1.0f + e;
        const float silu = g / den;
        store(c->y, i, silu * load(c->u, i, c->dtype), c->dtype);
    }
}

int ako_oracle_swiglu(const void* g, const void* u, void* y, int64_t rows, int64_t h, int dtype, int threads) {
    swiglu_ctx c = {g, u, y, h, dtype};
    parallel_rows(swiglu_rows, &c, rows, threads);
    return 0;
}
