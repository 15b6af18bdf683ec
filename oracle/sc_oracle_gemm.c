/*
 * sc_oracle_gemm.c -- CPU oracle (test infrastructure only) for the Q8_0
 * GEMM of she-workss/stealcode `audio_engine`: f16 decode, activation
 * quantisation, the scalar test-oracle GEMM, the SIMD kernel's accumulation
 * order, and an AVX2 + threaded twin of the SIMD dispatcher that serves as
 * the timed CPU baseline. Built with -ffp-contract=off (see sc_oracle.h).
 */
#include "sc_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* f16 decode: gguf.rs:365-397                                         */
static __thread int g_exp_cr;

void orc_set_exp_mode(int correctly_rounded) { g_exp_cr = correctly_rounded ? 1 : 0; }

int orc_get_exp_mode(void) { return g_exp_cr; }

float orc_expf(float x) { return g_exp_cr ? (float)exp((double)x) : expf(x); }

float orc_tanhf(float x) { return g_exp_cr ? (float)tanh((double)x) : tanhf(x); }

/* ------------------------------------------------------------------ */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15);
    uint32_t exp = (uint32_t)((h >> 10) & 0x1f);
    uint32_t man = (uint32_t)(h & 0x3ff);
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign << 31;
        } else {
            /* subnormal: normalise the mantissa */
            int32_t e = 127 - 15 + 1;
            uint32_t m = man << 13;
            while ((m & 0x00800000u) == 0) {
                m <<= 1;
                e -= 1;
            }
            m &= 0x007fffffu;
            bits = (sign << 31) | ((uint32_t)e << 23) | m;
        }
    } else if (exp == 0x1f) {
        bits = man == 0 ? ((sign << 31) | 0x7f800000u)
                        : ((sign << 31) | 0x7fc00000u | (man << 13));
    } else {
        bits = (sign << 31) | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* sgemm_kernel.rs:209-221: truncating f32 -> f16 used by the reference's
 * GEMM test generator (flush to signed zero below the normal range). */
uint16_t orc_half_from_f32_trunc(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t exp = (int32_t)((bits >> 23) & 0xff) - 127 + 15;
    uint32_t mant = (bits >> 13) & 0x3ff;
    if (exp <= 0) return sign;
    if (exp >= 31) return (uint16_t)(sign | 0x7c00);
    return (uint16_t)(sign | ((uint16_t)exp << 10) | (uint16_t)mant);
}

/* sgemm_kernel.rs:46-53 */
float orc_read_q8_scale(const uint8_t *w, size_t base, size_t block_bytes) {
    if (block_bytes == 34) {
        return orc_f16_to_f32((uint16_t)(w[base] | (w[base + 1] << 8)));
    }
    float f;
    memcpy(&f, w + base, 4);
    return f;
}

/* Rust `f32 as i8`: saturating, NaN -> 0. */
static inline int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v; /* v already integral (rounded) */
}

/* ------------------------------------------------------------------ */
/* quantize_col: sgemm_kernel.rs:57-90                                 */
/* ------------------------------------------------------------------ */
void orc_quantize_col(const float *x, size_t nj, size_t k, size_t n,
                      size_t nblocks, int8_t *xqrow, float *dxrow) {
    for (size_t b = 0; b < nblocks; b++) {
        size_t k0 = b * 32;
        size_t len = (k - k0) < 32 ? (k - k0) : 32;
        float maxv = 0.0f;
        for (size_t j = 0; j < len; j++) {
            float v = fabsf(x[(k0 + j) * n + nj]);
            if (v > maxv) maxv = v;
        }
        float s = maxv == 0.0f ? 1.0f : maxv / 127.0f;
        dxrow[b] = s;
        if (maxv != 0.0f) {
            float inv = 1.0f / s;
            for (size_t j = 0; j < len; j++) {
                /* f32::round = half away from zero = C roundf */
                xqrow[k0 + j] = sat_i8(roundf(x[(k0 + j) * n + nj] * inv));
            }
        } else {
            for (size_t j = 0; j < len; j++) xqrow[k0 + j] = 0;
        }
    }
}

static void quantize_all(const float *x, size_t k, size_t n, size_t nblocks,
                         int8_t *xq, float *dx) {
    for (size_t nj = 0; nj < n; nj++) {
        orc_quantize_col(x, nj, k, n, nblocks, xq + nj * k, dx + nj * nblocks);
    }
}

/* ------------------------------------------------------------------ */
/* q8_gemm_scalar: sgemm_kernel.rs:132-202                             */
/* ------------------------------------------------------------------ */
static void scalar_rows(size_t i0, size_t i1, size_t k, size_t n,
                        const uint8_t *w, size_t padded_row,
                        size_t block_bytes, size_t qoff, const int8_t *xq,
                        const float *dx, size_t nblocks, float *y) {
    for (size_t i = i0; i < i1; i++) {
        for (size_t nj = 0; nj < n; nj++) {
            float acc = 0.0f;
            for (size_t b = 0; b < nblocks; b++) {
                size_t wbase = i * padded_row + b * block_bytes;
                float dw = orc_read_q8_scale(w, wbase, block_bytes);
                float s = dw * dx[nj * nblocks + b];
                size_t k0 = b * 32;
                size_t len = (k - k0) < 32 ? (k - k0) : 32;
                const uint8_t *wb = w + wbase + qoff;
                const int8_t *xb = xq + nj * k + k0;
                float dot = 0.0f;
                for (size_t j = 0; j < len; j++) {
                    dot += (float)(int8_t)wb[j] * (float)xb[j];
                }
                acc += s * dot;
            }
            y[i * n + nj] = acc;
        }
    }
}

void orc_q8_gemm_scalar(size_t m, size_t k, size_t n, const uint8_t *w,
                        size_t padded_row, size_t block_bytes, size_t qoff,
                        const float *x, float *y) {
    if (m == 0 || k == 0 || n == 0) return;
    size_t nblocks = (k + 31) / 32;
    int8_t *xq = calloc(n * k, 1);
    float *dx = calloc(n * nblocks, sizeof(float));
    quantize_all(x, k, n, nblocks, xq, dx);
    scalar_rows(0, m, k, n, w, padded_row, block_bytes, qoff, xq, dx, nblocks,
                y);
    free(xq);
    free(dx);
}

void orc_q8_block_dots(size_t m, size_t k, size_t n, const uint8_t *w,
                       size_t padded_row, size_t block_bytes, size_t qoff,
                       const float *x, int32_t *dots) {
    if (m == 0 || k == 0 || n == 0) return;
    size_t nblocks = (k + 31) / 32;
    int8_t *xq = calloc(n * k, 1);
    float *dx = calloc(n * nblocks, sizeof(float));
    quantize_all(x, k, n, nblocks, xq, dx);
    for (size_t i = 0; i < m; i++)
        for (size_t nj = 0; nj < n; nj++)
            for (size_t b = 0; b < nblocks; b++) {
                size_t k0 = b * 32;
                size_t len = (k - k0) < 32 ? (k - k0) : 32;
                const uint8_t *wb = w + i * padded_row + b * block_bytes + qoff;
                const int8_t *xb = xq + nj * k + k0;
                int32_t dot = 0;
                for (size_t j = 0; j < len; j++)
                    dot += (int32_t)(int8_t)wb[j] * (int32_t)xb[j];
                dots[(i * n + nj) * nblocks + b] = dot;
            }
    free(xq);
    free(dx);
}

/* ------------------------------------------------------------------ */
/* SIMD accumulation order: simd_kernel.rs:276-394 (portable C)        */
/* ------------------------------------------------------------------ */
/* One 32-wide block: lane j of the 8 f32 partials gets
 *   (w[j]x[j] + w[j+16]x[j+16]) + (w[j+8]x[j+8] + w[j+24]x[j+24])
 * -- the i16 pair fold (:357-360) then the f32 lane fold (:361-364). */
static inline void block_partials(const int8_t *wq, const int8_t *xqb,
                                  float s8[8]) {
    int16_t p[16];
    for (int j = 0; j < 16; j++) {
        p[j] = (int16_t)((int16_t)(wq[j] * xqb[j]) +
                         (int16_t)(wq[j + 16] * xqb[j + 16]));
    }
    for (int j = 0; j < 8; j++) s8[j] = (float)p[j] + (float)p[j + 8];
}

static float reduce8(const float a[8]) {
    /* Simd::reduce_sum: ordered lane sum */
    float r = a[0];
    for (int j = 1; j < 8; j++) r += a[j];
    return r;
}

static void simd_order_rows(size_t i0, size_t i1, size_t k, size_t n,
                            const uint8_t *w, size_t padded_row,
                            size_t block_bytes, size_t qoff, const int8_t *xq,
                            const float *dx, size_t nblocks, float *y) {
    for (size_t i = i0; i < i1; i++) {
        size_t rowbase = i * padded_row;
        for (size_t nj = 0; nj < n; nj++) {
            float acc[8] = {0};
            for (size_t b = 0; b < nblocks; b++) {
                size_t wbase = rowbase + b * block_bytes;
                float dw = orc_read_q8_scale(w, wbase, block_bytes);
                float s8[8];
                block_partials((const int8_t *)(w + wbase + qoff),
                               xq + nj * k + b * 32, s8);
                float s = dw * dx[nj * nblocks + b];
                for (int j = 0; j < 8; j++) acc[j] = fmaf(s8[j], s, acc[j]);
            }
            y[i * n + nj] = reduce8(acc);
        }
    }
}

void orc_q8_gemm_simd_order(size_t m, size_t k, size_t n, const uint8_t *w,
                            size_t padded_row, size_t block_bytes,
                            size_t qoff, const float *x, float *y) {
    if (m == 0 || k == 0 || n == 0) return;
    if (m % 8 != 0 || k % 32 != 0 || n > 16) {
        orc_q8_gemm_scalar(m, k, n, w, padded_row, block_bytes, qoff, x, y);
        return;
    }
    size_t nblocks = k / 32;
    int8_t *xq = calloc(n * k, 1);
    float *dx = calloc(n * nblocks, sizeof(float));
    quantize_all(x, k, n, nblocks, xq, dx);
    simd_order_rows(0, m, k, n, w, padded_row, block_bytes, qoff, xq, dx,
                    nblocks, y);
    free(xq);
    free(dx);
}

/* ------------------------------------------------------------------ */
/* AVX2 + threads: the timed CPU baseline (same bits as above)         */
/* ------------------------------------------------------------------ */
__attribute__((target("avx2,fma"))) static void
avx2_rows(size_t i0, size_t i1, size_t k, size_t n, const uint8_t *w,
          size_t padded_row, size_t block_bytes, size_t qoff,
          const int8_t *xq, const float *dx, size_t nblocks, float *y) {
    __m256 acc[16];
    for (size_t i = i0; i < i1; i++) {
        size_t rowbase = i * padded_row;
        if (i + 1 < i1) __builtin_prefetch(w + rowbase + padded_row);
        for (size_t nj = 0; nj < n; nj++) acc[nj] = _mm256_setzero_ps();
        for (size_t b = 0; b < nblocks; b++) {
            size_t wbase = rowbase + b * block_bytes;
            float dw = orc_read_q8_scale(w, wbase, block_bytes);
            const uint8_t *wp = w + wbase + qoff;
            __m256i w16lo = _mm256_cvtepi8_epi16(
                _mm_loadu_si128((const __m128i *)wp));
            __m256i w16hi = _mm256_cvtepi8_epi16(
                _mm_loadu_si128((const __m128i *)(wp + 16)));
            for (size_t nj = 0; nj < n; nj++) {
                const int8_t *xp = xq + nj * k + b * 32;
                __m256i x16lo = _mm256_cvtepi8_epi16(
                    _mm_loadu_si128((const __m128i *)xp));
                __m256i x16hi = _mm256_cvtepi8_epi16(
                    _mm_loadu_si128((const __m128i *)(xp + 16)));
                __m256i p = _mm256_add_epi16(_mm256_mullo_epi16(w16lo, x16lo),
                                             _mm256_mullo_epi16(w16hi, x16hi));
                __m256 pa = _mm256_cvtepi32_ps(
                    _mm256_cvtepi16_epi32(_mm256_castsi256_si128(p)));
                __m256 pb = _mm256_cvtepi32_ps(
                    _mm256_cvtepi16_epi32(_mm256_extracti128_si256(p, 1)));
                __m256 s8 = _mm256_add_ps(pa, pb);
                float s = dw * dx[nj * nblocks + b];
                acc[nj] = _mm256_fmadd_ps(s8, _mm256_set1_ps(s), acc[nj]);
            }
        }
        for (size_t nj = 0; nj < n; nj++) {
            float a[8];
            _mm256_storeu_ps(a, acc[nj]);
            y[i * n + nj] = reduce8(a);
        }
    }
}

/* A small persistent worker pool with dynamic chunk claiming (rayon's
 * par_chunks_mut schedules chunks dynamically on a persistent pool). */
typedef void (*chunk_fn)(void *ctx, size_t chunk);

typedef struct {
    pthread_mutex_t mu;
    pthread_cond_t cv_work, cv_done;
    int nthreads;        /* worker threads (excluding the caller) */
    unsigned long gen;   /* job generation */
    int active;          /* workers still inside the current job */
    chunk_fn fn;
    void *ctx;
    size_t nchunks;
    atomic_size_t next;
    int stop;
    int limit;           /* workers taking part in the current job */
    pthread_t *th;
    int *ids;
} pool_t;

static pool_t g_pool;
static pthread_once_t g_pool_once = PTHREAD_ONCE_INIT;

int orc_num_cpus(void) {
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c > 0 ? (int)c : 1;
}

static void run_chunks(pool_t *p) {
    for (;;) {
        size_t c = atomic_fetch_add(&p->next, 1);
        if (c >= p->nchunks) break;
        p->fn(p->ctx, c);
    }
}

static void *worker(void *arg) {
    int id = *(int *)arg;
    pool_t *p = &g_pool;
    unsigned long seen = 0;
    pthread_mutex_lock(&p->mu);
    for (;;) {
        while (p->gen == seen && !p->stop) pthread_cond_wait(&p->cv_work, &p->mu);
        if (p->stop) break;
        seen = p->gen;
        int take_part = id < p->limit;
        pthread_mutex_unlock(&p->mu);
        if (take_part) run_chunks(p);
        pthread_mutex_lock(&p->mu);
        if (--p->active == 0) pthread_cond_signal(&p->cv_done);
    }
    pthread_mutex_unlock(&p->mu);
    return NULL;
}

static void pool_init(void) {
    pool_t *p = &g_pool;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_work, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    p->nthreads = orc_num_cpus() - 1;
    if (p->nthreads < 0) p->nthreads = 0;
    p->th = calloc((size_t)(p->nthreads > 0 ? p->nthreads : 1), sizeof(pthread_t));
    p->ids = calloc((size_t)(p->nthreads > 0 ? p->nthreads : 1), sizeof(int));
    for (int t = 0; t < p->nthreads; t++) {
        p->ids[t] = t;
        pthread_create(&p->th[t], NULL, worker, &p->ids[t]);
    }
}

/* Run fn over nchunks chunks on up to `threads` threads (caller included). */
static void parallel_chunks(int threads, size_t nchunks, chunk_fn fn, void *ctx) {
    if (threads <= 1 || nchunks <= 1) {
        for (size_t c = 0; c < nchunks; c++) fn(ctx, c);
        return;
    }
    pthread_once(&g_pool_once, pool_init);
    pool_t *p = &g_pool;
    static pthread_mutex_t call_mu = PTHREAD_MUTEX_INITIALIZER;
    pthread_mutex_lock(&call_mu);
    int workers = threads - 1 < p->nthreads ? threads - 1 : p->nthreads;
    if (workers <= 0) {
        for (size_t c = 0; c < nchunks; c++) fn(ctx, c);
        pthread_mutex_unlock(&call_mu);
        return;
    }
    pthread_mutex_lock(&p->mu);
    p->fn = fn;
    p->ctx = ctx;
    p->nchunks = nchunks;
    atomic_store(&p->next, 0);
    /* every pool worker wakes and reports back; only the first `workers`
     * of them claim chunks, so the job runs on exactly `threads` threads. */
    p->limit = workers;
    p->active = p->nthreads;
    p->gen++;
    pthread_cond_broadcast(&p->cv_work);
    pthread_mutex_unlock(&p->mu);
    run_chunks(p);
    pthread_mutex_lock(&p->mu);
    while (p->active > 0) pthread_cond_wait(&p->cv_done, &p->mu);
    pthread_mutex_unlock(&p->mu);
    pthread_mutex_unlock(&call_mu);
}

/* The reference's threading and SIMD kernels outside the Q8 GEMM (rayon over
 * spatial positions, queries and 256-row chunks; AVX2 lanes for score_dot,
 * softmax_v and the f32 GEMM) compute every output in the same order as the
 * serial scalar restatement, so the switch changes speed only. */
static atomic_int g_fast = 1;

void orc_set_fast(int on) { atomic_store(&g_fast, on ? 1 : 0); }

int orc_get_fast(void) { return atomic_load(&g_fast); }

int orc_have_avx2(void) {
    static int have = -1;
    if (have < 0) {
        __builtin_cpu_init();
        have = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
    return have;
}

void orc_parallel(size_t nchunks, void (*fn)(void *ctx, size_t chunk), void *ctx) {
    parallel_chunks(atomic_load(&g_fast) ? orc_num_cpus() : 1, nchunks, fn, ctx);
}

typedef struct {
    size_t m, k, n, padded_row, block_bytes, qoff, nblocks, chunk_rows;
    const uint8_t *w;
    const int8_t *xq;
    const float *dx;
    const float *x;
    int8_t *xq_out;
    float *dx_out;
    float *y;
} gemm_ctx;

static void simd_chunk(void *vctx, size_t c) {
    gemm_ctx *g = (gemm_ctx *)vctx;
    size_t i0 = c * g->chunk_rows;
    size_t i1 = i0 + g->chunk_rows < g->m ? i0 + g->chunk_rows : g->m;
    avx2_rows(i0, i1, g->k, g->n, g->w, g->padded_row, g->block_bytes,
              g->qoff, g->xq, g->dx, g->nblocks, g->y);
}

static void scalar_chunk(void *vctx, size_t c) {
    gemm_ctx *g = (gemm_ctx *)vctx;
    scalar_rows(c, c + 1, g->k, g->n, g->w, g->padded_row, g->block_bytes,
                g->qoff, g->xq, g->dx, g->nblocks, g->y);
}

static void quant_chunk(void *vctx, size_t nj) {
    gemm_ctx *g = (gemm_ctx *)vctx;
    orc_quantize_col(g->x, nj, g->k, g->n, g->nblocks, g->xq_out + nj * g->k,
                     g->dx_out + nj * g->nblocks);
}

void orc_q8_gemm(size_t m, size_t k, size_t n, const uint8_t *w,
                 size_t padded_row, size_t block_bytes, size_t qoff,
                 const float *x, float *y, int nthreads) {
    orc_q8_gemm_order(m, k, n, w, padded_row, block_bytes, qoff, x, y, nthreads, 0);
}

void orc_q8_gemm_order(size_t m, size_t k, size_t n, const uint8_t *w,
                       size_t padded_row, size_t block_bytes, size_t qoff,
                       const float *x, float *y, int nthreads, int scalar) {
    if (m == 0 || k == 0 || n == 0) return;
    int threads = nthreads > 0 ? nthreads : orc_num_cpus();
    size_t nblocks = (k + 31) / 32;
    int8_t *xq = calloc(n * k, 1);
    float *dx = calloc(n * nblocks, sizeof(float));
    gemm_ctx g = {m, k, n, padded_row, block_bytes, qoff, nblocks, 0,
                  w, xq, dx, x, xq, dx, y};
    int fast = !scalar && (m % 8 == 0) && (k % 32 == 0) && (n <= 16);
    /* simd_kernel.rs:129-144: columns quantised in parallel when
     * n*nblocks >= 1024; the scalar path quantises serially. */
    if (fast && n * nblocks >= 1024)
        parallel_chunks(threads, n, quant_chunk, &g);
    else
        quantize_all(x, k, n, nblocks, xq, dx);
    if (fast) {
        size_t per_thread = (m + (size_t)threads - 1) / (size_t)threads;
        size_t cr = per_thread < 32 ? 32 : (per_thread > 96 ? 96 : per_thread);
        cr = (cr + 7) / 8 * 8;
        g.chunk_rows = cr;
        parallel_chunks(threads, (m + cr - 1) / cr, simd_chunk, &g);
    } else if (m * nblocks <= 4096) {
        scalar_rows(0, m, k, n, w, padded_row, block_bytes, qoff, xq, dx,
                    nblocks, y);
    } else {
        parallel_chunks(threads, m, scalar_chunk, &g);
    }
    free(xq);
    free(dx);
}
