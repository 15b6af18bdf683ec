/*
 * sc_oracle_sgemm.c -- CPU oracle (test infrastructure only): the
 * reference's f32 GEMM `sgemm_kernel::gemm_into` -> `simd_kernel::
 * gemm_simd_into` (sgemm_kernel.rs:17-33, simd_kernel.rs:448-727), which
 * the pre-encode's pointwise convolutions run through
 * (nemotron/weights.rs:399-443).  Built with -ffp-contract=off: every
 * `mul_add` of the reference is an explicit fmaf, every `a * b` + `+=` is a
 * product and a sum rounded separately.
 *
 * Rounding per output c[i][j] (S = 16 lanes, simd_kernel.rs:47), with
 * k_main = (k / 16) * 16:
 *  - rows in whole 8-row tiles of a 256-row chunk (gemm_tile8, :560-627),
 *    columns in whole 16-column blocks: one fused multiply-add chain
 *    acc = fma(a[i][kk], b[kk][j], acc) for kk = 0 .. k_main - 1 from 0,
 *    a separately rounded tail ktail += a * b over kk >= k_main, then
 *    c = acc + ktail;
 *  - the same rows' last n % 16 columns (gemm_cols_tail, :688-727), and
 *    every column of rows outside whole 8-row tiles (gemm_row, :637-682):
 *    16 lane accumulators, lane l a fused chain over kk = l, l + 16, ...,
 *    < k_main; the separately rounded ktail; then
 *    c = reduce_sum(lanes) + ktail, reduce_sum being the ordered lane sum
 *    of std::simd (start -0.0, lanes 0..15 in order).  Starting from +0.0
 *    instead gives the same c, because `+ ktail` (ktail starts at +0.0)
 *    turns a -0.0 sum into +0.0 either way.
 */
#include <immintrin.h>
#include <math.h>
#include <stddef.h>

#include "sc_oracle.h"

#define SG_S 16

static float lanes_dot(const float *arow, const float *bt_col, size_t k) {
    float lane[SG_S];
    for (int l = 0; l < SG_S; l++) lane[l] = 0.0f;
    size_t kk = 0;
    for (; kk + SG_S <= k; kk += SG_S)
        for (int l = 0; l < SG_S; l++) lane[l] = fmaf(arow[kk + l], bt_col[kk + l], lane[l]);
    float ktail = 0.0f;
    for (; kk < k; kk++) ktail += arow[kk] * bt_col[kk];
    float r = -0.0f;
    for (int l = 0; l < SG_S; l++) r += lane[l];
    return r + ktail;
}

/* ---- AVX2 lanes (the reference's gemm_simd_chunk_avx2 build): the same
 * chains, eight outputs (whole-block columns) or eight k lanes per vector.
 * An explicit _mm256_fmadd_ps is one fused multiply-add per lane, like
 * fmaf; _mm256_mul_ps then _mm256_add_ps round twice, like `ktail += a*b`. */
__attribute__((target("avx2,fma"))) static float lanes_dot_avx2(const float *arow, const float *bt_col,
                                                                 size_t k) {
    __m256 l0 = _mm256_setzero_ps(), l1 = _mm256_setzero_ps();
    size_t kk = 0;
    for (; kk + SG_S <= k; kk += SG_S) {
        l0 = _mm256_fmadd_ps(_mm256_loadu_ps(arow + kk), _mm256_loadu_ps(bt_col + kk), l0);
        l1 = _mm256_fmadd_ps(_mm256_loadu_ps(arow + kk + 8), _mm256_loadu_ps(bt_col + kk + 8), l1);
    }
    float ktail = 0.0f;
    for (; kk < k; kk++) ktail += arow[kk] * bt_col[kk];
    float lane[SG_S];
    _mm256_storeu_ps(lane, l0);
    _mm256_storeu_ps(lane + 8, l1);
    float r = -0.0f;
    for (int l = 0; l < SG_S; l++) r += lane[l];
    return r + ktail;
}

/* rows [i0, i0 + rows) of one 256-row chunk */
__attribute__((target("avx2,fma"))) static void gemm_chunk_avx2(size_t i0, size_t rows, size_t k, size_t n,
                                                                 const float *a, const float *b,
                                                                 const float *bt, float *c) {
    const size_t k_main = k / SG_S * SG_S, n_main = n / SG_S * SG_S, tiled = rows / 8 * 8;
    for (size_t r0 = 0; r0 < tiled; r0 += 4) {
        const float *ar[4];
        for (int r = 0; r < 4; r++) ar[r] = a + (i0 + r0 + r) * k;
        for (size_t j = 0; j < n_main; j += SG_S) {
            __m256 acc[4][2], kt[4][2];
            for (int r = 0; r < 4; r++) {
                acc[r][0] = acc[r][1] = _mm256_setzero_ps();
                kt[r][0] = kt[r][1] = _mm256_setzero_ps();
            }
            for (size_t kk = 0; kk < k_main; kk++) {
                const __m256 b0 = _mm256_loadu_ps(b + kk * n + j), b1 = _mm256_loadu_ps(b + kk * n + j + 8);
                for (int r = 0; r < 4; r++) {
                    const __m256 av = _mm256_set1_ps(ar[r][kk]);
                    acc[r][0] = _mm256_fmadd_ps(av, b0, acc[r][0]);
                    acc[r][1] = _mm256_fmadd_ps(av, b1, acc[r][1]);
                }
            }
            for (size_t kk = k_main; kk < k; kk++) {
                const __m256 b0 = _mm256_loadu_ps(b + kk * n + j), b1 = _mm256_loadu_ps(b + kk * n + j + 8);
                for (int r = 0; r < 4; r++) {
                    const __m256 av = _mm256_set1_ps(ar[r][kk]);
                    kt[r][0] = _mm256_add_ps(kt[r][0], _mm256_mul_ps(av, b0));
                    kt[r][1] = _mm256_add_ps(kt[r][1], _mm256_mul_ps(av, b1));
                }
            }
            for (int r = 0; r < 4; r++) {
                float *cr = c + (i0 + r0 + r) * n + j;
                _mm256_storeu_ps(cr, _mm256_add_ps(acc[r][0], kt[r][0]));
                _mm256_storeu_ps(cr + 8, _mm256_add_ps(acc[r][1], kt[r][1]));
            }
        }
        for (int r = 0; r < 4; r++)
            for (size_t j = n_main; j < n; j++) c[(i0 + r0 + r) * n + j] = lanes_dot_avx2(ar[r], bt + j * k, k);
    }
    for (size_t r = tiled; r < rows; r++)
        for (size_t j = 0; j < n; j++) c[(i0 + r) * n + j] = lanes_dot_avx2(a + (i0 + r) * k, bt + j * k, k);
}

typedef struct {
    size_t m, k, n, chunk_rows;
    const float *a, *b, *bt;
    float *c;
} sgemm_ctx;

static void sgemm_chunk(void *vctx, size_t ci) {
    const sgemm_ctx *g = (const sgemm_ctx *)vctx;
    const size_t i0 = ci * g->chunk_rows;
    const size_t rows = g->m - i0 < g->chunk_rows ? g->m - i0 : g->chunk_rows;
    gemm_chunk_avx2(i0, rows, g->k, g->n, g->a, g->b, g->bt, g->c);
}

/* c[m, n] = a[m, k] @ b[k, n], all row-major (the reference's layouts);
 * bt is scratch of n * k floats (the [n, k] transpose the reference builds
 * when n % 16 != 0 or m % 8 != 0).  The reference's rayon split over
 * 256-row chunks (simd_kernel.rs:475-497) changes only which thread
 * computes an output; the fast path runs it on the oracle's pool with AVX2
 * lanes, the serial path below is the scalar restatement. */
void orc_gemm_simd_into(size_t m, size_t k, size_t n, const float *a, const float *b, float *c,
                        float *bt) {
    if (m == 0 || k == 0 || n == 0) return;
    for (size_t kk = 0; kk < k; kk++)
        for (size_t j = 0; j < n; j++) bt[j * k + kk] = b[kk * n + j];
    const size_t chunk_rows = m < 256 ? m : 256;
    if (orc_get_fast() && orc_have_avx2()) {
        sgemm_ctx g = {m, k, n, chunk_rows, a, b, bt, c};
        orc_parallel((m + chunk_rows - 1) / chunk_rows, sgemm_chunk, &g);
        return;
    }
    const size_t k_main = k / SG_S * SG_S, n_main = n / SG_S * SG_S;
    for (size_t i0 = 0; i0 < m; i0 += chunk_rows) {
        size_t rows = m - i0 < chunk_rows ? m - i0 : chunk_rows;
        size_t tiled = rows / 8 * 8;
        for (size_t r = 0; r < rows; r++) {
            size_t i = i0 + r;
            const float *arow = a + i * k;
            if (r < tiled) {
                for (size_t j = 0; j < n_main; j++) {
                    float acc = 0.0f;
                    for (size_t kk = 0; kk < k_main; kk++) acc = fmaf(arow[kk], b[kk * n + j], acc);
                    float ktail = 0.0f;
                    for (size_t kk = k_main; kk < k; kk++) ktail += arow[kk] * b[kk * n + j];
                    c[i * n + j] = acc + ktail;
                }
                for (size_t j = n_main; j < n; j++) c[i * n + j] = lanes_dot(arow, bt + j * k, k);
            } else {
                for (size_t j = 0; j < n; j++) c[i * n + j] = lanes_dot(arow, bt + j * k, k);
            }
        }
    }
}
