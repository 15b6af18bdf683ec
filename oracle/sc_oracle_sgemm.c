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

/* c[m, n] = a[m, k] @ b[k, n], all row-major (the reference's layouts);
 * bt is scratch of n * k floats (the [n, k] transpose the reference builds
 * when n % 16 != 0 or m % 8 != 0). Serial: the reference's rayon split
 * over 256-row chunks (simd_kernel.rs:483-497) does not change any
 * output's arithmetic, only which thread computes it. */
void orc_gemm_simd_into(size_t m, size_t k, size_t n, const float *a, const float *b, float *c,
                        float *bt) {
    if (m == 0 || k == 0 || n == 0) return;
    for (size_t kk = 0; kk < k; kk++)
        for (size_t j = 0; j < n; j++) bt[j * k + kk] = b[kk * n + j];
    const size_t chunk_rows = m < 256 ? m : 256;
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
