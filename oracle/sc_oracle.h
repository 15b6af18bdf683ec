/*
 * sc_oracle.h -- CPU oracle for the Q8_0 GEMM and streaming attention hot
 * path of she-workss/stealcode's `audio_engine` crate.
 *
 * TEST INFRASTRUCTURE ONLY. This library is a plain-C restatement of the
 * reference's CPU operators. It is the parity checker for the CUDA library
 * and the timed CPU baseline; nothing in the product links or calls it.
 *
 * Floating-point semantics follow the Rust reference: no implicit FMA
 * contraction (the library is built with -ffp-contract=off), explicit
 * fmaf() wherever the reference calls `mul_add`, libm expf/sinf/cosf
 * (Rust's f32::exp/sin/cos lower to the same glibc routines on Linux),
 * and lane-ordered horizontal sums where the reference calls
 * `Simd::reduce_sum` (an ordered reduction).
 *
 * Every function cites the reference file:line it restates; paths are
 * relative to crates/audio_engine/src/.
 */
#ifndef SC_ORACLE_H
#define SC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* exp as the oracle evaluates it: mode 0 (default) is libm expf, what the
 * reference's f32::exp and Simd::exp call on Linux/glibc; mode 1 is the
 * correctly rounded exp, (float)exp((double)x), which differs from glibc's
 * expf by one ulp for about 6 inputs in 10^4.  The mode is per thread. */
void orc_set_exp_mode(int correctly_rounded);
int orc_get_exp_mode(void);
float orc_expf(float x);
/* tanh under the same mode: libm tanhf (the reference's f32::tanh), or
 * (float)tanh((double)x). */
float orc_tanhf(float x);

/* gguf.rs:365-397 */
float orc_f16_to_f32(uint16_t h);
/* sgemm_kernel.rs:209-221 (test helper half_f32_to_u16: truncating) */
uint16_t orc_half_from_f32_trunc(float v);

/* sgemm_kernel.rs:46-53 */
float orc_read_q8_scale(const uint8_t *w, size_t base, size_t block_bytes);

/* sgemm_kernel.rs:57-90. x is feature-major [k, n]; column nj. */
void orc_quantize_col(const float *x, size_t nj, size_t k, size_t n,
                      size_t nblocks, int8_t *xqrow, float *dxrow);

/* sgemm_kernel.rs:132-202 -- the reference's own test oracle. Single thread;
 * the reference's rayon split does not change results. */
void orc_q8_gemm_scalar(size_t m, size_t k, size_t n, const uint8_t *w,
                        size_t padded_row, size_t block_bytes, size_t qoff,
                        const float *x, float *y);

/* simd_kernel.rs:96-158 + 276-394: the SIMD kernel's accumulation order
 * (i16 pair fold, 8 f32 partial lanes per (row, column), mul_add per block,
 * ordered reduce_sum), written in portable C. Falls back to the scalar path
 * for shapes outside the fast path (m % 8, k % 32, n > 16), as the reference
 * dispatcher does. */
void orc_q8_gemm_simd_order(size_t m, size_t k, size_t n, const uint8_t *w,
                            size_t padded_row, size_t block_bytes,
                            size_t qoff, const float *x, float *y);

/* sgemm_kernel.rs:99-127 dispatcher as the timed CPU baseline: the SIMD
 * path uses AVX2+FMA intrinsics (the reference's only vector tier,
 * simd_kernel.rs:5-14) and splits rows across `nthreads` threads in chunks
 * of 32..96 rows (simd_kernel.rs:178-189); other shapes take the scalar
 * path, row-parallel when m*nblocks > 4096 (sgemm_kernel.rs:156-201).
 * nthreads <= 0 means all online cores. Results equal
 * orc_q8_gemm_simd_order / orc_q8_gemm_scalar bit for bit. */
void orc_q8_gemm(size_t m, size_t k, size_t n, const uint8_t *w,
                 size_t padded_row, size_t block_bytes, size_t qoff,
                 const float *x, float *y, int nthreads);
/* orc_q8_gemm with the dispatch pinned: scalar = 0 is the reference's own
 * dispatch (above); scalar = 1 always takes q8_gemm_scalar's arithmetic
 * (sgemm_kernel.rs:185-196), threaded over rows. */
void orc_q8_gemm_order(size_t m, size_t k, size_t n, const uint8_t *w,
                       size_t padded_row, size_t block_bytes, size_t qoff,
                       const float *x, float *y, int nthreads, int scalar);

/* Per-block integer dot products dots[(i*n + nj)*nblocks + b] =
 * sum_j w[i, 32b+j] * xq[nj, 32b+j] (the exact integer that the scalar
 * path accumulates in f32, sgemm_kernel.rs:171-174). */
void orc_q8_block_dots(size_t m, size_t k, size_t n, const uint8_t *w,
                       size_t padded_row, size_t block_bytes, size_t qoff,
                       const float *x, int32_t *dots);

/* simd_kernel.rs:919-999 (S = 16 lanes). */
float orc_score_dot(const float *qu, const float *uh, const float *qv,
                    const float *vh, const float *kk, const float *p,
                    size_t hd, float scale);

/* simd_kernel.rs:1010-1152. v rows: vrows[kk] points at head_dim floats for
 * band index kk (kk in [k0, k1)). */
void orc_softmax_v(const float *srow, size_t k0, size_t k1, size_t n_heads,
                   size_t h, const float *const *vrows, size_t head_dim,
                   float *out);

/* Streaming attention of one stream as block_new computes it
 * (streaming.rs:492-589), in the parameter list of the reference GPU
 * operator AttnStreamKernel::forward (gpu/kernels.rs:1137-1156): kv/vv hold
 * the band frames [k_lo, k_hi) row-major [band, d]; q is [c, d]; the pos row
 * for query qq and frame fr is pos_p[qq - fr + pos_off]. out is [c, d]. */
void orc_attn_stream(const float *q, const float *kv, const float *vv,
                     const float *pos_p, const float *q_bias,
                     const float *v_bias, size_t c, size_t d, size_t n_heads,
                     float scale, size_t s, size_t k_lo, size_t band,
                     size_t chunk, size_t left_chunks, size_t k_hi,
                     size_t pos_off, float *out);

/* The CPU loop of the reference's own GPU attention test
 * (gpu/kernels.rs:1920-1960): plain sequential sums, used to pin
 * orc_attn_stream against the reference's test oracle. */
void orc_attn_stream_testloop(const float *q, const float *kv,
                              const float *vv, const float *pos_p,
                              const float *q_bias, const float *v_bias,
                              size_t c, size_t d, size_t n_heads, float scale,
                              size_t s, size_t k_lo, size_t chunk,
                              size_t left_chunks, size_t k_hi, size_t pos_off,
                              float *out);

/* The reference's f32 GEMM (sgemm_kernel.rs:17-33 -> simd_kernel.rs:448-727,
 * gemm_simd_into): c[m, n] = a[m, k] @ b[k, n] row-major with its rounding
 * (fused chains for whole 8-row x 16-column tiles, 16-lane partial sums
 * and an ordered lane sum for the remaining columns and rows). bt: n * k
 * floats of scratch. */
void orc_gemm_simd_into(size_t m, size_t k, size_t n, const float *a, const float *b, float *c,
                        float *bt);

/* Online CPU count used by nthreads <= 0. */
int orc_num_cpus(void);

/* 1 (default): the reference's threading (rayon over 256-row chunks,
 * spatial positions and queries) and AVX2 lanes for the f32 GEMM,
 * score_dot and softmax_v; 0: every operator serial and scalar.  Both give
 * bit-identical outputs; the switch exists so tests can check that. */
void orc_set_fast(int on);
int orc_get_fast(void);
int orc_have_avx2(void);
/* Runs fn(ctx, 0 .. nchunks-1) on the oracle's persistent worker pool (all
 * host threads when fast, else on the caller); chunks are claimed
 * dynamically, like rayon's par_chunks_mut.  Not reentrant: fn must not
 * call orc_parallel. */
void orc_parallel(size_t nchunks, void (*fn)(void *ctx, size_t chunk), void *ctx);

#ifdef __cplusplus
}
#endif
#endif
