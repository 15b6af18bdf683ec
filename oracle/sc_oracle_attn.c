/*
 * sc_oracle_attn.c -- CPU oracle (test infrastructure only) for the
 * cache-aware streaming rel-pos attention of she-workss/stealcode
 * `audio_engine`: score_dot, softmax_v and the band loop of block_new.
 * Built with -ffp-contract=off (see sc_oracle.h).
 */
#include "sc_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>

#define S_LANES 16 /* simd_kernel.rs:44 `const S: usize = 16` */

/* AVX2 build of score_dot (two 8-lane vectors = the 16 SIMD lanes): the
 * same two fused multiply-adds per lane and the same ordered lane sum. */
__attribute__((target("avx2,fma"))) static float score_dot_avx2(const float *qu, const float *uh,
                                                                 const float *qv, const float *vh,
                                                                 const float *kk, const float *p,
                                                                 size_t hd, float scale) {
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + S_LANES <= hd; i += S_LANES) {
        for (int h = 0; h < 2; h++) {
            const size_t o = i + 8 * (size_t)h;
            const __m256 quv = _mm256_add_ps(_mm256_loadu_ps(qu + o), _mm256_loadu_ps(uh + o));
            const __m256 qvv = _mm256_add_ps(_mm256_loadu_ps(qv + o), _mm256_loadu_ps(vh + o));
            __m256 *acc = h ? &a1 : &a0;
            const __m256 inner = _mm256_fmadd_ps(qvv, _mm256_loadu_ps(p + o), *acc);
            *acc = _mm256_fmadd_ps(quv, _mm256_loadu_ps(kk + o), inner);
        }
    }
    float acc[S_LANES];
    _mm256_storeu_ps(acc, a0);
    _mm256_storeu_ps(acc + 8, a1);
    float sum = acc[0];
    for (int l = 1; l < S_LANES; l++) sum += acc[l];
    for (; i < hd; i++) sum += (qu[i] + uh[i]) * kk[i] + (qv[i] + vh[i]) * p[i];
    return sum * scale;
}

/* the P.V lanes of softmax_v over 16-dim blocks, AVX2 */
__attribute__((target("avx2,fma"))) static size_t softmax_pv_avx2(const float *e, float inv, size_t k0,
                                                                   size_t k1, const float *const *vrows,
                                                                   size_t head_dim, float *out) {
    size_t j = 0;
    for (; j + S_LANES <= head_dim; j += S_LANES) {
        __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
        for (size_t kk = k0, ii = 0; kk < k1; kk++, ii++) {
            const __m256 w = _mm256_set1_ps(e[ii] * inv);
            a0 = _mm256_fmadd_ps(w, _mm256_loadu_ps(vrows[kk] + j), a0);
            a1 = _mm256_fmadd_ps(w, _mm256_loadu_ps(vrows[kk] + j + 8), a1);
        }
        _mm256_storeu_ps(out + j, a0);
        _mm256_storeu_ps(out + j + 8, a1);
    }
    return j;
}

/* simd_kernel.rs:919-983 */
float orc_score_dot(const float *qu, const float *uh, const float *qv,
                    const float *vh, const float *kk, const float *p,
                    size_t hd, float scale) {
    if (orc_get_fast() && orc_have_avx2()) return score_dot_avx2(qu, uh, qv, vh, kk, p, hd, scale);
    float acc[S_LANES] = {0};
    size_t i = 0;
    while (i + S_LANES <= hd) {
        for (int l = 0; l < S_LANES; l++) {
            /* (quv + uhv).mul_add(kkv, (qvv + vhv).mul_add(pv, acc)) */
            float inner = fmaf(qv[i + l] + vh[i + l], p[i + l], acc[l]);
            acc[l] = fmaf(qu[i + l] + uh[i + l], kk[i + l], inner);
        }
        i += S_LANES;
    }
    float sum = acc[0];
    for (int l = 1; l < S_LANES; l++) sum += acc[l];
    for (; i < hd; i++) {
        sum += (qu[i] + uh[i]) * kk[i] + (qv[i] + vh[i]) * p[i];
    }
    return sum * scale;
}

/* simd_kernel.rs:1010-1104 (both the stack-cache and heap branches compute
 * the same values; only where `e` lives differs). */
void orc_softmax_v(const float *srow, size_t k0, size_t k1, size_t n_heads,
                   size_t h, const float *const *vrows, size_t head_dim,
                   float *out) {
    float maxv = -INFINITY;
    for (size_t kk = k0; kk < k1; kk++) maxv = fmaxf(maxv, srow[kk * n_heads + h]);
    size_t band = k1 - k0;
    float *e = malloc((band ? band : 1) * sizeof(float));
    float sum = 0.0f;
    for (size_t kk = k0, i = 0; kk < k1; kk++, i++) {
        float val = orc_expf(srow[kk * n_heads + h] - maxv);
        e[i] = val;
        sum += val;
    }
    float inv = 1.0f / sum;
    size_t j = 0;
    if (orc_get_fast() && orc_have_avx2()) j = softmax_pv_avx2(e, inv, k0, k1, vrows, head_dim, out);
    while (j + S_LANES <= head_dim) {
        float acc[S_LANES] = {0};
        for (size_t kk = k0, ii = 0; kk < k1; kk++, ii++) {
            const float *v = vrows[kk];
            float wgt = e[ii] * inv;
            for (int l = 0; l < S_LANES; l++) acc[l] = fmaf(wgt, v[j + l], acc[l]);
        }
        for (int l = 0; l < S_LANES; l++) out[j + l] = acc[l];
        j += S_LANES;
    }
    for (; j < head_dim; j++) {
        float acc = 0.0f;
        for (size_t kk = k0, ii = 0; kk < k1; kk++, ii++) {
            acc += e[ii] * inv * vrows[kk][j];
        }
        out[j] = acc;
    }
    free(e);
}

/* streaming.rs:498-503: chunk-aligned band of query frame qq, clipped at
 * k_hi. */
static void band_of(size_t qq, size_t chunk, size_t left_chunks, size_t k_hi,
                    size_t *k_min, size_t *k_max) {
    size_t q_chunk = qq / chunk;
    size_t lo_chunk = q_chunk > left_chunks ? q_chunk - left_chunks : 0;
    *k_min = lo_chunk * chunk;
    size_t hi = (q_chunk + 1) * chunk;
    *k_max = hi < k_hi ? hi : k_hi;
}

/* streaming.rs:492-589 over a band buffer (AttnStreamKernel::forward's
 * parameter list, gpu/kernels.rs:1137-1156). */
void orc_attn_stream(const float *q, const float *kv, const float *vv,
                     const float *pos_p, const float *q_bias,
                     const float *v_bias, size_t c, size_t d, size_t n_heads,
                     float scale, size_t s, size_t k_lo, size_t band,
                     size_t chunk, size_t left_chunks, size_t k_hi,
                     size_t pos_off, float *out) {
    size_t head_dim = d / n_heads;
    float *srow = calloc((band ? band : 1) * n_heads, sizeof(float));
    const float **vrows = malloc((band ? band : 1) * sizeof(float *));
    for (size_t qi = 0; qi < c; qi++) {
        size_t qq = s + qi;
        size_t k_min, k_max;
        band_of(qq, chunk, left_chunks, k_hi, &k_min, &k_max);
        size_t k0 = k_min - k_lo, k1 = k_max - k_lo;
        for (size_t h = 0; h < n_heads; h++) {
            size_t hd = h * head_dim;
            const float *qh = q + qi * d + hd;
            for (size_t kk = k0; kk < k1; kk++) {
                size_t fr = k_lo + kk;
                size_t pr = qq + pos_off - fr;
                srow[kk * n_heads + h] =
                    orc_score_dot(qh, q_bias + hd, qh, v_bias + hd,
                                  kv + kk * d + hd, pos_p + pr * d + hd,
                                  head_dim, scale);
            }
        }
        for (size_t h = 0; h < n_heads; h++) {
            size_t hd = h * head_dim;
            for (size_t kk = k0; kk < k1; kk++) vrows[kk] = vv + kk * d + hd;
            orc_softmax_v(srow, k0, k1, n_heads, h, vrows, head_dim,
                          out + qi * d + hd);
        }
    }
    free(srow);
    free(vrows);
}

/* gpu/kernels.rs:1920-1960: the reference test's own CPU loop. */
void orc_attn_stream_testloop(const float *q, const float *kv,
                              const float *vv, const float *pos_p,
                              const float *q_bias, const float *v_bias,
                              size_t c, size_t d, size_t n_heads, float scale,
                              size_t s, size_t k_lo, size_t chunk,
                              size_t left_chunks, size_t k_hi, size_t pos_off,
                              float *out) {
    size_t head_dim = d / n_heads;
    for (size_t qi = 0; qi < c; qi++) {
        size_t qq = s + qi;
        size_t k_min, k_max;
        band_of(qq, chunk, left_chunks, k_hi, &k_min, &k_max);
        size_t k0 = k_min - k_lo, k1 = k_max - k_lo;
        for (size_t h = 0; h < n_heads; h++) {
            size_t hoff = h * head_dim;
            float maxv = -INFINITY, sum = 0.0f;
            float *exps = calloc(k1 ? k1 : 1, sizeof(float));
            for (size_t kk = k0; kk < k1; kk++) {
                size_t fr = k_lo + kk;
                size_t pr = qq + pos_off - fr;
                float acc = 0.0f;
                for (size_t i = 0; i < head_dim; i++) {
                    float qui = q[qi * d + hoff + i] + q_bias[hoff + i];
                    float qvi = q[qi * d + hoff + i] + v_bias[hoff + i];
                    acc += qui * kv[kk * d + hoff + i] +
                           qvi * pos_p[pr * d + hoff + i];
                }
                float sc = acc * scale;
                maxv = fmaxf(maxv, sc);
                exps[kk] = sc;
            }
            for (size_t kk = k0; kk < k1; kk++) {
                exps[kk] = orc_expf(exps[kk] - maxv);
                sum += exps[kk];
            }
            float inv = 1.0f / sum;
            for (size_t i = 0; i < head_dim; i++) {
                float acc = 0.0f;
                for (size_t kk = k0; kk < k1; kk++)
                    acc += exps[kk] * inv * vv[kk * d + hoff + i];
                out[qi * d + hoff + i] = acc;
            }
            free(exps);
        }
    }
}
