/*
 * sc_oracle_enc.c -- CPU oracle (test infrastructure only) for the
 * streaming FastConformer encoder step of she-workss/stealcode
 * `audio_engine`.  Built with -ffp-contract=off (see sc_oracle.h); every
 * function cites the reference file:line it restates.
 */
#include "sc_oracle_enc.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "sc_oracle.h"

#define S_LANES 16

/* ------------------------------------------------------------------ */
/* helper kernels                                                      */
/* ------------------------------------------------------------------ */

/* simd_kernel.rs:734-805 (ln_forward_impl) */
void orc_ln_forward(const float *x, const float *w, const float *b, float eps,
                    float *out, size_t d) {
    float sum = 0.0f;
    size_t i = 0;
    while (i + S_LANES <= d) {
        float cs = x[i];
        for (int l = 1; l < S_LANES; l++) cs += x[i + l];
        sum += cs;
        i += S_LANES;
    }
    for (; i < d; i++) sum += x[i];
    float mean = sum / (float)d;
    float var = 0.0f;
    i = 0;
    while (i + S_LANES <= d) {
        float diff = x[i] - mean;
        float cs = diff * diff;
        for (int l = 1; l < S_LANES; l++) {
            diff = x[i + l] - mean;
            cs += diff * diff;
        }
        var += cs;
        i += S_LANES;
    }
    for (; i < d; i++) {
        float diff = x[i] - mean;
        var += diff * diff;
    }
    float inv = 1.0f / sqrtf(var / (float)d + eps);
    i = 0;
    while (i + S_LANES <= d) {
        for (int l = 0; l < S_LANES; l++)
            out[i + l] = fmaf(x[i + l] - mean, w[i + l] * inv, b[i + l]);
        i += S_LANES;
    }
    for (; i < d; i++) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* simd_kernel.rs:817-839: v * (1 + exp(-v)).recip() */
void orc_silu_inplace(float *v, size_t n) {
    for (size_t i = 0; i < n; i++) v[i] = v[i] * (1.0f / (1.0f + orc_expf(-v[i])));
}

static void relu_inplace(float *v, size_t n) {
    for (size_t i = 0; i < n; i++) v[i] = fmaxf(v[i], 0.0f);
}

/* simd_kernel.rs:868-910: out[t, i] = h[t, i] * sigmoid(h[t, d + i]) */
void orc_glu_from(const float *h, size_t t, size_t d, float *out) {
    for (size_t tt = 0; tt < t; tt++)
        for (size_t i = 0; i < d; i++) {
            float gate = h[tt * 2 * d + i], val = h[tt * 2 * d + d + i];
            out[tt * d + i] = gate * (1.0f / (1.0f + orc_expf(-val)));
        }
}

/* simd_kernel.rs:1160-1235 (the S-lane body uses mul_add; the scalar tail
 * uses separate multiply and add) */
void orc_dwconv_forward(const float *x, size_t t, size_t dim, size_t kh,
                        size_t pad_left, size_t pad_right, const float *w,
                        float *out) {
    size_t t_out = t + pad_left + pad_right - kh + 1;
    size_t vec_dim = dim / S_LANES * S_LANES;
    for (size_t ot = 0; ot < t_out; ot++) {
        long t0 = (long)ot - (long)pad_left;
        for (size_t c = 0; c < dim; c++) {
            float acc = 0.0f;
            for (size_t k = 0; k < kh; k++) {
                long ti = t0 + (long)k;
                if (ti < 0 || ti >= (long)t) continue;
                float xv = x[(size_t)ti * dim + c], wv = w[c * kh + k];
                acc = c < vec_dim ? fmaf(xv, wv, acc) : acc + xv * wv;
            }
            out[ot * dim + c] = acc;
        }
    }
}

/* streaming.rs:236-249 */
void orc_pos_rows(size_t n_pos, size_t d, long pos_lo, float *out) {
    float ln10000 = logf(10000.0f);
    for (size_t i = 0; i < n_pos; i++) {
        float pos = (float)i + (float)pos_lo;
        for (size_t kk = 0; kk < d / 2; kk++) {
            float div = expf(-2.0f * (float)kk * ln10000 / (float)d);
            out[i * d + 2 * kk] = sinf(pos * div);
            out[i * d + 2 * kk + 1] = cosf(pos * div);
        }
    }
}

static void transpose(const float *x, size_t rows, size_t cols, float *out) {
    for (size_t r = 0; r < rows; r++)
        for (size_t c = 0; c < cols; c++) out[c * rows + r] = x[r * cols + c];
}

/* ------------------------------------------------------------------ */
/* weights                                                             */
/* ------------------------------------------------------------------ */
typedef struct {
    const uint8_t *w; /* Q8 blocks, rows x padded_row */
    size_t rows, row_len;
    const float *bias; /* optional */
} lin_t;

typedef struct {
    const float *w, *b;
} ln_t;

typedef struct {
    const float *w, *b;
    size_t out, inp, kh, kw, groups;
} conv2d_t;

typedef struct {
    ln_t norm_ff1, norm_att, norm_conv, conv_ln, norm_ff2, norm_out;
    lin_t ff1_1, ff1_2, q, k, v, pos, out, pw1, pw2, ff2_1, ff2_2;
    const float *pos_u, *pos_v, *dw;
} layer_t;

/* growable frame cache: frames [lo, lo + n) of width d */
typedef struct {
    float *data;
    size_t lo, n, cap, d;
} fcache;

struct orc_enc {
    orc_enc_config cfg;
    size_t chunk, left_chunks, n_pos, head_dim;
    layer_t *layers;
    conv2d_t conv0, conv2, conv3, conv5, conv6;
    lin_t pre_out;
    lin_t prompt0, prompt2; /* prompt MLP (optional): [d + n_prompts -> hidden], [hidden -> d] */
    size_t n_prompts;       /* 0: the model has no prompt MLP */
    int prompt_id;          /* -1: none */
    float **pos_p; /* per layer [n_pos, d], NULL until the first step */
    fcache *kc, *vc, *glu;
    fcache out;    /* last block output frames */
    size_t total;
    size_t last_c;
    int scalar_gemm; /* 1: every linear in q8_gemm_scalar's arithmetic */
    int exp_cr;      /* exp mode of this encoder's steps (orc_set_exp_mode) */
    float *last_pre; /* [c, d] */
    float **last_blk;
    int dump_layer;
    float *dump[8]; /* stages of dump_layer, [c, d] each */
    double *tm;     /* seconds: [0] pre-encode, [1] Q8 linears, [2] attention, [3] encode_new total,
                       [4] Q8 linears inside the pre-encode */
};

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static const orc_tensor *find(const orc_tensor *t, int n, const char *name) {
    for (int i = 0; i < n; i++)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

static int get_f32(const orc_tensor *t, int n, const char *name, size_t numel,
                   const float **out, char *err, size_t err_len, int optional) {
    const orc_tensor *x = find(t, n, name);
    if (!x) {
        if (optional) {
            *out = NULL;
            return 0;
        }
        snprintf(err, err_len, "tensor %s not found", name);
        return -1;
    }
    size_t cnt = 1;
    for (int i = 0; i < x->n_dims; i++) cnt *= (size_t)x->dims[i];
    if (x->dtype != 0 || cnt != numel) {
        snprintf(err, err_len, "tensor %s: dtype %d, %zu elements (want f32, %zu)", name, x->dtype, cnt, numel);
        return -1;
    }
    *out = (const float *)x->data;
    return 0;
}

/* nemotron/weights.rs:640-697 (load_lin for dtype 8, direct [out, in]) */
static int get_lin(const orc_tensor *t, int n, const char *base, size_t inp,
                   size_t out, lin_t *l, char *err, size_t err_len) {
    char name[256];
    snprintf(name, sizeof name, "%s.weight", base);
    const orc_tensor *x = find(t, n, name);
    if (!x || x->dtype != 8 || x->n_dims != 2 || (size_t)x->dims[0] != inp ||
        (size_t)x->dims[1] != out) {
        snprintf(err, err_len, "tensor %s missing or not Q8 [%zu -> %zu]", name, inp, out);
        return -1;
    }
    l->w = (const uint8_t *)x->data;
    l->rows = out;
    l->row_len = inp;
    snprintf(name, sizeof name, "%s.bias", base);
    return get_f32(t, n, name, out, &l->bias, err, err_len, 1);
}

static int get_ln(const orc_tensor *t, int n, const char *base, size_t d, ln_t *l,
                  char *err, size_t err_len) {
    char name[256];
    snprintf(name, sizeof name, "%s.weight", base);
    if (get_f32(t, n, name, d, &l->w, err, err_len, 0)) return -1;
    snprintf(name, sizeof name, "%s.bias", base);
    return get_f32(t, n, name, d, &l->b, err, err_len, 0);
}

static int get_conv(const orc_tensor *t, int n, const char *base, size_t inp,
                    size_t out, size_t k, size_t groups, conv2d_t *c, char *err,
                    size_t err_len) {
    char name[256];
    snprintf(name, sizeof name, "%s.weight", base);
    if (get_f32(t, n, name, out * (inp / groups) * k * k, &c->w, err, err_len, 0)) return -1;
    snprintf(name, sizeof name, "%s.bias", base);
    if (get_f32(t, n, name, out, &c->b, err, err_len, 0)) return -1;
    c->out = out;
    c->inp = inp;
    c->kh = c->kw = k;
    c->groups = groups;
    return 0;
}

/* Lin::forward_t (nemotron/weights.rs:305-337): y_t [out, t] = W x_t [inp, t] + b */
static void lin_forward_t(const orc_enc *e, const lin_t *l, const float *x_t, size_t t, float *y_t) {
    size_t padded_row = (l->row_len + 31) / 32 * 34;
    const double t0 = now_s();
    orc_q8_gemm_order(l->rows, l->row_len, t, l->w, padded_row, 34, 2, x_t, y_t, orc_get_fast() ? 0 : 1,
                      e->scalar_gemm);
    e->tm[1] += now_s() - t0;
    if (l->bias)
        for (size_t j = 0; j < l->rows; j++)
            for (size_t tt = 0; tt < t; tt++) y_t[j * t + tt] += l->bias[j];
}

/* time-major [t, inp] -> time-major [t, out] through forward_t's layout */
static void lin_tm(const orc_enc *e, const lin_t *l, const float *x, size_t t, float *y, float *scratch_a,
                   float *scratch_b) {
    transpose(x, t, l->row_len, scratch_a);
    lin_forward_t(e, l, scratch_a, t, scratch_b);
    transpose(scratch_b, l->rows, t, y);
}

/* ------------------------------------------------------------------ */
/* pre-encode: nemotron/weights.rs:386-524 (Conv2d::forward; pointwise  */
/* convs through simd_kernel.rs:448-727 gemm_simd_into),               */
/* nemotron/encoder.rs:400-482 (pre_encode_forward)                     */
/* ------------------------------------------------------------------ */
static size_t conv_dim(size_t in, size_t pad0, size_t pad1, size_t k, size_t stride) {
    return (in + pad0 + pad1 - k) / stride + 1;
}

typedef struct {
    const conv2d_t *cv;
    const float *x;
    float *out;
    size_t t_in, f_in, f_out, pad0, stride;
} conv_ctx;

/* every output channel of output position sp (the reference's par_chunks
 * slot): bias, then products summed over (ic, kt, kf) in order */
static void conv_position(void *vctx, size_t sp) {
    const conv_ctx *g = (const conv_ctx *)vctx;
    const conv2d_t *cv = g->cv;
    const size_t c_out = cv->out, c_in = cv->inp, in_groups = c_in / cv->groups;
    const size_t ot = sp / g->f_out, of = sp % g->f_out;
    for (size_t oc = 0; oc < c_out; oc++) {
        size_t ic0 = (oc % cv->groups) * in_groups;
        size_t wbase = oc * in_groups * cv->kh * cv->kw;
        float acc = cv->b[oc];
        for (size_t ic = 0; ic < in_groups; ic++)
            for (size_t kt = 0; kt < cv->kh; kt++) {
                long ti = (long)(ot * g->stride + kt) - (long)g->pad0;
                if (ti < 0 || ti >= (long)g->t_in) continue;
                for (size_t kf = 0; kf < cv->kw; kf++) {
                    long fi = (long)(of * g->stride + kf) - (long)g->pad0;
                    if (fi < 0 || fi >= (long)g->f_in) continue;
                    acc += g->x[((size_t)ti * g->f_in + (size_t)fi) * c_in + ic0 + ic] *
                           cv->w[wbase + (ic * cv->kh + kt) * cv->kw + kf];
                }
            }
        g->out[sp * c_out + oc] = acc;
    }
}

static float *conv2d_forward(const conv2d_t *cv, const float *x, size_t t_in, size_t f_in,
                             size_t pad0, size_t pad1, size_t stride, size_t *t_o, size_t *f_o) {
    size_t t_out = conv_dim(t_in, pad0, pad1, cv->kh, stride);
    size_t f_out = conv_dim(f_in, pad0, pad1, cv->kw, stride);
    size_t c_out = cv->out, c_in = cv->inp;
    float *out = calloc(t_out * f_out * c_out, sizeof(float));
    if (cv->kh == 1 && cv->kw == 1 && stride == 1) {
        /* pointwise (weights.rs:399-443): x [spatial, c_in] transposed to
         * [c_in, spatial], the f32 GEMM W [c_out, c_in] x [c_in, spatial]
         * (gemm_simd_into's rounding, sc_oracle_sgemm.c), bias added row by
         * row, transposed back */
        size_t spatial = t_in * f_in;
        float *xt = calloc(c_in * spatial + 1, sizeof(float));
        float *yt = malloc(c_out * spatial * sizeof(float));
        float *bt = malloc(c_in * spatial * sizeof(float));
        for (size_t sp = 0; sp < spatial; sp++)
            for (size_t ic = 0; ic < c_in; ic++) xt[ic * spatial + sp] = x[sp * c_in + ic];
        orc_gemm_simd_into(c_out, c_in, spatial, cv->w, xt, yt, bt);
        for (size_t oc = 0; oc < c_out; oc++)
            for (size_t sp = 0; sp < spatial; sp++) yt[oc * spatial + sp] += cv->b[oc];
        for (size_t sp = 0; sp < spatial; sp++)
            for (size_t oc = 0; oc < c_out; oc++) out[sp * c_out + oc] = yt[oc * spatial + sp];
        free(xt);
        free(yt);
        free(bt);
    } else {
        /* direct conv (weights.rs:444-524): rayon over output positions when
         * there are at least 8 of them (each position's channels are one
         * task), serial otherwise; either way every output is the same
         * ordered sum */
        conv_ctx g = {cv, x, out, t_in, f_in, f_out, pad0, stride};
        const size_t spatial = t_out * f_out;
        if (spatial >= 8)
            orc_parallel(spatial, conv_position, &g);
        else
            for (size_t sp = 0; sp < spatial; sp++) conv_position(&g, sp);
    }
    *t_o = t_out;
    *f_o = f_out;
    return out;
}

/* returns [t_out, d] */
static float *pre_encode_forward(const orc_enc *e, const float *mel, size_t t_mel,
                                 size_t n_mels, size_t *t_out) {
    size_t t = t_mel, f = n_mels, t2, f2;
    float *x0 = conv2d_forward(&e->conv0, mel, t, f, 2, 1, 2, &t2, &f2);
    relu_inplace(x0, t2 * f2 * e->conv0.out);
    t = t2, f = f2;
    float *x2 = conv2d_forward(&e->conv2, x0, t, f, 2, 1, 2, &t2, &f2);
    free(x0);
    t = t2, f = f2;
    float *x3 = conv2d_forward(&e->conv3, x2, t, f, 0, 0, 1, &t2, &f2);
    free(x2);
    relu_inplace(x3, t2 * f2 * e->conv3.out);
    float *x5 = conv2d_forward(&e->conv5, x3, t, f, 2, 1, 2, &t2, &f2);
    free(x3);
    t = t2, f = f2;
    float *x6 = conv2d_forward(&e->conv6, x5, t, f, 0, 0, 1, &t2, &f2);
    free(x5);
    relu_inplace(x6, t * f * e->conv6.out);
    size_t C = (size_t)e->cfg.conv_channels, flat = f * C, d = (size_t)e->cfg.d_model;
    float *flat_x = malloc(t * flat * sizeof(float));
    for (size_t tt = 0; tt < t; tt++)
        for (size_t c = 0; c < C; c++)
            for (size_t ff = 0; ff < f; ff++) flat_x[tt * flat + c * f + ff] = x6[(tt * f + ff) * C + c];
    free(x6);
    float *y = malloc(t * d * sizeof(float));
    float *sa = malloc(t * flat * sizeof(float)), *sb = malloc(t * d * sizeof(float));
    lin_tm(e, &e->pre_out, flat_x, t, y, sa, sb);
    free(sa);
    free(sb);
    free(flat_x);
    *t_out = t;
    return y;
}

/* ------------------------------------------------------------------ */
/* caches                                                              */
/* ------------------------------------------------------------------ */
static void fc_init(fcache *c, size_t d) {
    memset(c, 0, sizeof *c);
    c->d = d;
}
static void fc_drop_before(fcache *c, size_t frame) {
    if (frame <= c->lo) return;
    size_t drop = frame - c->lo;
    if (drop > c->n) drop = c->n;
    memmove(c->data, c->data + drop * c->d, (c->n - drop) * c->d * sizeof(float));
    c->n -= drop;
    c->lo += drop;
}
static void fc_append(fcache *c, const float *rows, size_t n) {
    if (c->n + n > c->cap) {
        c->cap = (c->n + n) * 2;
        c->data = realloc(c->data, c->cap * c->d * sizeof(float));
    }
    memcpy(c->data + c->n * c->d, rows, n * c->d * sizeof(float));
    c->n += n;
}
static const float *fc_row(const fcache *c, size_t frame) { return c->data + (frame - c->lo) * c->d; }

/* ------------------------------------------------------------------ */
/* create / destroy                                                     */
/* ------------------------------------------------------------------ */
orc_enc *orc_enc_create(const orc_enc_config *cfg, const orc_tensor *t, int n, char *err,
                        size_t err_len) {
    orc_enc *e = calloc(1, sizeof *e);
    e->cfg = *cfg;
    e->tm = calloc(5, sizeof(double));
    size_t d = (size_t)cfg->d_model, dff = (size_t)cfg->d_ff, C = (size_t)cfg->conv_channels;
    e->chunk = (size_t)cfg->att_right + 1;
    e->left_chunks = (size_t)cfg->att_left / e->chunk;
    e->n_pos = (e->left_chunks + 2) * e->chunk - 1;
    e->head_dim = d / (size_t)cfg->n_heads;
    e->layers = calloc((size_t)cfg->n_layers, sizeof(layer_t));
    char b[192], nm[256];
    int rc = 0;
    rc |= get_conv(t, n, "encoder.pre_encode.conv.0", 1, C, 3, 1, &e->conv0, err, err_len);
    rc |= get_conv(t, n, "encoder.pre_encode.conv.2", C, C, 3, C, &e->conv2, err, err_len);
    rc |= get_conv(t, n, "encoder.pre_encode.conv.3", C, C, 1, 1, &e->conv3, err, err_len);
    rc |= get_conv(t, n, "encoder.pre_encode.conv.5", C, C, 3, C, &e->conv5, err, err_len);
    rc |= get_conv(t, n, "encoder.pre_encode.conv.6", C, C, 1, 1, &e->conv6, err, err_len);
    size_t f_out = (size_t)cfg->feat_in;
    for (int i = 0; i < 3; i++) f_out = (f_out + 3 - 3) / 2 + 1;
    rc |= get_lin(t, n, "encoder.pre_encode.out", f_out * C, d, &e->pre_out, err, err_len);
    /* optional multilingual prompt MLP (nemotron/encoder.rs:260-270) */
    e->prompt_id = -1;
    {
        const orc_tensor *p0 = find(t, n, "prompt_kernel.0.weight");
        if (p0 && p0->n_dims == 2 && (size_t)p0->dims[0] > d) {
            size_t np = (size_t)p0->dims[0] - d, hid = (size_t)p0->dims[1];
            rc |= get_lin(t, n, "prompt_kernel.0", d + np, hid, &e->prompt0, err, err_len);
            rc |= get_lin(t, n, "prompt_kernel.2", hid, d, &e->prompt2, err, err_len);
            e->n_prompts = np;
        }
    }
    for (int i = 0; i < cfg->n_layers && !rc; i++) {
        layer_t *L = &e->layers[i];
        snprintf(b, sizeof b, "encoder.layers.%d", i);
#define LN(f, s) (snprintf(nm, sizeof nm, "%s.%s", b, s), get_ln(t, n, nm, d, &L->f, err, err_len))
#define LIN(f, s, in, out) (snprintf(nm, sizeof nm, "%s.%s", b, s), get_lin(t, n, nm, in, out, &L->f, err, err_len))
        rc |= LN(norm_ff1, "norm_feed_forward1");
        rc |= LIN(ff1_1, "feed_forward1.linear1", d, dff);
        rc |= LIN(ff1_2, "feed_forward1.linear2", dff, d);
        rc |= LN(norm_att, "norm_self_att");
        rc |= LIN(q, "self_attn.linear_q", d, d);
        rc |= LIN(k, "self_attn.linear_k", d, d);
        rc |= LIN(v, "self_attn.linear_v", d, d);
        rc |= LIN(pos, "self_attn.linear_pos", d, d);
        rc |= LIN(out, "self_attn.linear_out", d, d);
        snprintf(nm, sizeof nm, "%s.self_attn.pos_bias_u", b);
        rc |= get_f32(t, n, nm, d, &L->pos_u, err, err_len, 0);
        snprintf(nm, sizeof nm, "%s.self_attn.pos_bias_v", b);
        rc |= get_f32(t, n, nm, d, &L->pos_v, err, err_len, 0);
        rc |= LN(norm_conv, "norm_conv");
        rc |= LIN(pw1, "conv.pointwise_conv1", d, 2 * d);
        snprintf(nm, sizeof nm, "%s.conv.depthwise_conv.weight", b);
        rc |= get_f32(t, n, nm, d * (size_t)cfg->conv_kernel, &L->dw, err, err_len, 0);
        rc |= LN(conv_ln, "conv.batch_norm");
        rc |= LIN(pw2, "conv.pointwise_conv2", d, d);
        rc |= LN(norm_ff2, "norm_feed_forward2");
        rc |= LIN(ff2_1, "feed_forward2.linear1", d, dff);
        rc |= LIN(ff2_2, "feed_forward2.linear2", dff, d);
        rc |= LN(norm_out, "norm_out");
#undef LN
#undef LIN
    }
    if (rc) {
        orc_enc_destroy(e);
        return NULL;
    }
    size_t nl = (size_t)cfg->n_layers;
    e->pos_p = calloc(nl, sizeof(float *));
    e->kc = calloc(nl, sizeof(fcache));
    e->vc = calloc(nl, sizeof(fcache));
    e->glu = calloc(nl, sizeof(fcache));
    e->last_blk = calloc(nl, sizeof(float *));
    for (size_t i = 0; i < nl; i++) {
        fc_init(&e->kc[i], d);
        fc_init(&e->vc[i], d);
        fc_init(&e->glu[i], d);
    }
    fc_init(&e->out, d);
    e->dump_layer = -1;
    return e;
}

void orc_enc_destroy(orc_enc *e) {
    if (!e) return;
    free(e->tm);
    size_t nl = (size_t)e->cfg.n_layers;
    for (size_t i = 0; e->pos_p && i < nl; i++) free(e->pos_p[i]);
    for (size_t i = 0; e->kc && i < nl; i++) {
        free(e->kc[i].data);
        free(e->vc[i].data);
        free(e->glu[i].data);
        free(e->last_blk[i]);
    }
    free(e->pos_p);
    free(e->kc);
    free(e->vc);
    free(e->glu);
    free(e->last_blk);
    free(e->out.data);
    free(e->last_pre);
    free(e->layers);
    for (int i = 0; i < 8; i++) free(e->dump[i]);
    free(e);
}

/* ------------------------------------------------------------------ */
/* block_new: streaming.rs:395-680                                      */
/* ------------------------------------------------------------------ */
static void dump_stage(orc_enc *e, size_t li, int stage, const float *src, size_t c, size_t width) {
    if ((int)li != e->dump_layer) return;
    size_t d = (size_t)e->cfg.d_model;
    free(e->dump[stage]);
    e->dump[stage] = malloc(c * d * sizeof(float));
    for (size_t j = 0; j < c; j++) memcpy(e->dump[stage] + j * d, src + j * width, d * sizeof(float));
}

typedef struct {
    const orc_enc *e;
    const layer_t *L;
    size_t li, s, k_lo, k_hi;
    long pos_lo;
    size_t band;
    const float *q_new, *k_new, *v_new;
    float *scores, *attn;
    float scale;
    int exp_cr;
} attn_ctx;

static void attn_band_of(const attn_ctx *g, size_t qi, size_t *k0, size_t *k1) {
    const orc_enc *e = g->e;
    size_t qq = g->s + qi, q_chunk = qq / e->chunk;
    size_t k_min = (q_chunk > e->left_chunks ? q_chunk - e->left_chunks : 0) * e->chunk;
    size_t k_max = (q_chunk + 1) * e->chunk < g->k_hi ? (q_chunk + 1) * e->chunk : g->k_hi;
    *k0 = k_min - g->k_lo;
    *k1 = k_max - g->k_lo;
}

/* score row of query qi: every head and band key (streaming.rs:505-523) */
static void attn_scores_row(void *vctx, size_t qi) {
    const attn_ctx *g = (const attn_ctx *)vctx;
    const orc_enc *e = g->e;
    const size_t d = (size_t)e->cfg.d_model, nh = (size_t)e->cfg.n_heads, hd = e->head_dim;
    size_t k0, k1;
    attn_band_of(g, qi, &k0, &k1);
    float *row = g->scores + qi * g->band * nh;
    const size_t qq = g->s + qi;
    for (size_t hh = 0; hh < nh; hh++) {
        size_t ho = hh * hd;
        const float *qh = g->q_new + qi * d + ho;
        for (size_t kk = k0; kk < k1; kk++) {
            size_t fr = g->k_lo + kk;
            const float *kd = fr < g->s ? fc_row(&e->kc[g->li], fr) + ho : g->k_new + (fr - g->s) * d + ho;
            size_t pr = (size_t)((long)qq - (long)fr - g->pos_lo);
            const float *prow = e->pos_p[g->li] + pr * d + ho;
            row[kk * nh + hh] =
                orc_score_dot(qh, g->L->pos_u + ho, qh, g->L->pos_v + ho, kd, prow, hd, g->scale);
        }
    }
}

/* softmax over the band + P.V of query qi, every head (streaming.rs:542-577);
 * the exp mode is per thread, so the task sets the encoder's */
static void attn_softmax_row(void *vctx, size_t qi) {
    const attn_ctx *g = (const attn_ctx *)vctx;
    const orc_enc *e = g->e;
    const size_t d = (size_t)e->cfg.d_model, nh = (size_t)e->cfg.n_heads, hd = e->head_dim;
    const int saved = orc_get_exp_mode();
    orc_set_exp_mode(g->exp_cr);
    size_t k0, k1;
    attn_band_of(g, qi, &k0, &k1);
    const float **vrows = malloc((g->band ? g->band : 1) * sizeof(float *));
    const float *row = g->scores + qi * g->band * nh;
    for (size_t hh = 0; hh < nh; hh++) {
        size_t ho = hh * hd;
        for (size_t kk = k0; kk < k1; kk++) {
            size_t fr = g->k_lo + kk;
            vrows[kk] = fr < g->s ? fc_row(&e->vc[g->li], fr) + ho : g->v_new + (fr - g->s) * d + ho;
        }
        orc_softmax_v(row, k0, k1, nh, hh, vrows, hd, g->attn + qi * d + ho);
    }
    free(vrows);
    orc_set_exp_mode(saved);
}

static void block_new(orc_enc *e, size_t li, const float *input, size_t s, size_t t_new,
                      size_t k_lo, size_t k_hi, long pos_lo, float *out) {
    const layer_t *L = &e->layers[li];
    size_t d = (size_t)e->cfg.d_model, dff = (size_t)e->cfg.d_ff, c = t_new - s;
    size_t nh = (size_t)e->cfg.n_heads, hd = e->head_dim;
    float eps = e->cfg.ln_eps, scale = 1.0f / sqrtf((float)hd);
    size_t big = (dff > 2 * d ? dff : 2 * d) * c;
    float *sa = malloc(big * sizeof(float)), *sb = malloc(big * sizeof(float));
    float *y = malloc(c * d * sizeof(float)), *tmp = malloc(c * d * sizeof(float));
    float *h = malloc(c * dff * sizeof(float)), *f = malloc(c * d * sizeof(float));

    /* macaron FF1 (:436-462) */
    for (size_t j = 0; j < c; j++) orc_ln_forward(input + j * d, L->norm_ff1.w, L->norm_ff1.b, eps, y + j * d, d);
    transpose(y, c, d, sa);
    lin_forward_t(e, &L->ff1_1, sa, c, h); /* [dff, c] */
    orc_silu_inplace(h, dff * c);
    lin_forward_t(e, &L->ff1_2, h, c, sb); /* [d, c] */
    transpose(sb, d, c, f);
    for (size_t i = 0; i < c * d; i++) y[i] = input[i] + 0.5f * f[i];
    dump_stage(e, li, 0, y, c, d);

    /* rel-pos MHSA (:464-600) */
    float *ln_new = malloc(c * d * sizeof(float));
    float *k_new = malloc(c * d * sizeof(float)), *v_new = malloc(c * d * sizeof(float)),
          *q_new = malloc(c * d * sizeof(float));
    for (size_t j = 0; j < c; j++) orc_ln_forward(y + j * d, L->norm_att.w, L->norm_att.b, eps, ln_new + j * d, d);
    lin_tm(e, &L->k, ln_new, c, k_new, sa, sb);
    lin_tm(e, &L->v, ln_new, c, v_new, sa, sb);
    lin_tm(e, &L->q, ln_new, c, q_new, sa, sb);
    dump_stage(e, li, 1, ln_new, c, d);
    dump_stage(e, li, 4, q_new, c, d);
    size_t band = k_hi - k_lo;
    float *scores = calloc(c * band * nh, sizeof(float));
    float *attn = calloc(c * d, sizeof(float));
    {
        /* streaming.rs:492-589: the score rows, then softmax + P.V, each
         * over queries on rayon when c * band * n_heads >= 2048 */
        const double t0 = now_s();
        attn_ctx g = {e, L, li, s, k_lo, k_hi, pos_lo, band, q_new, k_new, v_new, scores, attn, scale,
                      e->exp_cr};
        if (c * band * nh >= 2048) {
            orc_parallel(c, attn_scores_row, &g);
            orc_parallel(c, attn_softmax_row, &g);
        } else {
            for (size_t qi = 0; qi < c; qi++) attn_scores_row(&g, qi);
            for (size_t qi = 0; qi < c; qi++) attn_softmax_row(&g, qi);
        }
        e->tm[2] += now_s() - t0;
    }
    dump_stage(e, li, 2, attn, c, d);
    lin_tm(e, &L->out, attn, c, tmp, sa, sb);
    for (size_t i = 0; i < c * d; i++) y[i] += tmp[i];
    dump_stage(e, li, 3, y, c, d);

    /* conv module (:602-646) */
    size_t conv_left = (size_t)e->cfg.conv_left, kh = (size_t)e->cfg.conv_kernel;
    size_t conv_lo = s > conv_left ? s - conv_left : 0, n_glu = t_new - conv_lo, old_glu = s - conv_lo;
    float *lnc = malloc(c * d * sizeof(float)), *h2 = malloc(c * 2 * d * sizeof(float));
    float *glu_new = malloc(c * d * sizeof(float));
    for (size_t j = 0; j < c; j++) orc_ln_forward(y + j * d, L->norm_conv.w, L->norm_conv.b, eps, lnc + j * d, d);
    lin_tm(e, &L->pw1, lnc, c, h2, sa, sb);
    orc_glu_from(h2, c, d, glu_new);
    float *glu = malloc(n_glu * d * sizeof(float));
    for (size_t fr = conv_lo; fr < s; fr++) memcpy(glu + (fr - conv_lo) * d, fc_row(&e->glu[li], fr), d * sizeof(float));
    memcpy(glu + old_glu * d, glu_new, c * d * sizeof(float));
    size_t t_out = n_glu + conv_left + 0 - kh + 1;
    float *conv = malloc(t_out * d * sizeof(float));
    orc_dwconv_forward(glu, n_glu, d, kh, conv_left, 0, L->dw, conv);
    float *o2 = malloc(c * d * sizeof(float));
    for (size_t j = 0; j < c; j++) {
        orc_ln_forward(conv + (old_glu + j) * d, L->conv_ln.w, L->conv_ln.b, eps, o2 + j * d, d);
        orc_silu_inplace(o2 + j * d, d);
    }
    dump_stage(e, li, 5, o2, c, d);
    lin_tm(e, &L->pw2, o2, c, tmp, sa, sb);
    for (size_t i = 0; i < c * d; i++) y[i] += tmp[i];
    dump_stage(e, li, 6, y, c, d);

    /* macaron FF2 + final LN (:648-679) */
    float *y2 = malloc(c * d * sizeof(float));
    for (size_t j = 0; j < c; j++) orc_ln_forward(y + j * d, L->norm_ff2.w, L->norm_ff2.b, eps, y2 + j * d, d);
    transpose(y2, c, d, sa);
    lin_forward_t(e, &L->ff2_1, sa, c, h);
    orc_silu_inplace(h, dff * c);
    lin_forward_t(e, &L->ff2_2, h, c, sb);
    transpose(sb, d, c, f);
    for (size_t i = 0; i < c * d; i++) y2[i] = y[i] + 0.5f * f[i];
    for (size_t j = 0; j < c; j++) orc_ln_forward(y2 + j * d, L->norm_out.w, L->norm_out.b, eps, out + j * d, d);
    dump_stage(e, li, 7, out, c, d);

    /* caches: the caller appends K/V and GLU after the block (:307-312) */
    fc_append(&e->kc[li], k_new, c);
    fc_append(&e->vc[li], v_new, c);
    fc_append(&e->glu[li], glu_new, c);

    free(sa), free(sb), free(y), free(tmp), free(h), free(f), free(ln_new), free(k_new), free(v_new);
    free(q_new), free(scores), free(attn), free(lnc), free(h2), free(glu_new), free(glu);
    free(conv), free(o2), free(y2);
}

/* ------------------------------------------------------------------ */
/* encode_new: streaming.rs:137-383                                     */
/* ------------------------------------------------------------------ */
static int encode_new(orc_enc *e, const float *mel, size_t mel_frames, size_t n_mels, size_t t0,
                      size_t t1, int fin);

int orc_enc_encode_new(orc_enc *e, const float *mel, size_t mel_frames, size_t n_mels, size_t t0,
                       size_t t1, int fin) {
    int saved = orc_get_exp_mode();
    orc_set_exp_mode(e->exp_cr);
    const double ts = now_s();
    int rc = encode_new(e, mel, mel_frames, n_mels, t0, t1, fin);
    e->tm[3] += now_s() - ts;
    orc_set_exp_mode(saved);
    return rc;
}

void orc_enc_phase_times(const orc_enc *e, double *out) {
    out[0] = e->tm[0];
    out[1] = e->tm[1] - e->tm[4];
    out[2] = e->tm[2];
    out[3] = e->tm[3];
}

static int encode_new(orc_enc *e, const float *mel, size_t mel_frames, size_t n_mels, size_t t0,
                      size_t t1, int fin) {
    size_t d = (size_t)e->cfg.d_model, nl = (size_t)e->cfg.n_layers;
    size_t s = t0 / 8, ecount = s + (t1 - t0 + 7) / 8;
    if (s != e->total) return -6;
    size_t tail = t1 - t0;
    size_t t_new = fin ? s + (((tail / 2 + 1) / 2 + 1) / 2 + 1) : ecount;
    if (t_new <= s) return 0;
    size_t c = t_new - s;

    /* pre_encode window (:182-218) */
    size_t mel_lo = s * 8, win_start = mel_lo > 24 ? mel_lo - 24 : 0;
    size_t start_rel = (mel_lo - win_start) / 8, rel_max = start_rel + c - 1;
    size_t avail = mel_frames > win_start ? mel_frames - win_start : 0;
    size_t want = 8 * rel_max + 1 > t_new * 8 - win_start ? 8 * rel_max + 1 : t_new * 8 - win_start;
    size_t t_mel = avail < want ? avail : want;
    float *win = calloc((t_mel ? t_mel : 1) * n_mels, sizeof(float));
    size_t take = avail < t_mel ? avail : t_mel;
    memcpy(win, mel + win_start * n_mels, take * n_mels * sizeof(float));
    size_t t_pe;
    const double tp = now_s(), tg = e->tm[1];
    float *pe = pre_encode_forward(e, win, t_mel, n_mels, &t_pe);
    e->tm[0] += now_s() - tp;
    e->tm[4] += e->tm[1] - tg;
    free(win);
    if (t_pe < start_rel + c) {
        free(pe);
        return -1;
    }
    free(e->last_pre);
    e->last_pre = malloc(c * d * sizeof(float));
    memcpy(e->last_pre, pe + start_rel * d, c * d * sizeof(float));
    free(pe);

    /* band and pos rows (:226-261) */
    size_t k_lo = (s / e->chunk > e->left_chunks ? s / e->chunk - e->left_chunks : 0) * e->chunk;
    size_t k_hi = t_new;
    long pos_lo = 1 - (long)e->chunk;
    if (!e->pos_p[0]) {
        float *pet = malloc(e->n_pos * d * sizeof(float));
        orc_pos_rows(e->n_pos, d, pos_lo, pet);
        float *sa = malloc(e->n_pos * d * sizeof(float)), *sb = malloc(e->n_pos * d * sizeof(float));
        for (size_t b = 0; b < nl; b++) {
            e->pos_p[b] = malloc(e->n_pos * d * sizeof(float));
            lin_tm(e, &e->layers[b].pos, pet, e->n_pos, e->pos_p[b], sa, sb);
        }
        free(sa), free(sb), free(pet);
    }
    /* slide the band caches (:263-277) */
    for (size_t b = 0; b < nl; b++) {
        fc_drop_before(&e->kc[b], k_lo);
        fc_drop_before(&e->vc[b], k_lo);
        if (e->kc[b].n == 0) e->kc[b].lo = e->vc[b].lo = k_lo > s ? s : k_lo;
    }
    /* blocks (:279-318) */
    float *in = malloc(c * d * sizeof(float)), *outb = malloc(c * d * sizeof(float));
    memcpy(in, e->last_pre, c * d * sizeof(float));
    for (size_t b = 0; b < nl; b++) {
        if (e->kc[b].n == 0) e->kc[b].lo = e->vc[b].lo = s;
        if (e->glu[b].n == 0) e->glu[b].lo = s;
        block_new(e, b, in, s, t_new, k_lo, k_hi, pos_lo, outb);
        free(e->last_blk[b]);
        e->last_blk[b] = malloc(c * d * sizeof(float));
        memcpy(e->last_blk[b], outb, c * d * sizeof(float));
        float *tswap = in;
        in = outb;
        outb = tswap;
        size_t keep = t_new > (size_t)e->cfg.conv_left ? t_new - (size_t)e->cfg.conv_left : 0;
        fc_drop_before(&e->glu[b], keep);
    }
    /* prompt MLP on the new frames (streaming.rs:320-342):
     * out = prompt2(relu(prompt0([x ; onehot(prompt_id)]))) */
    if (e->n_prompts && e->prompt_id >= 0 && (size_t)e->prompt_id < e->n_prompts) {
        size_t np = e->n_prompts, cat_in = d + np, hid = e->prompt0.rows;
        float *cat = calloc(cat_in * c, sizeof(float));
        for (size_t j = 0; j < c; j++) {
            memcpy(cat + j * cat_in, in + j * d, d * sizeof(float));
            cat[j * cat_in + d + (size_t)e->prompt_id] = 1.0f;
        }
        float *sa = malloc((cat_in > hid ? cat_in : hid) * c * sizeof(float));
        float *sb = malloc((hid > d ? hid : d) * c * sizeof(float));
        float *h = malloc(hid * c * sizeof(float));
        transpose(cat, c, cat_in, sa);
        lin_forward_t(e, &e->prompt0, sa, c, h); /* [hid, c] */
        for (size_t i = 0; i < hid * c; i++) h[i] = h[i] > 0.0f ? h[i] : 0.0f; /* relu_into: v.max(0) */
        lin_forward_t(e, &e->prompt2, h, c, sb); /* [d, c] */
        transpose(sb, d, c, in);
        free(cat), free(sa), free(sb), free(h);
    }
    if (e->out.n == 0) e->out.lo = s;
    fc_append(&e->out, in, c);
    free(in), free(outb);
    e->total = t_new;
    e->last_c = c;
    return 0;
}

size_t orc_enc_total(const orc_enc *e) { return e->total; }

int orc_enc_frames(const orc_enc *e, size_t from, size_t to, float *out) {
    if (from < e->out.lo || to > e->out.lo + e->out.n || to <= from) return -1;
    memcpy(out, fc_row(&e->out, from), (to - from) * e->out.d * sizeof(float));
    return 0;
}

int orc_enc_last(const orc_enc *e, int which, float *out, size_t *c_out) {
    size_t d = (size_t)e->cfg.d_model;
    *c_out = e->last_c;
    const float *src = which == 0 ? e->last_pre : (which - 1 < e->cfg.n_layers ? e->last_blk[which - 1] : NULL);
    if (!src) return -1;
    memcpy(out, src, e->last_c * d * sizeof(float));
    return 0;
}

void orc_enc_set_gemm_order(orc_enc *e, int scalar) { e->scalar_gemm = scalar ? 1 : 0; }

int orc_enc_set_prompt(orc_enc *e, int prompt_id) {
    if (prompt_id >= 0 && (!e->n_prompts || (size_t)prompt_id >= e->n_prompts)) return -1;
    e->prompt_id = prompt_id;
    return 0;
}

void orc_enc_set_exp_mode(orc_enc *e, int correctly_rounded) { e->exp_cr = correctly_rounded ? 1 : 0; }

void orc_enc_set_dump(orc_enc *e, int layer) { e->dump_layer = layer; }

int orc_enc_dump(const orc_enc *e, int stage, float *out, size_t *c_out) {
    if (stage < 0 || stage >= 8 || !e->dump[stage]) return -1;
    *c_out = e->last_c;
    memcpy(out, e->dump[stage], e->last_c * (size_t)e->cfg.d_model * sizeof(float));
    return 0;
}
