/*
 * sc_oracle_rnnt.c -- CPU oracle (TEST INFRASTRUCTURE ONLY) of the RNN-T
 * greedy decoder of the streaming transcriber: the predictor (embedding +
 * LSTM layers with the ih/hh matrices merged per row, nemotron/decoder.rs:
 * 75-205), the joint network (decoder.rs:207-235) and live.rs:56-145
 * `decode_frames` with the carried per-stream state.  Linears go through
 * orc_q8_gemm_order (the reference's q8_gemm dispatch, or q8_gemm_scalar's
 * order), exp/tanh through orc_expf/orc_tanhf (libm, or correctly
 * rounded).  Paths are relative to the reference's crates/audio_engine/src/.
 */
#include "sc_oracle_enc.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sc_oracle.h"

typedef struct {
    uint8_t *w; /* owned copy (merged rows) or NULL */
    const uint8_t *wp;
    size_t rows, row_len;
    const float *bias;
} rlin_t;

struct orc_rnnt {
    orc_rnnt_config cfg;
    const float *embed;   /* [vocab][hidden] */
    rlin_t *merged;       /* per layer [4H][2H]: row j = ih row j ++ hh row j */
    float **bias;         /* per layer ih_b + hh_b */
    rlin_t jenc, jpred, jout;
    int scalar_gemm, exp_cr;
};

struct orc_rnnt_state {
    size_t L, H;
    float *h, *c, *nh, *nc; /* [L][H] */
    int32_t last_token;
};

static const orc_tensor *rfind(const orc_tensor *t, int n, const char *name) {
    for (int i = 0; i < n; i++)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

static size_t numel(const orc_tensor *x) {
    size_t c = 1;
    for (int i = 0; i < x->n_dims; i++) c *= (size_t)x->dims[i];
    return c;
}

/* load_lin (weights.rs:640-697) for a Q8_0 tensor with GGUF dims [in, out] */
static int rlin(const orc_tensor *t, int n, const char *base, size_t inp, size_t out, rlin_t *l, char *err,
                size_t err_len) {
    char name[256];
    snprintf(name, sizeof name, "%s.weight", base);
    const orc_tensor *x = rfind(t, n, name);
    if (!x || x->dtype != 8 || x->n_dims != 2 || (size_t)x->dims[0] != inp || (size_t)x->dims[1] != out) {
        snprintf(err, err_len, "tensor %s missing or not Q8 [%zu -> %zu]", name, inp, out);
        return -1;
    }
    l->w = NULL;
    l->wp = (const uint8_t *)x->data;
    l->rows = out;
    l->row_len = inp;
    snprintf(name, sizeof name, "%s.bias", base);
    const orc_tensor *b = rfind(t, n, name);
    if (b && (b->dtype != 0 || numel(b) != out)) {
        snprintf(err, err_len, "tensor %s mis-shaped", name);
        return -1;
    }
    l->bias = b ? (const float *)b->data : NULL;
    return 0;
}

orc_rnnt *orc_rnnt_create(const orc_rnnt_config *cfg, const orc_tensor *t, int n, char *err, size_t err_len) {
    orc_rnnt *r = calloc(1, sizeof *r);
    r->cfg = *cfg;
    size_t H = (size_t)cfg->hidden, L = (size_t)cfg->n_layers, J = (size_t)cfg->joint;
    int rc = 0;
    const orc_tensor *emb = rfind(t, n, "decoder.prediction.embed.weight");
    if (!emb || emb->dtype != 0 || numel(emb) != (size_t)cfg->vocab * H) {
        snprintf(err, err_len, "decoder.prediction.embed.weight missing or not f32 [vocab x hidden]");
        rc = -1;
    } else {
        r->embed = (const float *)emb->data;
    }
    r->merged = calloc(L, sizeof(rlin_t));
    r->bias = calloc(L, sizeof(float *));
    for (size_t i = 0; i < L && !rc; i++) {
        char a[128], b[128];
        snprintf(a, sizeof a, "decoder.prediction.dec_rnn.lstm.ih_l%zu", i);
        snprintf(b, sizeof b, "decoder.prediction.dec_rnn.lstm.hh_l%zu", i);
        rlin_t ih, hh;
        rc |= rlin(t, n, a, H, 4 * H, &ih, err, err_len);
        rc |= rlin(t, n, b, H, 4 * H, &hh, err, err_len);
        if (rc) break;
        if (!ih.bias || !hh.bias) {
            snprintf(err, err_len, "LSTM layer %zu: ih/hh bias missing", i);
            rc = -1;
            break;
        }
        /* Q8Mat::concat_rows (weights.rs:132-147): row j = ih row j ++ hh row j */
        size_t prow = H / 32 * 34;
        rlin_t *m = &r->merged[i];
        m->w = malloc(4 * H * 2 * prow);
        for (size_t j = 0; j < 4 * H; j++) {
            memcpy(m->w + j * 2 * prow, ih.wp + j * prow, prow);
            memcpy(m->w + j * 2 * prow + prow, hh.wp + j * prow, prow);
        }
        m->wp = m->w;
        m->rows = 4 * H;
        m->row_len = 2 * H;
        m->bias = NULL;
        r->bias[i] = malloc(4 * H * sizeof(float));
        for (size_t k = 0; k < 4 * H; k++) r->bias[i][k] = ih.bias[k] + hh.bias[k]; /* decoder.rs:93-111 */
    }
    if (!rc) rc |= rlin(t, n, "joint.enc", (size_t)cfg->d_enc, J, &r->jenc, err, err_len);
    if (!rc) rc |= rlin(t, n, "joint.pred", H, J, &r->jpred, err, err_len);
    if (!rc) rc |= rlin(t, n, "joint.joint_net.2", J, (size_t)cfg->vocab, &r->jout, err, err_len);
    if (!rc && (H % 32 || (size_t)cfg->d_enc % 32 || J % 32)) {
        snprintf(err, err_len, "hidden, d_enc and joint must be multiples of 32");
        rc = -1;
    }
    if (rc) {
        orc_rnnt_destroy(r);
        return NULL;
    }
    return r;
}

void orc_rnnt_destroy(orc_rnnt *r) {
    if (!r) return;
    for (size_t i = 0; r->merged && i < (size_t)r->cfg.n_layers; i++) free(r->merged[i].w);
    for (size_t i = 0; r->bias && i < (size_t)r->cfg.n_layers; i++) free(r->bias[i]);
    free(r->merged);
    free(r->bias);
    free(r);
}

void orc_rnnt_set_order(orc_rnnt *r, int scalar_gemm, int exp_cr) {
    r->scalar_gemm = scalar_gemm ? 1 : 0;
    r->exp_cr = exp_cr ? 1 : 0;
}

orc_rnnt_state *orc_rnnt_state_new(const orc_rnnt *r) {
    orc_rnnt_state *s = calloc(1, sizeof *s);
    s->L = (size_t)r->cfg.n_layers;
    s->H = (size_t)r->cfg.hidden;
    s->h = calloc(s->L * s->H, sizeof(float));
    s->c = calloc(s->L * s->H, sizeof(float));
    s->nh = calloc(s->L * s->H, sizeof(float));
    s->nc = calloc(s->L * s->H, sizeof(float));
    s->last_token = -1;
    return s;
}

void orc_rnnt_state_free(orc_rnnt_state *s) {
    if (!s) return;
    free(s->h), free(s->c), free(s->nh), free(s->nc);
    free(s);
}

void orc_rnnt_state_get(const orc_rnnt_state *s, float *h, float *c, int32_t *last_token) {
    memcpy(h, s->h, s->L * s->H * sizeof(float));
    memcpy(c, s->c, s->L * s->H * sizeof(float));
    *last_token = s->last_token;
}

/* Lin::matvec (weights.rs:157-182, 264-282): q8_gemm with n = 1, then bias */
static void matvec(const orc_rnnt *r, const rlin_t *l, const float *x, const float *bias, float *y) {
    size_t prow = l->row_len / 32 * 34;
    orc_q8_gemm_order(l->rows, l->row_len, 1, l->wp, prow, 34, 2, x, y, 0, r->scalar_gemm);
    if (bias)
        for (size_t j = 0; j < l->rows; j++) y[j] += bias[j];
}

static float sigmoid(float x) { return 1.0f / (1.0f + orc_expf(-x)); }

/* Predictor::step (decoder.rs:142-205): last_token < 0 feeds zeros */
static void predictor_step(const orc_rnnt *r, orc_rnnt_state *s) {
    size_t H = s->H;
    float *x = calloc(H, sizeof(float)), *xh = malloc(2 * H * sizeof(float));
    float *gates = malloc(4 * H * sizeof(float));
    if (s->last_token >= 0) memcpy(x, r->embed + (size_t)s->last_token * H, H * sizeof(float));
    for (size_t l = 0; l < s->L; l++) {
        const float *input = l == 0 ? x : s->nh + (l - 1) * H;
        memcpy(xh, input, H * sizeof(float));
        memcpy(xh + H, s->h + l * H, H * sizeof(float));
        matvec(r, &r->merged[l], xh, NULL, gates);
        for (size_t k = 0; k < 4 * H; k++) gates[k] += r->bias[l][k];
        const float *gi = gates, *gf = gates + H, *gg = gates + 2 * H, *go = gates + 3 * H;
        for (size_t k = 0; k < H; k++) {
            float ig = sigmoid(gi[k]), fg = sigmoid(gf[k]), g = orc_tanhf(gg[k]), og = sigmoid(go[k]);
            float cn = fg * s->c[l * H + k] + ig * g;
            s->nc[l * H + k] = cn;
            s->nh[l * H + k] = og * orc_tanhf(cn);
        }
    }
    free(x), free(xh), free(gates);
}

int orc_rnnt_decode_frames(orc_rnnt *r, orc_rnnt_state *st, const float *frames, size_t n, int32_t *ids,
                           int32_t *steps, int cap) {
    int saved = orc_get_exp_mode();
    orc_set_exp_mode(r->exp_cr);
    size_t d = (size_t)r->cfg.d_enc, J = (size_t)r->cfg.joint, V = (size_t)r->cfg.vocab;
    size_t H = st->H, L = st->L;
    /* enc_proj = joint.enc over the n frames (live.rs:73-81) */
    float *xt = malloc(d * n * sizeof(float)), *y = malloc(J * n * sizeof(float));
    for (size_t t = 0; t < n; t++)
        for (size_t i = 0; i < d; i++) xt[i * n + t] = frames[t * d + i];
    {
        size_t prow = d / 32 * 34;
        orc_q8_gemm_order(J, d, n, r->jenc.wp, prow, 34, 2, xt, y, 0, r->scalar_gemm);
        if (r->jenc.bias)
            for (size_t j = 0; j < J; j++)
                for (size_t t = 0; t < n; t++) y[j * n + t] += r->jenc.bias[j];
    }
    float *pred = malloc(J * sizeof(float)), *sum = malloc(J * sizeof(float)), *logits = malloc(V * sizeof(float));
    size_t max_iters = 16 * n + 64, step = 0, new_symbols = 0, iter = 0;
    int dirty = 1, emitted = 0;
    while (step < n && iter < max_iters) {
        iter++;
        if (dirty) {
            predictor_step(r, st);
            dirty = 0;
        }
        matvec(r, &r->jpred, st->nh + (L - 1) * H, r->jpred.bias, pred);
        for (size_t j = 0; j < J; j++) {
            float v = y[j * n + step] + pred[j];
            sum[j] = v > 0.0f ? v : 0.0f; /* (e + p).max(0.0) */
        }
        matvec(r, &r->jout, sum, r->jout.bias, logits);
        size_t best = 0;
        float bv = logits[0];
        for (size_t i = 1; i < V; i++)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        if ((int)best == r->cfg.blank) {
            step++;
            new_symbols = 0;
        } else {
            if (emitted < cap) {
                ids[emitted] = (int32_t)best;
                steps[emitted] = (int32_t)step;
            }
            emitted++;
            st->last_token = (int32_t)best;
            float *tmp = st->h;
            st->h = st->nh;
            st->nh = tmp;
            tmp = st->c;
            st->c = st->nc;
            st->nc = tmp;
            dirty = 1;
            new_symbols++;
            if (r->cfg.max_symbols > 0 && new_symbols >= (size_t)r->cfg.max_symbols) {
                step++;
                new_symbols = 0;
            }
        }
    }
    free(xt), free(y), free(pred), free(sum), free(logits);
    orc_set_exp_mode(saved);
    return iter >= max_iters ? -1 : emitted;
}
