/*
 * sc_oracle_enc.h -- CPU oracle (TEST INFRASTRUCTURE ONLY) for the streaming
 * Nemotron/FastConformer encoder step: a plain-C restatement of the
 * reference's StreamingEncoder (streaming.rs:42-383), block_new
 * (streaming.rs:395-680), the causal pre-encode stack
 * (nemotron/encoder.rs:400-482) and the helper kernels they call
 * (simd_kernel.rs:734-910, 1160-1235; nemotron/weights.rs:345-579).
 * Paths are relative to the reference's crates/audio_engine/src/.
 *
 * Weights come as a table of named tensors using the GGUF tensor names the
 * reference loads (nemotron/encoder.rs:89-245): f32 tensors (dtype 0) and
 * Q8_0 tensors with f16 block scales (dtype 8, 34-byte blocks).
 */
#ifndef SC_ORACLE_ENC_H
#define SC_ORACLE_ENC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const char *name;
    int32_t dtype;      /* 0 = f32, 8 = Q8_0 (f16 scale, 34-byte blocks) */
    int32_t n_dims;
    int64_t dims[4];    /* GGUF order: fastest axis first */
    const void *data;
} orc_tensor;

typedef struct {
    int32_t d_model, n_layers, n_heads, d_ff;
    int32_t feat_in;        /* mel bins */
    int32_t conv_channels;  /* pre-encode channels */
    int32_t conv_kernel;    /* conformer depthwise kernel */
    int32_t conv_left;      /* causal left context = kernel - 1 */
    int32_t att_left;       /* att_context_left (frames) */
    int32_t att_right;      /* att_context_right; chunk = att_right + 1 */
    float ln_eps;
} orc_enc_config;

typedef struct orc_enc orc_enc;

/* Returns NULL (and fills err) when a tensor is missing or mis-shaped. */
orc_enc *orc_enc_create(const orc_enc_config *cfg, const orc_tensor *tensors,
                        int n_tensors, char *err, size_t err_len);
void orc_enc_destroy(orc_enc *e);
/* streaming.rs:137-383.  mel is time-major [mel_frames, n_mels] (all mel
 * frames of the stream so far); returns 0, -6 when t0 is out of sync. */
int orc_enc_encode_new(orc_enc *e, const float *mel, size_t mel_frames,
                       size_t n_mels, size_t t0, size_t t1, int fin);
size_t orc_enc_total(const orc_enc *e);
/* streaming.rs:111-127: copy frames [from, to) of the last block output. */
int orc_enc_frames(const orc_enc *e, size_t from, size_t to, float *out);
/* Stage outputs of the last step, for debugging parity: which = 0 pre-encode
 * output of the new frames [c, d]; 1 + b = block b output [c, d]. */
int orc_enc_last(const orc_enc *e, int which, float *out, size_t *c_out);

/* Arithmetic of the Q8_0 linears: 0 (default) the reference's dispatch
 * (the 8-lane SIMD order for 7-frame chunks, simd_kernel.rs:93-230),
 * 1 the scalar oracle's order (sgemm_kernel.rs:185-196) for every linear. */
void orc_enc_set_gemm_order(orc_enc *e, int scalar);
/* exp of this encoder's SiLU, GLU and softmax: 0 (default) libm expf as the
 * reference on glibc, 1 correctly rounded (orc_set_exp_mode). */
void orc_enc_set_exp_mode(orc_enc *e, int correctly_rounded);

/* Prompt of the multilingual prompt MLP applied to every new frame
 * (streaming.rs:320-342; tensors prompt_kernel.0 / prompt_kernel.2, whose
 * input width d + n_prompts gives n_prompts).  -1 = none (the default).
 * Returns -1 when the model has no prompt MLP or the id is out of range. */
int orc_enc_set_prompt(orc_enc *e, int prompt_id);

/* Stage dumps of one layer of the last step (the reference's
 * STEALCODE_DUMP_DIR block dumps): 0 after FF1, 1 attention LN, 2 attention
 * output, 3 after the attention residual, 4 q projection, 5 conv module
 * after dw + LN + SiLU, 6 after the conv residual, 7 block output. */
void orc_enc_set_dump(orc_enc *e, int layer);
int orc_enc_dump(const orc_enc *e, int stage, float *out, size_t *c_out);

/* Host seconds this encoder has spent in encode_new since it was created:
 * out[0] the pre-encode (convs and its linear), out[1] the Q8 linears of the
 * blocks and the prompt MLP, out[2] the attention (scores, softmax, P.V),
 * out[3] the whole of encode_new. */
void orc_enc_phase_times(const orc_enc *e, double *out);
/* Helper kernels, exposed for unit checks. */
void orc_ln_forward(const float *x, const float *w, const float *b,
                    float eps, float *out, size_t d);
void orc_silu_inplace(float *v, size_t n);
void orc_glu_from(const float *h, size_t t, size_t d, float *out);
void orc_dwconv_forward(const float *x, size_t t, size_t dim, size_t kh,
                        size_t pad_left, size_t pad_right, const float *w,
                        float *out);
/* streaming.rs:236-261: pos rows for pos in [1-chunk, (left_chunks+1)*chunk-1]
 * before the linear_pos projection: [n_pos, d] sin/cos rows. */
void orc_pos_rows(size_t n_pos, size_t d, long pos_lo, float *out);

/* ------------------------------------------------------------------ */
/* RNN-T greedy decoder (sc_oracle_rnnt.c): predictor LSTM + joint +
 * live.rs:56-145 decode_frames with a carried per-stream state.  Tensors:
 * decoder.prediction.embed.weight (f32 [vocab][hidden]),
 * decoder.prediction.dec_rnn.lstm.{ih,hh}_l<i>.{weight,bias} (Q8 [hidden ->
 * 4 hidden], f32 biases), joint.enc / joint.pred / joint.joint_net.2 (Q8,
 * optional f32 biases). */
typedef struct {
    int32_t d_enc, hidden, n_layers, joint, vocab, blank, max_symbols;
} orc_rnnt_config;

typedef struct orc_rnnt orc_rnnt;
typedef struct orc_rnnt_state orc_rnnt_state;

orc_rnnt *orc_rnnt_create(const orc_rnnt_config *cfg, const orc_tensor *tensors,
                          int n_tensors, char *err, size_t err_len);
void orc_rnnt_destroy(orc_rnnt *r);
/* scalar_gemm: every matvec in q8_gemm_scalar's order instead of the
 * reference's dispatch; exp_cr: correctly rounded exp/tanh. */
void orc_rnnt_set_order(orc_rnnt *r, int scalar_gemm, int exp_cr);
/* StreamState::new (live.rs:35-50): zero h/c, last_token -1. */
orc_rnnt_state *orc_rnnt_state_new(const orc_rnnt *r);
void orc_rnnt_state_free(orc_rnnt_state *s);
/* h, c: [n_layers][hidden] */
void orc_rnnt_state_get(const orc_rnnt_state *s, float *h, float *c, int32_t *last_token);
/* decode_frames over n frames [n][d_enc]: writes up to cap (id, step)
 * pairs and returns the number emitted, or -1 when the iteration cap
 * 16 n + 64 is hit (the reference's bail). */
int orc_rnnt_decode_frames(orc_rnnt *r, orc_rnnt_state *st, const float *frames, size_t n,
                           int32_t *ids, int32_t *steps, int cap);

#ifdef __cplusplus
}
#endif
#endif
