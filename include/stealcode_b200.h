/*
 * stealcode_b200.h -- C ABI of libstealcode_cuda.so, the B200 (sm_100a)
 * implementation of the streaming Nemotron/FastConformer encoder hot path of
 * she-workss/stealcode: the Q8_0 weight x f32 activation GEMM and the
 * cache-aware chunked streaming rel-pos self-attention.
 *
 * Conventions
 *   - Every function returns SC_OK (0) or a negative SC_ERR_* code and never
 *     aborts; sc_last_error() returns the calling thread's last message.
 *   - `stream` arguments are cudaStream_t values passed as void* (NULL = the
 *     legacy default stream).  Device-pointer entry points are asynchronous on
 *     that stream; *_host entry points are synchronous.
 *   - Reference citations are paths inside the reference's
 *     crates/audio_engine/src/ directory.
 *
 * Dimension names: the reference's CPU operator q8_gemm(m, k, n, ...) uses
 * m = output features (weight rows), k = input features, n = frames; the
 * device API below calls the frame count `t` and the weight rows `rows`.
 */
#ifndef STEALCODE_B200_H
#define STEALCODE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 1

#define SC_OK 0
#define SC_ERR_INVALID (-1)     /* bad argument or shape */
#define SC_ERR_ALLOC (-2)       /* device or host allocation failed */
#define SC_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define SC_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up */
#define SC_ERR_UNSUPPORTED (-5) /* valid input outside what the kernels take */
#define SC_ERR_STATE (-6)       /* call out of order (e.g. encoder out of sync) */

/* Activation / output layouts.
 * FEATURE_MAJOR: x is [k, t] (element (frame j, feature i) at x[i*ld + j]) and
 *   y is [rows, t] -- the reference CPU layout of q8_gemm / Lin::forward_t
 *   (sgemm_kernel.rs:92-97, nemotron/weights.rs:299-305).
 * TIME_MAJOR: x is [t, k] (x[j*ld + i]) and y is [t, rows] -- the layout of
 *   the reference wgpu kernel (gpu/shaders/q8_gemm.wgsl:1-8) and of the
 *   device encoder. */
#define SC_LAYOUT_FEATURE_MAJOR 0
#define SC_LAYOUT_TIME_MAJOR 1

/* Repacked Q8_0 weight matrix resident in device memory (opaque). */
typedef struct sc_q8w sc_q8w;

const char *sc_last_error(void);
int sc_abi_version(void);

/* Status bits that kernels set on the current device when a bounded
 * device-side wait gave up (SC_STATUS_WAIT_TIMEOUT); reading clears them.
 * Synchronous.  New in this library (the reference has no device waits). */
#define SC_STATUS_WAIT_TIMEOUT 1u
int sc_device_status(uint32_t *flags);

/* Number of CUDA kernel launches this library has issued in this process
 * (all devices, all entry points).  Diagnostic; no counterpart in the
 * reference. */
long long sc_launch_count(void);

/* Test hook for the allocation-failure paths: after this call the library's
 * device allocations fail (the entry point that needed one returns
 * SC_ERR_ALLOC and frees what it had allocated) once their total since the
 * call would exceed `bytes`; bytes < 0 removes the cap.  No counterpart in
 * the reference. */
int sc_debug_set_device_alloc_cap(int64_t bytes);

/* ---- weights --------------------------------------------------------- */

/* Repack a GGUF Q8_0 tensor once into the device layout: int8 quants in
 * 128-row x 32-column tiles plus a separate f16 scale array.  `blocks` (host)
 * holds `rows` rows of ceil(k/32) blocks of `block_bytes` bytes, scale at byte
 * 0 and quants at byte `qoff` -- exactly Q8Mat's bytes
 * (nemotron/weights.rs:91-111, as load_lin copies them from the GGUF,
 * nemotron/weights.rs:640-697).  Replaces the reference GPU backend's
 * load-time repack pack_q8 (gpu/kernels.rs:44-78).  Only the 34-byte
 * f16-scale block (GGUF dtype 8, qoff 2) is accepted; the 36-byte f32-scale
 * variant returns SC_ERR_UNSUPPORTED (pack_q8 has the same restriction: it
 * reads quants at byte 2).  Synchronous. */
int sc_q8_repack(const uint8_t *blocks, int64_t rows, int64_t k,
                 int64_t block_bytes, int64_t qoff, sc_q8w **out);
/* Same, from GGUF block bytes already in device memory; async on stream. */
int sc_q8_repack_device(const uint8_t *blocks_dev, int64_t rows, int64_t k,
                        int64_t block_bytes, int64_t qoff, void *stream,
                        sc_q8w **out);
int sc_q8w_free(sc_q8w *w);
/* Q8Mat::rows / Q8Mat::row_len (nemotron/weights.rs:113-119). */
int sc_q8w_shape(const sc_q8w *w, int64_t *rows, int64_t *k);
/* Device pointers of the repacked layout (for tests and tooling). */
int sc_q8w_device_layout(const sc_q8w *w, const int8_t **quants,
                         const uint16_t **scales, int64_t *rows_pad,
                         int64_t *nblocks);

/* ---- Q8_0 GEMM ------------------------------------------------------- */

/* Bytes of workspace sc_q8_gemm needs for t frames of k features. */
int64_t sc_q8_gemm_workspace_bytes(int64_t t, int64_t k);

/* y = W x (+ bias), device pointers: the device twin of q8_gemm
 * (sgemm_kernel.rs:99-127) and Lin::forward_t (nemotron/weights.rs:305-337).
 * Each activation frame is quantised per 32-block exactly as quantize_col
 * (sgemm_kernel.rs:57-90) does, then multiplied with exact int8 block dots
 * and an f32 per-block scale.  ldx/ldy <= 0 select the packed leading
 * dimension of the layout.  `workspace` (256-byte aligned, at least
 * sc_q8_gemm_workspace_bytes) may be NULL to use a per-device library
 * workspace, which is then shared by all NULL-workspace calls on that device
 * and must not be used from two streams at once.  t == 0 is a no-op, as in
 * the reference. */
int sc_q8_gemm(const sc_q8w *w, const float *x, int64_t t, int32_t x_layout,
               int64_t ldx, const float *bias, float *y, int32_t y_layout,
               int64_t ldy, void *workspace, int64_t workspace_bytes,
               void *stream);

/* Kernel half over pre-quantised activations -- q8_gemm_simd_q
 * (simd_kernel.rs:160-234), which lets callers that feed one input to several
 * matrices (the attention's Q/K/V) quantise once.  xq [t_pad][32*nblocks] and
 * dx [nblocks][t_pad] are what sc_q8_quantize writes with m = t_pad; frames
 * t .. t_pad-1 are ignored.  xq must be 16-byte aligned. */
int sc_q8_gemm_q(const sc_q8w *w, const int8_t *xq, const float *dx,
                 int64_t t, int64_t t_pad, const float *bias, float *y,
                 int32_t y_layout, int64_t ldy, void *stream);

/* n independent GEMMs y[i] = W[i] x[i] (+ bias[i]) of the same frame count
 * t (0..16) in one streaming pass over their weights (1 <= n <= 128; host
 * arrays of handles and device pointers; bias may be NULL or hold NULLs):
 * the batched form of q8_gemm (sgemm_kernel.rs:99-127) for the streaming
 * chunk's small M, where one GEMM's weights take HBM well under a
 * microsecond and a launch per GEMM would cost more than the weights.  Each
 * output agrees with sc_q8_gemm's within the same f32 tolerance (both use
 * the per-block fused multiply-add of the streaming kernel).  Packed leading
 * dimensions.  workspace (256-byte aligned, sc_q8_gemm_batch_workspace_bytes)
 * may be NULL for the per-device library workspace.  No counterpart in the
 * reference, which calls q8_gemm once per matrix.  Async on stream. */
int64_t sc_q8_gemm_batch_workspace_bytes(const sc_q8w *const *w, int32_t n);
int sc_q8_gemm_batch(const sc_q8w *const *w, const float *const *x,
                     const float *const *bias, float *const *y, int32_t n,
                     int64_t t, int32_t x_layout, int32_t y_layout,
                     void *workspace, int64_t workspace_bytes, void *stream);

/* Size of the fixed device array behind sc_q8_gemm_noalloc (4 MiB). */
#define SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES (4u << 20)

/* sc_q8_gemm for callers that must not allocate device memory; this entry
 * point has no counterpart in the reference.  Such callers are plugins that
 * run inside another framework's CUDA-graph capture (a cudaMalloc there
 * breaks the capture), real-time audio callbacks (cudaMalloc and cudaFree can
 * synchronise the device and stall the callback), and hosts that own all
 * device memory.  The quantised-activation scratch lives in a file-scope
 * device array of SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES, which every GPU that
 * loads the library holds until the process exits.  Calls whose scratch need
 * (sc_q8_gemm_workspace_bytes(t, k)) exceeds it return SC_ERR_INVALID; split
 * the frames over several calls.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current,
 * and does the one-time set-up of every GEMM kernel this entry point can
 * run (their status words' addresses and shared-memory limits), so later
 * calls of any frame count make no such host calls; make that first call
 * before any stream capture.  All calls share the one
 * array, so calls that overlap on the GPU (different streams, or different
 * host threads) race and corrupt each other's results; serialise them.  The
 * array keeps the previous call's contents, but every byte a call reads is
 * written earlier in that same call.  Arguments as sc_q8_gemm. */
int sc_q8_gemm_noalloc(const sc_q8w *w, const float *x, int64_t t,
                       int32_t x_layout, int64_t ldx, const float *bias,
                       float *y, int32_t y_layout, int64_t ldy, void *stream);

/* Q8Mat::gemm_t (nemotron/weights.rs:186-202) with host activations and
 * outputs: x_host is [k, t], y_host is [rows, t] (feature-major).  Copies
 * through a per-device staging buffer on the legacy default stream and
 * returns when y_host is written (pinned host buffers copy fastest). */
int sc_q8mat_gemm_t(const sc_q8w *w, const float *x_host, int64_t t,
                    float *y_host);

/* Byte-for-byte twin of q8_gemm (sgemm_kernel.rs:99-109): host weight
 * blocks, host x [k, n], host y [m, n]; repacks the weights on every call
 * (use sc_q8_repack + sc_q8mat_gemm_t to keep them resident). */
int sc_q8_gemm_host(size_t m, size_t k, size_t n, const uint8_t *w,
                    size_t padded_row, size_t block_bytes, size_t qoff,
                    const float *x, float *y);

/* The activation quantiser alone (quantize_col, sgemm_kernel.rs:57-90), for
 * bit-exact checks: xq is [m][32*ceil(k/32)] int8, dx is [ceil(k/32)][m]. */
int sc_q8_quantize(const float *x, int64_t m, int64_t k, int32_t x_layout,
                   int64_t ldx, int8_t *xq, float *dx, void *stream);

/* The GEMM's integer path alone: dots[(row*t + frame)*nblocks + b] = the
 * int32 dot of weight row `row` and quantised frame `frame` over block b --
 * the exact integer the reference accumulates (sgemm_kernel.rs:171-174). */
int sc_q8_block_dots(const sc_q8w *w, const float *x, int64_t t,
                     int32_t x_layout, int64_t ldx, int32_t *dots,
                     void *stream);

/* ---- streaming attention --------------------------------------------- */

/* AttnStreamKernel::forward (gpu/kernels.rs:1137-1156) on device pointers:
 * q [c, d], kv/vv the band frames [k_lo, k_hi) as [band, d], pos_p [n_pos, d],
 * q_bias/v_bias = pos_bias_u/pos_bias_v [d]; out [c, d].  Semantics of the CPU
 * path: block_new's score/softmax loops (streaming.rs:492-589) with score_dot
 * and softmax_v (simd_kernel.rs:919-1152).  band must equal k_hi - k_lo (1 ..
 * 256), c is 1..16, head_dim = d / n_heads is 64 or 128.  n_pos is new (the
 * reference passes pos_p as a slice) and is used to reject out-of-range pos
 * rows. */
int sc_attn_stream(const float *q, const float *kv, const float *vv,
                   const float *pos_p, int64_t n_pos, const float *q_bias,
                   const float *v_bias, int64_t c, int64_t d, int64_t n_heads,
                   float scale, int64_t s, int64_t k_lo, int64_t band,
                   int64_t chunk, int64_t left_chunks, int64_t k_hi,
                   int64_t pos_off, float *out, void *stream);

/* Host-buffer twin of AttnStreamKernel::forward (returns out in a host
 * buffer, as forward returns Vec<f32>); synchronous. */
int sc_attn_stream_host(const float *q, const float *kv, const float *vv,
                        const float *pos_p, int64_t n_pos,
                        const float *q_bias, const float *v_bias, int64_t c,
                        int64_t d, int64_t n_heads, float scale, int64_t s,
                        int64_t k_lo, int64_t band, int64_t chunk,
                        int64_t left_chunks, int64_t k_hi, int64_t pos_off,
                        float *out);

/* Batched streaming attention over per-stream HBM ring caches: the
 * device-resident replacement for block_new's band caches k_v/v_v and their
 * drain/extend slide (streaming.rs:263-277, 307-312), over n_streams streams in
 * lockstep.  Stream z's queries are rows z*c .. z*c+c-1 of q (row stride
 * ldq), its new frames' K/V rows z*c.. of k_new/v_new (stride ld_new); frame
 * fr of stream z lives in ring row z*cap + fr % cap (row stride d).  The
 * call appends the new frames [s, s+c) to the rings and attends over
 * [k_lo, k_hi = s + c); cap must be >= k_hi - k_lo.  out rows z*c + j (stride
 * ldo).  Leading dimensions <= 0 mean d. */
int sc_attn_stream_ring(const float *q, int64_t ldq, const float *k_new,
                        const float *v_new, int64_t ld_new, float *k_ring,
                        float *v_ring, int64_t cap, int64_t n_streams,
                        const float *pos_p, int64_t n_pos,
                        const float *q_bias, const float *v_bias, int64_t c,
                        int64_t d, int64_t n_heads, float scale, int64_t s,
                        int64_t k_lo, int64_t chunk, int64_t left_chunks,
                        int64_t k_hi, int64_t pos_off, float *out,
                        int64_t ldo, void *stream);

/* ---- streaming encoder (StreamEncoder) --------------------------------- */

/* A named tensor of the model, with the GGUF tensor names the reference
 * loads (nemotron/encoder.rs:89-245, e.g. "encoder.layers.3.self_attn.linear_q
 * .weight").  dtype 0 = f32, 8 = Q8_0 with f16 block scales (34-byte blocks);
 * dims in GGUF order (fastest axis first); data is host memory. */
typedef struct {
  const char *name;
  int32_t dtype;
  int32_t n_dims;
  int64_t dims[4];
  const void *data;
} sc_tensor;

/* EncoderConfig (nemotron/config.rs:19-39) plus max_frames, the largest
 * number of encoder frames one encode_new call may add (1..64): 7 for
 * streaming chunks, more to encode a longer stretch of audio per call (a
 * prefill); the output is the same either way.
 * att_right is the chunk's right context: chunk = att_right + 1 (the
 * reference fixes it to 6, nemotron/config.rs:164). */
typedef struct {
  int32_t d_model, n_layers, n_heads, d_ff;
  int32_t feat_in;        /* mel bins */
  int32_t conv_channels;  /* pre-encode channels */
  int32_t conv_kernel;    /* conformer depthwise kernel */
  int32_t conv_left;      /* causal left context = conv_kernel - 1 */
  int32_t att_left;       /* attention left context in frames */
  int32_t att_right;
  float ln_eps;
  int32_t max_frames;
} sc_encoder_config;

typedef struct sc_stream_encoder sc_stream_encoder;

/* relu(Conv2d::forward(x)) for the pre-encode's pointwise convs conv.3 and
 * conv.6 (1x1, stride 1; nemotron/weights.rs:399-443, the ReLU that follows
 * each of them in pre_encode_forward, nemotron/encoder.rs:400-482), over
 * n_streams windows at once, device pointers.  x is [n_streams *
 * rows_per_stream][c_in] (channels last), y the same rows x c_out; w is
 * [c_out][c_in], bias [c_out].  Row r of stream z is position sp_base + r
 * of a window of `spatial` (time x frequency) positions: the reference runs
 * the conv as one f32 GEMM per window (sgemm_kernel::gemm_into, with
 * spatial as its column count), and its rounding depends on the position's
 * column (one fused chain per output for whole 16-column blocks, 16 lane
 * sums for the last spatial % 16 columns; simd_kernel.rs:560-727), which
 * this call reproduces bit for bit.  c_in a multiple of 16 (<= 4096), c_out
 * a multiple of 8, else SC_ERR_UNSUPPORTED.  Async on stream. */
int sc_pre_encode_pointwise_relu(const float *x, const float *w,
                                 const float *bias, float *y,
                                 int64_t n_streams, int64_t rows_per_stream,
                                 int64_t sp_base, int64_t spatial,
                                 int64_t c_out, int64_t c_in, void *stream);

/* Build a device streaming encoder for n_streams streams from the model's
 * tensors (Encoder::load, nemotron/encoder.rs:249-282, then the weights'
 * one-time device repack).  Synchronous. */
int sc_stream_encoder_create(const sc_encoder_config *cfg,
                             const sc_tensor *tensors, int n_tensors,
                             int64_t n_streams, sc_stream_encoder **out);
/* StreamEncoder::encode_new (streaming.rs:687-699, 137-383) for every
 * stream at once: mel_new (device) holds each stream's new mel frames
 * [t0, t1) as [n_streams][t1 - t0][feat_in]; the encoder keeps the mel left
 * context itself, so the whole mel history is not passed.  t0 must equal 8 *
 * the frames encoded so far (else SC_ERR_STATE, as the reference's "out of
 * sync" bail); fin marks a stream's last batch.  Async on stream, except
 * the first call, which also computes every layer's positional rows
 * (streaming.rs:236-261) from host sinusoids and synchronises the stream.
 * With enough streams the call runs half of them on the encoder's own CUDA
 * stream, joined back into `stream` before it returns
 * (sc_stream_encoder_set_concurrency). */
int sc_stream_encoder_encode_new(sc_stream_encoder *e, const float *mel_new,
                                 int64_t t0, int64_t t1, int32_t fin,
                                 void *stream);
/* StreamEncoder::encode_new with host buffers, the twin of the reference's
 * call (which takes the mel frames in host memory): mel_host holds
 * [n_streams][t1 - t0][feat_in] floats (at most 8 * max_frames frames); the
 * call's output frames, [n_streams * c][d_model] stream-major as
 * sc_stream_encoder_output gives them, go to out_host (if not NULL; room for
 * n_streams * max_frames rows) and *rows (if not NULL) receives
 * n_streams * c.  Each half of the streams is copied in, encoded and copied
 * out on its own CUDA stream, so one half's copies overlap the other half's
 * kernels (page-locked host buffers let the copies run asynchronously).
 * Synchronous: out_host is filled when the call returns. */
int sc_stream_encoder_encode_new_host(sc_stream_encoder *e,
                                      const float *mel_host, int64_t t0,
                                      int64_t t1, int32_t fin, float *out_host,
                                      int64_t *rows, void *stream);
/* StreamEncoder::total (streaming.rs:702-703). */
int64_t sc_stream_encoder_total(const sc_stream_encoder *e);
/* StreamEncoder::frames (streaming.rs:700-701, 111-127) for one stream,
 * copied to a host buffer [to - from][d_model]; the last 64 frames are kept.
 * Synchronous. */
int sc_stream_encoder_frames(const sc_stream_encoder *e, int64_t stream_idx,
                             int64_t from, int64_t to, float *out_host);
/* Device pointer to the last call's output frames, [n_streams * c][d]
 * (stream-major); valid until the next encode_new. */
int sc_stream_encoder_output(const sc_stream_encoder *e, const float **frames,
                             int64_t *rows, int64_t *d);
/* Prompt of each stream for the multilingual prompt MLP that encode_new
 * applies to the new frames (streaming.rs:320-342, the prompt_id argument of
 * StreamEncoder::encode_new): prompt_ids is a host array [n_streams]; an id
 * < 0 or >= n_prompts means no prompt, as the reference.  Models without
 * the prompt_kernel.* tensors ignore it.  Applies to later encode_new calls;
 * synchronous. */
int sc_stream_encoder_set_prompts(sc_stream_encoder *e, const int32_t *prompt_ids);
/* Number of prompts of the model's prompt MLP (0: none). */
int64_t sc_stream_encoder_n_prompts(const sc_stream_encoder *e);
/* Stage dumps of one layer, the device twin of the reference's
 * STEALCODE_DUMP_DIR block dumps (streaming.rs:426-434, 462-631): after
 * set_dump(layer) (-1 = off) every encode_new records, for that layer and
 * all rows [n_streams * c][d]: 0 after FF1, 1 attention LayerNorm, 2
 * attention output, 3 after the attention residual, 4 q projection, 5 conv
 * module after dw conv + LN + SiLU, 6 after the conv residual, 7 block
 * output.  dump() copies one stage to a host buffer; synchronous. */
int sc_stream_encoder_set_dump(sc_stream_encoder *e, int32_t layer);
int sc_stream_encoder_dump(const sc_stream_encoder *e, int32_t stage,
                           float *out_host, int64_t *rows);
/* How many sub-batches of streams one encode_new keeps in flight: 2 (the
 * default) splits the streams into two halves at a 128-frame boundary of
 * the GEMM inputs and runs the second half on a stream the encoder owns,
 * forked from and joined back to the caller's stream, so one half's kernels
 * fill the SMs the other half's last GEMM wave leaves idle; 1 runs every
 * kernel on the caller's stream.  Both give the same bits.  Steps whose
 * stream count has no such boundary, and steps with stage dumps on, run as
 * one batch.  No counterpart in the reference, which encodes one stream at
 * a time. */
int sc_stream_encoder_set_concurrency(sc_stream_encoder *e, int32_t n_batches);
/* Step graphs (on by default), the counterpart of the reference GPU
 * backend's one submission per step (gpu/batch.rs:50,163,
 * gpu/streaming.rs:259-298).  A step whose geometry (streams, frames, mel
 * window, attention bands relative to the step, entry point) repeats the
 * previous step's is captured into a CUDA graph; later steps with that
 * geometry replay it as one launch after a one-thread store of their frame
 * shift, with its copy nodes pointed at the call's own mel and output
 * buffers.  Steady streaming steps all share one geometry (two graphs: the
 * mel history alternates between two buffers).  At most four graphs are
 * kept; capturing a fifth drops the least recently used one after a device
 * synchronise (a caller that alternates between more than two step
 * geometries sees that synchronise).  Host buffers of
 * encode_new_host must be page-locked for a step to use a graph; stage dumps
 * turn graphs off.  Same bits as separate launches.  enable 0 drops the
 * graphs (after a device synchronise) and launches every kernel separately. */
int sc_stream_encoder_set_graphs(sc_stream_encoder *e, int32_t enable);
/* Step graphs captured and graph launches so far; returns 1 while graphs
 * are on, 0 when off (set_graphs(0), or a capture that failed, after which
 * the encoder launches separately), <0 on error. */
int sc_stream_encoder_graph_stats(const sc_stream_encoder *e, int64_t *captures, int64_t *launches);
int sc_stream_encoder_destroy(sc_stream_encoder *e);

/* ---- RNN-T greedy decoder --------------------------------------------------
 * The streaming transcriber's decode loop (nemotron/live.rs:56-145,
 * decode_frames) with the predictor LSTM and the joint network
 * (nemotron/decoder.rs:75-235) for n_streams streams, each with its own
 * carried StreamState (live.rs:24-50).  Tensors (GGUF names, as the
 * reference loads them): decoder.prediction.embed.weight f32 [vocab x
 * hidden]; decoder.prediction.dec_rnn.lstm.{ih,hh}_l<i>.weight Q8_0
 * [hidden -> 4 hidden] with f32 .bias; joint.enc [d_enc -> joint],
 * joint.pred [hidden -> joint], joint.joint_net.2 [joint -> vocab], Q8_0
 * with optional f32 biases.  hidden, joint, d_enc: multiples of 32. */
typedef struct {
  int32_t d_enc, hidden, n_layers, joint;
  int32_t vocab;        /* classes including blank (RnntConfig::vocab_size) */
  int32_t blank;        /* blank_id */
  int32_t max_symbols;  /* max_symbols_per_step; 0 = no per-frame cap */
  int32_t max_frames;   /* largest n of one decode_frames call (1..256) */
} sc_rnnt_config;

typedef struct sc_rnnt_decoder sc_rnnt_decoder;

/* GreedyDecoder::load (decoder.rs:238-247) plus StreamState::new for every
 * stream; weights are repacked once for the device.  Synchronous. */
int sc_rnnt_create(const sc_rnnt_config *cfg, const sc_tensor *tensors,
                   int n_tensors, int64_t n_streams, sc_rnnt_decoder **out);
/* decode_frames (live.rs:56-145) for every stream at once: frames (device)
 * is [n_streams][n][d_enc], e.g. sc_stream_encoder_output's frames.  Each
 * stream's state carries over to the next call.  Synchronises `stream`
 * (the loop length depends on the tokens).  SC_ERR_STATE when a stream
 * hits the iteration cap 16 n + 64 (the reference's bail). */
int sc_rnnt_decode_frames(sc_rnnt_decoder *r, const float *frames, int64_t n,
                          void *stream);
/* Tokens the last decode_frames emitted for one stream: (id, frame step
 * within that call) pairs, the reference's Token {id, step} with p = 1;
 * up to cap of them are written, *count gets how many were emitted. */
int sc_rnnt_tokens(const sc_rnnt_decoder *r, int64_t stream_idx, int32_t *ids,
                   int32_t *steps, int32_t cap, int32_t *count);
/* How many tokens each stream emitted in the last call, [n_streams] (host). */
int sc_rnnt_emitted(const sc_rnnt_decoder *r, int32_t *counts);
/* Loop rounds the last decode_frames ran (each round is one iteration of
 * every still-active stream; no reference counterpart, for diagnostics). */
int64_t sc_rnnt_last_rounds(const sc_rnnt_decoder *r);
/* Device arrays of the last call's tokens: ids/steps [n_streams][*cap],
 * counts [n_streams]; valid until the next decode_frames. */
int sc_rnnt_tokens_device(const sc_rnnt_decoder *r, const int32_t **ids,
                          const int32_t **steps, const int32_t **counts,
                          int32_t *cap);
/* StreamState::new for one stream (-1: all streams). */
int sc_rnnt_reset(sc_rnnt_decoder *r, int64_t stream_idx);
/* A stream's LSTM state h, c ([n_layers][hidden] each, host) and its last
 * emitted token (-1 before the first). */
int sc_rnnt_state(const sc_rnnt_decoder *r, int64_t stream_idx, float *h,
                  float *c, int32_t *last_token);
int sc_rnnt_destroy(sc_rnnt_decoder *r);

#ifdef __cplusplus
}
#endif
#endif
