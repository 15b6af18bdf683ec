// sc_encoder.cu -- the device streaming encoder: the B200 counterpart of the
// reference's StreamEncoder trait (streaming.rs:687-729) and its CPU
// implementation StreamingEncoder::encode_new (streaming.rs:137-383) with
// block_new (streaming.rs:395-680) and the causal pre-encode stack
// (nemotron/encoder.rs:400-482), for n_streams streams advanced in lockstep.
//
// One encode_new call is one streaming step for every stream: M = n_streams x
// c frames flow through the 24 conformer blocks as time-major [M, d] rows.
// All per-stream state lives in HBM: per layer a K ring and a V ring
// (cap >= the attention band), a GLU ring (the depthwise conv's causal
// context), the last 24 mel frames for the next pre-encode window and an
// output ring for frames().  The reference's Vec caches with drain/extend
// (streaming.rs:263-277, 307-312, 345-361) become ring slots, so no per-step
// host<->device traffic remains besides the new mel frames.
//
// Weights come as a table of named tensors with the reference's GGUF names
// (nemotron/encoder.rs:89-245); linear_q/k/v are fused row-wise into one Q8
// matrix (each output row is computed independently, so the result is the
// same as three GEMMs over the same quantised input).

#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <algorithm>
#include <functional>
#include <vector>

#include "sc_kernels.cuh"
#include "../../include/stealcode_b200.h"

namespace sc {

int repack_q8_device(const uint8_t *raw_dev, int64_t rows, int64_t k, int64_t block_bytes, int64_t qoff,
                     Q8Weights *w, cudaStream_t st);
int launch_ln_rows(const float *x, int64_t ldx, const float *w, const float *b, float eps, float *out, int64_t ldo,
                   int64_t rows, int d, cudaStream_t st);
// shift (in the ring launchers below): device frame shift of a replayed step
// graph, added to frame numbers before they become ring slots; nullptr none.
int launch_glu_ring(const float *h2, int64_t rows, int c, int d, float *ring, int cap, int64_t s,
                    const int64_t *shift, cudaStream_t st);
int launch_mel_window(const float *hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                      int n_mels, int t_mel, float *win, int64_t n_streams, cudaStream_t st);
int launch_mel_hist(const float *old_hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                    int n_mels, float *new_hist, int64_t n_streams, cudaStream_t st);
int launch_conv2d_3x3s2(const float *x, int64_t n_streams, int t_in, int x_row0, int x_rows, int f_in, int c_in,
                        const float *w, const float *b, int c_out, int out_row0, int out_rows, int f_out, int relu,
                        float *out, cudaStream_t st);
int launch_conv02_fused(const float *win, int64_t n_streams, int t_mel, int f_mel, const float *w0, const float *b0,
                        const float *w2, const float *b2, int C, int ta, int fa, int out_row0, int out_rows, int fb,
                        float *out, cudaStream_t st);
// Rows of stream z are window positions sp_base .. sp_base + rows_per_stream
// - 1 of a conv input with `spatial` positions (time x frequency).
int launch_pw_conv_relu(const float *x, const float *w, const float *b, float *y, int64_t n_streams,
                        int rows_per_stream, int64_t sp_base, int64_t spatial, int n, int k, cudaStream_t st);
int launch_flatten(const float *x, int64_t n_streams, int t, int f, int C, int start_rel, int c, float *out,
                   cudaStream_t st, QOut qo);
int launch_ln2_quant(const float *x, int64_t ldx, const float *w0, const float *b0, float *out0, int64_t ld0,
                     const float *w, const float *b, float eps, int d, int64_t rows, const QOut &qo, float *out,
                     int64_t ldo, cudaStream_t st);
int launch_ln_quant(const float *x, int64_t ldx, const float *w, const float *b, float eps, int d, int64_t rows,
                    const QOut &qo, float *out, int64_t ldo, cudaStream_t st);
int launch_dwconv_ln_silu_quant(const float *ring, int cap, int64_t rows, int c, int d, int kh, int64_t s,
                                const int64_t *shift, const float *wt, const float *lnw, const float *lnb, float eps,
                                const QOut &qo, float *out, cudaStream_t st);
int launch_out_ring(const float *x, int64_t rows, int c, int d, float *ring, int cap, int64_t s,
                    const int64_t *shift, cudaStream_t st);
int launch_store_i64(int64_t *dst, int64_t v, cudaStream_t st);
int launch_prompt_cat_quant(const float *x, int64_t rows, int c, int d, int n_prompts, const int32_t *pids,
                            const QOut &qo, cudaStream_t st);
int launch_prompt_select(float *x, const float *y, int64_t rows, int c, int d, const int32_t *pids,
                         cudaStream_t st);

constexpr int kMelHistory = 24;  // mel frames of left context (streaming.rs:188)
constexpr int kDumpStages = 8;

// Position of head element i in the attention's lane-major row order:
// element 16*ch + l at (ch/4)*64 + 4l + ch%4 (head_dim a multiple of 64).
static int64_t lane_major_h(int64_t i) { return (i >> 6) * 64 + (i & 15) * 4 + ((i >> 4) & 3); }

struct Lin {
  Q8Weights w{};
  float *bias = nullptr;
};

struct Layer {
  float *ln_ff1_w, *ln_ff1_b, *ln_att_w, *ln_att_b, *ln_conv_w, *ln_conv_b, *conv_ln_w, *conv_ln_b;
  float *ln_ff2_w, *ln_ff2_b, *ln_out_w, *ln_out_b;
  Lin ff1_1, ff1_2, qkv, pos, out, pw1, pw2, ff2_1, ff2_2;
  float *pos_u, *pos_v, *dw;
  float *dw_t = nullptr;               // depthwise weight transposed to [kh][d]
  float *pos_p = nullptr;              // [n_pos][d], after the first step
  float *k_ring, *v_ring, *glu_ring;   // [n_streams][cap][d]
};

struct Conv {
  float *w, *b;
};

}  // namespace sc

using namespace sc;

// A copy node of a step graph: the mel of streams [za, za + nz) into the
// staging buffer (dir 0) or their output frames to the caller (dir 1).
// Replays point it at the call's own buffers.
struct StepCopy {
  cudaGraphNode_t node;
  int64_t za, nz;
  int dir;
};

// One captured encode_new step (both sub-batches, fork and join included).
struct StepGraph {
  std::vector<int64_t> key;  // step geometry + mel-history buffer parity
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int64_t s = 0;             // first frame of the captured step
  long long kernels = 0;     // kernel nodes (launches per replay)
  std::vector<StepCopy> copies;
  uint64_t used = 0;         // last use, for eviction
};

struct sc_stream_encoder {
  sc_encoder_config cfg{};
  int64_t n_streams = 0;
  int device = 0;
  int64_t chunk = 0, left_chunks = 0, n_pos = 0, kv_cap = 0, glu_cap = 0, out_cap = 0, t_mel_max = 0;
  std::vector<Layer> layers;
  Conv c0{}, c2{}, c3{}, c5{}, c6{};
  Lin pre_out;
  // multilingual prompt MLP (nemotron/encoder.rs:260-270), optional:
  // prompt0 [d + n_prompts -> hidden], prompt2 [hidden -> d]
  Lin prompt0, prompt2;
  int64_t n_prompts = 0, prompt_hidden = 0;
  int32_t *pids = nullptr;  // [n_streams] device: prompt of each stream, -1 none
  bool any_prompt = false;
  std::vector<void *> allocs;
  // state
  int64_t total = 0;
  int64_t last_c = 0;
  int hist_frames = 0;
  float *hist[2] = {nullptr, nullptr};
  int hist_cur = 0;
  bool pos_ready = false;
  // scratch
  float *x, *y, *xn, *h, *qkv, *attn, *h2, *o2, *out_ring;
  float *win, *p0, *p1, *p2, *flat, *pos_in;
  // GEMM inputs as codes in the tensor-core tiled layout (two, so that a
  // GEMM can write its successor's codes while reading its own)
  __half *qx[2] = {nullptr, nullptr};  // f16 codes of the GEMM inputs (QOut layout)
  float *qd[2] = {nullptr, nullptr};
  void *ws = nullptr;
  size_t ws_bytes = 0;
  // second sub-batch's stream and the fork / join events
  cudaStream_t side = nullptr;
  // per-stream sizes of the pre-encode buffers and the code buffers' widest
  // row (features), as allocated
  int64_t win_stride = 0, conv_stride = 0, code_k = 0;
  float *mel_stage = nullptr;   // [n_streams][mel_stage_frames][feat_in]: host-entry mel
  int64_t mel_stage_frames = 0;
  int max_batches = 2;  // sub-batches of streams in flight (1 or 2)
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // stage dumps of one layer (the reference's STEALCODE_DUMP_DIR senc_b*_*
  // files, streaming.rs:426-434): -1 = off
  int dump_layer = -1;
  float *dump = nullptr;  // [kDumpStages][M][2d]
  int64_t dump_rows = 0;
  // Step graphs: a step whose geometry repeats the previous step's is
  // captured into a CUDA graph (on cap_stream, which runs nothing); later
  // steps with the same geometry and history parity replay it as one
  // submission, after one store of their frame shift (s minus the captured
  // s) into shift_dev, which the ring kernels add to frame numbers.
  bool graphs = true;
  int64_t *shift_dev = nullptr;
  const int64_t *shift_arg = nullptr;  // what the step's ring kernels get: shift_dev while capturing
  cudaStream_t cap_stream = nullptr;
  std::vector<StepGraph> step_graphs;
  std::vector<int64_t> prev_geom;      // geometry of the previous step (empty: none to compare)
  int64_t graph_captures = 0, graph_launches = 0;
  uint64_t graph_clock = 0;

  void drop_graph(StepGraph &g) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.graph) cudaGraphDestroy(g.graph);
    g.exec = nullptr;
    g.graph = nullptr;
  }

  ~sc_stream_encoder() {
    for (auto &g : step_graphs) drop_graph(g);
    if (cap_stream) cudaStreamDestroy(cap_stream);
    for (auto &l : layers)
      for (Lin *q : {&l.ff1_1, &l.ff1_2, &l.qkv, &l.pos, &l.out, &l.pw1, &l.pw2, &l.ff2_1, &l.ff2_2}) {
        cudaFree(q->w.qs);
        cudaFree(q->w.sc);
        cudaFree(q->w.qh);
      }
    for (Lin *q : {&pre_out, &prompt0, &prompt2}) {
      cudaFree(q->w.qs);
      cudaFree(q->w.sc);
      cudaFree(q->w.qh);
    }
    for (void *p : allocs) cudaFree(p);
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (side) cudaStreamDestroy(side);
  }
};

namespace {

struct Loader {
  const sc_tensor *t;
  int n;
  sc_stream_encoder *e;
  std::string err;

  const sc_tensor *find(const std::string &name) const {
    for (int i = 0; i < n; i++)
      if (name == t[i].name) return &t[i];
    return nullptr;
  }
  static int64_t numel(const sc_tensor *x) {
    int64_t c = 1;
    for (int i = 0; i < x->n_dims; i++) c *= x->dims[i];
    return c;
  }
  float *dev_alloc(size_t bytes) {
    void *p = nullptr;
    if (dev_malloc(&p, bytes < 16 ? 16 : bytes) != cudaSuccess) {
      cudaGetLastError();
      err = "cudaMalloc failed";
      return nullptr;
    }
    e->allocs.push_back(p);
    return (float *)p;
  }
  // Rows (or elements) of a [.., d] part permuted into lane-major order
  // within each head: source index h*hd + i goes to h*hd + lane_major(i).
  static int64_t head_perm(int64_t n, int64_t hd) {
    return hd > 0 ? (n / hd) * hd + lane_major_h(n % hd) : n;
  }
  float *f32(const std::string &name, int64_t count, bool optional = false, int64_t perm_hd = 0) {
    const sc_tensor *x = find(name);
    if (!x) {
      if (!optional && err.empty()) err = "tensor " + name + " not found";
      return nullptr;
    }
    if (x->dtype != 0 || numel(x) != count) {
      if (err.empty()) err = "tensor " + name + " is not f32 with " + std::to_string(count) + " elements";
      return nullptr;
    }
    float *d = dev_alloc((size_t)count * 4);
    const float *src = (const float *)x->data;
    std::vector<float> perm;
    if (perm_hd > 0) {
      perm.resize((size_t)count);
      for (int64_t i = 0; i < count; i++) perm[(size_t)head_perm(i, perm_hd)] = src[i];
      src = perm.data();
    }
    if (d && cudaMemcpy(d, src, (size_t)count * 4, cudaMemcpyHostToDevice) != cudaSuccess) err = "upload failed";
    return d;
  }
  // Q8 linear [out, inp] (GGUF dims [inp, out]); `parts` tensors are stacked
  // row-wise (QKV fusion).  Parts listed in perm_parts get their output rows
  // (and bias) permuted lane-major within each head of perm_hd rows: the
  // same per-row arithmetic, outputs in the attention's staging order.
  bool lin(const std::vector<std::string> &bases, int64_t inp, int64_t out_each, Lin *l, bool bias_optional,
           const std::vector<int> &perm_parts = {}, int64_t perm_hd = 0) {
    const int64_t nb = (inp + 31) / 32, padded = nb * 34, rows = out_each * (int64_t)bases.size();
    std::vector<uint8_t> raw((size_t)(rows * padded));
    std::vector<float> bias((size_t)rows, 0.0f);
    bool have_bias = false;  // missing parts of a fused bias are zero
    for (size_t p = 0; p < bases.size(); p++) {
      const sc_tensor *x = find(bases[p] + ".weight");
      if (!x || x->dtype != 8 || x->n_dims != 2 || x->dims[0] != inp || x->dims[1] != out_each) {
        if (err.empty()) err = "tensor " + bases[p] + ".weight missing or not Q8_0 [" + std::to_string(inp) + " -> " +
                               std::to_string(out_each) + "]";
        return false;
      }
      const bool perm = std::find(perm_parts.begin(), perm_parts.end(), (int)p) != perm_parts.end();
      const int64_t hd = perm ? perm_hd : 0;
      for (int64_t r = 0; r < out_each; r++)
        memcpy(raw.data() + (p * out_each + head_perm(r, hd)) * padded, (const uint8_t *)x->data + r * padded,
               (size_t)padded);
      const sc_tensor *b = find(bases[p] + ".bias");
      if (b) {
        if (b->dtype != 0 || numel(b) != out_each) {
          if (err.empty()) err = "tensor " + bases[p] + ".bias mis-shaped";
          return false;
        }
        for (int64_t r = 0; r < out_each; r++)
          bias[(size_t)(p * out_each + head_perm(r, hd))] = ((const float *)b->data)[r];
        have_bias = true;
      }
    }
    (void)bias_optional;  // a linear without bias is allowed (Lin::bias is optional)
    uint8_t *draw = nullptr;
    if (dev_malloc((void **)&draw, raw.size()) != cudaSuccess) {
      cudaGetLastError();
      err = "cudaMalloc failed";
      return false;
    }
    Q8Weights &w = l->w;
    w.rows = rows;
    w.k = inp;
    w.nb = nb;
    w.rows_pad = (rows + SC_GROUP_ROWS - 1) / SC_GROUP_ROWS * SC_GROUP_ROWS;
    w.device = e->device;
    const bool allocated = dev_malloc((void **)&w.qs, (size_t)w.rows_pad * nb * 32) == cudaSuccess &&
                           dev_malloc((void **)&w.sc, (size_t)w.rows_pad * nb * 2) == cudaSuccess &&
                           dev_malloc((void **)&w.qh, (size_t)w.rows_pad * nb * 64) == cudaSuccess;
    if (!allocated) err = "cudaMalloc failed";
    bool ok = allocated && cudaMemcpy(draw, raw.data(), raw.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
              repack_q8_device(draw, rows, inp, 34, 2, &w, 0) == kOk && cudaDeviceSynchronize() == cudaSuccess;
    cudaFree(draw);
    if (!ok) {
      cudaGetLastError();
      if (err.empty()) err = "Q8 upload/repack failed";
      return false;
    }
    if (have_bias) {
      l->bias = dev_alloc(bias.size() * 4);
      if (!l->bias || cudaMemcpy(l->bias, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return false;
    }
    return true;
  }
};

#define TRY(call)         \
  do {                    \
    int _rc = (call);     \
    if (_rc) return _rc;  \
  } while (0)

int64_t conv_out(int64_t in) { return (in + 3 - 3) / 2 + 1; }  // k 3, pads (2, 1), stride 2

}  // namespace

extern "C" {

int sc_stream_encoder_create(const sc_encoder_config *cfg, const sc_tensor *tensors, int n_tensors,
                             int64_t n_streams, sc_stream_encoder **out) {
  if (!cfg || !tensors || !out || n_tensors <= 0 || n_streams <= 0) {
    set_error("stream_encoder_create: invalid argument");
    return kErrInvalid;
  }
  *out = nullptr;
  const sc_encoder_config &c = *cfg;
  if (c.d_model % 256 || c.d_model > 4096 || c.n_heads <= 0 || c.d_model % c.n_heads || c.att_right < 0 ||
      c.conv_kernel < 1 || c.conv_left != c.conv_kernel - 1 || c.max_frames < 1 || c.max_frames > 64 ||
      c.feat_in <= 0 || c.conv_channels <= 0 || c.n_layers < 0 ||
      (c.d_model / c.n_heads != 64 && c.d_model / c.n_heads != 128) || (c.d_model & (c.d_model - 1)) ||
      c.d_ff % 128) {
    set_error("stream_encoder_create: unsupported config (d_model %d (a power of two, 256..4096), heads %d "
              "(head_dim 64 or 128), d_ff a multiple of 128, conv %d/%d, max_frames %d (1..64))",
              c.d_model, c.n_heads, c.conv_kernel, c.conv_left, c.max_frames);
    return kErrUnsupported;
  }
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  sc_stream_encoder *e = new (std::nothrow) sc_stream_encoder();
  if (!e) {
    set_error("stream_encoder_create: host allocation failed");
    return kErrAlloc;
  }
  e->cfg = c;
  e->n_streams = n_streams;
  e->device = dev;
  e->chunk = c.att_right + 1;
  e->left_chunks = c.att_left / e->chunk;
  e->n_pos = (e->left_chunks + 2) * e->chunk - 1;
  e->kv_cap = e->left_chunks * e->chunk + (e->chunk - 1) + c.max_frames;
  e->glu_cap = c.conv_left + c.max_frames;
  e->out_cap = std::max<int64_t>(64, c.max_frames);
  e->t_mel_max = kMelHistory + 8 * (int64_t)c.max_frames + 8;
  const int64_t d = c.d_model, dff = c.d_ff, C = c.conv_channels, hd = d / c.n_heads;
  Loader L{tensors, n_tensors, e, {}};
  // pre-encode (nemotron/encoder.rs:89-160)
  const std::string pc = "encoder.pre_encode.conv.";
  e->c0 = {L.f32(pc + "0.weight", C * 9), L.f32(pc + "0.bias", C)};
  e->c2 = {L.f32(pc + "2.weight", C * 9), L.f32(pc + "2.bias", C)};
  e->c3 = {L.f32(pc + "3.weight", C * C), L.f32(pc + "3.bias", C)};
  e->c5 = {L.f32(pc + "5.weight", C * 9), L.f32(pc + "5.bias", C)};
  e->c6 = {L.f32(pc + "6.weight", C * C), L.f32(pc + "6.bias", C)};
  const int64_t f_final = conv_out(conv_out(conv_out(c.feat_in)));
  bool ok = L.err.empty() && L.lin({"encoder.pre_encode.out"}, f_final * C, d, &e->pre_out, true);
  // conformer blocks (nemotron/encoder.rs:171-245)
  e->layers.resize(c.n_layers);
  for (int i = 0; ok && i < c.n_layers; i++) {
    Layer &ly = e->layers[i];
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    ly.ln_ff1_w = L.f32(p + "norm_feed_forward1.weight", d);
    ly.ln_ff1_b = L.f32(p + "norm_feed_forward1.bias", d);
    ly.ln_att_w = L.f32(p + "norm_self_att.weight", d);
    ly.ln_att_b = L.f32(p + "norm_self_att.bias", d);
    ly.ln_conv_w = L.f32(p + "norm_conv.weight", d);
    ly.ln_conv_b = L.f32(p + "norm_conv.bias", d);
    ly.conv_ln_w = L.f32(p + "conv.batch_norm.weight", d);
    ly.conv_ln_b = L.f32(p + "conv.batch_norm.bias", d);
    ly.ln_ff2_w = L.f32(p + "norm_feed_forward2.weight", d);
    ly.ln_ff2_b = L.f32(p + "norm_feed_forward2.bias", d);
    ly.ln_out_w = L.f32(p + "norm_out.weight", d);
    ly.ln_out_b = L.f32(p + "norm_out.bias", d);
    // q, k, pos rows and the pos biases live in lane-major head order (the
    // attention kernel's staging order); v and everything else stay natural
    ly.pos_u = L.f32(p + "self_attn.pos_bias_u", d, false, hd);
    ly.pos_v = L.f32(p + "self_attn.pos_bias_v", d, false, hd);
    ly.dw = L.f32(p + "conv.depthwise_conv.weight", d * c.conv_kernel);
    if (const sc_tensor *dwx = L.find(p + "conv.depthwise_conv.weight")) {
      if (dwx->dtype == 0 && L.numel(dwx) == d * c.conv_kernel) {
        std::vector<float> tr((size_t)(d * c.conv_kernel));
        const float *src = (const float *)dwx->data;
        for (int64_t ch = 0; ch < d; ch++)
          for (int64_t t = 0; t < c.conv_kernel; t++) tr[(size_t)(t * d + ch)] = src[ch * c.conv_kernel + t];
        ly.dw_t = L.dev_alloc(tr.size() * 4);
        if (ly.dw_t && cudaMemcpy(ly.dw_t, tr.data(), tr.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
          L.err = "upload failed";
      }
    }
    ok = L.err.empty() && L.lin({p + "feed_forward1.linear1"}, d, dff, &ly.ff1_1, true) &&
         L.lin({p + "feed_forward1.linear2"}, dff, d, &ly.ff1_2, true) &&
         L.lin({p + "self_attn.linear_q", p + "self_attn.linear_k", p + "self_attn.linear_v"}, d, d, &ly.qkv, true,
               {0, 1}, hd) &&
         L.lin({p + "self_attn.linear_pos"}, d, d, &ly.pos, true, {0}, hd) &&
         L.lin({p + "self_attn.linear_out"}, d, d, &ly.out, true) &&
         L.lin({p + "conv.pointwise_conv1"}, d, 2 * d, &ly.pw1, true) &&
         L.lin({p + "conv.pointwise_conv2"}, d, d, &ly.pw2, true) &&
         L.lin({p + "feed_forward2.linear1"}, d, dff, &ly.ff2_1, true) &&
         L.lin({p + "feed_forward2.linear2"}, dff, d, &ly.ff2_2, true);
    if (ok) {
      ly.pos_p = L.dev_alloc((size_t)(e->n_pos * d * 4));
      ly.k_ring = L.dev_alloc((size_t)(n_streams * e->kv_cap * d * 4));
      ly.v_ring = L.dev_alloc((size_t)(n_streams * e->kv_cap * d * 4));
      ly.glu_ring = L.dev_alloc((size_t)(n_streams * e->glu_cap * d * 4));
      ok = L.err.empty();
    }
  }
  // optional prompt MLP: its input width d + n_prompts gives n_prompts
  if (const sc_tensor *p0 = ok ? L.find("prompt_kernel.0.weight") : nullptr) {
    if (p0->n_dims == 2 && p0->dims[0] > d && (p0->dims[0] - d) % 32 == 0 && p0->dims[1] % 128 == 0) {
      e->n_prompts = p0->dims[0] - d;
      e->prompt_hidden = p0->dims[1];
      ok = L.lin({"prompt_kernel.0"}, d + e->n_prompts, e->prompt_hidden, &e->prompt0, true) &&
           L.lin({"prompt_kernel.2"}, e->prompt_hidden, d, &e->prompt2, true);
      if (ok) {
        e->pids = (int32_t *)L.dev_alloc((size_t)n_streams * 4);
        std::vector<int32_t> none((size_t)n_streams, -1);
        ok = e->pids && cudaMemcpy(e->pids, none.data(), none.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        if (!ok && L.err.empty()) L.err = "upload failed";
      }
    } else {
      L.err = "prompt_kernel.0.weight: dims [d + n_prompts, hidden] with n_prompts and hidden multiples of 32 and "
              "128 expected";
      ok = false;
    }
  }
  const int64_t M = n_streams * c.max_frames;
  if (ok) {
    e->x = L.dev_alloc(M * d * 4);
    e->y = L.dev_alloc(M * d * 4);
    e->xn = L.dev_alloc(M * d * 4);
    e->h = L.dev_alloc(M * dff * 4);
    e->qkv = L.dev_alloc(M * 3 * d * 4);
    e->attn = L.dev_alloc(M * d * 4);
    e->h2 = L.dev_alloc(M * 2 * d * 4);
    e->o2 = L.dev_alloc(M * d * 4);
    e->out_ring = L.dev_alloc((size_t)(n_streams * e->out_cap * d * 4));
    e->hist[0] = L.dev_alloc((size_t)(n_streams * kMelHistory * c.feat_in * 4));
    e->hist[1] = L.dev_alloc((size_t)(n_streams * kMelHistory * c.feat_in * 4));
    // the pre-encode buffers hold conv.2's (and conv.3's) output rows at
    // most, [tb][fb][C] per stream (conv.0's output is never stored: the
    // fused conv.0 + conv.2 kernel rebuilds the rows it reads)
    const int64_t tb_max = conv_out(conv_out(e->t_mel_max)), fb = conv_out(conv_out(c.feat_in));
    e->win = L.dev_alloc((size_t)(n_streams * e->t_mel_max * c.feat_in * 4));
    e->p0 = L.dev_alloc((size_t)(n_streams * tb_max * fb * C * 4));
    e->p1 = L.dev_alloc((size_t)(n_streams * tb_max * fb * C * 4));
    e->p2 = L.dev_alloc((size_t)(n_streams * tb_max * fb * C * 4));
    e->flat = L.dev_alloc((size_t)(M * f_final * C * 4));
    e->pos_in = L.dev_alloc((size_t)(e->n_pos * d * 4));
    const int64_t kmax = std::max<int64_t>(std::max<int64_t>(std::max<int64_t>(dff, f_final * C), d),
                                           std::max<int64_t>(d + e->n_prompts, e->prompt_hidden));
    const int64_t tmax = std::max<int64_t>(M, e->n_pos);
    e->ws_bytes = gemm_ws_bytes(tmax, kmax);
    e->ws = L.dev_alloc(e->ws_bytes);
    const int64_t tp = std::max<int64_t>(ceil_div(M, 128) * 128, 64), kp = ceil_div(kmax, 32) * 32;
    e->mel_stage_frames = 8 * (int64_t)c.max_frames;
    e->mel_stage = L.dev_alloc((size_t)(n_streams * e->mel_stage_frames * c.feat_in * 4));
    e->shift_dev = (int64_t *)L.dev_alloc(sizeof(int64_t));
    e->win_stride = e->t_mel_max * c.feat_in;
    e->conv_stride = tb_max * fb * C;
    e->code_k = kp;
    for (int i = 0; i < 2; i++) {
      e->qx[i] = (__half *)L.dev_alloc((size_t)(tp * kp * 2));
      e->qd[i] = L.dev_alloc((size_t)(kp / 32 * tp * 4));
    }
    ok = L.err.empty();
  }
  if (ok && (cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking) != cudaSuccess ||
             cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking) != cudaSuccess ||
             cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
             cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming) != cudaSuccess)) {
    L.err = "side stream / event creation failed";
    ok = false;
  }
  if (!ok) {
    set_error("stream_encoder_create: %s", L.err.c_str());
    delete e;
    return L.err.find("cudaMalloc") != std::string::npos ? kErrAlloc : kErrInvalid;
  }
  *out = e;
  return kOk;
}

int sc_stream_encoder_destroy(sc_stream_encoder *e) {
  if (e) {
    cudaDeviceSynchronize();
    delete e;
  }
  return kOk;
}

int64_t sc_stream_encoder_total(const sc_stream_encoder *e) { return e ? e->total : -1; }

int sc_stream_encoder_frames(const sc_stream_encoder *e, int64_t stream_idx, int64_t from, int64_t to,
                             float *out_host) {
  if (!e || !out_host || stream_idx < 0 || stream_idx >= e->n_streams) {
    set_error("stream_encoder_frames: invalid argument");
    return kErrInvalid;
  }
  if (e->total == 0) {
    set_error("stream_encoder_frames: nothing encoded yet");
    return kErrState;
  }
  if (to <= from || to > e->total || from < e->total - e->out_cap || from < 0) {
    set_error("frames [%lld, %lld) outside cache [%lld, %lld)", (long long)from, (long long)to,
              (long long)std::max<int64_t>(0, e->total - e->out_cap), (long long)e->total);
    return kErrInvalid;
  }
  const int64_t d = e->cfg.d_model;
  SC_CUDA(cudaDeviceSynchronize());
  for (int64_t f = from; f < to; f++)
    SC_CUDA(cudaMemcpy(out_host + (f - from) * d, e->out_ring + (stream_idx * e->out_cap + f % e->out_cap) * d,
                       d * 4, cudaMemcpyDeviceToHost));
  return kOk;
}

// Sizes of one encode_new step, shared by its sub-batches.
struct StepGeom {
  int64_t s, n_new, t_new, cf, t_mel, start_rel;
  int64_t ta, fa, tb, fb, fc, r3, e3, r5, n5;
};

// One attention launch of a call's frames from a: frames [a, b) inside one
// attention chunk, keys from k_lo (left_chunks whole chunks back, clamped at
// frame 0; streaming.rs:227, 501).
static void attn_span(const sc_stream_encoder *e, int64_t a, int64_t t_new, int64_t &b, int64_t &k_lo) {
  b = std::min<int64_t>(t_new, (a / e->chunk + 1) * e->chunk);
  k_lo = (a / e->chunk > e->left_chunks ? a / e->chunk - e->left_chunks : 0) * e->chunk;
}

// One step for streams [z0, z0 + nz) on stream st.  Every buffer is indexed
// by stream (or by row = stream * cf + frame) with per-stream strides that
// depend only on the step's sizes, so a sub-batch is the same launches over
// offset base pointers.  Its GEMM-input codes start at frame z0 * cf of the
// code buffers, which is a whole number of 128-frame tiles (or 0).
static int encode_streams(sc_stream_encoder *e, const StepGeom &g, const float *mel_new, int64_t z0, int64_t nz,
                          cudaStream_t st) {
  const sc_encoder_config &c = e->cfg;
  const int64_t d = c.d_model, dff = c.d_ff, C = c.conv_channels, Z = nz;
  const float eps = c.ln_eps;
  const int64_t s = g.s, cf = g.cf, t_new = g.t_new, t_mel = g.t_mel;
  const int64_t M = Z * cf, f0 = z0 * cf;
  const int64_t fin_ = c.feat_in;
  // Per-stream regions of the pre-encode buffers start at z0 times the
  // allocated per-stream size: the kernels index each buffer with this
  // step's (smaller) strides, so a half stays inside its own streams'
  // regions whichever stage the other half is at.
  float *win = e->win + z0 * e->win_stride;
  float *hist_cur = e->hist[e->hist_cur] + z0 * kMelHistory * fin_;
  float *hist_nxt = e->hist[e->hist_cur ^ 1] + z0 * kMelHistory * fin_;
  const float *mel = mel_new ? mel_new + z0 * g.n_new * fin_ : nullptr;
  float *p0 = e->p0 + z0 * e->conv_stride, *p1 = e->p1 + z0 * e->conv_stride, *p2 = e->p2 + z0 * e->conv_stride;
  float *x = e->x + f0 * d, *y = e->y + f0 * d, *qkv = e->qkv + f0 * 3 * d, *h2 = e->h2 + f0 * 2 * d;
  float *xn = e->xn + f0 * d, *attn = e->attn + f0 * d, *o2 = e->o2 + f0 * d;
  TRY(launch_mel_window(hist_cur, kMelHistory, e->hist_frames, mel, (int)g.n_new, c.feat_in, (int)t_mel, win, Z,
                        st));
  // ---- pre-encode stack (nemotron/encoder.rs:400-482) ----
  // conv0 + ReLU and the depthwise conv2 in one kernel (the conv0 rows that
  // conv2 reads are rebuilt where it reads them)
  TRY(launch_conv02_fused(win, Z, (int)t_mel, c.feat_in, e->c0.w, e->c0.b, e->c2.w, e->c2.b, (int)C, (int)g.ta,
                          (int)g.fa, (int)g.r3, (int)(g.e3 - g.r3), (int)g.fb, p1, st));
  TRY(launch_pw_conv_relu(p1, e->c3.w, e->c3.b, p2, Z, (int)((g.e3 - g.r3) * g.fb), g.r3 * g.fb, g.tb * g.fb,
                          (int)C, (int)C, st));
  TRY(launch_conv2d_3x3s2(p2, Z, (int)g.tb, (int)g.r3, (int)(g.e3 - g.r3), (int)g.fb, (int)C, e->c5.w, e->c5.b,
                          (int)C, (int)g.r5, (int)g.n5, (int)g.fc, 0, p1, st));
  TRY(launch_pw_conv_relu(p1, e->c6.w, e->c6.b, p0, Z, (int)(g.n5 * g.fc), g.r5 * g.fc,
                          conv_out(g.tb) * g.fc, (int)C, (int)C, st));
  // GEMM inputs are quantised by their producers straight into the
  // tensor-core operand layout (code buffers qx/qd, ping-pong)
  const int ft = tc_frame_tile(M);
  const int64_t t_pad = ceil_div(M, ft) * ft;
  // a half's codes start at frame f0 times the buffers' widest row, so the
  // halves' regions stay apart for every feature width
  auto qbuf = [&](int i, int64_t k) {
    return QOut{e->qx[i] + f0 * e->code_k, e->qd[i] + f0 * (e->code_k / 32), ceil_div(k, 32), t_pad, ft};
  };
  auto gemm_q = [&](const Lin &l, const QOut &in, float *out, int64_t ldo, Epilogue epi, QOut next) {
    TcGemmArgs ta{&l.w, in.xq, in.dx, M, t_pad, l.bias, out, 1, ldo, epi, next};
    return gemm_tc(ta, st);
  };
  TRY(launch_flatten(p0, Z, (int)g.n5, (int)g.fc, (int)C, 0, (int)cf, nullptr, st, qbuf(0, C * g.fc)));
  TRY(gemm_q(e->pre_out, qbuf(0, C * g.fc), x, d, Epilogue{}, QOut{}));
  // history for the next window
  TRY(launch_mel_hist(hist_cur, kMelHistory, e->hist_frames, mel, (int)g.n_new, c.feat_in, hist_nxt, Z, st));
  // ---- conformer blocks (streaming.rs:279-318, block_new :395-680) ----
  const int64_t pos_off = e->chunk - 1;
  Epilogue silu{kEpiSilu, nullptr, 1.0f};
  for (size_t li = 0; li < e->layers.size(); li++) {
    Layer &ly = e->layers[li];
    float *k_ring = ly.k_ring + z0 * e->kv_cap * d, *v_ring = ly.v_ring + z0 * e->kv_cap * d;
    float *glu_ring = ly.glu_ring + z0 * e->glu_cap * d;
    auto dump = [&](int stage, const float *src, int64_t width) -> int {
      if ((int)li != e->dump_layer || !e->dump) return kOk;
      SC_CUDA(cudaMemcpy2DAsync(e->dump + (size_t)stage * M * 2 * d, 2 * d * 4, src, width * 4, d * 4, M,
                                cudaMemcpyDeviceToDevice, st));
      return kOk;
    };
    const bool dumping = (int)li == e->dump_layer && e->dump;
    const QOut qa = qbuf(0, d), qb_ff = qbuf(1, dff), qb_d = qbuf(1, d);
    // macaron FF1: y = x + 0.5 * FF(LN(x)); the SiLU output goes to ff1_2 as codes
    if (li == 0)  // later layers get these codes from the previous block's output LayerNorm
      TRY(launch_ln_quant(x, d, ly.ln_ff1_w, ly.ln_ff1_b, eps, (int)d, M, qa, nullptr, d, st));
    TRY(gemm_q(ly.ff1_1, qa, nullptr, dff, silu, qb_ff));
    TRY(gemm_q(ly.ff1_2, qb_ff, y, d, Epilogue{kEpiResidual, x, 0.5f}, QOut{}));
    TRY(dump(0, y, d));
    // rel-pos MHSA over the band, K/V from the rings; its output goes to
    // the out projection as codes
    TRY(launch_ln_quant(y, d, ly.ln_att_w, ly.ln_att_b, eps, (int)d, M, qa, dumping ? xn : nullptr, d, st));
    TRY(dump(1, xn, d));
    TRY(gemm_q(ly.qkv, qa, qkv, 3 * d, Epilogue{}, QOut{}));
    // the call's frames [s, t_new) in sub-ranges that stay inside one
    // attention chunk, in order: each launch writes its frames' K/V rows to
    // the rings before the next one reads them, and every band stays within
    // left context + one chunk however many frames the call brings
    for (int64_t a = s; a < t_new;) {
      int64_t b, k_lo;
      attn_span(e, a, t_new, b, k_lo);
      AttnParams p{};
      p.q = qkv;
      p.ldq = 3 * d;
      p.k_new = qkv + d;
      p.v_new = qkv + 2 * d;
      p.ld_new = 3 * d;
      p.rows_new = b - a;
      p.new_lo = a;
      p.k_ring = k_ring;
      p.v_ring = v_ring;
      p.cap = e->kv_cap;
      p.pos_p = ly.pos_p;
      p.u = ly.pos_u;
      p.v = ly.pos_v;
      p.out = dumping ? attn : nullptr;
      p.ldo = d;
      p.qout = qb_d;
      p.c = (int)(b - a);
      p.d = (int)d;
      p.n_heads = c.n_heads;
      p.scale = 1.0f / sqrtf((float)(d / c.n_heads));
      p.s = a;
      p.k_lo = k_lo;
      p.k_hi = b;
      p.chunk = e->chunk;
      p.left_chunks = e->left_chunks;
      p.pos_off = pos_off;
      p.lane_major = 1;  // q, k, pos rows and biases in lane-major head order
      p.zrows = cf;      // rows of stream z: z * cf + (frame - s)
      p.r0 = a - s;
      p.frame_shift = e->shift_arg;
      TRY(attn_prepare(p, e->n_pos));
      TRY(launch_attn(p, Z, st));
      a = b;
    }
    TRY(dump(2, attn, d));
    TRY(gemm_q(ly.out, qb_d, y, d, Epilogue{kEpiResidual, y, 1.0f}, QOut{}));
    TRY(dump(3, y, d));
    // conv module: LN, pw1, GLU (ring), causal dw conv + LN + SiLU (codes), pw2
    TRY(launch_ln_quant(y, d, ly.ln_conv_w, ly.ln_conv_b, eps, (int)d, M, qa, nullptr, d, st));
    TRY(gemm_q(ly.pw1, qa, h2, 2 * d, Epilogue{}, QOut{}));
    TRY(launch_glu_ring(h2, M, (int)cf, (int)d, glu_ring, (int)e->glu_cap, s, e->shift_arg, st));
    TRY(launch_dwconv_ln_silu_quant(glu_ring, (int)e->glu_cap, M, (int)cf, (int)d, c.conv_kernel, s, e->shift_arg,
                                    ly.dw_t, ly.conv_ln_w, ly.conv_ln_b, eps, qb_d, dumping ? o2 : nullptr, st));
    TRY(dump(4, qkv, 3 * d));  // q of the new frames
    TRY(dump(5, o2, d));
    TRY(gemm_q(ly.pw2, qb_d, y, d, Epilogue{kEpiResidual, y, 1.0f}, QOut{}));
    TRY(dump(6, y, d));
    // macaron FF2 and the block's final LN
    TRY(launch_ln_quant(y, d, ly.ln_ff2_w, ly.ln_ff2_b, eps, (int)d, M, qa, nullptr, d, st));
    TRY(gemm_q(ly.ff2_1, qa, nullptr, dff, silu, qb_ff));
    TRY(gemm_q(ly.ff2_2, qb_ff, y, d, Epilogue{kEpiResidual, y, 0.5f}, QOut{}));
    if (li + 1 < e->layers.size()) {  // the block's output LN and the next block's FF1 LN in one pass
      const Layer &nx = e->layers[li + 1];
      TRY(launch_ln2_quant(y, d, ly.ln_out_w, ly.ln_out_b, x, d, nx.ln_ff1_w, nx.ln_ff1_b, eps, (int)d, M, qa,
                           nullptr, d, st));
    } else {
      TRY(launch_ln_rows(y, d, ly.ln_out_w, ly.ln_out_b, eps, x, d, M, (int)d, st));
    }
    TRY(dump(7, x, d));
  }
  // ---- prompt MLP on the new frames (streaming.rs:320-342) ----
  if (e->any_prompt) {
    const QOut qcat = qbuf(0, d + e->n_prompts), qh = qbuf(1, e->prompt_hidden);
    TRY(launch_prompt_cat_quant(x, M, (int)cf, (int)d, (int)e->n_prompts, e->pids + z0, qcat, st));
    TRY(gemm_q(e->prompt0, qcat, nullptr, e->prompt_hidden, Epilogue{kEpiRelu, nullptr, 1.0f}, qh));
    TRY(gemm_q(e->prompt2, qh, y, d, Epilogue{}, QOut{}));
    TRY(launch_prompt_select(x, y, M, (int)cf, (int)d, e->pids + z0, st));
  }
  TRY(launch_out_ring(x, M, (int)cf, (int)d, e->out_ring + z0 * e->out_cap * d, (int)e->out_cap, s, e->shift_arg,
                      st));
  return kOk;
}

// First stream of the second sub-batch, or 0 for one batch: the halves are
// split where the code buffers' 128-frame tiles split (z0 * cf a multiple of
// 128), so the two halves' GEMM inputs never share a tile.  Stage dumps keep
// one batch (their buffer holds the whole step).
static int64_t split_point(const sc_stream_encoder *e, int64_t cf) {
  const int64_t Z = e->n_streams;
  if (!e->side || e->max_batches < 2 || e->dump_layer >= 0 || Z < 2) return 0;
  int64_t gcd = 128, v = cf;
  while (v) {
    const int64_t r = gcd % v;
    gcd = v;
    v = r;
  }
  const int64_t unit = 128 / gcd;  // streams per 128-frame tile boundary
  const int64_t z0 = (Z / 2) / unit * unit;
  return z0 > 0 && z0 < Z ? z0 : 0;
}

// ---- step graphs ----------------------------------------------------------
//
// The reference's GPU backend records a whole step into one submission
// (gpu/batch.rs:50,163; gpu/streaming.rs:259-298).  Here a step is captured
// by stream capture into a CUDA graph and replayed by later steps with the
// same launches.  Two steps issue the same launches with the same arguments
// when their geometry below is equal, except for
//  - frame numbers, which differ by a whole number of attention chunks:
//    bands, masks, pos rows and the conv taps depend only on frame
//    differences (and on chunk indices, which shift together), so only ring
//    slots move, and the ring kernels add the device frame shift;
//  - the caller's mel and output buffers: the mel always passes through the
//    staging buffer in a graph step, and replays re-point the copy nodes.
// The mel-history buffer pair alternates between steps; its parity is part
// of a graph's key.
constexpr size_t kMaxStepGraphs = 4;

static std::vector<int64_t> step_geometry(const sc_stream_encoder *e, const StepGeom &g, int64_t z0, bool host_io,
                                          bool has_out) {
  std::vector<int64_t> k = {e->n_streams, z0, g.cf, g.n_new, g.t_mel, g.start_rel, e->hist_frames,
                            g.s % e->chunk,
                            // depthwise taps before frame 0 are skipped until s >= kernel - 1
                            std::min<int64_t>(g.s, e->cfg.conv_kernel - 1), host_io, has_out, e->any_prompt};
  for (int64_t a = g.s; a < g.t_new;) {
    int64_t b, k_lo;
    attn_span(e, a, g.t_new, b, k_lo);
    k.insert(k.end(), {a - g.s, b - g.s, k_lo - g.s});
    a = b;
  }
  return k;
}

static bool page_locked(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

static StepGraph *find_step_graph(sc_stream_encoder *e, const std::vector<int64_t> &key) {
  for (auto &g : e->step_graphs)
    if (g.exec && g.key == key) return &g;
  return nullptr;
}

// Captures the launches issue(stream) makes into a new step graph.  Nothing
// runs.  On any failure the encoder stops using graphs (its steps run as
// separate launches, which report errors of their own) and nullptr returns.
static StepGraph *capture_step(sc_stream_encoder *e, std::vector<int64_t> key, int64_t s, int64_t n_new,
                               int64_t cf, int64_t z0, const std::function<int(cudaStream_t)> &issue) {
  const long long n0 = sc_launch_count();
  e->shift_arg = e->shift_dev;
  cudaGraph_t graph = nullptr;
  int rc = kOk;
  cudaError_t ce = cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal);
  if (ce == cudaSuccess) {
    rc = issue(e->cap_stream);
    ce = cudaStreamEndCapture(e->cap_stream, &graph);
  }
  e->shift_arg = nullptr;
  note_launches(-(sc_launch_count() - n0));  // captured, not run
  StepGraph sg;
  sg.key = std::move(key);
  sg.s = s;
  sg.graph = graph;
  bool ok = !rc && ce == cudaSuccess && graph;
  if (ok) {
    // kernel nodes, and which copy each copy node is (by its device-side
    // address: the staging buffer for mel in, the frames for frames out)
    const int64_t fi = e->cfg.feat_in, d = e->cfg.d_model, Z = e->n_streams;
    const int64_t halves[2][2] = {{0, z0 ? z0 : Z}, {z0, Z - z0}};
    size_t n = 0;
    ok = cudaGraphGetNodes(graph, nullptr, &n) == cudaSuccess;
    std::vector<cudaGraphNode_t> nodes(n);
    if (ok && n) ok = cudaGraphGetNodes(graph, nodes.data(), &n) == cudaSuccess;
    for (size_t i = 0; ok && i < n; i++) {
      cudaGraphNodeType t;
      ok = cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess;
      if (!ok) break;
      if (t == cudaGraphNodeTypeKernel) {
        sg.kernels++;
      } else if (t == cudaGraphNodeTypeMemcpy) {
        cudaMemcpy3DParms p{};
        ok = cudaGraphMemcpyNodeGetParams(nodes[i], &p) == cudaSuccess;
        const char *dst = (const char *)p.dstPtr.ptr + p.dstPos.x, *src = (const char *)p.srcPtr.ptr + p.srcPos.x;
        bool found = false;
        for (int h = 0; ok && !found && h < (z0 ? 2 : 1); h++) {
          const int64_t za = halves[h][0], nz = halves[h][1];
          if (n_new > 0 && dst == (const char *)(e->mel_stage + za * n_new * fi)) {
            sg.copies.push_back(StepCopy{nodes[i], za, nz, 0});
            found = true;
          } else if (src == (const char *)(e->x + za * cf * d)) {
            sg.copies.push_back(StepCopy{nodes[i], za, nz, 1});
            found = true;
          }
        }
        ok = ok && found;
      }
    }
  }
  if (ok) ok = cudaGraphInstantiate(&sg.exec, graph, 0) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    e->drop_graph(sg);
    e->graphs = false;
    return nullptr;
  }
  if (e->step_graphs.size() >= kMaxStepGraphs) {
    // the least recently used one goes; wait until no launch of it is queued
    size_t lru = 0;
    for (size_t i = 1; i < e->step_graphs.size(); i++)
      if (e->step_graphs[i].used < e->step_graphs[lru].used) lru = i;
    cudaDeviceSynchronize();
    e->drop_graph(e->step_graphs[lru]);
    e->step_graphs.erase(e->step_graphs.begin() + (std::ptrdiff_t)lru);
  }
  e->graph_captures++;
  e->step_graphs.push_back(std::move(sg));
  return &e->step_graphs.back();
}

// Replays a step graph on st for the step at frame s: copy nodes pointed at
// this call's buffers, the frame shift stored, one graph launch.  Returns 1
// (nothing issued) when the graph cannot serve this step.
static int replay_step(sc_stream_encoder *e, StepGraph &g, int64_t s, const float *mel_new, int64_t n_new,
                       float *out_host, int64_t cf, bool host_io, cudaStream_t st) {
  const int64_t fi = e->cfg.feat_in, d = e->cfg.d_model;
  if (s < g.s || (s - g.s) % e->chunk) return 1;  // the shift must be whole chunks forward
  for (const StepCopy &c : g.copies) {
    cudaError_t ce;
    if (c.dir == 0) {
      const int64_t off = c.za * n_new * fi;
      ce = cudaGraphExecMemcpyNodeSetParams1D(g.exec, c.node, e->mel_stage + off, mel_new + off,
                                              (size_t)(c.nz * n_new * fi) * 4,
                                              host_io ? cudaMemcpyHostToDevice : cudaMemcpyDefault);
    } else {
      const int64_t off = c.za * cf * d;
      ce = cudaGraphExecMemcpyNodeSetParams1D(g.exec, c.node, out_host + off, e->x + off, (size_t)(c.nz * cf * d) * 4,
                                              cudaMemcpyDeviceToHost);
    }
    if (ce != cudaSuccess) {
      cudaGetLastError();
      return 1;
    }
  }
  TRY(launch_store_i64(e->shift_dev, s - g.s, st));
  SC_CUDA(cudaGraphLaunch(g.exec, st));
  note_launches(g.kernels);
  g.used = ++e->graph_clock;
  e->graph_launches++;
  return kOk;
}

// One encode_new step.  host_io: mel_new is host memory, copied per half
// into the encoder's staging buffer on that half's stream, and each half's
// output frames are copied to out_host (if given) on its stream, so one
// half's copies overlap the other half's kernels; the call then waits for
// the caller's stream.
static int encode_call(sc_stream_encoder *e, const float *mel_new, int64_t t0, int64_t t1, int32_t fin,
                       cudaStream_t st, bool host_io, float *out_host, int64_t *rows_out) {
  if (!e || (!mel_new && t1 > t0) || t0 < 0 || t1 < t0 || t0 % 8) {
    set_error("stream_encoder_encode_new: invalid argument (t0 must be a multiple of 8)");
    return kErrInvalid;
  }
  const sc_encoder_config &c = e->cfg;
  const int64_t d = c.d_model, Z = e->n_streams;
  StepGeom g{};
  // ---- frames of this step (streaming.rs:160-180) ----
  const int64_t s = t0 / 8, n_new = t1 - t0, ecount = s + (n_new + 7) / 8;
  if (s != e->total) {
    set_error("streaming encoder out of sync: expected frame %lld, cache has %lld", (long long)s,
              (long long)e->total);
    return kErrState;
  }
  const int64_t t_new = fin ? s + (((n_new / 2 + 1) / 2 + 1) / 2 + 1) : ecount;
  if (rows_out) *rows_out = 0;
  if (t_new <= s) return kOk;
  if (host_io && n_new > e->mel_stage_frames) {
    set_error("stream_encoder_encode_new_host: %lld mel frames exceed the staging buffer's %lld",
              (long long)n_new, (long long)e->mel_stage_frames);
    return kErrUnsupported;
  }
  const int64_t cf = t_new - s;
  if (cf > c.max_frames) {
    set_error("stream_encoder_encode_new: %lld new frames exceed max_frames %d", (long long)cf, c.max_frames);
    return kErrUnsupported;
  }
  // ---- pre-encode window (streaming.rs:182-218) ----
  const int64_t mel_lo = s * 8, win_start = mel_lo > kMelHistory ? mel_lo - kMelHistory : 0;
  const int64_t start_rel = (mel_lo - win_start) / 8, rel_max = start_rel + cf - 1;
  const int64_t avail = t1 - win_start;
  const int64_t want = std::max<int64_t>(8 * rel_max + 1, t_new * 8 - win_start);
  const int64_t t_mel = std::min<int64_t>(avail, want);
  if (mel_lo - win_start != e->hist_frames || t_mel > e->t_mel_max) {
    set_error("stream_encoder_encode_new: window of %lld mel frames unsupported", (long long)t_mel);
    return kErrUnsupported;
  }
  g.s = s;
  g.n_new = n_new;
  g.t_new = t_new;
  g.cf = cf;
  g.t_mel = t_mel;
  g.start_rel = start_rel;
  g.ta = conv_out(t_mel);
  g.fa = conv_out(c.feat_in);
  g.tb = conv_out(g.ta);
  g.fb = conv_out(g.fa);
  const int64_t tc = conv_out(g.tb);
  g.fc = conv_out(g.fb);
  if (tc < start_rel + cf) {
    set_error("pre_encode produced too few frames: %lld < %lld", (long long)tc, (long long)(start_rel + cf));
    return kErrInvalid;
  }
  // Rows each pre-encode stage must produce for output frames
  // [start_rel, start_rel + cf) (a 3x3 stride-2 conv with top pad 2 maps
  // output row r to input rows 2r - 2 .. 2r); the convs compute only those.
  g.r5 = start_rel;
  g.n5 = cf;
  g.r3 = std::max<int64_t>(2 * g.r5 - 2, 0);
  g.e3 = std::min<int64_t>(2 * (g.r5 + g.n5 - 1) + 1, g.tb);
  // ---- pos rows, once (streaming.rs:236-261) ----
  if (!e->pos_ready) {
    // sinusoid rows computed on the host in f32 exactly as the reference does
    std::vector<float> pet((size_t)(e->n_pos * d));
    const float ln10000 = logf(10000.0f);
    for (int64_t i = 0; i < e->n_pos; i++) {
      const float pos = (float)i + (float)(1 - e->chunk);
      for (int64_t k = 0; k < d / 2; k++) {
        const float div = expf(-2.0f * (float)k * ln10000 / (float)d);
        pet[i * d + 2 * k] = sinf(pos * div);
        pet[i * d + 2 * k + 1] = cosf(pos * div);
      }
    }
    SC_CUDA(cudaMemcpyAsync(e->pos_in, pet.data(), pet.size() * 4, cudaMemcpyHostToDevice, st));
    for (auto &ly : e->layers)
      TRY(gemm_impl(&ly.pos.w, e->pos_in, e->n_pos, SC_LAYOUT_TIME_MAJOR, 0, ly.pos.bias, ly.pos_p,
                    SC_LAYOUT_TIME_MAJOR, d, e->ws, e->ws_bytes, nullptr, st, Epilogue{}, true));
    SC_CUDA(cudaStreamSynchronize(st));  // pet must outlive the copy
    e->pos_ready = true;
  }
  e->dump_rows = Z * cf;
  // ---- the streams, as one batch or as two halves in flight at once on the
  // caller's stream and the encoder's side stream (each half's GEMMs are
  // under two waves of CTAs, so the other half's kernels fill the SMs their
  // last wave leaves idle) ----
  const int64_t fi = c.feat_in;
  // streams [za, za + nz) on sa; stage: the mel goes through the staging
  // buffer (the host entry point, and every graph step)
  auto run = [&](int64_t za, int64_t nz, cudaStream_t sa, bool stage) -> int {
    const float *mel = mel_new;
    if (stage && n_new > 0) {
      SC_CUDA(cudaMemcpyAsync(e->mel_stage + za * n_new * fi, mel_new + za * n_new * fi,
                              (size_t)(nz * n_new * fi) * 4, host_io ? cudaMemcpyHostToDevice : cudaMemcpyDefault,
                              sa));
      mel = e->mel_stage;
    }
    TRY(encode_streams(e, g, mel, za, nz, sa));
    if (host_io && out_host)
      SC_CUDA(cudaMemcpyAsync(out_host + za * cf * d, e->x + za * cf * d, (size_t)(nz * cf * d) * 4,
                              cudaMemcpyDeviceToHost, sa));
    return kOk;
  };
  const int64_t z0 = split_point(e, cf);
  auto run_all = [&](cudaStream_t s0, bool stage) -> int {
    if (z0 == 0) return run(0, Z, s0, stage);
    SC_CUDA(cudaEventRecord(e->ev_fork, s0));
    SC_CUDA(cudaStreamWaitEvent(e->side, e->ev_fork, 0));
    int r = run(0, z0, s0, stage);
    if (!r) r = run(z0, Z - z0, e->side, stage);
    // join even after an error, so the caller's stream never runs ahead of
    // work left on the side stream
    SC_CUDA(cudaEventRecord(e->ev_join, e->side));
    SC_CUDA(cudaStreamWaitEvent(s0, e->ev_join, 0));
    return r;
  };
  // a step graph when this step's geometry was seen before (replay) or
  // repeats the previous step's (capture, then replay); separate launches
  // otherwise
  const bool graph_ok = e->graphs && e->dump_layer < 0 && n_new <= e->mel_stage_frames &&
                        (!host_io || ((n_new == 0 || page_locked(mel_new)) && (!out_host || page_locked(out_host))));
  std::vector<int64_t> geom;
  StepGraph *gr = nullptr;
  if (graph_ok) {
    geom = step_geometry(e, g, z0, host_io, out_host != nullptr);
    std::vector<int64_t> key = geom;
    key.push_back(e->hist_cur);
    gr = find_step_graph(e, key);
    if (!gr && geom == e->prev_geom)
      gr = capture_step(e, std::move(key), s, n_new, cf, z0, [&](cudaStream_t cs) { return run_all(cs, true); });
  }
  e->prev_geom = std::move(geom);
  int rc = 1;
  if (gr) rc = replay_step(e, *gr, s, mel_new, n_new, out_host, cf, host_io, st);
  if (rc == 1) rc = run_all(st, host_io);
  if (host_io) {
    // even after an error: copies already queued may still be reading the
    // caller's mel buffer or writing its output buffer
    const cudaError_t se = cudaStreamSynchronize(st);
    if (!rc && se != cudaSuccess) return cuda_fail(se, "cudaStreamSynchronize");
  }
  if (rc) return rc;
  if (rows_out) *rows_out = Z * cf;
  e->hist_cur ^= 1;
  e->hist_frames = (int)std::min<int64_t>(kMelHistory, e->hist_frames + n_new);
  e->total = t_new;
  e->last_c = cf;
  return kOk;
}

int sc_stream_encoder_encode_new(sc_stream_encoder *e, const float *mel_new, int64_t t0, int64_t t1, int32_t fin,
                                 void *stream) {
  return encode_call(e, mel_new, t0, t1, fin, (cudaStream_t)stream, false, nullptr, nullptr);
}

int sc_stream_encoder_encode_new_host(sc_stream_encoder *e, const float *mel_host, int64_t t0, int64_t t1,
                                      int32_t fin, float *out_host, int64_t *rows, void *stream) {
  return encode_call(e, mel_host, t0, t1, fin, (cudaStream_t)stream, true, out_host, rows);
}

int sc_stream_encoder_set_concurrency(sc_stream_encoder *e, int32_t n_batches) {
  if (!e || n_batches < 1 || n_batches > 2) {
    set_error("stream_encoder_set_concurrency: n_batches must be 1 or 2");
    return kErrInvalid;
  }
  e->max_batches = n_batches;
  return kOk;
}

int sc_stream_encoder_set_graphs(sc_stream_encoder *e, int32_t enable) {
  if (!e || (enable != 0 && enable != 1)) {
    set_error("stream_encoder_set_graphs: enable must be 0 or 1");
    return kErrInvalid;
  }
  if (!enable && !e->step_graphs.empty()) {
    SC_CUDA(cudaDeviceSynchronize());  // no replay of them may still be queued
    for (auto &g : e->step_graphs) e->drop_graph(g);
    e->step_graphs.clear();
  }
  e->graphs = enable != 0;
  e->prev_geom.clear();
  return kOk;
}

int sc_stream_encoder_graph_stats(const sc_stream_encoder *e, int64_t *captures, int64_t *launches) {
  if (!e || !captures || !launches) {
    set_error("stream_encoder_graph_stats: invalid argument");
    return kErrInvalid;
  }
  *captures = e->graph_captures;
  *launches = e->graph_launches;
  return e->graphs ? 1 : 0;
}

int sc_stream_encoder_set_prompts(sc_stream_encoder *e, const int32_t *prompt_ids) {
  if (!e || !prompt_ids) {
    set_error("stream_encoder_set_prompts: invalid argument");
    return kErrInvalid;
  }
  if (!e->n_prompts) return kOk;  // no prompt MLP: the output is left unchanged
  // an id out of range means no prompt, as the reference's `pid < num_prompts`
  std::vector<int32_t> ids((size_t)e->n_streams);
  bool any = false;
  for (int64_t i = 0; i < e->n_streams; i++) {
    const int32_t p = prompt_ids[i];
    ids[(size_t)i] = p >= 0 && p < e->n_prompts ? p : -1;
    any |= ids[(size_t)i] >= 0;
  }
  SC_CUDA(cudaMemcpy(e->pids, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice));
  e->any_prompt = any;
  return kOk;
}

int64_t sc_stream_encoder_n_prompts(const sc_stream_encoder *e) { return e ? e->n_prompts : 0; }

int sc_stream_encoder_set_dump(sc_stream_encoder *e, int32_t layer) {
  if (!e || layer >= (int32_t)e->layers.size()) {
    set_error("stream_encoder_set_dump: invalid layer");
    return kErrInvalid;
  }
  if (layer >= 0 && !e->dump) {
    const size_t bytes = (size_t)kDumpStages * e->n_streams * e->cfg.max_frames * 2 * e->cfg.d_model * 4;
    if (dev_malloc((void **)&e->dump, bytes) != cudaSuccess) {
      cudaGetLastError();
      set_error("stream_encoder_set_dump: cudaMalloc failed");
      return kErrAlloc;
    }
    e->allocs.push_back(e->dump);
  }
  e->dump_layer = layer;
  return kOk;
}

int sc_stream_encoder_dump(const sc_stream_encoder *e, int32_t stage, float *out_host, int64_t *rows) {
  if (!e || !e->dump || stage < 0 || stage >= kDumpStages || !out_host) {
    set_error("stream_encoder_dump: no dump recorded or bad stage");
    return kErrInvalid;
  }
  SC_CUDA(cudaDeviceSynchronize());
  const int64_t d = e->cfg.d_model;
  SC_CUDA(cudaMemcpy2D(out_host, d * 4, e->dump + (size_t)stage * e->dump_rows * 2 * d, 2 * d * 4, d * 4,
                       e->dump_rows, cudaMemcpyDeviceToHost));
  if (stage == 4) {  // q is held in lane-major head order: back to natural
    const int64_t hd = d / e->cfg.n_heads;
    std::vector<float> row((size_t)d);
    for (int64_t r = 0; r < e->dump_rows; r++) {
      float *q = out_host + r * d;
      for (int64_t i = 0; i < d; i++) row[(size_t)i] = q[(i / hd) * hd + lane_major_h(i % hd)];
      memcpy(q, row.data(), (size_t)d * 4);
    }
  }
  if (rows) *rows = e->dump_rows;
  return kOk;
}

int sc_stream_encoder_output(const sc_stream_encoder *e, const float **frames, int64_t *rows, int64_t *d) {
  if (!e || !frames) {
    set_error("stream_encoder_output: invalid argument");
    return kErrInvalid;
  }
  *frames = e->x;
  if (rows) *rows = e->n_streams * e->last_c;
  if (d) *d = e->cfg.d_model;
  return kOk;
}

int sc_pre_encode_pointwise_relu(const float *x, const float *w, const float *bias, float *y, int64_t n_streams,
                                 int64_t rows_per_stream, int64_t sp_base, int64_t spatial, int64_t c_out,
                                 int64_t c_in, void *stream) {
  if (!x || !w || !bias || !y || n_streams < 0 || rows_per_stream < 0 || c_out <= 0 || c_in <= 0 ||
      c_out > (1 << 20) || rows_per_stream > (1 << 24)) {
    set_error("pre_encode_pointwise_relu: invalid argument");
    return kErrInvalid;
  }
  if (n_streams == 0 || rows_per_stream == 0) return kOk;
  return launch_pw_conv_relu(x, w, bias, y, n_streams, (int)rows_per_stream, sp_base, spatial, (int)c_out,
                             (int)c_in, (cudaStream_t)stream);
}

}  // extern "C"
