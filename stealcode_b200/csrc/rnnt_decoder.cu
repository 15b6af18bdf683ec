// rnnt_decoder.cu -- the device greedy RNN-T decoder: the B200 counterpart of
// the reference's streaming decode loop (nemotron/live.rs:56-145,
// decode_frames) with its predictor LSTM (nemotron/decoder.rs:75-205) and
// joint network (decoder.rs:207-235), for n_streams streams at once.
//
// Every stream runs the reference's loop; the device runs the loops of all
// streams in lockstep rounds.  One round is one loop iteration of every
// stream that is still decoding:
//   1. predictor step (one launch per LSTM layer) for the streams that
//      emitted in the previous round (the reference's `predictor_dirty`);
//   2. joint.pred over the new predictor output, for the same streams;
//   3. joint.out over relu(enc_proj[step] + pred) for every active stream;
//   4. per stream: greedy argmax, token append, the step / max_symbols
//      bookkeeping, and the stream lists of the next round.
// The host stops launching rounds once no stream is active (it reads the
// count one round behind, so the GPU never idles on the check).
//
// Arithmetic follows the reference's CPU path to the bit.  Every linear is a
// q8_gemm call with n = 1 (n = frames for joint.enc) and the reference
// dispatches it by shape (simd_kernel.rs:106-125): rows % 8 == 0, k % 32 ==
// 0 and n <= 16 take the 8-lane SIMD order (lane l sums the products of
// elements l, l+8, l+16, l+24 of a block exactly, then fma(lane sum, dw*dx,
// acc) per block and an ordered sum of the 8 lanes, simd_kernel.rs:292-330),
// anything else q8_gemm_scalar's (acc += (dw*dx) * dot, sgemm_kernel.rs:
// 132-202).  The device stores each block with element l + 8j at byte 4l + j
// (weights at load, activation codes at quantisation), so one dp4a gives a
// SIMD lane's exact integer sum.  exp and tanh are correctly rounded (f32
// from the double functions); the reference calls glibc's expf/tanhf.

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "sc_device.cuh"
#include "sc_kernels.cuh"
#include "../../include/stealcode_b200.h"

namespace sc {
namespace {

constexpr int kRows = 128;    // output rows of a tile: one per thread
constexpr int kCols = 8;      // input vectors (columns) of a tile
constexpr int kThreads = 128;
constexpr int kCtasPerSm = 4;

// A Q8_0 matrix in the decoder's lane order: int8 [rows_pad][k] with the
// element l + 8j of every 32-block at byte 4l + j, f32 block scales
// [rows_pad][nb] (the f16 scales converted exactly).  Padding rows are zero.
struct LaneMat {
  int8_t *qs = nullptr;
  float *sc = nullptr;
  float *bias = nullptr;  // [rows] or nullptr (Lin::bias is optional)
  int rows = 0, rows_pad = 0, k = 0, nb = 0;
  bool simd = false;      // the reference's SIMD order for an n <= 16 GEMM
};

// Device state of all streams (StreamState, live.rs:24-50, plus the loop
// variables of decode_frames).
struct DecState {
  const float *embed;  // [vocab][H]
  float *hc;           // [S][2 bufs][h, c][L][H]; buf cur[z] is (h, c), the other (nh, nc)
  int32_t *cur, *last_tok, *pred_valid;  // [S]
  float *pred;         // [S][J] joint.pred of the current predictor output
  float *enc;          // [S][n][J] joint.enc of this call's frames
  float *logits;       // [S][V]
  const float *frames; // [S][n][d_enc]
  int32_t *step, *nsym, *iter, *emitted, *status;  // [S]
  int32_t *ids, *steps;                            // [S][cap]
  int32_t *lists;      // [2 parities][dirty, active][S]
  int32_t *counts;     // [2 parities][dirty, active]
  int S, H, L, J, V, n, cap, blank, max_symbols, max_iters, d_enc;
};

__device__ __forceinline__ float *hc_at(const DecState &s, int z, int buf, int which, int l) {
  return s.hc + ((((int64_t)z * 2 + buf) * 2 + which) * s.L + l) * s.H;
}
__device__ __forceinline__ int32_t *list_at(const DecState &s, int parity, int which) {
  return s.lists + (int64_t)(parity * 2 + which) * s.S;
}

// sigmoid and tanh as decoder.rs:431-433 and f32::tanh write them, with
// correctly rounded exp/tanh.
__device__ __forceinline__ float sigmoid_ref(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-x)));
}
__device__ __forceinline__ float tanh_rn(float x) { return (float)tanh((double)x); }

// ---- the column sources and sinks of each linear -------------------------
// LSTM layer l of the predictor step (decoder.rs:158-190): input [x ; h_l]
// with x the embedding of the last token (zeros before the first) or the new
// h of layer l-1; rows in gate-interleaved order 4k + g (g = i, f, g, o), so
// the 4 gates of a cell sit in 4 adjacent lanes.
struct LstmOp {
  int l, parity;
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 0)[j]; }
  __device__ float input(const DecState &s, int z, int i) const {
    const int H = s.H;
    if (i >= H) return hc_at(s, z, s.cur[z], 0, l)[i - H];
    if (l > 0) return hc_at(s, z, s.cur[z] ^ 1, 0, l - 1)[i];
    const int tok = s.last_tok[z];
    return tok >= 0 ? s.embed[(int64_t)tok * H + i] : 0.0f;
  }
  __device__ void output(const DecState &s, const LaneMat &w, int z, int row, float y) const {
    // gates[k] += bias[k] (decoder.rs:176-178), then the cell (:185-194)
    const float g = __fadd_rn(y, w.bias[row < w.rows ? row : 0]);
    const int lane = threadIdx.x & 31, base = lane & ~3;
    const float gi = __shfl_sync(0xffffffffu, g, base), gf = __shfl_sync(0xffffffffu, g, base + 1);
    const float gg = __shfl_sync(0xffffffffu, g, base + 2), go = __shfl_sync(0xffffffffu, g, base + 3);
    const int k = row >> 2;
    if (z < 0 || (lane & 3) || k >= s.H) return;
    const int nb = s.cur[z] ^ 1;
    const float ig = sigmoid_ref(gi), fg = sigmoid_ref(gf), gt = tanh_rn(gg), og = sigmoid_ref(go);
    const float cold = hc_at(s, z, nb ^ 1, 1, l)[k];
    const float cn = __fadd_rn(__fmul_rn(fg, cold), __fmul_rn(ig, gt));
    hc_at(s, z, nb, 1, l)[k] = cn;
    hc_at(s, z, nb, 0, l)[k] = __fmul_rn(og, tanh_rn(cn));
  }
};

// joint.pred over the last layer's new h (live.rs:100-101, Lin::matvec).
struct PredOp {
  int parity;
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 0)[j]; }
  __device__ float input(const DecState &s, int z, int i) const {
    return hc_at(s, z, s.cur[z] ^ 1, 0, s.L - 1)[i];
  }
  __device__ void output(const DecState &s, const LaneMat &w, int z, int row, float y) const {
    if (z < 0 || row >= w.rows) return;
    s.pred[(int64_t)z * s.J + row] = w.bias ? __fadd_rn(y, w.bias[row]) : y;
    if (row == 0) s.pred_valid[z] = 1;
  }
};

// joint.out over relu(enc_proj[step] + pred) (live.rs:102-106), every
// active stream.
struct OutOp {
  int parity;
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2 + 1]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 1)[j]; }
  __device__ float input(const DecState &s, int z, int i) const {
    const float v = __fadd_rn(s.enc[((int64_t)z * s.n + s.step[z]) * s.J + i], s.pred[(int64_t)z * s.J + i]);
    return v > 0.0f ? v : 0.0f;  // (e + p).max(0.0): NaN -> 0
  }
  __device__ void output(const DecState &s, const LaneMat &w, int z, int row, float y) const {
    if (z < 0 || row >= w.rows) return;
    s.logits[(int64_t)z * s.V + row] = w.bias ? __fadd_rn(y, w.bias[row]) : y;
  }
};

// joint.enc over the call's frames (live.rs:71-81, Lin::forward_t with n
// frames): column z * n + t.
struct EncOp {
  __device__ int n_cols(const DecState &s) const { return s.S * s.n; }
  __device__ int col_id(const DecState &, int j) const { return j; }
  __device__ float input(const DecState &s, int col, int i) const {
    return s.frames[(int64_t)col * s.d_enc + i];
  }
  __device__ void output(const DecState &s, const LaneMat &w, int col, int row, float y) const {
    if (col < 0 || row >= w.rows) return;
    s.enc[(int64_t)col * s.J + row] = w.bias ? __fadd_rn(y, w.bias[row]) : y;
  }
};

// y = W x for tiles of 128 rows x 8 columns, grid-stride over the tiles
// the column count (read on the device) needs.  The columns' codes are
// quantised per 32-block in the prologue (quantize_col, one warp per block)
// into shared memory in lane order; every thread owns one row.
template <bool kSimd, class Op>
__global__ void __launch_bounds__(kThreads) lane_gemv_kernel(LaneMat w, DecState s, Op op) {
  extern __shared__ __align__(16) unsigned char smem[];
  int8_t *xs = reinterpret_cast<int8_t *>(smem);                // [kCols][k]
  float *dxs = reinterpret_cast<float *>(smem + kCols * w.k);   // [kCols][nb]
  int *ids = reinterpret_cast<int *>(dxs + kCols * w.nb);       // [kCols]
  const int ncols = op.n_cols(s);
  const int row_tiles = w.rows_pad / kRows, col_tiles = (ncols + kCols - 1) / kCols;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int tile = blockIdx.x; tile < row_tiles * col_tiles; tile += gridDim.x) {
    const int rt = tile % row_tiles, ct = tile / row_tiles;
    __syncthreads();  // the previous tile's reads of xs/dxs/ids are done
    for (int c = warp; c < kCols; c += kThreads / 32) {
      const int j = ct * kCols + c;
      const int id = j < ncols ? op.col_id(s, j) : -1;
      if (lane == 0) ids[c] = id;
      for (int b = 0; b < w.nb; b++) {
        const float v = id >= 0 ? op.input(s, id, b * 32 + lane) : 0.0f;
        float sc;
        const int8_t q = warp_quantize_block(v, true, sc);
        xs[c * w.k + b * 32 + (lane & 7) * 4 + (lane >> 3)] = q;
        if (lane == 0) dxs[c * w.nb + b] = sc;
      }
    }
    __syncthreads();
    const int row = rt * kRows + threadIdx.x;
    const int4 *wq = reinterpret_cast<const int4 *>(w.qs + (int64_t)row * w.k);
    const float *wsc = w.sc + (int64_t)row * w.nb;
    float acc[kCols][kSimd ? 8 : 1];
#pragma unroll
    for (int c = 0; c < kCols; c++)
#pragma unroll
      for (int l = 0; l < (kSimd ? 8 : 1); l++) acc[c][l] = 0.0f;
    for (int b = 0; b < w.nb; b++) {
      const int4 lo = __ldg(wq + 2 * b), hi = __ldg(wq + 2 * b + 1);
      const int wv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      const float dw = __ldg(wsc + b);
#pragma unroll
      for (int c = 0; c < kCols; c++) {
        const int4 *xb = reinterpret_cast<const int4 *>(xs + c * w.k + b * 32);
        const int4 xlo = xb[0], xhi = xb[1];
        const int xv[8] = {xlo.x, xlo.y, xlo.z, xlo.w, xhi.x, xhi.y, xhi.z, xhi.w};
        const float scale = __fmul_rn(dw, dxs[c * w.nb + b]);
        if (kSimd) {
#pragma unroll
          for (int l = 0; l < 8; l++) acc[c][l] = __fmaf_rn((float)__dp4a(wv[l], xv[l], 0), scale, acc[c][l]);
        } else {
          int dot = 0;
#pragma unroll
          for (int l = 0; l < 8; l++) dot = __dp4a(wv[l], xv[l], dot);
          acc[c][0] = __fadd_rn(acc[c][0], __fmul_rn(scale, (float)dot));
        }
      }
    }
#pragma unroll
    for (int c = 0; c < kCols; c++) {
      float y = acc[c][0];
      if (kSimd) {
#pragma unroll
        for (int l = 1; l < 8; l++) y = __fadd_rn(y, acc[c][l]);  // reduce_sum: lanes in order
      }
      op.output(s, w, ids[c], row, y);
    }
  }
}

// Start of a decode_frames call: the loop variables of every stream, the
// first round's lists (every stream active; the predictor runs where its
// output is not already current).  One CTA.
__global__ void rnnt_init_kernel(DecState s) {
  if (threadIdx.x == 0)
    for (int i = 0; i < 4; i++) s.counts[i] = 0;
  __syncthreads();
  for (int z = threadIdx.x; z < s.S; z += blockDim.x) {
    s.step[z] = 0;
    s.nsym[z] = 0;
    s.iter[z] = 0;
    s.emitted[z] = 0;
    s.status[z] = 0;
    list_at(s, 0, 1)[atomicAdd(&s.counts[1], 1)] = z;
    if (!s.pred_valid[z]) list_at(s, 0, 0)[atomicAdd(&s.counts[0], 1)] = z;
  }
}

// Clears the next round's list counts (their last readers, the previous
// round's kernels, have finished).
__global__ void rnnt_clear_kernel(DecState s, int parity) {
  s.counts[(parity ^ 1) * 2] = 0;
  s.counts[(parity ^ 1) * 2 + 1] = 0;
}

// One loop iteration's decision per active stream (live.rs:107-140): the
// first index of the largest logit (NaNs never win; a NaN logit 0 keeps
// index 0), then blank -> next frame, else emit, swap the LSTM state and
// count symbols against max_symbols.  One warp per stream.
__global__ void rnnt_update_kernel(DecState s, int parity) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= s.counts[parity * 2 + 1]) return;
  const int z = list_at(s, parity, 1)[wid];
  const float *lg = s.logits + (int64_t)z * s.V;
  float bv = 0.0f;
  int bi = INT_MAX;
  for (int i = lane; i < s.V; i += 32) {
    const float v = lg[i];
    if (v == v && (bi == INT_MAX || v > bv)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane) return;
  const float v0 = lg[0];
  const int best = (v0 != v0 || bi == INT_MAX) ? 0 : bi;
  int step = s.step[z], ns = s.nsym[z], em = s.emitted[z];
  const int it = s.iter[z] + 1;
  bool dirty = false;
  if (best == s.blank) {
    step++;
    ns = 0;
  } else {
    if (em < s.cap) {
      s.ids[(int64_t)z * s.cap + em] = best;
      s.steps[(int64_t)z * s.cap + em] = step;
    }
    em++;
    s.last_tok[z] = best;
    s.cur[z] ^= 1;  // std::mem::swap(h, nh), (c, nc)
    s.pred_valid[z] = 0;
    dirty = true;
    ns++;
    if (s.max_symbols > 0 && ns >= s.max_symbols) {
      step++;
      ns = 0;
    }
  }
  s.step[z] = step;
  s.nsym[z] = ns;
  s.iter[z] = it;
  s.emitted[z] = em;
  const bool active = step < s.n && it < s.max_iters;
  if (!active && it >= s.max_iters) s.status[z] = 1;  // "rnnt decode: iteration cap hit"
  if (active) {
    const int np = parity ^ 1;
    list_at(s, np, 1)[atomicAdd(&s.counts[np * 2 + 1], 1)] = z;
    if (dirty) list_at(s, np, 0)[atomicAdd(&s.counts[np * 2], 1)] = z;
  }
}

float half_to_float_host(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, ex = (h >> 10) & 0x1f, man = h & 0x3ff;
  uint32_t bits;
  if (ex == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      uint32_t m = man;
      do {
        e++;
        m <<= 1;
      } while (!(m & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((ex + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

}  // namespace
}  // namespace sc

using namespace sc;

struct sc_rnnt_decoder {
  sc_rnnt_config cfg{};
  int64_t S = 0;
  int device = 0, sm_count = 148;
  int cap = 0;
  std::vector<LaneMat> lstm;
  LaneMat jenc, jpred, jout;
  DecState st{};
  int32_t *pinned = nullptr;  // [2] active counts read back
  cudaEvent_t ev[2] = {nullptr, nullptr};
  int64_t last_n = 0;
  std::vector<void *> allocs;
  ~sc_rnnt_decoder() {
    for (void *p : allocs) cudaFree(p);
    if (pinned) cudaFreeHost(pinned);
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
  }
};

namespace {

struct RLoader {
  const sc_tensor *t;
  int n;
  sc_rnnt_decoder *r;
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
  void *dev(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes < 16 ? 16 : bytes) != cudaSuccess) {
      cudaGetLastError();
      if (err.empty()) err = "cudaMalloc failed";
      return nullptr;
    }
    r->allocs.push_back(p);
    return p;
  }
  template <class T>
  T *upload(const std::vector<T> &v) {
    T *d = (T *)dev(v.size() * sizeof(T));
    if (d && cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess && err.empty())
      err = "upload failed";
    return d;
  }
  const float *f32(const std::string &name, int64_t count) {
    const sc_tensor *x = find(name);
    if (!x || x->dtype != 0 || numel(x) != count) {
      if (err.empty()) err = "tensor " + name + " missing or not f32 with " + std::to_string(count) + " elements";
      return nullptr;
    }
    return (const float *)x->data;
  }
  // Q8_0 tensor `base`.weight, GGUF dims [inp, out] (load_lin,
  // nemotron/weights.rs:640-697): rows out, row length inp.
  const uint8_t *q8(const std::string &base, int64_t inp, int64_t out) {
    const sc_tensor *x = find(base + ".weight");
    if (!x || x->dtype != 8 || x->n_dims != 2 || x->dims[0] != inp || x->dims[1] != out) {
      if (err.empty())
        err = "tensor " + base + ".weight missing or not Q8_0 [" + std::to_string(inp) + " -> " +
              std::to_string(out) + "]";
      return nullptr;
    }
    return (const uint8_t *)x->data;
  }
  // Builds a LaneMat from `parts` Q8 row-sources concatenated along K per
  // row (Q8Mat::concat_rows, weights.rs:132-147), with output row p taken
  // from source row src_row(p).
  template <class F>
  bool lane_mat(const std::vector<const uint8_t *> &parts, int64_t k_each, int64_t rows, F src_row,
                const std::vector<float> *bias, LaneMat *m) {
    const int64_t nb_each = k_each / 32, k = k_each * (int64_t)parts.size(), nb = k / 32;
    const int64_t rows_pad = (rows + kRows - 1) / kRows * kRows;
    std::vector<int8_t> qs((size_t)(rows_pad * k), 0);
    std::vector<float> sc((size_t)(rows_pad * nb), 0.0f);
    for (int64_t p = 0; p < rows; p++) {
      const int64_t srow = src_row(p);
      for (size_t part = 0; part < parts.size(); part++)
        for (int64_t b = 0; b < nb_each; b++) {
          const uint8_t *blk = parts[part] + (srow * nb_each + b) * 34;
          const int64_t ob = (int64_t)part * nb_each + b;
          sc[(size_t)(p * nb + ob)] = half_to_float_host((uint16_t)(blk[0] | (blk[1] << 8)));
          for (int e = 0; e < 32; e++)
            qs[(size_t)(p * k + ob * 32 + (e & 7) * 4 + (e >> 3))] = (int8_t)blk[2 + e];
        }
    }
    m->rows = (int)rows;
    m->rows_pad = (int)rows_pad;
    m->k = (int)k;
    m->nb = (int)nb;
    m->simd = rows % 8 == 0 && k % 32 == 0;
    m->qs = upload(qs);
    m->sc = upload(sc);
    m->bias = bias ? upload(*bias) : nullptr;
    return err.empty();
  }
  bool linear(const std::string &base, int64_t inp, int64_t out, LaneMat *m) {
    const uint8_t *w = q8(base, inp, out);
    if (!w) return false;
    std::vector<float> bias;
    const sc_tensor *b = find(base + ".bias");
    if (b) {
      if (b->dtype != 0 || numel(b) != out) {
        if (err.empty()) err = "tensor " + base + ".bias mis-shaped";
        return false;
      }
      bias.assign((const float *)b->data, (const float *)b->data + out);
    }
    return lane_mat({w}, inp, out, [](int64_t p) { return p; }, b ? &bias : nullptr, m);
  }
};

int launch_gemv(const sc_rnnt_decoder *r, const LaneMat &w, int64_t max_cols, bool simd, int kind, int arg,
                cudaStream_t st) {
  const int64_t tiles = (w.rows_pad / kRows) * ((max_cols + kCols - 1) / kCols);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)r->sm_count * kCtasPerSm));
  const size_t smem = (size_t)kCols * w.k + (size_t)kCols * w.nb * 4 + kCols * 4;
  const DecState &s = r->st;
#define SC_GEMV(OP)                                                                        \
  do {                                                                                     \
    if (simd)                                                                              \
      lane_gemv_kernel<true, OP><<<grid, kThreads, smem, st>>>(w, s, op);                  \
    else                                                                                   \
      lane_gemv_kernel<false, OP><<<grid, kThreads, smem, st>>>(w, s, op);                 \
  } while (0)
  switch (kind) {
    case 0: {
      LstmOp op{arg >> 1, arg & 1};
      SC_GEMV(LstmOp);
      break;
    }
    case 1: {
      PredOp op{arg};
      SC_GEMV(PredOp);
      break;
    }
    case 2: {
      OutOp op{arg};
      SC_GEMV(OutOp);
      break;
    }
    default: {
      EncOp op{};
      SC_GEMV(EncOp);
      break;
    }
  }
#undef SC_GEMV
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

#define TRY(call)         \
  do {                    \
    int _rc = (call);     \
    if (_rc) return _rc;  \
  } while (0)

}  // namespace

extern "C" {

int sc_rnnt_create(const sc_rnnt_config *cfg, const sc_tensor *tensors, int n_tensors, int64_t n_streams,
                   sc_rnnt_decoder **out) {
  if (!cfg || !tensors || !out || n_tensors <= 0 || n_streams <= 0 || n_streams > (1 << 24)) {
    set_error("rnnt_create: invalid argument");
    return kErrInvalid;
  }
  *out = nullptr;
  const sc_rnnt_config &c = *cfg;
  if (c.hidden <= 0 || c.hidden % 32 || c.hidden > 2048 || c.n_layers < 1 || c.n_layers > 8 || c.joint <= 0 ||
      c.joint % 32 || c.joint > 4096 || c.d_enc <= 0 || c.d_enc % 32 || c.d_enc > 4096 || c.vocab < 1 ||
      c.blank < 0 || c.blank >= c.vocab || c.max_symbols < 0 || c.max_frames < 1 || c.max_frames > 256 ||
      n_streams * (c.max_frames + (int64_t)c.vocab) > (int64_t)1 << 30) {
    set_error("rnnt_create: unsupported config (hidden %d, joint %d and d_enc %d: multiples of 32 up to "
              "2048/4096/4096; layers %d in 1..8; blank %d < vocab %d; max_frames %d in 1..256)",
              c.hidden, c.joint, c.d_enc, c.n_layers, c.blank, c.vocab, c.max_frames);
    return kErrUnsupported;
  }
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  sc_rnnt_decoder *r = new (std::nothrow) sc_rnnt_decoder();
  if (!r) {
    set_error("rnnt_create: host allocation failed");
    return kErrAlloc;
  }
  r->cfg = c;
  r->S = n_streams;
  r->device = dev;
  cudaDeviceGetAttribute(&r->sm_count, cudaDevAttrMultiProcessorCount, dev);
  r->cap = 16 * c.max_frames + 64;
  const int64_t H = c.hidden, L = c.n_layers, J = c.joint, V = c.vocab, S = n_streams;
  RLoader ld{tensors, n_tensors, r, {}};
  // predictor (decoder.rs:75-140): embedding, LSTM layers with ih|hh merged
  // per row and the two biases summed in f32
  const float *embed = ld.f32("decoder.prediction.embed.weight", V * H);
  r->lstm.resize((size_t)L);
  for (int64_t l = 0; l < L && ld.err.empty(); l++) {
    const std::string p = "decoder.prediction.dec_rnn.lstm.ih_l" + std::to_string(l);
    const std::string q = "decoder.prediction.dec_rnn.lstm.hh_l" + std::to_string(l);
    const uint8_t *ih = ld.q8(p, H, 4 * H), *hh = ld.q8(q, H, 4 * H);
    const float *bi = ld.f32(p + ".bias", 4 * H), *bh = ld.f32(q + ".bias", 4 * H);
    if (!ih || !hh || !bi || !bh) break;
    std::vector<float> bias((size_t)(4 * H));
    for (int64_t p4 = 0; p4 < 4 * H; p4++) {  // gate-interleaved row 4k + g <- row g*H + k
      const int64_t src = (p4 & 3) * H + (p4 >> 2);
      bias[(size_t)p4] = bi[src] + bh[src];
    }
    ld.lane_mat({ih, hh}, H, 4 * H, [H](int64_t p4) { return (p4 & 3) * H + (p4 >> 2); }, &bias,
                &r->lstm[(size_t)l]);
  }
  if (ld.err.empty()) ld.linear("joint.enc", c.d_enc, J, &r->jenc);
  if (ld.err.empty()) ld.linear("joint.pred", H, J, &r->jpred);
  if (ld.err.empty()) ld.linear("joint.joint_net.2", J, V, &r->jout);
  DecState &s = r->st;
  if (ld.err.empty()) {
    s.embed = ld.upload(std::vector<float>(embed, embed + V * H));
    s.hc = (float *)ld.dev((size_t)(S * 4 * L * H * 4));
    s.cur = (int32_t *)ld.dev((size_t)S * 4);
    s.last_tok = (int32_t *)ld.dev((size_t)S * 4);
    s.pred_valid = (int32_t *)ld.dev((size_t)S * 4);
    s.pred = (float *)ld.dev((size_t)(S * J * 4));
    s.enc = (float *)ld.dev((size_t)(S * c.max_frames * J * 4));
    s.logits = (float *)ld.dev((size_t)(S * V * 4));
    s.step = (int32_t *)ld.dev((size_t)S * 4);
    s.nsym = (int32_t *)ld.dev((size_t)S * 4);
    s.iter = (int32_t *)ld.dev((size_t)S * 4);
    s.emitted = (int32_t *)ld.dev((size_t)S * 4);
    s.status = (int32_t *)ld.dev((size_t)S * 4);
    s.ids = (int32_t *)ld.dev((size_t)(S * r->cap * 4));
    s.steps = (int32_t *)ld.dev((size_t)(S * r->cap * 4));
    s.lists = (int32_t *)ld.dev((size_t)(S * 4 * 4));
    s.counts = (int32_t *)ld.dev(16);
  }
  if (ld.err.empty() && (cudaHostAlloc(&r->pinned, 8, cudaHostAllocDefault) != cudaSuccess ||
                         cudaEventCreateWithFlags(&r->ev[0], cudaEventDisableTiming) != cudaSuccess ||
                         cudaEventCreateWithFlags(&r->ev[1], cudaEventDisableTiming) != cudaSuccess)) {
    cudaGetLastError();
    ld.err = "cudaMalloc failed (pinned buffer or events)";
  }
  if (!ld.err.empty()) {
    set_error("rnnt_create: %s", ld.err.c_str());
    const bool alloc = ld.err.find("cudaMalloc") != std::string::npos;
    delete r;
    return alloc ? kErrAlloc : kErrInvalid;
  }
  s.S = (int)S;
  s.H = (int)H;
  s.L = (int)L;
  s.J = (int)J;
  s.V = (int)V;
  s.cap = r->cap;
  s.blank = c.blank;
  s.max_symbols = c.max_symbols;
  s.d_enc = c.d_enc;
  *out = r;
  rc = sc_rnnt_reset(r, -1);
  if (rc) {
    *out = nullptr;
    delete r;
  }
  return rc;
}

int sc_rnnt_reset(sc_rnnt_decoder *r, int64_t stream_idx) {
  if (!r || stream_idx < -1 || stream_idx >= r->S) {
    set_error("rnnt_reset: invalid argument");
    return kErrInvalid;
  }
  const DecState &s = r->st;
  const int64_t lo = stream_idx < 0 ? 0 : stream_idx, cnt = stream_idx < 0 ? r->S : 1;
  const size_t per = (size_t)4 * s.L * s.H * 4;
  SC_CUDA(cudaDeviceSynchronize());
  SC_CUDA(cudaMemset(s.hc + lo * 4 * s.L * s.H, 0, per * cnt));
  SC_CUDA(cudaMemset(s.cur + lo, 0, cnt * 4));
  SC_CUDA(cudaMemset(s.pred_valid + lo, 0, cnt * 4));
  SC_CUDA(cudaMemset(s.emitted + lo, 0, cnt * 4));
  std::vector<int32_t> neg((size_t)cnt, -1);
  SC_CUDA(cudaMemcpy(s.last_tok + lo, neg.data(), cnt * 4, cudaMemcpyHostToDevice));
  return kOk;
}

int sc_rnnt_decode_frames(sc_rnnt_decoder *r, const float *frames, int64_t n, void *stream) {
  if (!r || n < 0 || n > r->cfg.max_frames || (n > 0 && !frames)) {
    set_error("rnnt_decode_frames: invalid argument (n %lld, max_frames %d)", (long long)n,
              r ? r->cfg.max_frames : 0);
    return kErrInvalid;
  }
  cudaStream_t st = (cudaStream_t)stream;
  DecState &s = r->st;
  r->last_n = n;
  if (n == 0) {  // the loop does not run: nothing is emitted
    SC_CUDA(cudaMemsetAsync(s.emitted, 0, r->S * 4, st));
    SC_CUDA(cudaStreamSynchronize(st));
    return kOk;
  }
  s.n = (int)n;
  s.frames = frames;
  s.max_iters = (int)(16 * n + 64);
  rnnt_init_kernel<<<1, 1024, 0, st>>>(s);
  note_launch();
  SC_CUDA(cudaGetLastError());
  // joint.enc over every stream's frames: the SIMD order for n <= 16
  TRY(launch_gemv(r, r->jenc, r->S * n, r->jenc.simd && n <= 16, 3, 0, st));
  const int L = (int)r->lstm.size();
  const unsigned upd_blocks = (unsigned)ceil_div(r->S, 8);  // 8 warps per CTA
  int64_t rounds = 0;
  bool done = false;
  for (int64_t it = 0; it < s.max_iters && !done; it++) {
    const int parity = (int)(it & 1);
    for (int l = 0; l < L; l++)
      TRY(launch_gemv(r, r->lstm[(size_t)l], r->S, true, 0, (l << 1) | parity, st));
    TRY(launch_gemv(r, r->jpred, r->S, r->jpred.simd, 1, parity, st));
    TRY(launch_gemv(r, r->jout, r->S, r->jout.simd, 2, parity, st));
    rnnt_clear_kernel<<<1, 1, 0, st>>>(s, parity);
    note_launch();
    rnnt_update_kernel<<<upd_blocks, 256, 0, st>>>(s, parity);
    note_launch();
    SC_CUDA(cudaGetLastError());
    rounds++;
    // every stream needs n iterations; from then on read the active count
    // of the round before (the GPU keeps working on this one meanwhile)
    if (it >= n - 1) {
      SC_CUDA(cudaMemcpyAsync(r->pinned + parity, s.counts + (parity ^ 1) * 2 + 1, 4, cudaMemcpyDeviceToHost, st));
      SC_CUDA(cudaEventRecord(r->ev[parity], st));
      if (it >= n) {
        SC_CUDA(cudaEventSynchronize(r->ev[parity ^ 1]));
        done = r->pinned[parity ^ 1] == 0;
      }
    }
  }
  SC_CUDA(cudaStreamSynchronize(st));
  std::vector<int32_t> status((size_t)r->S);
  SC_CUDA(cudaMemcpy(status.data(), s.status, r->S * 4, cudaMemcpyDeviceToHost));
  for (int64_t z = 0; z < r->S; z++)
    if (status[(size_t)z]) {
      set_error("rnnt decode: iteration cap hit (stream %lld)", (long long)z);
      return kErrState;
    }
  (void)rounds;
  return kOk;
}

int sc_rnnt_tokens(const sc_rnnt_decoder *r, int64_t stream_idx, int32_t *ids, int32_t *steps, int32_t cap,
                   int32_t *count) {
  if (!r || stream_idx < 0 || stream_idx >= r->S || cap < 0 || (cap > 0 && (!ids || !steps)) || !count) {
    set_error("rnnt_tokens: invalid argument");
    return kErrInvalid;
  }
  int32_t em = 0;
  SC_CUDA(cudaDeviceSynchronize());
  SC_CUDA(cudaMemcpy(&em, r->st.emitted + stream_idx, 4, cudaMemcpyDeviceToHost));
  *count = em;
  const int32_t k = std::min(std::min(em, cap), (int32_t)r->cap);
  if (k > 0) {
    SC_CUDA(cudaMemcpy(ids, r->st.ids + stream_idx * r->cap, (size_t)k * 4, cudaMemcpyDeviceToHost));
    SC_CUDA(cudaMemcpy(steps, r->st.steps + stream_idx * r->cap, (size_t)k * 4, cudaMemcpyDeviceToHost));
  }
  return kOk;
}

int sc_rnnt_emitted(const sc_rnnt_decoder *r, int32_t *counts) {
  if (!r || !counts) {
    set_error("rnnt_emitted: invalid argument");
    return kErrInvalid;
  }
  SC_CUDA(cudaDeviceSynchronize());
  SC_CUDA(cudaMemcpy(counts, r->st.emitted, (size_t)r->S * 4, cudaMemcpyDeviceToHost));
  return kOk;
}

int sc_rnnt_tokens_device(const sc_rnnt_decoder *r, const int32_t **ids, const int32_t **steps,
                          const int32_t **counts, int32_t *cap) {
  if (!r || !ids || !steps || !counts || !cap) {
    set_error("rnnt_tokens_device: invalid argument");
    return kErrInvalid;
  }
  *ids = r->st.ids;
  *steps = r->st.steps;
  *counts = r->st.emitted;
  *cap = r->cap;
  return kOk;
}

int sc_rnnt_state(const sc_rnnt_decoder *r, int64_t stream_idx, float *h, float *c, int32_t *last_token) {
  if (!r || stream_idx < 0 || stream_idx >= r->S || !h || !c || !last_token) {
    set_error("rnnt_state: invalid argument");
    return kErrInvalid;
  }
  const DecState &s = r->st;
  int32_t cur = 0;
  SC_CUDA(cudaDeviceSynchronize());
  SC_CUDA(cudaMemcpy(&cur, s.cur + stream_idx, 4, cudaMemcpyDeviceToHost));
  SC_CUDA(cudaMemcpy(last_token, s.last_tok + stream_idx, 4, cudaMemcpyDeviceToHost));
  const size_t lh = (size_t)s.L * s.H;
  const float *base = s.hc + ((stream_idx * 2 + cur) * 2) * lh;
  SC_CUDA(cudaMemcpy(h, base, lh * 4, cudaMemcpyDeviceToHost));
  SC_CUDA(cudaMemcpy(c, base + lh, lh * 4, cudaMemcpyDeviceToHost));
  return kOk;
}

int sc_rnnt_destroy(sc_rnnt_decoder *r) {
  if (!r) return kOk;
  cudaDeviceSynchronize();
  delete r;
  return kOk;
}

}  // extern "C"
