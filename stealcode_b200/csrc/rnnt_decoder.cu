// rnnt_decoder.cu -- the device greedy RNN-T decoder: the B200 counterpart of
// the reference's streaming decode loop (nemotron/live.rs:56-145,
// decode_frames) with its predictor LSTM (nemotron/decoder.rs:75-205) and
// joint network (decoder.rs:207-235), for n_streams streams at once.
//
// Every stream runs the reference's loop; the device runs the loops of all
// streams in lockstep rounds.  One round is one loop iteration of every
// stream that is still decoding, five kernels:
//   1. predictor step, one launch per LSTM layer, for the streams that
//      emitted in the previous round (the reference's `predictor_dirty`);
//   2. joint.pred over the new predictor output, for the same streams;
//   3. joint.out over relu(enc_proj[step] + pred) for every active stream;
//   4. per stream: greedy argmax, token append, the step / max_symbols
//      bookkeeping, and the stream lists of the next round.
// Every linear reads its input as int8 codes that the producer of the input
// quantised once (quantize_col per 32-block): the embedding rows at load,
// each LSTM layer's new h in that layer's epilogue (it is both the next
// layer's input and, after an emission, the layer's h input), relu(enc +
// pred) in joint.pred's epilogue or, for streams whose predictor output did
// not change, in the update.  The round's kernels are captured once into a
// CUDA graph (two rounds, one per list parity); the host replays it and
// stops once no stream is active, reading the count one replay behind so the
// GPU never idles on the check.
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

constexpr int kLsRows = 128;  // rows of a lane-split tile: 8 threads per row, one per SIMD lane
constexpr int kLsLanes = 8;
constexpr int kLsThreads = kLsRows * kLsLanes;
constexpr int kLsCols = 4;    // columns of a lane-split tile

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

// Per-call parameters, in device memory so that the captured round graph
// serves every call.
struct CallParams {
  int n, max_iters;
};

// Device state of all streams (StreamState, live.rs:24-50, plus the loop
// variables of decode_frames).  Codes are in lane order, one f32 scale per
// 32-block (dx arrays hold k / 32 scales per vector).
struct DecState {
  const int8_t *emb_q;  // [vocab][H] codes of the embedding rows
  const float *emb_dx;  // [vocab][H / 32]
  const int8_t *zq;     // [H] zero codes (the zero input before the first token)
  const float *zdx;     // [H / 32] ones (quantize_col's scale of a zero block)
  float *hc;            // [S][2 bufs][h, c][L][H]; buf cur[z] is (h, c), the other (nh, nc)
  int8_t *qh;           // [S][2 bufs][L][H] codes of each buffer's h
  float *qh_dx;         // [S][2 bufs][L][H / 32]
  int32_t *cur, *last_tok, *pred_valid;  // [S]
  float *pred;          // [S][J] joint.pred of the current predictor output
  float *enc;           // [S][max_frames][J] joint.enc of this call's frames
  float *logits;        // [S][V]
  int8_t *qo;           // [S][J] codes of relu(enc[step] + pred), joint.out's input
  float *qo_dx;         // [S][J / 32]
  int8_t *qf;           // [S * max_frames][d_enc] codes of this call's frames
  float *qf_dx;         // [S * max_frames][d_enc / 32]
  const float *frames;  // this call's frames (set per call; used outside the graph)
  int32_t *step, *nsym, *iter, *emitted, *status;  // [S]
  int32_t *ids, *steps;                            // [S][cap]
  int32_t *lists;       // [2 parities][dirty, active][S]
  int32_t *counts;      // [2 parities][dirty, active]
  const CallParams *call;
  int S, H, L, J, V, cap, blank, max_symbols, d_enc;
};

__device__ __forceinline__ float *hc_at(const DecState &s, int z, int buf, int which, int l) {
  return s.hc + ((((int64_t)z * 2 + buf) * 2 + which) * s.L + l) * s.H;
}
__device__ __forceinline__ int8_t *qh_at(const DecState &s, int z, int buf, int l) {
  return s.qh + (((int64_t)z * 2 + buf) * s.L + l) * s.H;
}
__device__ __forceinline__ float *qhdx_at(const DecState &s, int z, int buf, int l) {
  return s.qh_dx + (((int64_t)z * 2 + buf) * s.L + l) * (s.H / 32);
}
__device__ __forceinline__ int32_t *list_at(const DecState &s, int parity, int which) {
  return s.lists + (int64_t)(parity * 2 + which) * s.S;
}

// Lane-order position of element e within its 32-block.
__device__ __forceinline__ int lane_pos(int e) { return (e & 7) * 4 + (e >> 3); }

// quantize_col of one 32-block, one warp, lane e holding element e: codes
// (lane order) and the block's scale.
__device__ __forceinline__ void warp_store_block(float v, int8_t *codes, float *dx, int blk) {
  const int lane = threadIdx.x & 31;
  float sc;
  const int8_t q = warp_quantize_block(v, true, sc);
  codes[blk * 32 + lane_pos(lane)] = q;
  if (lane == 0) dx[blk] = sc;
}

// joint.out's input for stream z at its current step, all J/32 blocks, by
// one warp: relu(enc_proj[step] + pred) (live.rs:102-105).
__device__ void warp_store_out_codes(const DecState &s, int z) {
  const int lane = threadIdx.x & 31;
  const float *e = s.enc + ((int64_t)z * s.call->n + s.step[z]) * s.J;
  const float *p = s.pred + (int64_t)z * s.J;
  for (int b = 0; b < s.J / 32; b++) {
    const float v = __fadd_rn(e[b * 32 + lane], p[b * 32 + lane]);
    warp_store_block(v > 0.0f ? v : 0.0f, s.qo + (int64_t)z * s.J, s.qo_dx + (int64_t)z * (s.J / 32), b);
  }
}

// sigmoid and tanh as decoder.rs:431-433 and f32::tanh write them, with
// correctly rounded exp/tanh.
__device__ __forceinline__ float sigmoid_ref(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-x)));
}
__device__ __forceinline__ float tanh_rn(float x) { return (float)tanh((double)x); }

// ---- lane-split GEMV ------------------------------------------------------
// Thread (row, l) of a tile of 128 rows handles SIMD lane l of its row (the
// products of elements l, l+8, l+16, l+24 of every block: one dp4a) for
// kLsCols input vectors.  kSimd: the reference's 8-lane order, per block
// fma(dp4a, dw * dx, acc) and at the end the row's 8 lane sums added in lane
// order (reduce_sum); otherwise q8_gemm_scalar's order, the 8 lanes' exact
// integer parts summed per block and acc += (dw * dx) * dot.  The tile's
// weight rows stream through shared memory in double-buffered chunks of
// kChunk blocks (cp.async), its input codes are staged once, so the loop
// never waits on a dependent global load.  Op supplies the column list, the
// input codes (in up to two parts along K) and the epilogue.
constexpr int kChunk = 8;                 // K blocks per staged weight chunk
constexpr int kRing = 4;                  // chunks in flight (a ring of shared-memory buffers)
constexpr int kWRow = kChunk * 32 + 32;   // staged bytes per row (padded: conflict-free reads)

__device__ __forceinline__ void dec_cp16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void dec_cp4(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void dec_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void dec_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__host__ __device__ inline size_t lane_split_smem(int k, int nb) {
  return (size_t)kRing * kLsRows * kWRow + (size_t)kRing * kLsRows * kChunk * 4 + (size_t)kLsCols * k +
         (size_t)kLsCols * nb * 4 + (size_t)kLsCols * kLsRows * 4 + 2 * kLsCols * 2 * sizeof(void *);
}

template <class Op, bool kSimd>
__global__ void __launch_bounds__(kLsThreads, 1) lane_split_kernel(LaneMat w, DecState s, Op op) {
  extern __shared__ __align__(16) unsigned char smem[];
  int8_t *wsm = reinterpret_cast<int8_t *>(smem);                            // [kRing][128][kWRow]
  float *ssm = reinterpret_cast<float *>(smem + kRing * kLsRows * kWRow);    // [kRing][128][kChunk]
  int8_t *xs = reinterpret_cast<int8_t *>(ssm + kRing * kLsRows * kChunk);   // [kLsCols][k]
  float *xds = reinterpret_cast<float *>(xs + kLsCols * w.k);                // [kLsCols][nb]
  float(&vals)[kLsCols][kLsRows] = *reinterpret_cast<float(*)[kLsCols][kLsRows]>(xds + kLsCols * w.nb);
  const int8_t **srcx = reinterpret_cast<const int8_t **>(&vals[kLsCols][0]);  // [kLsCols][2]
  const float **srcd = reinterpret_cast<const float **>(srcx + 2 * kLsCols);
  const int t = threadIdx.x, rloc = t >> 3, l = t & 7;
  op.prologue(s);
  const int ncols = op.n_cols(s);
  const int row_tiles = w.rows_pad / kLsRows, col_tiles = (ncols + kLsCols - 1) / kLsCols;
  const int nbx = Op::kParts == 2 ? op.nbx(s) : w.nb;  // blocks of part 0
  const int nch = (w.nb + kChunk - 1) / kChunk;
  for (int tile = blockIdx.x; tile < row_tiles * col_tiles; tile += gridDim.x) {
    const int rt = tile % row_tiles, ct = tile / row_tiles;
    int id[kLsCols];
#pragma unroll
    for (int c = 0; c < kLsCols; c++) {
      const int j = ct * kLsCols + c;
      id[c] = j < ncols ? op.col_id(s, j) : -1;
    }
    __syncthreads();  // the previous tile's shared-memory reads are done
    if (t < kLsCols * Op::kParts && id[t / Op::kParts] >= 0)
      op.src(s, id[t / Op::kParts], t % Op::kParts, srcx[t / Op::kParts * 2 + t % Op::kParts],
             srcd[t / Op::kParts * 2 + t % Op::kParts]);
    __syncthreads();
    // group 0: the input codes and scales of the tile's columns, and chunk 0
    for (int i = t; i < kLsCols * (w.k / 16); i += kLsThreads) {
      const int c = i / (w.k / 16), off = (i % (w.k / 16)) * 16, b = off / 32;
      if (id[c] < 0) continue;
      const int part = b >= nbx;
      dec_cp16(xs + c * w.k + off, srcx[c * 2 + part] + off - (part ? nbx * 32 : 0));
    }
    for (int i = t; i < kLsCols * w.nb; i += kLsThreads) {
      const int c = i / w.nb, b = i % w.nb;
      if (id[c] < 0) continue;
      const int part = b >= nbx;
      dec_cp4(xds + c * w.nb + b, srcd[c * 2 + part] + b - (part ? nbx : 0));
    }
    // each iteration commits one group (empty past the last chunk), so
    // waiting for all but the kRing - 1 newest groups lands chunk ch
    auto stage = [&](int ch) {
      if (ch < nch) {
        const int buf = ch % kRing, b0 = ch * kChunk, nbk = w.nb - b0 < kChunk ? w.nb - b0 : kChunk;
        const int per_row = nbk * 2;
        for (int i = t; i < kLsRows * per_row; i += kLsThreads) {
          const int r = i / per_row, q = i % per_row;
          dec_cp16(wsm + (buf * kLsRows + r) * kWRow + q * 16,
                   w.qs + (int64_t)(rt * kLsRows + r) * w.k + b0 * 32 + q * 16);
        }
        for (int i = t; i < kLsRows * nbk; i += kLsThreads) {
          const int r = i / nbk, q = i % nbk;
          dec_cp4(ssm + (buf * kLsRows + r) * kChunk + q, w.sc + (int64_t)(rt * kLsRows + r) * w.nb + b0 + q);
        }
      }
      dec_cp_commit();
    };
#pragma unroll
    for (int ch = 0; ch < kRing - 1; ch++) stage(ch);
    float acc[kLsCols];
#pragma unroll
    for (int c = 0; c < kLsCols; c++) acc[c] = 0.0f;
    for (int ch = 0; ch < nch; ch++) {
      stage(ch + kRing - 1);
      dec_cp_wait<kRing - 1>();
      __syncthreads();
      const int buf = ch % kRing, b0 = ch * kChunk, nbk = w.nb - b0 < kChunk ? w.nb - b0 : kChunk;
      const int8_t *wr = wsm + (buf * kLsRows + rloc) * kWRow + 4 * l;
      const float *sr = ssm + (buf * kLsRows + rloc) * kChunk;
      for (int q = 0; q < nbk; q++) {
        const int b = b0 + q;
        const int wv = *reinterpret_cast<const int *>(wr + q * 32);
        const float dw = sr[q];
#pragma unroll
        for (int c = 0; c < kLsCols; c++) {
          if (id[c] < 0) continue;
          const int xw = *reinterpret_cast<const int *>(xs + c * w.k + b * 32 + 4 * l);
          const float scale = __fmul_rn(dw, xds[c * w.nb + b]);
          if (kSimd) {
            acc[c] = __fmaf_rn((float)__dp4a(wv, xw, 0), scale, acc[c]);
          } else {  // the block's exact dot: the 8 lanes' integer parts
            int d = __dp4a(wv, xw, 0);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            d += __shfl_xor_sync(0xffffffffu, d, 4);
            acc[c] = __fadd_rn(acc[c], __fmul_rn(scale, (float)d));
          }
        }
      }
      __syncthreads();  // the chunk's buffer may be restaged
    }
    dec_cp_wait<0>();  // no copy of this tile still in flight (the trailing groups are empty)
    if (kSimd) {
      // reduce_sum over the row's 8 lanes, in lane order (every lane of the
      // row computes the same sum from the same values)
      const int base = (threadIdx.x & 31) & ~7;
#pragma unroll
      for (int c = 0; c < kLsCols; c++) {
        float y = __shfl_sync(0xffffffffu, acc[c], base);
#pragma unroll
        for (int q = 1; q < kLsLanes; q++) y = __fadd_rn(y, __shfl_sync(0xffffffffu, acc[c], base + q));
        acc[c] = y;
      }
    }
    op.epilogue(s, w, id, rt, rloc, l, acc, vals);
  }
}

// LSTM layer l of the predictor step (decoder.rs:158-195) for the streams
// that emitted: input [x ; h_l], x the embedding of the last token (zeros
// before the first) or layer l-1's new h; rows in gate-interleaved order
// 4k + g (g = i, f, g, o), so a warp (4 rows) holds one cell's gates.  The
// epilogue adds the merged bias, runs the cell, stores nc/nh, and quantises
// the tile's 32 new h values (one 32-block) for the next layer and for the
// next step's h input.
struct LstmOp {
  static constexpr int kParts = 2;
  int l_, parity;  // layer, list parity
  __device__ void prologue(const DecState &) const {}
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 0)[j]; }
  __device__ int nbx(const DecState &s) const { return s.H / 32; }
  __device__ void src(const DecState &s, int z, int part, const int8_t *&x, const float *&dx) const {
    if (part) {
      x = qh_at(s, z, s.cur[z], l_);
      dx = qhdx_at(s, z, s.cur[z], l_);
    } else if (l_ > 0) {
      x = qh_at(s, z, s.cur[z] ^ 1, l_ - 1);
      dx = qhdx_at(s, z, s.cur[z] ^ 1, l_ - 1);
    } else {
      const int tok = s.last_tok[z];
      x = tok >= 0 ? s.emb_q + (int64_t)tok * s.H : s.zq;
      dx = tok >= 0 ? s.emb_dx + (int64_t)tok * (s.H / 32) : s.zdx;
    }
  }
  __device__ void epilogue(const DecState &s, const LaneMat &w, const int (&id)[kLsCols], int rt, int rloc, int l,
                           const float (&y)[kLsCols], float (&vals)[kLsCols][kLsRows]) const {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = rt * kLsRows + rloc, k = rt * 32 + warp;  // warp = cell of the tile
    const int gate = lane >> 3;                               // this thread's row = gate `gate` of the cell
    // gates[k] += bias[k] (decoder.rs:176-178); lane (gate, l < kLsCols)
    // applies its gate's activation for column l
    float a = 0.0f;
    {
      const float bias = w.bias[row];
      float g = 0.0f;
#pragma unroll
      for (int c = 0; c < kLsCols; c++)
        if (c == l) g = __fadd_rn(y[c], bias);
      if (l < kLsCols) a = gate == 2 ? tanh_rn(g) : sigmoid_ref(g);
    }
    const float ig = __shfl_sync(0xffffffffu, a, l & 7), fg = __shfl_sync(0xffffffffu, a, 8 + (l & 7));
    const float gt = __shfl_sync(0xffffffffu, a, 16 + (l & 7)), og = __shfl_sync(0xffffffffu, a, 24 + (l & 7));
    // the cell (decoder.rs:185-194), lane l < kLsCols of row group 0 for column l
    int z = -1;
#pragma unroll
    for (int c = 0; c < kLsCols; c++)
      if (c == l) z = id[c];
    if (gate == 0 && l < kLsCols && z >= 0) {
      const int nb = s.cur[z] ^ 1;
      const float cn = __fadd_rn(__fmul_rn(fg, hc_at(s, z, nb ^ 1, 1, l_)[k]), __fmul_rn(ig, gt));
      const float hn = __fmul_rn(og, tanh_rn(cn));
      hc_at(s, z, nb, 1, l_)[k] = cn;
      hc_at(s, z, nb, 0, l_)[k] = hn;
      vals[l][warp] = hn;
    }
    __syncthreads();
    if (warp < kLsCols && id[warp] >= 0) {
      const int zz = id[warp], nb = s.cur[zz] ^ 1;
      warp_store_block(vals[warp][lane], qh_at(s, zz, nb, l_), qhdx_at(s, zz, nb, l_), rt);
    }
    __syncthreads();
  }
};

// joint.pred over the last layer's new h (live.rs:100-101, Lin::matvec) for
// the streams whose predictor ran; the epilogue stores pred and quantises
// joint.out's input relu(enc_proj[step] + pred) for them.  Block 0 also
// clears the next round's list counts (their last readers, the previous
// round's kernels, have finished).
struct PredOp {
  static constexpr int kParts = 1;
  int parity;
  __device__ void prologue(const DecState &s) const {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      s.counts[(parity ^ 1) * 2] = 0;
      s.counts[(parity ^ 1) * 2 + 1] = 0;
    }
  }
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 0)[j]; }
  __device__ int nbx(const DecState &s) const { return 0; }
  __device__ void src(const DecState &s, int z, int, const int8_t *&x, const float *&dx) const {
    x = qh_at(s, z, s.cur[z] ^ 1, s.L - 1);
    dx = qhdx_at(s, z, s.cur[z] ^ 1, s.L - 1);
  }
  __device__ void epilogue(const DecState &s, const LaneMat &w, const int (&id)[kLsCols], int rt, int rloc, int l,
                           const float (&y)[kLsCols], float (&vals)[kLsCols][kLsRows]) const {
    const int row = rt * kLsRows + rloc;
#pragma unroll
    for (int c = 0; c < kLsCols; c++) {
      const int z = id[c];
      if (l == 0 && z >= 0) {
        float v = 0.0f;
        if (row < w.rows) {
          const float p = w.bias ? __fadd_rn(y[c], w.bias[row]) : y[c];
          s.pred[(int64_t)z * s.J + row] = p;
          v = __fadd_rn(s.enc[((int64_t)z * s.call->n + s.step[z]) * s.J + row], p);
          v = v > 0.0f ? v : 0.0f;  // (e + p).max(0.0): NaN -> 0
          if (row == 0) s.pred_valid[z] = 1;
        }
        vals[c][rloc] = v;
      }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < kLsCols * (kLsRows / 32)) {
      const int c = warp / (kLsRows / 32), blk = warp % (kLsRows / 32), gb = rt * (kLsRows / 32) + blk;
      const int z = id[c];
      if (z >= 0 && gb < s.J / 32)
        warp_store_block(vals[c][blk * 32 + lane], s.qo + (int64_t)z * s.J, s.qo_dx + (int64_t)z * (s.J / 32),
                         gb);
    }
    __syncthreads();
  }
};

// joint.out (live.rs:106, Lin::matvec) for every active stream: logits.
struct OutOp {
  static constexpr int kParts = 1;
  int parity;
  __device__ void prologue(const DecState &) const {}
  __device__ int n_cols(const DecState &s) const { return s.counts[parity * 2 + 1]; }
  __device__ int col_id(const DecState &s, int j) const { return list_at(s, parity, 1)[j]; }
  __device__ int nbx(const DecState &) const { return 0; }
  __device__ void src(const DecState &s, int z, int, const int8_t *&x, const float *&dx) const {
    x = s.qo + (int64_t)z * s.J;
    dx = s.qo_dx + (int64_t)z * (s.J / 32);
  }
  __device__ void epilogue(const DecState &s, const LaneMat &w, const int (&id)[kLsCols], int rt, int rloc, int l,
                           const float (&y)[kLsCols], float (&)[kLsCols][kLsRows]) const {
    const int row = rt * kLsRows + rloc;
    if (l || row >= w.rows) return;
#pragma unroll
    for (int c = 0; c < kLsCols; c++)
      if (id[c] >= 0) s.logits[(int64_t)id[c] * s.V + row] = w.bias ? __fadd_rn(y[c], w.bias[row]) : y[c];
  }
};

// joint.enc over the call's frames (live.rs:71-81, Lin::forward_t with n
// frames, bias added after): column z * n + t.
struct EncOp {
  static constexpr int kParts = 1;
  __device__ void prologue(const DecState &) const {}
  __device__ int n_cols(const DecState &s) const { return s.S * s.call->n; }
  __device__ int col_id(const DecState &, int j) const { return j; }
  __device__ int nbx(const DecState &) const { return 0; }
  __device__ void src(const DecState &s, int col, int, const int8_t *&x, const float *&dx) const {
    x = s.qf + (int64_t)col * s.d_enc;
    dx = s.qf_dx + (int64_t)col * (s.d_enc / 32);
  }
  __device__ void epilogue(const DecState &s, const LaneMat &w, const int (&id)[kLsCols], int rt, int rloc, int l,
                           const float (&y)[kLsCols], float (&)[kLsCols][kLsRows]) const {
    const int row = rt * kLsRows + rloc;
    if (l || row >= w.rows) return;
#pragma unroll
    for (int c = 0; c < kLsCols; c++)
      if (id[c] >= 0) s.enc[(int64_t)id[c] * s.J + row] = w.bias ? __fadd_rn(y[c], w.bias[row]) : y[c];
  }
};

// quantize_col of every frame of the call (one warp per frame and block).
__global__ void rnnt_quant_frames_kernel(DecState s, int64_t cols) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nbk = s.d_enc / 32;
  if (wid >= cols * nbk) return;
  const int64_t col = wid / nbk;
  const int b = (int)(wid % nbk);
  warp_store_block(s.frames[col * s.d_enc + b * 32 + (threadIdx.x & 31)], s.qf + col * s.d_enc,
                   s.qf_dx + col * nbk, b);
}

// Embedding rows -> codes, once at load (one warp per row and block).
__global__ void rnnt_quant_embed_kernel(const float *emb, int64_t rows, int H, int8_t *q, float *dx) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nbk = H / 32;
  if (wid >= rows * nbk) return;
  const int64_t r = wid / nbk;
  const int b = (int)(wid % nbk);
  warp_store_block(emb[r * H + b * 32 + (threadIdx.x & 31)], q + r * H, dx + r * nbk, b);
}

// Start of a decode_frames call: the loop variables of every stream, the
// first round's lists (every stream active; the predictor runs where its
// output is not already current) and joint.out's input for the streams
// whose predictor output is current.  One warp per stream; the list counts
// were cleared before.
__global__ void rnnt_init_kernel(DecState s) {
  const int z = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (z >= s.S) return;
  if (lane == 0) {
    s.step[z] = 0;
    s.nsym[z] = 0;
    s.iter[z] = 0;
    s.emitted[z] = 0;
    s.status[z] = 0;
    list_at(s, 0, 1)[atomicAdd(&s.counts[1], 1)] = z;
    if (!s.pred_valid[z]) list_at(s, 0, 0)[atomicAdd(&s.counts[0], 1)] = z;
  }
  __syncwarp();
  if (s.pred_valid[z]) warp_store_out_codes(s, z);
}

// One loop iteration's decision per active stream (live.rs:107-140): the
// first index of the largest logit (NaNs never win; a NaN logit 0 keeps
// index 0), then blank -> next frame, else emit, swap the LSTM state and
// count symbols against max_symbols.  A stream that stays active without
// emitting gets joint.out's input for its new step here.  One CTA per
// stream: the argmax over the whole CTA, the input codes one warp per block.
constexpr int kUpdThreads = 512;
__global__ void __launch_bounds__(kUpdThreads) rnnt_update_kernel(DecState s, int parity) {
  __shared__ float sv[kUpdThreads / 32];
  __shared__ int si[kUpdThreads / 32];
  __shared__ int keep_s;
  if ((int)blockIdx.x >= s.counts[parity * 2 + 1]) return;
  const int z = list_at(s, parity, 1)[blockIdx.x];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float *lg = s.logits + (int64_t)z * s.V;
  float bv = 0.0f;
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < s.V; i += kUpdThreads) {
    const float v = lg[i];
    if (v == v && (bi == INT_MAX || v > bv)) {
      bv = v;
      bi = i;
    }
  }
  // (value, index) order: larger value first, then the smaller index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int q = 1; q < kUpdThreads / 32; q++) {
      const float ov = sv[q];
      const int oi = si[q];
      if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
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
    const bool active = step < s.call->n && it < s.call->max_iters;
    if (!active && it >= s.call->max_iters) s.status[z] = 1;  // "rnnt decode: iteration cap hit"
    if (active) {
      const int np = parity ^ 1;
      list_at(s, np, 1)[atomicAdd(&s.counts[np * 2 + 1], 1)] = z;
      if (dirty) list_at(s, np, 0)[atomicAdd(&s.counts[np * 2], 1)] = z;
    }
    keep_s = active && !dirty;
  }
  __syncthreads();  // thread 0's stores of the loop variables are visible to the CTA
  if (!keep_s) return;
  const float *e = s.enc + ((int64_t)z * s.call->n + s.step[z]) * s.J;
  const float *p = s.pred + (int64_t)z * s.J;
  for (int b = warp; b < s.J / 32; b += kUpdThreads / 32) {
    const float v = __fadd_rn(e[b * 32 + lane], p[b * 32 + lane]);
    warp_store_block(v > 0.0f ? v : 0.0f, s.qo + (int64_t)z * s.J, s.qo_dx + (int64_t)z * (s.J / 32), b);
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
  CallParams *call = nullptr;     // device
  int32_t *pinned = nullptr;      // [2] active counts read back; [2..3] call parameters staging
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaGraphExec_t rounds = nullptr;  // two rounds (list parities 0, 1)
  int round_launches = 0;
  int64_t last_n = 0, last_rounds = 0;
  std::vector<void *> allocs;
  ~sc_rnnt_decoder() {
    if (rounds) cudaGraphExecDestroy(rounds);
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
    if (dev_malloc(&p, bytes < 16 ? 16 : bytes) != cudaSuccess) {
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
    const int64_t rows_pad = (rows + kLsRows - 1) / kLsRows * kLsRows;
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

template <class Op, bool kSimd>
int launch_lane_split_t(const sc_rnnt_decoder *r, const LaneMat &w, Op op, int64_t max_cols, cudaStream_t st) {
  const int64_t tiles = (w.rows_pad / kLsRows) * ceil_div(max_cols, kLsCols);
  // one wave at most: CTAs past the live columns' tiles exit at once, and
  // a second wave of them would only add scheduling time
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)r->sm_count));
  const size_t smem = lane_split_smem(w.k, w.nb);
  lane_split_kernel<Op, kSimd><<<grid, kLsThreads, smem, st>>>(w, r->st, op);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

template <class Op>
int launch_lane_split(const sc_rnnt_decoder *r, const LaneMat &w, Op op, int64_t max_cols, bool simd,
                      cudaStream_t st) {
  return simd ? launch_lane_split_t<Op, true>(r, w, op, max_cols, st)
              : launch_lane_split_t<Op, false>(r, w, op, max_cols, st);
}

// Shared-memory limit of every lane-split instantiation, raised before the
// round graph is captured.  The limits only grow, so a decoder built later
// with smaller matrices never lowers them under an earlier decoder.
template <class Op, bool SIMD>
static int raise_lane_split(size_t smem) {
  static std::atomic<size_t> smem_limit[64];
  return raise_smem_limit((const void *)lane_split_kernel<Op, SIMD>, smem, smem_limit);
}

int configure_lane_split(size_t smem) {
  int rc = raise_lane_split<LstmOp, true>(smem);
  if (!rc) rc = raise_lane_split<LstmOp, false>(smem);
  if (!rc) rc = raise_lane_split<PredOp, true>(smem);
  if (!rc) rc = raise_lane_split<PredOp, false>(smem);
  if (!rc) rc = raise_lane_split<OutOp, true>(smem);
  if (!rc) rc = raise_lane_split<OutOp, false>(smem);
  if (!rc) rc = raise_lane_split<EncOp, true>(smem);
  if (!rc) rc = raise_lane_split<EncOp, false>(smem);
  return rc;
}

// One round of the decode loop for list parity `parity` (its launches are
// captured into the round graph).
int launch_round(const sc_rnnt_decoder *r, int parity, cudaStream_t st) {
  for (int l = 0; l < (int)r->lstm.size(); l++) {
    int rc = launch_lane_split(r, r->lstm[(size_t)l], LstmOp{l, parity}, r->S, true, st);
    if (rc) return rc;
  }
  int rc = launch_lane_split(r, r->jpred, PredOp{parity}, r->S, r->jpred.simd, st);
  if (rc) return rc;
  rc = launch_lane_split(r, r->jout, OutOp{parity}, r->S, r->jout.simd, st);
  if (rc) return rc;
  rnnt_update_kernel<<<(unsigned)r->S, kUpdThreads, 0, st>>>(r->st, parity);  // one CTA per stream
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

// Captures two rounds (parities 0 and 1) into a graph on a private stream.
int build_round_graph(sc_rnnt_decoder *r) {
  cudaStream_t cs;
  SC_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  cudaGraph_t g = nullptr;
  int rc = kOk;
  if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    cudaStreamDestroy(cs);
    set_error("rnnt_create: stream capture failed");
    return kErrCuda;
  }
  rc = launch_round(r, 0, cs);
  if (!rc) rc = launch_round(r, 1, cs);
  const cudaError_t e = cudaStreamEndCapture(cs, &g);
  if (!rc && e != cudaSuccess) rc = cuda_fail(e, "cudaStreamEndCapture");
  if (!rc && cudaGraphInstantiate(&r->rounds, g, 0) != cudaSuccess) {
    cudaGetLastError();
    set_error("rnnt_create: graph instantiation failed");
    rc = kErrCuda;
  }
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(cs);
  r->round_launches = 2 * ((int)r->lstm.size() + 3);
  return rc;
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
  float *emb_dev = nullptr;
  if (ld.err.empty()) {
    emb_dev = ld.upload(std::vector<float>(embed, embed + V * H));
    s.emb_q = (int8_t *)ld.dev((size_t)(V * H));
    s.emb_dx = (float *)ld.dev((size_t)(V * H / 32 * 4));
    s.zq = (int8_t *)ld.dev((size_t)H);
    s.zdx = ld.upload(std::vector<float>((size_t)(H / 32), 1.0f));
    s.hc = (float *)ld.dev((size_t)(S * 4 * L * H * 4));
    s.qh = (int8_t *)ld.dev((size_t)(S * 2 * L * H));
    s.qh_dx = (float *)ld.dev((size_t)(S * 2 * L * H / 32 * 4));
    s.cur = (int32_t *)ld.dev((size_t)S * 4);
    s.last_tok = (int32_t *)ld.dev((size_t)S * 4);
    s.pred_valid = (int32_t *)ld.dev((size_t)S * 4);
    s.pred = (float *)ld.dev((size_t)(S * J * 4));
    s.enc = (float *)ld.dev((size_t)(S * c.max_frames * J * 4));
    s.logits = (float *)ld.dev((size_t)(S * V * 4));
    s.qo = (int8_t *)ld.dev((size_t)(S * J));
    s.qo_dx = (float *)ld.dev((size_t)(S * J / 32 * 4));
    s.qf = (int8_t *)ld.dev((size_t)(S * c.max_frames * c.d_enc));
    s.qf_dx = (float *)ld.dev((size_t)(S * c.max_frames * c.d_enc / 32 * 4));
    s.step = (int32_t *)ld.dev((size_t)S * 4);
    s.nsym = (int32_t *)ld.dev((size_t)S * 4);
    s.iter = (int32_t *)ld.dev((size_t)S * 4);
    s.emitted = (int32_t *)ld.dev((size_t)S * 4);
    s.status = (int32_t *)ld.dev((size_t)S * 4);
    s.ids = (int32_t *)ld.dev((size_t)(S * r->cap * 4));
    s.steps = (int32_t *)ld.dev((size_t)(S * r->cap * 4));
    s.lists = (int32_t *)ld.dev((size_t)(S * 4 * 4));
    s.counts = (int32_t *)ld.dev(16);
    r->call = (CallParams *)ld.dev(sizeof(CallParams));
    s.call = r->call;
  }
  if (ld.err.empty() && (cudaHostAlloc(&r->pinned, 16, cudaHostAllocDefault) != cudaSuccess ||
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
  // the embedding rows' codes (the predictor's layer-0 input), once
  SC_CUDA(cudaMemset((void *)s.zq, 0, (size_t)H));
  rnnt_quant_embed_kernel<<<(unsigned)ceil_div(V * (H / 32) * 32, 256), 256>>>(emb_dev, V, (int)H,
                                                                                 (int8_t *)s.emb_q,
                                                                                 (float *)s.emb_dx);
  note_launch();
  const cudaError_t ce = cudaDeviceSynchronize();
  rc = ce == cudaSuccess ? kOk : cuda_fail(ce, "rnnt_create: embedding codes");
  if (rc == kOk) {
    size_t smem = 0;
    for (const LaneMat *m : {&r->jenc, &r->jpred, &r->jout}) smem = std::max(smem, lane_split_smem(m->k, m->nb));
    for (const LaneMat &m : r->lstm) smem = std::max(smem, lane_split_smem(m.k, m.nb));
    rc = configure_lane_split(smem);
  }
  if (rc == kOk) rc = build_round_graph(r);
  if (rc == kOk) rc = sc_rnnt_reset(r, -1);
  if (rc) {
    delete r;
    return rc;
  }
  *out = r;
  return kOk;
}

int sc_rnnt_reset(sc_rnnt_decoder *r, int64_t stream_idx) {
  if (!r || stream_idx < -1 || stream_idx >= r->S) {
    set_error("rnnt_reset: invalid argument");
    return kErrInvalid;
  }
  const DecState &s = r->st;
  const int64_t lo = stream_idx < 0 ? 0 : stream_idx, cnt = stream_idx < 0 ? r->S : 1;
  const int64_t lh = (int64_t)s.L * s.H;
  SC_CUDA(cudaDeviceSynchronize());
  SC_CUDA(cudaMemset(s.hc + lo * 4 * lh, 0, (size_t)(cnt * 4 * lh * 4)));
  // h = 0 in both buffers: zero codes with quantize_col's scale 1 for a zero block
  SC_CUDA(cudaMemset(s.qh + lo * 2 * lh, 0, (size_t)(cnt * 2 * lh)));
  std::vector<float> ones((size_t)(cnt * 2 * lh / 32), 1.0f);
  SC_CUDA(cudaMemcpy(s.qh_dx + lo * 2 * lh / 32, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice));
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
  s.frames = frames;
  const int max_iters = (int)(16 * n + 64);
  r->pinned[2] = (int32_t)n;
  r->pinned[3] = max_iters;
  SC_CUDA(cudaMemcpyAsync(r->call, r->pinned + 2, sizeof(CallParams), cudaMemcpyHostToDevice, st));
  // joint.enc over every stream's frames (the SIMD order for n <= 16), then
  // the first round's lists and inputs
  const int64_t cols = r->S * n;
  rnnt_quant_frames_kernel<<<(unsigned)ceil_div(cols * (s.d_enc / 32) * 32, 256), 256, 0, st>>>(s, cols);
  note_launch();
  SC_CUDA(cudaGetLastError());
  TRY(launch_lane_split(r, r->jenc, EncOp{}, cols, r->jenc.simd && n <= 16, st));
  SC_CUDA(cudaMemsetAsync(s.counts, 0, 16, st));
  rnnt_init_kernel<<<(unsigned)ceil_div(r->S, 8), 256, 0, st>>>(s);
  note_launch();
  SC_CUDA(cudaGetLastError());
  // two rounds per replay; every stream needs n iterations, so from then on
  // the host reads the active count left by the replay before (the GPU is
  // busy with the current one meanwhile)
  const int64_t pairs = (max_iters + 1) / 2;
  r->last_rounds = 0;
  for (int64_t pr = 0; pr < pairs; pr++) {
    SC_CUDA(cudaGraphLaunch(r->rounds, st));
    r->last_rounds += 2;
    for (int i = 0; i < r->round_launches; i++) note_launch();
    const int slot = (int)(pr & 1);
    if (2 * (pr + 1) >= n) {
      SC_CUDA(cudaMemcpyAsync(r->pinned + slot, s.counts + 1, 4, cudaMemcpyDeviceToHost, st));
      SC_CUDA(cudaEventRecord(r->ev[slot], st));
      if (2 * pr >= n) {
        SC_CUDA(cudaEventSynchronize(r->ev[slot ^ 1]));
        if (r->pinned[slot ^ 1] == 0) break;
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

int64_t sc_rnnt_last_rounds(const sc_rnnt_decoder *r) { return r ? r->last_rounds : 0; }

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
