// encoder_kernels.cu -- the non-GEMM kernels of the device streaming
// encoder step (everything in block_new and pre_encode_forward except the
// Q8_0 linears and the attention):
//   ln_rows_kernel            LayerNorm per frame row   (simd_kernel.rs:734-813)
//   ln_quant_kernel           LayerNorm (or two in a row) + the next GEMM's
//                             activation codes
//   glu_ring_kernel           GLU into the per-stream conv ring
//                                                       (simd_kernel.rs:868-910)
//   dwconv_ln_silu_quant_kernel  causal depthwise conv over the ring +
//                             LayerNorm + SiLU + codes  (streaming.rs:608-638,
//                             simd_kernel.rs:1160-1235, 817-839)
//   mel_window_kernel, mel_hist_kernel  pre-encode mel window and the mel
//                             history kept for the next step
//                                                       (streaming.rs:182-207)
//   conv02_fused_kernel       conv0 + ReLU and the depthwise conv2, fused
//   conv2d_3x3s2_kernel       the depthwise conv5       (nemotron/weights.rs:418-523)
//   pw_conv_relu_kernel, pw_conv_tail_kernel  pointwise convs 3/6 as an f32
//                             GEMM + bias + ReLU in the reference GEMM's order
//                                                       (nemotron/weights.rs:345-417)
//   flatten_kernel            [t, f, C] -> [t, C*f] of the needed frames
//                                                       (nemotron/encoder.rs:460-470)
//   prompt_cat_quant_kernel, prompt_select_kernel  the prompt MLP's input
//                             and output                (streaming.rs:320-342)
//   out_ring_kernel           output frames into the per-stream output ring
// Frame rows are time-major [stream][frame][d].
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

constexpr int kRowThreads = 256;
constexpr int kMaxRowVals = 16;  // d up to 4096

constexpr int kLnLanes = 16;  // the reference's SIMD width for ln_forward

// Shared scratch of the row kernels: the row padded to 17 floats per
// 16-element chunk (conflict-free chunk walks), the chunk sums and the
// broadcast scalar.
struct RowScratch {
  float row[kMaxRowVals * kRowThreads / kLnLanes * (kLnLanes + 1)];
  float part[kMaxRowVals * kRowThreads / kLnLanes];
  float bcast;
};

__device__ __forceinline__ int row_slot(int i) { return i + i / kLnLanes; }

// Sum of the row's 16-element chunk sums in the reference's order
// (simd_kernel.rs:734-776): each chunk summed lane 0..15 in sequence, then
// the chunk sums in sequence.  sq = true sums (x - mean)^2 with the square
// rounded before the add, as the reference's (diff * diff).reduce_sum().
template <bool kSq>
__device__ __forceinline__ float ordered_row_sum(RowScratch &sh, int d, float mean) {
  const int nchunks = d / kLnLanes;
  for (int ci = threadIdx.x; ci < nchunks; ci += kRowThreads) {
    const float *r = sh.row + ci * (kLnLanes + 1);
    float cs;
    if (kSq) {
      float df = __fsub_rn(r[0], mean);
      cs = __fmul_rn(df, df);
#pragma unroll
      for (int q = 1; q < kLnLanes; q++) {
        df = __fsub_rn(r[q], mean);
        cs = __fadd_rn(cs, __fmul_rn(df, df));
      }
    } else {
      cs = r[0];
#pragma unroll
      for (int q = 1; q < kLnLanes; q++) cs = __fadd_rn(cs, r[q]);
    }
    sh.part[ci] = cs;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int ci = 0; ci < nchunks; ci++) t = __fadd_rn(t, sh.part[ci]);
    sh.bcast = t;
  }
  __syncthreads();
  const float t = sh.bcast;
  __syncthreads();  // bcast and part are reused by the next call
  return t;
}

// LayerNorm of the row values held by this thread (element i = tid + k*256),
// rounded as the reference's ln_forward (simd_kernel.rs:734-805):
// mean = sum/d, var = sum (x-mean)^2 / d, inv = 1 / sqrt(var/d + eps),
// out = fma(x - mean, w * inv, b).
__device__ __forceinline__ void ln_vals(float (&v)[kMaxRowVals], int d, const float *w, const float *b, float eps,
                                        RowScratch &sh) {
  const int nv = d / kRowThreads;
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) sh.row[row_slot(threadIdx.x + k * kRowThreads)] = v[k];
  __syncthreads();
  const float mean = __fdiv_rn(ordered_row_sum<false>(sh, d, 0.0f), (float)d);
  const float var = ordered_row_sum<true>(sh, d, mean);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, (float)d), eps)));
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) {
      const int i = threadIdx.x + k * kRowThreads;
      v[k] = __fmaf_rn(__fsub_rn(v[k], mean), __fmul_rn(w[i], inv), b[i]);
    }
}

__global__ void __launch_bounds__(kRowThreads) ln_rows_kernel(const float *__restrict__ x, int64_t ldx,
                                                              const float *__restrict__ w,
                                                              const float *__restrict__ b, float eps,
                                                              float *__restrict__ out, int64_t ldo, int d) {
  __shared__ RowScratch sh;
  const int64_t row = blockIdx.x;
  const int nv = d / kRowThreads;
  float v[kMaxRowVals];
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) v[k] = x[row * ldx + threadIdx.x + k * kRowThreads];
  ln_vals(v, d, w, b, eps, sh);
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) out[row * ldo + threadIdx.x + k * kRowThreads] = v[k];
}

// ---- row kernels with fused quantisation (one row per L lanes) -----------
// A row of d = 32 * L * ... floats is held by L lanes of a warp, lane l of
// the group owning the E = d / L consecutive elements [l*E, l*E + E), E a
// multiple of 32: its E/16 LayerNorm chunks and E/32 quantisation blocks are
// lane-local, and the reference's ordered chunk sums become a walk over the
// group's lanes in order (every lane computes the same total).
template <int E, int L>
__device__ __forceinline__ float ordered_group_sum(const float (&cs)[E / 16], int lead) {
  float t = 0.0f;
#pragma unroll
  for (int l = 0; l < L; l++)
#pragma unroll
    for (int c = 0; c < E / 16; c++) t = __fadd_rn(t, __shfl_sync(0xffffffffu, cs[c], lead + l));
  return t;
}

// LayerNorm of v (the lane's E elements) in ln_forward's rounding
// (simd_kernel.rs:734-805).
template <int E, int L>
__device__ __forceinline__ void ln_lane(float (&v)[E], int lead, const float *w, const float *b, float eps,
                                        int i0) {
  constexpr int d = E * L;
  // up to 32 features a lane: the weight and bias loaded before the two
  // ordered sums so that their latency overlaps them (more would spill)
  constexpr bool kEarly = E <= 32;
  float4 w4[kEarly ? E / 4 : 1], b4[kEarly ? E / 4 : 1];
  if constexpr (kEarly) {
#pragma unroll
    for (int e4 = 0; e4 < E / 4; e4++) {
      w4[e4] = __ldg(reinterpret_cast<const float4 *>(w + i0 + 4 * e4));
      b4[e4] = __ldg(reinterpret_cast<const float4 *>(b + i0 + 4 * e4));
    }
  }
  float cs[E / 16];
#pragma unroll
  for (int c = 0; c < E / 16; c++) {
    cs[c] = v[16 * c];
#pragma unroll
    for (int q = 1; q < 16; q++) cs[c] = __fadd_rn(cs[c], v[16 * c + q]);
  }
  const float mean = __fdiv_rn(ordered_group_sum<E, L>(cs, lead), (float)d);
#pragma unroll
  for (int c = 0; c < E / 16; c++) {
    float df = __fsub_rn(v[16 * c], mean);
    cs[c] = __fmul_rn(df, df);
#pragma unroll
    for (int q = 1; q < 16; q++) {
      df = __fsub_rn(v[16 * c + q], mean);
      cs[c] = __fadd_rn(cs[c], __fmul_rn(df, df));
    }
  }
  const float var = ordered_group_sum<E, L>(cs, lead);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, (float)d), eps)));
#pragma unroll
  for (int e4 = 0; e4 < E / 4; e4++) {
    const float4 wq = kEarly ? w4[kEarly ? e4 : 0] : *reinterpret_cast<const float4 *>(w + i0 + 4 * e4);
    const float4 bq = kEarly ? b4[kEarly ? e4 : 0] : *reinterpret_cast<const float4 *>(b + i0 + 4 * e4);
    const float wv[4] = {wq.x, wq.y, wq.z, wq.w}, bv[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      float &x = v[4 * e4 + q];
      x = __fmaf_rn(__fsub_rn(x, mean), __fmul_rn(wv[q], inv), bv[q]);
    }
  }
}

// quantize_col of the lane's E elements (features i0 .. i0 + E - 1 of frame
// f), E/32 whole blocks, into the tiled codes of qo.
template <int E>
__device__ __forceinline__ void quant_lane(const float (&v)[E], const QOut &qo, int64_t f, int i0) {
#pragma unroll
  for (int blk = 0; blk < E / 32; blk++) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; e++) amax = fmaxf(amax, fabsf(v[32 * blk + e]));
    const float sc = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    const int i = i0 + 32 * blk;
    __half *dst = qo.xq + qout_code_index(qo, f, i);
#pragma unroll
    for (int c8 = 0; c8 < 4; c8++) {  // four 8-feature chunks, 16 bytes each
      __half h8[8];
#pragma unroll
      for (int q = 0; q < 8; q++)
        h8[q] = code_half(amax != 0.0f ? rust_round_i8(__fmul_rn(v[32 * blk + 8 * c8 + q], inv)) : (int8_t)0);
      uint4 u;
      memcpy(&u, h8, 16);
      *reinterpret_cast<uint4 *>(dst + (int64_t)c8 * qo.ft * 8) = u;
    }
    qo.dx[qout_dx_index(qo, f, i / 32)] = sc;
  }
}

// LayerNorm of each row, written as codes for the next GEMM (and as f32
// when out != nullptr).  rows_per_warp = 32 / L.
template <int E, int L>
__global__ void __launch_bounds__(128) ln_quant_kernel(const float *__restrict__ x, int64_t ldx,
                                                       const float *__restrict__ w, const float *__restrict__ b,
                                                       float eps, int64_t rows, QOut qo, float *__restrict__ out,
                                                       int64_t ldo, const float *__restrict__ w0,
                                                       const float *__restrict__ b0, float *__restrict__ out0,
                                                       int64_t ld0) {
  const int lane = threadIdx.x & 31, sub = lane / L, lead = sub * L, l = lane % L;
  const int64_t row = ((int64_t)blockIdx.x * 4 + (threadIdx.x >> 5)) * (32 / L) + sub;
  const bool live = row < rows;
  const int i0 = l * E;
  float v[E];
  if constexpr (E == 32 && L == 32) {
    // d = 1024, one row per warp: coalesced 512-byte loads, then through
    // shared memory (element i at i + 4 * (i / 32), conflict-free both
    // ways) to the lane-contiguous split
    __shared__ __align__(16) float s_row[4][1024 + 128];
    float *sr = s_row[threadIdx.x >> 5];
    const float *xr = x + (live ? row : 0) * ldx + 4 * lane;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = 4 * lane + 128 * k;
      *reinterpret_cast<float4 *>(sr + i + 4 * (i >> 5)) = *reinterpret_cast<const float4 *>(xr + 128 * k);
    }
    __syncwarp();
#pragma unroll
    for (int e4 = 0; e4 < 8; e4++) {
      const float4 t = *reinterpret_cast<const float4 *>(sr + 36 * lane + 4 * e4);
      v[4 * e4] = t.x, v[4 * e4 + 1] = t.y, v[4 * e4 + 2] = t.z, v[4 * e4 + 3] = t.w;
    }
  } else {
    const float *xr = x + (live ? row : 0) * ldx + i0;
#pragma unroll
    for (int e4 = 0; e4 < E / 4; e4++) {
      const float4 t = *reinterpret_cast<const float4 *>(xr + 4 * e4);
      v[4 * e4] = t.x, v[4 * e4 + 1] = t.y, v[4 * e4 + 2] = t.z, v[4 * e4 + 3] = t.w;
    }
  }
  if (w0) {  // a first LayerNorm (the previous block's output LN), written to out0
    ln_lane<E, L>(v, lead, w0, b0, eps, i0);
    if (live)
#pragma unroll
      for (int e4 = 0; e4 < E / 4; e4++)
        *reinterpret_cast<float4 *>(out0 + row * ld0 + i0 + 4 * e4) =
            make_float4(v[4 * e4], v[4 * e4 + 1], v[4 * e4 + 2], v[4 * e4 + 3]);
  }
  ln_lane<E, L>(v, lead, w, b, eps, i0);  // all lanes take part in the shuffles
  if (!live) return;
  if (out)
#pragma unroll
    for (int e4 = 0; e4 < E / 4; e4++)
      *reinterpret_cast<float4 *>(out + row * ldo + i0 + 4 * e4) =
          make_float4(v[4 * e4], v[4 * e4 + 1], v[4 * e4 + 2], v[4 * e4 + 3]);
  quant_lane<E>(v, qo, row, i0);
}

// Causal depthwise conv over the GLU ring (taps in order, fused multiply-
// adds as the reference's S-lane loop), the conv module's LayerNorm and
// SiLU, then codes for pw2.  wt is the depthwise weight transposed to
// [kh][d].  rows = n_streams * c, frame of row r: s + r % c.  Taps before
// frame 0 are skipped; a tap's ring slot is (frame + shift) % cap (shift:
// the step graph's device frame shift, nullptr for none).
template <int E, int L, int KH>
__global__ void __launch_bounds__(128)
    dwconv_ln_silu_quant_kernel(const float *__restrict__ ring, int cap, int c, int kh_rt, int64_t s,
                                const int64_t *shift, const float *__restrict__ wt, const float *__restrict__ lnw,
                                const float *__restrict__ lnb, float eps, int64_t rows, QOut qo,
                                float *__restrict__ out) {
  constexpr int d = E * L;
  const int kh = KH > 0 ? KH : kh_rt;
  const int lane = threadIdx.x & 31, sub = lane / L, lead = sub * L, l = lane % L;
  const int64_t row = ((int64_t)blockIdx.x * 4 + (threadIdx.x >> 5)) * (32 / L) + sub;
  const bool live = row < rows;
  const int64_t rr = live ? row : 0;
  const int64_t z = rr / c, fr = s + rr % c;
  const int64_t sh = shift ? *shift : 0;
  const int i0 = l * E;
  float v[E];
  if constexpr (E == 32 && L == 32) {
    // d = 1024, one row per warp: the taps are read coalesced (lane l owns
    // elements 4l + 128k, one 512-byte run per warp load), then the row
    // passes through shared memory to the LayerNorm's split (lane l owns
    // [32l, 32l + 32)).  Element i sits at i + 4 * (i / 32) there, so both
    // the scattered float4 writes and the lane-contiguous reads are free of
    // bank conflicts.  Per element the same ordered chain of fused
    // multiply-adds over the taps.
    __shared__ __align__(16) float s_row[4][1024 + 128];
    float *sr = s_row[threadIdx.x >> 5];
    float4 a4[8];
#pragma unroll
    for (int k = 0; k < 8; k++) a4[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int t = 0; t < (KH > 0 ? KH : 64); t++) {
      if (KH == 0 && t >= kh) break;
      const int64_t ti = fr - (kh - 1) + t;
      if (ti < 0) continue;
      const float *rw = ring + (z * cap + (ti + sh) % cap) * (int64_t)d + 4 * lane;
      const float *ww = wt + (int64_t)t * d + 4 * lane;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float4 a = *reinterpret_cast<const float4 *>(rw + 128 * k);
        const float4 w = *reinterpret_cast<const float4 *>(ww + 128 * k);
        a4[k].x = __fmaf_rn(a.x, w.x, a4[k].x);
        a4[k].y = __fmaf_rn(a.y, w.y, a4[k].y);
        a4[k].z = __fmaf_rn(a.z, w.z, a4[k].z);
        a4[k].w = __fmaf_rn(a.w, w.w, a4[k].w);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = 4 * lane + 128 * k;
      *reinterpret_cast<float4 *>(sr + i + 4 * (i >> 5)) = a4[k];
    }
    __syncwarp();
#pragma unroll
    for (int e4 = 0; e4 < 8; e4++) {
      const float4 t4 = *reinterpret_cast<const float4 *>(sr + 36 * lane + 4 * e4);
      v[4 * e4] = t4.x, v[4 * e4 + 1] = t4.y, v[4 * e4 + 2] = t4.z, v[4 * e4 + 3] = t4.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; e++) v[e] = 0.0f;
#pragma unroll
    for (int t = 0; t < (KH > 0 ? KH : 64); t++) {
      if (KH == 0 && t >= kh) break;
      const int64_t ti = fr - (kh - 1) + t;
      if (ti < 0) continue;
      const float *rw = ring + (z * cap + (ti + sh) % cap) * (int64_t)d + i0;
      const float *ww = wt + (int64_t)t * d + i0;
#pragma unroll
      for (int e4 = 0; e4 < E / 4; e4++) {
        const float4 a = *reinterpret_cast<const float4 *>(rw + 4 * e4);
        const float4 k = *reinterpret_cast<const float4 *>(ww + 4 * e4);
        v[4 * e4] = __fmaf_rn(a.x, k.x, v[4 * e4]);
        v[4 * e4 + 1] = __fmaf_rn(a.y, k.y, v[4 * e4 + 1]);
        v[4 * e4 + 2] = __fmaf_rn(a.z, k.z, v[4 * e4 + 2]);
        v[4 * e4 + 3] = __fmaf_rn(a.w, k.w, v[4 * e4 + 3]);
      }
    }
  }
  ln_lane<E, L>(v, lead, lnw, lnb, eps, i0);
  if (!live) return;
#pragma unroll
  for (int e = 0; e < E; e++) v[e] = silu_ref(v[e]);
  if (out)
#pragma unroll
    for (int e4 = 0; e4 < E / 4; e4++)
      *reinterpret_cast<float4 *>(out + row * d + i0 + 4 * e4) =
          make_float4(v[4 * e4], v[4 * e4 + 1], v[4 * e4 + 2], v[4 * e4 + 3]);
  quant_lane<E>(v, qo, row, i0);
}

// GLU of the new frames (h2 = [M][2d] time-major, gate first, value second)
// stored into ring slot (s + shift + j) % cap of stream z (shift: the step
// graph's device frame shift, nullptr for none).
__global__ void glu_ring_kernel(const float *__restrict__ h2, int c, int d, float *__restrict__ ring, int cap,
                                int64_t s, const int64_t *shift) {
  const int64_t row = blockIdx.x;  // z * c + j
  const int64_t z = row / c, j = row % c;
  if (shift) s += *shift;
  float *dst = ring + (z * cap + (s + j) % cap) * (int64_t)d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float gate = h2[row * 2 * d + i], val = h2[row * 2 * d + d + i];
    dst[i] = __fmul_rn(gate, __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-val))));
  }
}

// Pre-encode window of stream z: `hist` held frames of history (the last
// mel frames before this batch) then the new frames; rows past both are the
// zero padding of a short final batch.
__global__ void mel_window_kernel(const float *__restrict__ hist, int hist_cap, int hist_frames,
                                  const float *__restrict__ mel_new, int n_new, int n_mels, int t_mel,
                                  float *__restrict__ win) {
  const int64_t z = blockIdx.y;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)t_mel * n_mels) return;
  const int t = (int)(i / n_mels), f = (int)(i % n_mels);
  float v = 0.0f;
  if (t < hist_frames)
    v = hist[(z * hist_cap + (hist_cap - hist_frames + t)) * n_mels + f];
  else if (t - hist_frames < n_new)
    v = mel_new[(z * n_new + (t - hist_frames)) * n_mels + f];
  win[(z * t_mel + t) * n_mels + f] = v;
}

// History update: keep the last hist_cap frames of (history ++ new frames).
__global__ void mel_hist_kernel(const float *__restrict__ old_hist, int hist_cap, int hist_frames,
                                const float *__restrict__ mel_new, int n_new, int n_mels,
                                float *__restrict__ new_hist) {
  const int64_t z = blockIdx.y;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)hist_cap * n_mels) return;
  const int slot = (int)(i / n_mels), f = (int)(i % n_mels);
  const int total = hist_frames + n_new;
  const int src = total - hist_cap + slot;  // index into (history ++ new)
  float v = 0.0f;
  if (src >= 0) {
    if (src < hist_frames)
      v = old_hist[(z * hist_cap + (hist_cap - hist_frames + src)) * n_mels + f];
    else
      v = mel_new[(z * n_new + (src - hist_frames)) * n_mels + f];
  }
  new_hist[(z * hist_cap + slot) * n_mels + f] = v;
}

// 3x3 stride-2 conv with causal pads (2, 1) on both axes, groups = c_in
// (depthwise, c_in == c_out) or c_in == 1 (conv0): acc = bias, then taps in
// (kt, kf) order, each product and sum rounded on its own (the reference's
// scalar loop, nemotron/weights.rs:418-523).  Only output rows
// [out_row0, out_row0 + out_rows) are computed -- the rows the step's new
// frames depend on; the input holds rows [x_row0, x_row0 + x_rows) of the
// t_in-row map, and rows outside [0, t_in) are the zero padding.
// Layouts: x [z][x_rows][f_in][c_in], out [z][out_rows][f_out][c_out].
// One CTA per (output row, stream), one thread per output channel, looping
// over the row's f_out positions: loads are coalesced over channels (conv0
// reads one broadcast mel value per tap).
__global__ void conv2d_3x3s2_kernel(const float *__restrict__ x, int t_in, int x_row0, int x_rows, int f_in,
                                    int c_in, const float *__restrict__ w, const float *__restrict__ b, int c_out,
                                    int out_row0, int out_rows, int f_out, int relu, float *__restrict__ out) {
  const int oc = threadIdx.x;
  if (oc >= c_out) return;
  const int r = blockIdx.x, z = blockIdx.y;
  const int ot = out_row0 + r;
  const int ic = c_in == 1 ? 0 : oc;  // depthwise: channel oc only
  float wr[9];
#pragma unroll
  for (int tap = 0; tap < 9; tap++) wr[tap] = w[oc * 9 + tap];
  const float bias = b[oc];
  const float *xz = x + (size_t)z * x_rows * f_in * c_in + ic;
  float *o = out + ((size_t)z * out_rows + r) * f_out * c_out + oc;
  bool row_ok[3];
  const float *xr[3];
#pragma unroll
  for (int kt = 0; kt < 3; kt++) {
    const int ti = ot * 2 + kt - 2;
    const int li = ti - x_row0;
    row_ok[kt] = ti >= 0 && ti < t_in && li >= 0 && li < x_rows;
    xr[kt] = xz + (size_t)(row_ok[kt] ? li : 0) * f_in * c_in;
  }
  for (int of = 0; of < f_out; of++) {
    float acc = bias;
#pragma unroll
    for (int kt = 0; kt < 3; kt++) {
      if (!row_ok[kt]) continue;
#pragma unroll
      for (int kf = 0; kf < 3; kf++) {
        const int fi = of * 2 + kf - 2;
        if (fi < 0 || fi >= f_in) continue;
        acc = __fadd_rn(acc, __fmul_rn(xr[kt][(size_t)fi * c_in], wr[kt * 3 + kf]));
      }
    }
    o[(size_t)of * c_out] = relu ? fmaxf(acc, 0.0f) : acc;
  }
}

// conv0 (1 -> C channels, 3x3 stride 2, ReLU) feeding the depthwise conv2
// (3x3 stride 2), fused: each conv2 output rebuilds the conv0 values it reads
// from the 7 mel rows it depends on (staged in shared memory), with the same
// taps in the same order as conv2d_3x3s2_kernel, so the result is the same
// as running the two convs apart -- and conv0's output, the largest tensor
// of the pre-encode stack, never goes to memory.  One CTA per conv2 output
// row and stream, one thread per channel.
__global__ void conv02_fused_kernel(const float *__restrict__ win, int t_mel, int f_mel,
                                    const float *__restrict__ w0, const float *__restrict__ b0,
                                    const float *__restrict__ w2, const float *__restrict__ b2, int C, int ta,
                                    int fa, int out_row0, int out_rows, int fb, float *__restrict__ out) {
  extern __shared__ float mel[];  // [7][f_mel]
  const int r = blockIdx.x, z = blockIdx.y;
  const int ot = out_row0 + r;    // conv2 output row
  const int m0 = 4 * ot - 6;      // first mel row any of its conv0 inputs reads
  for (int i = threadIdx.x; i < 7 * f_mel; i += blockDim.x) {
    const int mt = m0 + i / f_mel;
    mel[i] = (mt >= 0 && mt < t_mel) ? win[((size_t)z * t_mel + mt) * f_mel + i % f_mel] : 0.0f;
  }
  __syncthreads();
  // conv0 at (row 2*ot + kt - 2, frequency f0) for this thread's channel,
  // ReLU applied: mel rows 2 kt + kt0 of the tile
  auto conv0 = [&](const float (&w0r)[9], float bias0, int kt, int f0) -> float {
    float a0 = bias0;
#pragma unroll
    for (int kt0 = 0; kt0 < 3; kt0++) {
      const int mt = m0 + 2 * kt + kt0;
      if (mt < 0 || mt >= t_mel) continue;
      const float *mr = mel + (2 * kt + kt0) * f_mel;
#pragma unroll
      for (int kf0 = 0; kf0 < 3; kf0++) {
        const int mf = 2 * f0 + kf0 - 2;
        if (mf < 0 || mf >= f_mel) continue;
        a0 = __fadd_rn(a0, __fmul_rn(mr[mf], w0r[kt0 * 3 + kf0]));
      }
    }
    return fmaxf(a0, 0.0f);
  };
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float w0r[9], w2r[9];
#pragma unroll
    for (int tap = 0; tap < 9; tap++) {
      w0r[tap] = w0[c * 9 + tap];
      w2r[tap] = w2[c * 9 + tap];
    }
    const float bias0 = b0[c], bias2 = b2[c];
    bool rv[3];
#pragma unroll
    for (int kt = 0; kt < 3; kt++) {
      const int t0 = 2 * ot + kt - 2;
      rv[kt] = t0 >= 0 && t0 < ta;
    }
    float *o = out + ((size_t)z * out_rows + r) * fb * C + c;
    // conv0 columns 2 f2 - 2, 2 f2 - 1, 2 f2 of the 3 rows; the first is the
    // previous output's last, so each column is computed once
    float vl[3] = {0.0f, 0.0f, 0.0f};
    auto column = [&](int f2) {  // any column, every tap checked
      float vm[3], vr[3];
#pragma unroll
      for (int kt = 0; kt < 3; kt++) {
        vm[kt] = rv[kt] && 2 * f2 - 1 >= 0 && 2 * f2 - 1 < fa ? conv0(w0r, bias0, kt, 2 * f2 - 1) : 0.0f;
        vr[kt] = rv[kt] && 2 * f2 < fa ? conv0(w0r, bias0, kt, 2 * f2) : 0.0f;
      }
      float acc = bias2;
#pragma unroll
      for (int kt = 0; kt < 3; kt++) {
        if (!rv[kt]) continue;
        if (2 * f2 - 2 >= 0 && 2 * f2 - 2 < fa) acc = __fadd_rn(acc, __fmul_rn(vl[kt], w2r[kt * 3 + 0]));
        if (2 * f2 - 1 >= 0 && 2 * f2 - 1 < fa) acc = __fadd_rn(acc, __fmul_rn(vm[kt], w2r[kt * 3 + 1]));
        if (2 * f2 < fa) acc = __fadd_rn(acc, __fmul_rn(vr[kt], w2r[kt * 3 + 2]));
      }
      o[(size_t)f2 * C] = acc;
#pragma unroll
      for (int kt = 0; kt < 3; kt++) vl[kt] = vr[kt];
    };
    // Interior columns [1, f2b): all 7 mel rows and all 3 conv0 rows exist,
    // conv0 columns 2 f2 - 2 .. 2 f2 lie in [0, fa) and mel columns
    // 4 f2 - 4 .. 4 f2 in [0, f_mel), so no tap is skipped: the same sums in
    // the same order from a 7 x 5 window of mel values held in registers
    // (mel column 4 f2 - 4 + i at window column i), slid by 4 columns a step.
    const bool rows_ok = rv[0] && rv[1] && rv[2] && m0 >= 0 && m0 + 6 < t_mel;
    const int f2b = rows_ok ? min(min((fa - 1) / 2, (f_mel - 1) / 4) + 1, fb) : 1;
    column(0);
    if (f2b > 1) {
      float wv[7][5];
#pragma unroll
      for (int rr = 0; rr < 7; rr++)
#pragma unroll
        for (int i = 0; i < 5; i++) wv[rr][i] = mel[rr * f_mel + i];
      for (int f2 = 1; f2 < f2b; f2++) {
        float vm[3], vr[3];
#pragma unroll
        for (int kt = 0; kt < 3; kt++) {
          float am = bias0, ar = bias0;
#pragma unroll
          for (int kt0 = 0; kt0 < 3; kt0++)
#pragma unroll
            for (int kf0 = 0; kf0 < 3; kf0++) {
              am = __fadd_rn(am, __fmul_rn(wv[2 * kt + kt0][kf0], w0r[kt0 * 3 + kf0]));
              ar = __fadd_rn(ar, __fmul_rn(wv[2 * kt + kt0][2 + kf0], w0r[kt0 * 3 + kf0]));
            }
          vm[kt] = fmaxf(am, 0.0f);
          vr[kt] = fmaxf(ar, 0.0f);
        }
        float acc = bias2;
#pragma unroll
        for (int kt = 0; kt < 3; kt++) {
          acc = __fadd_rn(acc, __fmul_rn(vl[kt], w2r[kt * 3 + 0]));
          acc = __fadd_rn(acc, __fmul_rn(vm[kt], w2r[kt * 3 + 1]));
          acc = __fadd_rn(acc, __fmul_rn(vr[kt], w2r[kt * 3 + 2]));
        }
        o[(size_t)f2 * C] = acc;
#pragma unroll
        for (int kt = 0; kt < 3; kt++) vl[kt] = vr[kt];
        if (f2 + 1 < f2b) {  // the next window: mel columns 4 f2 .. 4 f2 + 4
#pragma unroll
          for (int rr = 0; rr < 7; rr++) {
            wv[rr][0] = wv[rr][4];
#pragma unroll
            for (int i = 1; i < 5; i++) wv[rr][i] = mel[rr * f_mel + 4 * f2 + i];
          }
        }
      }
    }
    for (int f2 = f2b; f2 < fb; f2++) column(f2);
  }
}

// Pointwise conv: Y[m][n] = max(sum_k W[n][k] X[m][k] + b[n], 0) over all
// spatial positions m of all streams (X, Y channels-last).  Each output's
// k-sum is one fused multiply-add chain from k = 0 upwards, then the bias
// is added -- the reference's rounding for its pointwise convs.  128 x 128
// tile per CTA, 8 x 8 outputs per thread, k staged 16 at a time (k is a
// multiple of 16: 16-byte loads of both operands).
constexpr int kPwBM = 128, kPwBN = 128, kPwBK = 16, kPwThreads = 256;

__global__ void __launch_bounds__(kPwThreads, 2)
    pw_conv_relu_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                        float *__restrict__ y, int64_t m_rows, int n, int k) {
  __shared__ __align__(16) float as[2][kPwBK][kPwBM];
  __shared__ __align__(16) float bs[2][kPwBK][kPwBN];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.x * kPwBM;
  const int n0 = blockIdx.y * kPwBN;
  // loader: thread -> (row tid / 2, k quads (tid % 2) * 8 .. + 7) of both tiles
  const int lr = tid >> 1, lk = (tid & 1) * 8;
  const int64_t am = m0 + lr;
  const int bn = n0 + lr;
  auto load = [&](int kb, float (&ra)[8], float (&rb)[8]) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const float4 a4 = am < m_rows ? *reinterpret_cast<const float4 *>(x + am * k + kb + lk + 4 * h)
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const float4 b4 = bn < n ? *reinterpret_cast<const float4 *>(w + (int64_t)bn * k + kb + lk + 4 * h)
                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      ra[4 * h] = a4.x, ra[4 * h + 1] = a4.y, ra[4 * h + 2] = a4.z, ra[4 * h + 3] = a4.w;
      rb[4 * h] = b4.x, rb[4 * h + 1] = b4.y, rb[4 * h + 2] = b4.z, rb[4 * h + 3] = b4.w;
    }
  };
  const int ty = tid / 16, tx = tid % 16;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
  float ra[8], rb[8];
  load(0, ra, rb);
  int buf = 0;
  for (int kb = 0; kb < k; kb += kPwBK) {
#pragma unroll
    for (int q = 0; q < 8; q++) {
      as[buf][lk + q][lr] = ra[q];
      bs[buf][lk + q][lr] = rb[q];
    }
    __syncthreads();
    if (kb + kPwBK < k) load(kb + kPwBK, ra, rb);
#pragma unroll
    for (int kq = 0; kq < kPwBK; kq++) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&as[buf][kq][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&as[buf][kq][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&bs[buf][kq][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&bs[buf][kq][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(bv[j], av[i], acc[i][j]);
    }
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= m_rows) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int nn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (nn < n) y[m * n + nn] = fmaxf(__fadd_rn(acc[i][j], b[nn]), 0.0f);
    }
  }
}

// The pointwise conv's positions that the reference's f32 GEMM sums in its
// column-tail order.  The reference runs a 1x1 conv as W [c_out, c_in] x
// X^T [c_in, spatial] per stream (nemotron/weights.rs:399-443); its GEMM
// (simd_kernel.rs:448-727) gives each output of a whole 16-column block one
// fused chain over k (pw_conv_relu_kernel above), but each of the last
// spatial % 16 columns (gemm_cols_tail, :688-727) 16 lane accumulators --
// lane l a fused chain over k = l, l + 16, ... -- summed in lane order from
// -0.0, then + the k tail (k % 16 == 0 here, so + 0.0), then the bias.
// One CTA per stream rewrites those positions' outputs (at most 15, all in
// the window's last time row, which the step computes): the stream's tail
// input rows are staged in shared memory, thread = output channel, four
// positions at a time.  Row r of a stream is window position sp_base + r.
__global__ void __launch_bounds__(256)
    pw_conv_tail_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                        float *__restrict__ y, int rows_per_stream, int tail_row0, int n, int k) {
  extern __shared__ __align__(16) float xs[];  // [rows_per_stream - tail_row0][k]
  const int nt = rows_per_stream - tail_row0;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_stream + tail_row0;
  for (int i = threadIdx.x; i < nt * k; i += blockDim.x) xs[i] = x[row0 * k + i];
  __syncthreads();
  for (int oc = threadIdx.x; oc < n; oc += blockDim.x) {
    const float *wr = w + (int64_t)oc * k;
    const float bias = b[oc];
    for (int p0 = 0; p0 < nt; p0 += 4) {
      const int np = min(4, nt - p0);
      float lane[4][16];
#pragma unroll
      for (int p = 0; p < 4; p++)
#pragma unroll
        for (int l = 0; l < 16; l++) lane[p][l] = 0.0f;
      for (int kk = 0; kk < k; kk += 16) {
        float wv[16];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 v = *reinterpret_cast<const float4 *>(wr + kk + 4 * q);
          wv[4 * q] = v.x, wv[4 * q + 1] = v.y, wv[4 * q + 2] = v.z, wv[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int p = 0; p < 4; p++) {
          if (p >= np) break;
          const float *xr = xs + (p0 + p) * k + kk;
#pragma unroll
          for (int l = 0; l < 16; l++) lane[p][l] = __fmaf_rn(wv[l], xr[l], lane[p][l]);
        }
      }
#pragma unroll
      for (int p = 0; p < 4; p++) {
        if (p >= np) break;
        float r = -0.0f;
#pragma unroll
        for (int l = 0; l < 16; l++) r = __fadd_rn(r, lane[p][l]);
        r = __fadd_rn(r, 0.0f);  // + the (empty) k tail
        y[(row0 + p0 + p) * n + oc] = fmaxf(__fadd_rn(r, bias), 0.0f);
      }
    }
  }
}

// [z][t][f][C] -> rows (z, j) of [C*f] (channel-major, frequency fastest)
// for frames start_rel .. start_rel + c - 1.
__global__ void flatten_kernel(const float *__restrict__ x, int t, int f, int C, int start_rel, int c,
                               float *__restrict__ out, QOut qo) {
  const int64_t row = blockIdx.y;  // z * c + j
  const int64_t z = row / c, j = row % c;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // blockDim 256: whole warps of one block
  const bool valid = i < C * f;
  const int ch = valid ? i / f : 0, ff = valid ? i % f : 0;
  const float v = valid ? x[((z * t + start_rel + j) * f + ff) * C + ch] : 0.0f;
  if (out && valid) out[row * C * f + i] = v;
  if (qo.xq) {  // one warp = one 32-feature block of the pre-encode linear
    float sblk;
    const int8_t q = warp_quantize_block(v, valid, sblk);
    if (i < (C * f + 31) / 32 * 32) {
      qo.xq[qout_code_index(qo, row, i)] = code_half(q);
      if ((threadIdx.x & 31) == 0) qo.dx[qout_dx_index(qo, row, i / 32)] = sblk;
    }
  }
}

// Input codes of the prompt MLP's first linear for every row: the row's d
// features followed by the one-hot of its stream's prompt (streaming.rs:
// 323-331, cat = [x ; onehot(prompt_id)]), quantised per 32-block as
// quantize_col does.  One warp per block; rows whose stream has no prompt
// get an all-zero one-hot (their MLP output is discarded).
__global__ void prompt_cat_quant_kernel(const float *__restrict__ x, int64_t rows, int c, int d, int n_prompts,
                                        const int32_t *__restrict__ pids, QOut qo) {
  const int64_t row = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // whole warps of one block
  const int k = d + n_prompts;
  if (row >= rows || (i & ~31) >= k) return;
  const int pid = pids[row / c];
  const bool valid = i < k;
  const float v = i < d ? x[row * d + i] : (valid && i - d == pid ? 1.0f : 0.0f);
  float sblk;
  const int8_t q = warp_quantize_block(v, valid, sblk);
  qo.xq[qout_code_index(qo, row, i)] = code_half(q);
  if ((threadIdx.x & 31) == 0) qo.dx[qout_dx_index(qo, row, i / 32)] = sblk;
}

// Rows of streams with a prompt take the prompt MLP's output
// (streaming.rs:337-341: the block output frames are replaced).
__global__ void prompt_select_kernel(float *__restrict__ x, const float *__restrict__ y, int c, int d,
                                     const int32_t *__restrict__ pids) {
  const int64_t row = blockIdx.x;
  if (pids[row / c] < 0) return;
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[row * d + i] = y[row * d + i];
}

// Output frames into the per-stream output ring (slot = (frame + shift) % cap).
__global__ void out_ring_kernel(const float *__restrict__ x, int c, int d, float *__restrict__ ring, int cap,
                                int64_t s, const int64_t *shift) {
  const int64_t row = blockIdx.x;
  const int64_t z = row / c, j = row % c;
  if (shift) s += *shift;
  float *dst = ring + (z * cap + (s + j) % cap) * (int64_t)d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = x[row * d + i];
}

// ---- launchers ------------------------------------------------------------
int launch_ln_rows(const float *x, int64_t ldx, const float *w, const float *b, float eps, float *out, int64_t ldo,
                   int64_t rows, int d, cudaStream_t st) {
  if (d % kRowThreads || d / kRowThreads > kMaxRowVals) {
    set_error("layernorm: d=%d must be a multiple of 256 up to 4096", d);
    return kErrUnsupported;
  }
  ln_rows_kernel<<<(unsigned)rows, kRowThreads, 0, st>>>(x, ldx, w, b, eps, out, ldo, d);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_glu_ring(const float *h2, int64_t rows, int c, int d, float *ring, int cap, int64_t s,
                    const int64_t *shift, cudaStream_t st) {
  glu_ring_kernel<<<(unsigned)rows, 256, 0, st>>>(h2, c, d, ring, cap, s, shift);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_mel_window(const float *hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                      int n_mels, int t_mel, float *win, int64_t n_streams, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div((int64_t)t_mel * n_mels, 256), (unsigned)n_streams);
  mel_window_kernel<<<grid, 256, 0, st>>>(hist, hist_cap, hist_frames, mel_new, n_new, n_mels, t_mel, win);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_mel_hist(const float *old_hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                    int n_mels, float *new_hist, int64_t n_streams, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div((int64_t)hist_cap * n_mels, 256), (unsigned)n_streams);
  mel_hist_kernel<<<grid, 256, 0, st>>>(old_hist, hist_cap, hist_frames, mel_new, n_new, n_mels, new_hist);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_conv02_fused(const float *win, int64_t n_streams, int t_mel, int f_mel, const float *w0, const float *b0,
                        const float *w2, const float *b2, int C, int ta, int fa, int out_row0, int out_rows, int fb,
                        float *out, cudaStream_t st) {
  if (C > 1024 || f_mel > 1024) {
    set_error("pre_encode conv: %d channels / %d mel bins unsupported (at most 1024)", C, f_mel);
    return kErrUnsupported;
  }
  if (out_rows <= 0 || n_streams <= 0) return kOk;
  conv02_fused_kernel<<<dim3((unsigned)out_rows, (unsigned)n_streams), (unsigned)C, 7 * f_mel * sizeof(float), st>>>(
      win, t_mel, f_mel, w0, b0, w2, b2, C, ta, fa, out_row0, out_rows, fb, out);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_conv2d_3x3s2(const float *x, int64_t n_streams, int t_in, int x_row0, int x_rows, int f_in, int c_in,
                        const float *w, const float *b, int c_out, int out_row0, int out_rows, int f_out, int relu,
                        float *out, cudaStream_t st) {
  if (c_out > 1024 || (c_in != 1 && c_in != c_out)) {
    set_error("pre_encode conv: c_in %d / c_out %d unsupported (c_out <= 1024, depthwise or c_in 1)", c_in, c_out);
    return kErrUnsupported;
  }
  if (out_rows <= 0 || n_streams <= 0) return kOk;
  conv2d_3x3s2_kernel<<<dim3((unsigned)out_rows, (unsigned)n_streams), (unsigned)c_out, 0, st>>>(
      x, t_in, x_row0, x_rows, f_in, c_in, w, b, c_out, out_row0, out_rows, f_out, relu, out);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_pw_conv_relu(const float *x, const float *w, const float *b, float *y, int64_t n_streams,
                        int rows_per_stream, int64_t sp_base, int64_t spatial, int n, int k, cudaStream_t st) {
  const int64_t m_rows = n_streams * rows_per_stream;
  if (m_rows <= 0) return kOk;
  // the reference's f32 GEMM order is restated for k a multiple of 16 (no k
  // tail) and whole 8-row tiles of output channels
  if (k % 16 || n % 8 || k > 4096 || sp_base < 0 || sp_base + rows_per_stream > spatial) {
    set_error("pw_conv: c_in %d (multiple of 16, <= 4096), c_out %d (multiple of 8), rows [%lld, %lld) of %lld",
              k, n, (long long)sp_base, (long long)(sp_base + rows_per_stream), (long long)spatial);
    return kErrUnsupported;
  }
  if (((uintptr_t)x | (uintptr_t)w) & 15) {
    set_error("pw_conv: input and weights must be 16-byte aligned");
    return kErrUnsupported;
  }
  dim3 grid((unsigned)ceil_div(m_rows, kPwBM), (unsigned)ceil_div(n, kPwBN));
  pw_conv_relu_kernel<<<grid, kPwThreads, 0, st>>>(x, w, b, y, m_rows, n, k);
  note_launch();
  SC_CUDA(cudaGetLastError());
  const int64_t sp_tail = spatial / 16 * 16;
  const int64_t tail_row0 = std::max<int64_t>(sp_tail - sp_base, 0);
  if (tail_row0 < rows_per_stream) {
    const size_t smem = (size_t)(rows_per_stream - tail_row0) * k * 4;
    if (smem > 48 * 1024) {
      set_error("pw_conv: %lld tail rows x %d channels exceed the staging buffer",
                (long long)(rows_per_stream - tail_row0), k);
      return kErrUnsupported;
    }
    pw_conv_tail_kernel<<<(unsigned)n_streams, 256, smem, st>>>(x, w, b, y, rows_per_stream, (int)tail_row0, n,
                                                                 k);
    note_launch();
    SC_CUDA(cudaGetLastError());
  }
  return kOk;
}

int launch_flatten(const float *x, int64_t n_streams, int t, int f, int C, int start_rel, int c, float *out,
                   cudaStream_t st, QOut qo) {
  dim3 grid((unsigned)ceil_div((int64_t)C * f, 256), (unsigned)(n_streams * c));
  flatten_kernel<<<grid, 256, 0, st>>>(x, t, f, C, start_rel, c, out, qo);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_prompt_cat_quant(const float *x, int64_t rows, int c, int d, int n_prompts, const int32_t *pids,
                            const QOut &qo, cudaStream_t st) {
  if (!qo.xq || (d % 32)) {
    set_error("prompt_cat_quant: codes output required and d a multiple of 32");
    return kErrInvalid;
  }
  dim3 grid((unsigned)ceil_div((int64_t)d + n_prompts, 256), (unsigned)rows);
  prompt_cat_quant_kernel<<<grid, 256, 0, st>>>(x, rows, c, d, n_prompts, pids, qo);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_prompt_select(float *x, const float *y, int64_t rows, int c, int d, const int32_t *pids,
                         cudaStream_t st) {
  prompt_select_kernel<<<(unsigned)rows, 256, 0, st>>>(x, y, c, d, pids);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

template <int E, int L>
static int launch_ln_quant_t(const float *x, int64_t ldx, const float *w, const float *b, float eps, int64_t rows,
                             const QOut &qo, float *out, int64_t ldo, const float *w0, const float *b0, float *out0,
                             int64_t ld0, cudaStream_t st) {
  const int64_t warps = ceil_div(rows, 32 / L);
  ln_quant_kernel<E, L><<<(unsigned)ceil_div(warps, 4), 128, 0, st>>>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0,
                                                                       out0, ld0);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

// LayerNorm (w0, b0) of x into out0 (ld0), then LayerNorm (w, b) of that
// into the codes qo (and out when given): two consecutive per-row LayerNorms
// in one pass over the rows.  w0 == nullptr: the second one only.
int launch_ln2_quant(const float *x, int64_t ldx, const float *w0, const float *b0, float *out0, int64_t ld0,
                     const float *w, const float *b, float eps, int d, int64_t rows, const QOut &qo, float *out,
                     int64_t ldo, cudaStream_t st) {
  if (w0 && (!out0 || (((uintptr_t)out0 | ((uintptr_t)ld0 * 4)) & 15))) {
    set_error("layernorm+quantise: the first LayerNorm's output must be 16-byte aligned");
    return kErrInvalid;
  }
  switch (d) {
    case 256: return launch_ln_quant_t<32, 8>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0, out0, ld0, st);
    case 512: return launch_ln_quant_t<32, 16>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0, out0, ld0, st);
    case 1024: return launch_ln_quant_t<32, 32>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0, out0, ld0, st);
    case 2048: return launch_ln_quant_t<64, 32>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0, out0, ld0, st);
    case 4096: return launch_ln_quant_t<128, 32>(x, ldx, w, b, eps, rows, qo, out, ldo, w0, b0, out0, ld0, st);
    default:
      set_error("layernorm+quantise: d=%d must be 256, 512, 1024, 2048 or 4096", d);
      return kErrUnsupported;
  }
}

int launch_ln_quant(const float *x, int64_t ldx, const float *w, const float *b, float eps, int d, int64_t rows,
                    const QOut &qo, float *out, int64_t ldo, cudaStream_t st) {
  return launch_ln2_quant(x, ldx, nullptr, nullptr, nullptr, 0, w, b, eps, d, rows, qo, out, ldo, st);
}

template <int E, int L>
static int launch_dwq_t(const float *ring, int cap, int64_t rows, int c, int kh, int64_t s, const int64_t *shift,
                        const float *wt, const float *lnw, const float *lnb, float eps, const QOut &qo, float *out,
                        cudaStream_t st) {
  const int64_t warps = ceil_div(rows, 32 / L);
  const unsigned grid = (unsigned)ceil_div(warps, 4);
  if (kh == 9)
    dwconv_ln_silu_quant_kernel<E, L, 9>
        <<<grid, 128, 0, st>>>(ring, cap, c, kh, s, shift, wt, lnw, lnb, eps, rows, qo, out);
  else if (kh <= 64)
    dwconv_ln_silu_quant_kernel<E, L, 0>
        <<<grid, 128, 0, st>>>(ring, cap, c, kh, s, shift, wt, lnw, lnb, eps, rows, qo, out);
  else {
    set_error("conv module: kernel %d > 64 unsupported", kh);
    return kErrUnsupported;
  }
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_dwconv_ln_silu_quant(const float *ring, int cap, int64_t rows, int c, int d, int kh, int64_t s,
                                const int64_t *shift, const float *wt, const float *lnw, const float *lnb, float eps,
                                const QOut &qo, float *out, cudaStream_t st) {
  switch (d) {
    case 256: return launch_dwq_t<32, 8>(ring, cap, rows, c, kh, s, shift, wt, lnw, lnb, eps, qo, out, st);
    case 512: return launch_dwq_t<32, 16>(ring, cap, rows, c, kh, s, shift, wt, lnw, lnb, eps, qo, out, st);
    case 1024: return launch_dwq_t<32, 32>(ring, cap, rows, c, kh, s, shift, wt, lnw, lnb, eps, qo, out, st);
    case 2048: return launch_dwq_t<64, 32>(ring, cap, rows, c, kh, s, shift, wt, lnw, lnb, eps, qo, out, st);
    case 4096: return launch_dwq_t<128, 32>(ring, cap, rows, c, kh, s, shift, wt, lnw, lnb, eps, qo, out, st);
    default:
      set_error("conv module: d=%d must be 256, 512, 1024, 2048 or 4096", d);
      return kErrUnsupported;
  }
}

int launch_out_ring(const float *x, int64_t rows, int c, int d, float *ring, int cap, int64_t s,
                    const int64_t *shift, cudaStream_t st) {
  out_ring_kernel<<<(unsigned)rows, 256, 0, st>>>(x, c, d, ring, cap, s, shift);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

__global__ void store_i64_kernel(int64_t *dst, int64_t v) { *dst = v; }

// One 64-bit value into device memory, in stream order (the step graph's
// frame shift, written before each replay).
int launch_store_i64(int64_t *dst, int64_t v, cudaStream_t st) {
  store_i64_kernel<<<1, 1, 0, st>>>(dst, v);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace sc
