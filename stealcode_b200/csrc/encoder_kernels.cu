// encoder_kernels.cu -- the non-GEMM kernels of the device streaming
// encoder step (everything in block_new and pre_encode_forward except the
// Q8_0 linears and the attention):
//   ln_rows_kernel            LayerNorm per frame row   (simd_kernel.rs:734-813)
//   glu_ring_kernel           GLU into the per-stream conv ring
//                                                       (simd_kernel.rs:868-910)
//   dwconv_ln_silu_kernel     causal depthwise conv over the ring + LayerNorm
//                             + SiLU, fused            (streaming.rs:608-638,
//                             simd_kernel.rs:1160-1235, 817-839)
//   mel_window_kernel         pre-encode mel window     (streaming.rs:182-207)
//   conv2d_3x3s2_kernel       conv0 and the depthwise convs 2/5
//                                                       (nemotron/weights.rs:418-523)
//   bias_relu_kernel          bias + ReLU after the pointwise convs
//   flatten_kernel            [t, f, C] -> [t, C*f] of the needed frames
//                                                       (nemotron/encoder.rs:460-470)
// Frame rows are time-major [stream][frame][d]; one CTA handles one row for
// the row-wise kernels (d = 1024: 4 elements per thread).
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

constexpr int kRowThreads = 256;
constexpr int kMaxRowVals = 16;  // d up to 4096

// Sum over the CTA (256 threads): warp shuffles, then the 8 warp sums.
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; w++) t += red[w];
  return t;
}

// LayerNorm of the row values held by this thread (element i = tid + k*256):
// mean = sum/d, var = sum (x-mean)^2 / d, out = (x-mean) * (w * inv) + b
// with inv = 1 / sqrt(var + eps) -- the reference's formula.
__device__ __forceinline__ void ln_vals(float (&v)[kMaxRowVals], int d, const float *w, const float *b, float eps,
                                        float *red) {
  const int nv = d / kRowThreads;
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) s += v[k];
  const float mean = block_sum(s, red) / (float)d;
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) {
      const float df = v[k] - mean;
      q += df * df;
    }
  const float var = block_sum(q, red);
  const float inv = 1.0f / sqrtf(var / (float)d + eps);
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) {
      const int i = threadIdx.x + k * kRowThreads;
      v[k] = fmaf(v[k] - mean, w[i] * inv, b[i]);
    }
}

__global__ void __launch_bounds__(kRowThreads) ln_rows_kernel(const float *__restrict__ x, int64_t ldx,
                                                              const float *__restrict__ w,
                                                              const float *__restrict__ b, float eps,
                                                              float *__restrict__ out, int64_t ldo, int d) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int nv = d / kRowThreads;
  float v[kMaxRowVals];
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) v[k] = x[row * ldx + threadIdx.x + k * kRowThreads];
  ln_vals(v, d, w, b, eps, red);
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) out[row * ldo + threadIdx.x + k * kRowThreads] = v[k];
}

// GLU of the new frames (h2 = [M][2d] time-major, gate first, value second)
// stored into ring slot (s + j) % cap of stream z.
__global__ void glu_ring_kernel(const float *__restrict__ h2, int c, int d, float *__restrict__ ring, int cap,
                                int64_t s) {
  const int64_t row = blockIdx.x;  // z * c + j
  const int64_t z = row / c, j = row % c;
  float *dst = ring + (z * cap + (s + j) % cap) * (int64_t)d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float gate = h2[row * 2 * d + i], val = h2[row * 2 * d + d + i];
    dst[i] = gate * (1.0f / (1.0f + expf(-val)));
  }
}

// Causal depthwise conv (kernel kh, left pad kh - 1) over the GLU ring, then
// the conv module's LayerNorm and SiLU, for new frame j of stream z.  Taps
// before frame 0 are the zero padding (as for the first batch of a stream).
__global__ void __launch_bounds__(kRowThreads)
    dwconv_ln_silu_kernel(const float *__restrict__ ring, int cap, int c, int d, int kh, int64_t s,
                          const float *__restrict__ w, const float *__restrict__ lnw,
                          const float *__restrict__ lnb, float eps, float *__restrict__ out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int64_t z = row / c, fr = s + row % c;
  const int nv = d / kRowThreads;
  float v[kMaxRowVals];
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) {
      const int ch = threadIdx.x + k * kRowThreads;
      float acc = 0.0f;
      for (int t = 0; t < kh; t++) {
        const int64_t ti = fr - (kh - 1) + t;
        if (ti < 0) continue;
        acc = fmaf(ring[(z * cap + ti % cap) * (int64_t)d + ch], w[ch * kh + t], acc);
      }
      v[k] = acc;
    }
  ln_vals(v, d, lnw, lnb, eps, red);
#pragma unroll
  for (int k = 0; k < kMaxRowVals; k++)
    if (k < nv) {
      const float a = v[k];
      out[row * d + threadIdx.x + k * kRowThreads] = a * (1.0f / (1.0f + expf(-a)));
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
// (kt, kf) order; input [z][t_in][f_in][c_in], output [z][t_out][f_out][c_out].
__global__ void conv2d_3x3s2_kernel(const float *__restrict__ x, int t_in, int f_in, int c_in,
                                    const float *__restrict__ w, const float *__restrict__ b, int c_out,
                                    int t_out, int f_out, int relu, float *__restrict__ out, int64_t n_total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_total) return;
  const int oc = (int)(i % c_out);
  const int64_t r = i / c_out;
  const int of = (int)(r % f_out);
  const int ot = (int)((r / f_out) % t_out);
  const int64_t z = r / ((int64_t)f_out * t_out);
  const int ic = c_in == 1 ? 0 : oc;  // depthwise: channel oc only
  float acc = b[oc];
#pragma unroll
  for (int kt = 0; kt < 3; kt++) {
    const int ti = ot * 2 + kt - 2;
    if (ti < 0 || ti >= t_in) continue;
#pragma unroll
    for (int kf = 0; kf < 3; kf++) {
      const int fi = of * 2 + kf - 2;
      if (fi < 0 || fi >= f_in) continue;
      acc += x[((z * t_in + ti) * f_in + fi) * c_in + ic] * w[oc * 9 + kt * 3 + kf];
    }
  }
  out[i] = relu ? fmaxf(acc, 0.0f) : acc;
}

__global__ void bias_relu_kernel(float *__restrict__ x, const float *__restrict__ b, int c, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = fmaxf(x[i] + b[i % c], 0.0f);
}

// [z][t][f][C] -> rows (z, j) of [C*f] (channel-major, frequency fastest)
// for frames start_rel .. start_rel + c - 1.
__global__ void flatten_kernel(const float *__restrict__ x, int t, int f, int C, int start_rel, int c,
                               float *__restrict__ out) {
  const int64_t row = blockIdx.y;  // z * c + j
  const int64_t z = row / c, j = row % c;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)C * f) return;
  const int ch = (int)(i / f), ff = (int)(i % f);
  out[row * C * f + i] = x[((z * t + start_rel + j) * f + ff) * C + ch];
}

// Output frames into the per-stream output ring (slot = frame % cap).
__global__ void out_ring_kernel(const float *__restrict__ x, int c, int d, float *__restrict__ ring, int cap,
                                int64_t s) {
  const int64_t row = blockIdx.x;
  const int64_t z = row / c, j = row % c;
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
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_glu_ring(const float *h2, int64_t rows, int c, int d, float *ring, int cap, int64_t s, cudaStream_t st) {
  glu_ring_kernel<<<(unsigned)rows, 256, 0, st>>>(h2, c, d, ring, cap, s);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_dwconv_ln_silu(const float *ring, int cap, int64_t rows, int c, int d, int kh, int64_t s, const float *w,
                          const float *lnw, const float *lnb, float eps, float *out, cudaStream_t st) {
  dwconv_ln_silu_kernel<<<(unsigned)rows, kRowThreads, 0, st>>>(ring, cap, c, d, kh, s, w, lnw, lnb, eps, out);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_mel_window(const float *hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                      int n_mels, int t_mel, float *win, int64_t n_streams, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div((int64_t)t_mel * n_mels, 256), (unsigned)n_streams);
  mel_window_kernel<<<grid, 256, 0, st>>>(hist, hist_cap, hist_frames, mel_new, n_new, n_mels, t_mel, win);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_mel_hist(const float *old_hist, int hist_cap, int hist_frames, const float *mel_new, int n_new,
                    int n_mels, float *new_hist, int64_t n_streams, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div((int64_t)hist_cap * n_mels, 256), (unsigned)n_streams);
  mel_hist_kernel<<<grid, 256, 0, st>>>(old_hist, hist_cap, hist_frames, mel_new, n_new, n_mels, new_hist);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_conv2d_3x3s2(const float *x, int64_t n_streams, int t_in, int f_in, int c_in, const float *w,
                        const float *b, int c_out, int t_out, int f_out, int relu, float *out, cudaStream_t st) {
  const int64_t n = n_streams * t_out * f_out * c_out;
  conv2d_3x3s2_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(x, t_in, f_in, c_in, w, b, c_out, t_out, f_out,
                                                                   relu, out, n);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_bias_relu(float *x, const float *b, int c, int64_t n, cudaStream_t st) {
  bias_relu_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(x, b, c, n);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_flatten(const float *x, int64_t n_streams, int t, int f, int C, int start_rel, int c, float *out,
                   cudaStream_t st) {
  dim3 grid((unsigned)ceil_div((int64_t)C * f, 256), (unsigned)(n_streams * c));
  flatten_kernel<<<grid, 256, 0, st>>>(x, t, f, C, start_rel, c, out);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_out_ring(const float *x, int64_t rows, int c, int d, float *ring, int cap, int64_t s, cudaStream_t st) {
  out_ring_kernel<<<(unsigned)rows, 256, 0, st>>>(x, c, d, ring, cap, s);
  SC_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace sc
