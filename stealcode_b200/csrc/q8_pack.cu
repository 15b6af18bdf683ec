// q8_pack.cu -- one-time repack of GGUF Q8_0 tensors into the row-group tile
// layout (sc_common.cuh) and the bit-exact activation quantiser.
//
// Reference: the GGUF loader keeps 34-byte blocks [f16 d][32 x i8] as stored
// (nemotron/weights.rs:91-111, load_lin :640-697); the reference GPU backend
// repacks once at load (gpu/kernels.rs:44-78 pack_q8).  The activation
// quantiser restates sgemm_kernel.rs:57-90 (quantize_col).
#include "sc_kernels.cuh"

namespace sc {

// One thread per (padded row, block): copy 32 quants into the tile layout and
// the raw f16 scale bits into the scale array; if qh is set, also write the
// quants as f16 tiles (sc_common.cuh).  raw holds `rows` rows of
// `padded_row` bytes; blocks are `block_bytes` long with the f16 scale at byte
// 0 and the quants at byte `qoff`.
__global__ void repack_q8f16_kernel(const uint8_t *__restrict__ raw, int64_t rows,
                                    int64_t k, int64_t padded_row,
                                    int64_t block_bytes, int64_t qoff,
                                    int64_t rows_pad, int64_t nb,
                                    int8_t *__restrict__ qs,
                                    __half *__restrict__ sc,
                                    __half *__restrict__ qh) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows_pad * nb) return;
  int64_t b = idx % nb;
  int64_t row = idx / nb;
  int64_t g = row / SC_GROUP_ROWS, r = row % SC_GROUP_ROWS;
  uint8_t q[32];
  uint16_t s16 = 0;
  if (row < rows) {
    const uint8_t *blk = raw + row * padded_row + b * block_bytes;
    s16 = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
    int64_t len = k - b * 32 < 32 ? k - b * 32 : 32;
#pragma unroll
    for (int i = 0; i < 32; i++) q[i] = i < len ? blk[qoff + i] : 0;
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++) q[i] = 0;
  }
  uint8_t *tile = (uint8_t *)qs + (g * nb + b) * SC_TILE_BYTES;
  uint4 lo, hi;
  memcpy(&lo, q, 16);
  memcpy(&hi, q + 16, 16);
  *(uint4 *)(tile + r * 16) = lo;
  *(uint4 *)(tile + 2048 + r * 16) = hi;
  sc[(g * nb + b) * SC_GROUP_ROWS + r] = __ushort_as_half(s16);
  if (qh) {  // the same quants as f16 tiles for the tensor-core path
    __half *th = qh + (g * nb + b) * 4096;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      __half h8[8];
#pragma unroll
      for (int e = 0; e < 8; e++) h8[e] = __short2half_rn((short)(int8_t)q[8 * c + e]);
      uint4 v;
      memcpy(&v, h8, 16);
      *(uint4 *)(th + c * 1024 + r * 8) = v;
    }
  }
}

int repack_q8_device(const uint8_t *raw_dev, int64_t rows, int64_t k,
                     int64_t block_bytes, int64_t qoff, Q8Weights *w,
                     cudaStream_t st) {
  int64_t nb = ceil_div(k, 32);
  int64_t padded_row = nb * block_bytes;
  int64_t rows_pad = ceil_div(rows, SC_GROUP_ROWS) * SC_GROUP_ROWS;
  int64_t n = rows_pad * nb;
  int threads = 256;
  repack_q8f16_kernel<<<(unsigned)ceil_div(n, threads), threads, 0, st>>>(
      raw_dev, rows, k, padded_row, block_bytes, qoff, rows_pad, nb, w->qs,
      w->sc, w->qh);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

// ---------------------------------------------------------------------------
// Activation quantisation (bit-exact restatement of quantize_col).
//
// Output: xq [m_pad][k_pad] int8 (row = activation column = frame), dx
// [nb][m_pad] f32 (block-major so a GEMM reads the scales of all frames of a
// block contiguously).  One warp per (frame, block); lane j owns element
// 32b + j.  x is time-major (element (m, kk) at x[m*ldx + kk]) or
// feature-major (x[kk*ldx + m], the reference CPU layout [k, n]).
//
// Semantics kept exactly: amax over |x| ignoring NaN (`v > maxv`), scale 1 and
// zero codes for an all-zero block, s = amax / 127 and inv = 1 / s with IEEE
// division, q = round-half-away(x * inv) with the saturating, NaN -> 0 cast of
// Rust's `as i8`.  No fast-math anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int8_t rust_round_i8(float v) {
  float r = roundf(v);  // half away from zero, like f32::round
  if (r != r) return 0;
  r = fminf(fmaxf(r, -128.0f), 127.0f);
  return (int8_t)(int)r;
}

template <bool kFeatureMajor>
__global__ void quantize_act_kernel(const float *__restrict__ x, int64_t m,
                                    int64_t k, int64_t ldx, int64_t nb,
                                    int64_t m_pad, int64_t k_pad,
                                    void *__restrict__ xq,
                                    float *__restrict__ dx, int tile_ft) {
  int lane = threadIdx.x & 31;
  int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= m_pad * nb) return;
  int64_t col = wid / nb, b = wid % nb;
  int64_t kk = b * 32 + lane;
  bool valid = col < m && kk < k;
  float v = 0.0f;
  if (valid) v = kFeatureMajor ? x[kk * ldx + col] : x[col * ldx + kk];
  // `if v > maxv { maxv = v }` over |x|: fmaxf drops NaN the same way; a block
  // of NaNs only leaves amax = 0, as the reference's maxv stays 0.
  float amax = valid ? fabsf(v) : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (amax != amax) amax = 0.0f;
  float s = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
  int8_t q = 0;
  if (amax != 0.0f && valid) {
    float inv = __fdiv_rn(1.0f, s);
    q = rust_round_i8(__fmul_rn(v, inv));
  }
  if (tile_ft)
    ((__half *)xq)[((col / tile_ft) * nb + b) * (int64_t)tile_ft * 32 + (lane >> 3) * tile_ft * 8 +
                   (col % tile_ft) * 8 + (lane & 7)] = __short2half_rn((short)q);
  else
    ((int8_t *)xq)[col * k_pad + kk] = q;
  if (lane == 0) dx[tile_ft ? ((col / tile_ft) * nb + b) * tile_ft + col % tile_ft : b * m_pad + col] = s;
}

// Time-major variant with 16-byte loads: one warp per (frame, 4 blocks); the
// 8 lanes of a block each hold 4 consecutive elements, reduce amax over the
// 8-lane group and store their 4 codes with one 32-bit store.  Same
// arithmetic per element as quantize_act_kernel.
__global__ void quantize_act_v4_kernel(const float *__restrict__ x, int64_t m, int64_t k, int64_t ldx,
                                       int64_t nb, int64_t m_pad, int64_t k_pad, void *__restrict__ xq,
                                       float *__restrict__ dx, int tile_ft) {
  const int lane = threadIdx.x & 31;
  const int64_t nq = ceil_div(nb, 4);
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= m_pad * nq) return;
  const int64_t col = wid / nq;
  const int64_t b = (wid % nq) * 4 + (lane >> 3);
  const int sub = lane & 7;
  const int64_t kk = b * 32 + sub * 4;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  bool valid[4];
  const bool blk_ok = b < nb;
  if (blk_ok && col < m && kk + 3 < k) {
    const float4 t4 = *(const float4 *)(x + col * ldx + kk);
    v[0] = t4.x, v[1] = t4.y, v[2] = t4.z, v[3] = t4.w;
#pragma unroll
    for (int e = 0; e < 4; e++) valid[e] = true;
  } else {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      valid[e] = blk_ok && col < m && kk + e < k;
      if (valid[e]) v[e] = x[col * ldx + kk + e];
    }
  }
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; e++) amax = fmaxf(amax, valid[e] ? fabsf(v[e]) : 0.0f);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (amax != amax) amax = 0.0f;
  const float s = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
  int8_t q[4] = {0, 0, 0, 0};
  if (amax != 0.0f) {
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int e = 0; e < 4; e++) q[e] = valid[e] ? rust_round_i8(__fmul_rn(v[e], inv)) : (int8_t)0;
  }
  if (!blk_ok) return;
  if (tile_ft) {  // 4 f16 codes: half of one 8-element chunk of the tile layout
    __half h4[4];
#pragma unroll
    for (int e = 0; e < 4; e++) h4[e] = __short2half_rn((short)q[e]);
    uint2 u;
    memcpy(&u, h4, 8);
    *(uint2 *)((__half *)xq + ((col / tile_ft) * nb + b) * (int64_t)tile_ft * 32 + (sub >> 1) * tile_ft * 8 +
               (col % tile_ft) * 8 + (sub & 1) * 4) = u;
  } else {
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) packed |= (uint32_t)(uint8_t)q[e] << (8 * e);
    *(uint32_t *)((int8_t *)xq + col * k_pad + kk) = packed;
  }
  if (sub == 0) dx[tile_ft ? ((col / tile_ft) * nb + b) * tile_ft + col % tile_ft : b * m_pad + col] = s;
}

int quantize_act(const float *x, int64_t m, int64_t k, int64_t ldx,
                 bool feature_major, int64_t m_pad, void *xq, float *dx,
                 cudaStream_t st, int tile_ft) {
  int64_t nb = ceil_div(k, 32);
  int64_t k_pad = nb * 32;
  if (!feature_major && ldx % 4 == 0 && ((uintptr_t)x & 15) == 0) {
    const int64_t warps = m_pad * ceil_div(nb, 4);
    const int threads = 256;
    quantize_act_v4_kernel<<<(unsigned)ceil_div(warps * 32, threads), threads, 0, st>>>(
        x, m, k, ldx, nb, m_pad, k_pad, xq, dx, tile_ft);
    note_launch();
    SC_CUDA(cudaGetLastError());
    return kOk;
  }
  int64_t warps = m_pad * nb;
  int threads = 256;
  unsigned grid = (unsigned)ceil_div(warps * 32, threads);
  if (feature_major)
    quantize_act_kernel<true><<<grid, threads, 0, st>>>(x, m, k, ldx, nb, m_pad, k_pad, xq, dx, tile_ft);
  else
    quantize_act_kernel<false><<<grid, threads, 0, st>>>(x, m, k, ldx, nb, m_pad, k_pad, xq, dx, tile_ft);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace sc
