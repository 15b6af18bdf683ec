// sc_kernels.cuh -- argument structs and launchers shared between the kernel
// translation units and the C ABI (sc_api.cu).
#pragma once

#include <atomic>

#include "sc_common.cuh"

namespace sc {

// GEMM epilogue applied to v = W x + bias, element-wise on the output,
// rounding like the reference's element loops (no fused multiply-add):
//   kEpiNone:     y = v
//   kEpiSilu:     y = v * (1 / (1 + exp(-v)))        (simd_kernel.rs:817-839)
//   kEpiResidual: y = res + alpha * v                 (res may alias y;
//                 streaming.rs:458-460, 596-598, 643-645, 667-669)
//   kEpiRelu:     y = max(v, 0), NaN -> 0             (simd_kernel.rs:843-861)
enum : int { kEpiNone = 0, kEpiSilu = 1, kEpiResidual = 2, kEpiRelu = 3 };
struct Epilogue {
  int op = kEpiNone;
  const float *res = nullptr;
  float alpha = 1.0f;
};

__device__ __forceinline__ float apply_epilogue(const Epilogue &e, float v, int64_t idx) {
  if (e.op == kEpiSilu) return silu_ref(v);
  if (e.op == kEpiResidual) return __fadd_rn(e.res[idx], __fmul_rn(e.alpha, v));
  if (e.op == kEpiRelu) return v > 0.0f ? v : 0.0f;
  return v;
}

// q8_pack.cu
int repack_q8_device(const uint8_t *raw_dev, int64_t rows, int64_t k, int64_t block_bytes,
                     int64_t qoff, Q8Weights *w, cudaStream_t st);
// tile_ft == 0: xq is int8 [m_pad][k_pad], dx [nb][m_pad]; tile_ft > 0: xq
// holds f16 codes in the tensor-core operand layout (the QOut layout with ft
// = tile_ft: [m_pad/tile_ft][nb][4][tile_ft][8]) and dx is
// [m_pad/tile_ft][nb][tile_ft].
int quantize_act(const float *x, int64_t m, int64_t k, int64_t ldx, bool feature_major,
                 int64_t m_pad, void *xq, float *dx, cudaStream_t st, int tile_ft = 0);

// q8_gemm_small.cu
struct SmallGemmArgs {
  const Q8Weights *w;
  const float *x;     // f32 activations quantised inside the kernel, or nullptr
  int64_t ldx;
  int x_feature_major;
  const int8_t *xq;   // else: pre-quantised [m_pad][k_pad] activations
  const float *dx;    // and their block scales [nb][m_pad]
  int64_t k_pad, m_pad, m;
  const float *bias;  // [rows] or nullptr
  float *y;
  int y_time_major;   // 1: y[col*ldy + n]; 0: y[n*ldy + col]
  int64_t ldy;
  int32_t *dots;      // non-null: write raw int32 block dots instead of y
  Epilogue epi;
};
int gemm_small(const SmallGemmArgs &a, int sm_count, cudaStream_t st);
int small_gemm_status(unsigned *out);  // read and clear the kernels' status word
// One-time per-device set-up of each GEMM path, done ahead of its first
// launch on the current device: the status word's device address and the
// kernels' largest shared-memory limits (otherwise done by the first call
// that needs them).
int small_gemm_prime();
int mid_gemm_prime();
int tc_gemm_prime();

// q8_gemm_batch.cu: up to kMaxBatch independent GEMMs of the same t <=
// kBatchFrames frames in one streaming pass.  The caller fills qs .. k,
// x_feature_major; gemm_batch sets xq, dx (workspace) and unit0.
constexpr int kMaxBatch = 128, kBatchFrames = 16;
struct BatchItem {
  const int8_t *qs;
  const __half *sc;
  const float *x;
  const float *bias;
  float *y;
  int8_t *xq;   // activation codes, per 8-block group 16 frames x 256 bytes (q8_gemm_batch.cu)
  float *dx;    // [nb][kBatchFrames] their block scales
  int64_t ldx, ldy;
  int32_t nb, rows, groups, unit0, k, x_feature_major;
};
size_t batch_ws_bytes(const BatchItem *items, int n);
int batch_gemm_status(unsigned *out);  // read and clear the batched kernel's status word
int gemm_batch(BatchItem *items, int n, int t, int y_time_major, void *ws, size_t ws_bytes, int sm_count,
               cudaStream_t st);

// q8_gemm_mid.cu: 16 < m <= 128 frames, q8_gemm_scalar's order (bit-exact)
struct MidGemmArgs {
  const Q8Weights *w;
  const int8_t *xq;   // [m_pad][k_pad] codes (quantize_act, tile_ft 0)
  const float *dx;    // [nb][m_pad]
  int64_t m, m_pad, k_pad;
  const float *bias;  // [rows] or nullptr
  float *y;
  int y_time_major;   // 1: y[col*ldy + n]; 0: y[n*ldy + col]
  int64_t ldy;
  Epilogue epi;
};
int gemm_mid(const MidGemmArgs &a, cudaStream_t st);

// q8_gemm_tc.cu
// Activation codes quantised by the kernel that produces them, written in
// the tensor-core GEMM's tiled operand layout (ft = tc_frame_tile(t)) as f16
// values (every int8 code is an f16 integer): the code of frame f, feature i
// at element
//   ((f / ft) * nb + i / 32) * ft * 32 + ((i % 32) / 8) * ft * 8 + (f % ft) * 8 + i % 8
// (per 32-wide block and frame tile: four 8-feature chunks, each the
// no-swizzle K-major core-matrix layout of ft rows x 16 bytes), and the
// block scale at dx[((f / ft) * nb + i / 32) * ft + f % ft] (a frame tile's
// scales for consecutive blocks are contiguous).  xq == nullptr: unused.
// ft is 64 or 128 (tc_frame_tile), so the indices take shifts, not divisions.
struct QOut {
  __half *xq;
  float *dx;
  int64_t nb, t_pad;
  int ft;
};
__host__ __device__ inline int qout_ft_shift(const QOut &q) { return q.ft == 128 ? 7 : 6; }
__host__ __device__ inline int64_t qout_dx_index(const QOut &q, int64_t f, int64_t blk) {
  const int sh = qout_ft_shift(q);
  return (((f >> sh) * q.nb + blk) << sh) + (f & (q.ft - 1));
}
__host__ __device__ inline int64_t qout_code_index(const QOut &q, int64_t f, int64_t i) {
  const int sh = qout_ft_shift(q);
  return (((f >> sh) * q.nb + (i >> 5)) << (sh + 5)) + (((i & 31) >> 3) << (sh + 3)) + ((f & (q.ft - 1)) << 3) +
         (i & 7);
}

struct TcGemmArgs {
  const Q8Weights *w;
  const __half *xq;   // tiled f16 activation codes (quantize_act with tile_ft = tc_frame_tile(t))
  const float *dx;    // [nb][t_pad]
  int64_t t, t_pad;   // t_pad: multiple of tc_frame_tile(t)
  const float *bias;
  float *y;
  int y_time_major;
  int64_t ldy;
  Epilogue epi;
  QOut qout;          // quantise the epilogue output for the next GEMM (rows % 128 == 0;
                      // y may then be nullptr)
};
int tc_frame_tile(int64_t t);
int gemm_tc(const TcGemmArgs &a, cudaStream_t st);
int tc_gemm_status(unsigned *out);

// sc_api.cu: the shared dispatch behind the Q8_0 GEMM entry points.
// t <= 16 frames run the weight-streaming kernel, more frames (or force_tc)
// the tensor-core kernel, whose accumulation follows the reference scalar
// oracle's order (sgemm_kernel.rs:185-196) -- the encoder's linears set
// force_tc so that every output is rounded the same way at any frame count.
size_t gemm_ws_bytes(int64_t m, int64_t k);
int current_device(int *dev, int *sm_count);
// Raises kernel `kern`'s dynamic shared-memory limit on the current device to
// at least `bytes` (a no-op up to the 48 KB default).  `limit` is the
// kernel's per-device record [64]: it only grows and changes under a lock,
// so no caller lowers the limit under another's launch.
int raise_smem_limit(const void *kern, size_t bytes, std::atomic<size_t> *limit);
int gemm_impl(const Q8Weights *w, const float *x, int64_t t, int32_t x_layout, int64_t ldx,
              const float *bias, float *y, int32_t y_layout, int64_t ldy, void *ws, size_t ws_bytes,
              int32_t *dots, cudaStream_t st, Epilogue epi, bool force_tc = false);

// attn_stream.cu
struct AttnParams {
  const float *q;       // query rows; stream z, query j at (z*c + j)*ldq
  int64_t ldq;
  const float *k_new;   // frames >= new_lo of stream z at (z*rows_new + fr - new_lo)*ld_new
  const float *v_new;
  int64_t ld_new, rows_new, new_lo;
  float *k_ring;        // nullptr in band mode; stream z, frame fr at (z*cap + fr % cap)*d
  float *v_ring;
  int64_t cap;
  const float *pos_p;   // [n_pos, d]
  const float *u;       // pos_bias_u [d]
  const float *v;       // pos_bias_v [d]
  float *out;           // (z*c + j)*ldo
  int64_t ldo;
  int c, d, n_heads;
  float scale;
  int64_t s, k_lo, k_hi, chunk, left_chunks, pos_off;
  int64_t pr_lo;        // first pos row the chunk touches (attn_prepare)
  int np;               // number of pos rows touched (attn_prepare)
  QOut qout;            // also write the output as codes for the next GEMM (out may be nullptr)
  int lane_major;       // q, k (new and ring), u, v and pos rows are stored
                        // lane-major within each head (element 16*ch + l
                        // at (ch/4)*64 + 4l + ch%4); v_new / v_ring natural
  // Sub-range of a longer call (staged kernel only): when zrows > 0 the
  // q / out / qout rows of stream z, query j are z*zrows + r0 + j and its new
  // K/V rows z*zrows + r0 + (fr - new_lo); 0 keeps the layouts above.
  int64_t zrows = 0, r0 = 0;
  // Device frame shift added to every frame number before it becomes a ring
  // slot (nullptr: none).  A replayed step graph runs its captured launches
  // at a later step whose frames are these plus a whole number of chunks:
  // bands, masks and pos rows depend only on frame differences and chunk
  // indices relative to the band, so only the ring slots move.
  const int64_t *frame_shift = nullptr;
};
int attn_prepare(AttnParams &p, int64_t n_pos);
int launch_attn(const AttnParams &p, int64_t n_streams, cudaStream_t st);

}  // namespace sc
