// q8_gemm_mid.cu -- Q8_0 GEMM for mid-size M (17 to 128 frames): a few
// streams' chunks, or one stream's short prefill.
//
// The reference runs every GEMM with more than 16 frames through
// q8_gemm_scalar (simd_kernel.rs:111-125, sgemm_kernel.rs:132-202): per
// output, over the K blocks in order, acc += (dw * dx) * dot with dot the
// block's exact integer dot.  This kernel computes exactly that, so its
// outputs are bit-equal to the reference's.  At these sizes the work is too
// small for the tensor-core path (whose every 32-deep block needs its own
// accumulator round trip) to fill the GPU, and the weight stream is the
// roofline: each CTA streams a 32-row slice of one 128-row group's weight
// tiles through a ring of shared-memory chunks (cp.async) and computes 32
// rows x 32 frames with dp4a on the CUDA cores.  Slicing the groups gives
// four times as many CTAs as groups without reading any weight twice
// (measured: 32-row slices beat 128- and 16-row ones on the layer shapes).
//
// Thread t: row t % 32 of the slice, frames 4 * (t / 32) .. + 3 of the CTA's
// 32.  In the row-group tile layout (sc_common.cuh) a slice's 32 rows of a
// tile are two 512-byte runs, and a warp (32 rows) reads 512 contiguous
// bytes per 16-byte load; the activation codes and scales of a frame are the
// same for every row, so their shared-memory reads are broadcasts.
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

constexpr int kMidRows = 32;              // rows per CTA: a quarter of a row group
constexpr int kMidSlices = SC_GROUP_ROWS / kMidRows;
constexpr int kMidCols = 32;              // frames per CTA
constexpr int kMidThreads = 256;
constexpr int kMidColsPerThread = kMidCols / (kMidThreads / kMidRows);
constexpr int kMidChunk = 8;              // K blocks per staged chunk
constexpr int kMidRing = 4;               // chunks in flight

struct MidSmem {
  static constexpr int kA = kMidChunk * kMidRows * 32;        // weight slices [block][2 halves][32 rows][16]
  static constexpr int kS = kMidChunk * kMidRows * 2;         // f16 weight scales [block][32 rows]
  static constexpr int kX = kMidCols * kMidChunk * 32;        // codes [frame][block][32]
  static constexpr int kD = kMidChunk * kMidCols * 4;         // scales [block][frame]
  static constexpr int kSlot = kA + kS + kX + kD;             // multiples of 16
  static constexpr int kBytes = kMidRing * kSlot;
};

__device__ __forceinline__ void mid_cp16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
template <int N>
__device__ __forceinline__ void mid_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ int mid_dot32(const int4 w0, const int4 w1, const int4 x0, const int4 x1) {
  int d = __dp4a(w0.x, x0.x, 0);
  d = __dp4a(w0.y, x0.y, d);
  d = __dp4a(w0.z, x0.z, d);
  d = __dp4a(w0.w, x0.w, d);
  d = __dp4a(w1.x, x1.x, d);
  d = __dp4a(w1.y, x1.y, d);
  d = __dp4a(w1.z, x1.z, d);
  d = __dp4a(w1.w, x1.w, d);
  return d;
}

// Kernel parameters: the weight descriptor's fields by value (MidGemmArgs
// holds a host pointer to it).
struct MidParams {
  const int8_t *qs;
  const __half *sc;
  int64_t nb, rows;
  const int8_t *xq;
  const float *dx;
  int64_t m, m_pad, k_pad;
  const float *bias;
  float *y;
  int y_time_major;
  int64_t ldy;
  Epilogue epi;
};

__global__ void __launch_bounds__(kMidThreads, 1) q8_gemm_mid_kernel(const __grid_constant__ MidParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int t = threadIdx.x, r = t & (kMidRows - 1), q = t / kMidRows;
  const int64_t g = blockIdx.x / kMidSlices, col0 = (int64_t)blockIdx.y * kMidCols;
  const int rs = blockIdx.x % kMidSlices;  // slice of the group
  const int nb = (int)p.nb;
  const int nch = (nb + kMidChunk - 1) / kMidChunk;
  const int8_t *qs = p.qs;
  const __half *sc = p.sc;

  // Each stage() commits one cp.async group (empty past the last chunk), so
  // waiting for all but the kMidRing - 1 newest groups lands chunk ch.
  auto stage = [&](int ch) {
    if (ch < nch) {
      unsigned char *slot = smem + (ch % kMidRing) * MidSmem::kSlot;
      const int b0 = ch * kMidChunk, nbk = nb - b0 < kMidChunk ? nb - b0 : kMidChunk;
      // tile (g, b): byte i of row rr at (i / 16) * 2048 + rr * 16 + i % 16;
      // the slice's rows of each half are 512 contiguous bytes
      const unsigned char *a = (const unsigned char *)qs + (g * nb + b0) * SC_TILE_BYTES + rs * kMidRows * 16;
      for (int i = t; i < nbk * 2 * (kMidRows * 16 / 16); i += kMidThreads) {
        const int bb = i / (2 * kMidRows), half = (i / kMidRows) & 1, piece = i % kMidRows;
        mid_cp16(slot + (bb * 2 + half) * kMidRows * 16 + piece * 16,
                 a + (int64_t)bb * SC_TILE_BYTES + half * 2048 + piece * 16);
      }
      const unsigned char *s = (const unsigned char *)(sc + (g * nb + b0) * SC_GROUP_ROWS + rs * kMidRows);
      for (int i = t; i < nbk * (kMidRows * 2 / 16); i += kMidThreads) {
        const int bb = i / (kMidRows * 2 / 16), piece = i % (kMidRows * 2 / 16);
        mid_cp16(slot + MidSmem::kA + bb * kMidRows * 2 + piece * 16, s + (int64_t)bb * SC_GROUP_ROWS * 2 + piece * 16);
      }
      for (int i = t; i < kMidCols * nbk * 2; i += kMidThreads) {
        const int j = i / (nbk * 2), piece = i % (nbk * 2);
        mid_cp16(slot + MidSmem::kA + MidSmem::kS + j * kMidChunk * 32 + piece * 16,
                 p.xq + (col0 + j) * p.k_pad + b0 * 32 + piece * 16);
      }
      for (int i = t; i < nbk * kMidCols / 4; i += kMidThreads) {
        const int bb = i / (kMidCols / 4), piece = i % (kMidCols / 4);
        mid_cp16(slot + MidSmem::kA + MidSmem::kS + MidSmem::kX + (bb * kMidCols + piece * 4) * 4,
                 p.dx + (int64_t)(b0 + bb) * p.m_pad + col0 + piece * 4);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

#pragma unroll
  for (int ch = 0; ch < kMidRing - 1; ch++) stage(ch);
  float acc[kMidColsPerThread];
#pragma unroll
  for (int j = 0; j < kMidColsPerThread; j++) acc[j] = 0.0f;
  for (int ch = 0; ch < nch; ch++) {
    stage(ch + kMidRing - 1);
    mid_cp_wait<kMidRing - 1>();
    __syncthreads();
    const unsigned char *slot = smem + (ch % kMidRing) * MidSmem::kSlot;
    const __half *ss = (const __half *)(slot + MidSmem::kA);
    const unsigned char *xs = slot + MidSmem::kA + MidSmem::kS;
    const float *ds = (const float *)(slot + MidSmem::kA + MidSmem::kS + MidSmem::kX);
    const int nbk = nb - ch * kMidChunk < kMidChunk ? nb - ch * kMidChunk : kMidChunk;
    for (int bb = 0; bb < nbk; bb++) {
      const unsigned char *tile = slot + bb * 2 * kMidRows * 16;
      const int4 w0 = *(const int4 *)(tile + r * 16), w1 = *(const int4 *)(tile + kMidRows * 16 + r * 16);
      const float dw = __half2float(ss[bb * kMidRows + r]);
#pragma unroll
      for (int j = 0; j < kMidColsPerThread; j++) {
        const int col = q * kMidColsPerThread + j;
        const int4 *xp = (const int4 *)(xs + (col * kMidChunk + bb) * 32);
        const int d = mid_dot32(w0, w1, xp[0], xp[1]);
        // acc += (dw * dx) * dot: three roundings, as q8_gemm_scalar
        acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmul_rn(dw, ds[bb * kMidCols + col]), (float)d));
      }
    }
    __syncthreads();  // the slot may be restaged
  }
  mid_cp_wait<0>();
  const int64_t n = g * SC_GROUP_ROWS + rs * kMidRows + r;
  if (n >= p.rows) return;
#pragma unroll
  for (int j = 0; j < kMidColsPerThread; j++) {
    const int64_t col = col0 + q * kMidColsPerThread + j;
    if (col >= p.m) continue;
    const float v = p.bias ? __fadd_rn(acc[j], p.bias[n]) : acc[j];
    const int64_t idx = p.y_time_major ? col * p.ldy + n : n * p.ldy + col;
    p.y[idx] = apply_epilogue(p.epi, v, idx);
  }
}

static std::atomic<size_t> g_mid_smem_limit[64];  // per device

int mid_gemm_prime() {
  return raise_smem_limit((const void *)q8_gemm_mid_kernel, MidSmem::kBytes, g_mid_smem_limit);
}

int gemm_mid(const MidGemmArgs &a, cudaStream_t st) {
  if (a.m <= 0) return kOk;
  if (a.m_pad % kMidCols || a.m_pad < a.m || a.k_pad != a.w->nb * 32) {
    set_error("q8_gemm_mid: codes must be [m_pad][k_pad] with m_pad a multiple of %d", kMidCols);
    return kErrInvalid;
  }
  const int rc = mid_gemm_prime();
  if (rc) return rc;
  MidParams p{a.w->qs, a.w->sc, a.w->nb, a.w->rows, a.xq, a.dx, a.m, a.m_pad, a.k_pad, a.bias, a.y,
              a.y_time_major, a.ldy, a.epi};
  const dim3 grid((unsigned)(a.w->rows_pad / kMidRows), (unsigned)ceil_div(a.m, kMidCols));  // (group, slice) x frames
  q8_gemm_mid_kernel<<<grid, kMidThreads, MidSmem::kBytes, st>>>(p);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace sc
