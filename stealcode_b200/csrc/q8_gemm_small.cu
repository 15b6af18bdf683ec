// q8_gemm_small.cu -- weight-streaming Q8_0 GEMM for small M (frames x
// streams up to a few dozen): the bandwidth-bound streaming-chunk case.
//
// Computes y[col, n] = sum_b dw[n, b] * dx[col, b] * sum_{i<32} w[n, 32b+i] *
// xq[col, 32b+i] (+ bias[n]) -- the arithmetic of sgemm_kernel.rs:156-201 and
// simd_kernel.rs:333-393: exact int8 x int8 block dots (dp4a, int32), one f32
// scale product per (row, column, block), f32 accumulation.
//
// Mapping: a CTA owns 32 weight rows (lane = row) and a slice of the K
// blocks; its 4 warps take interleaved blocks of that slice and each lane
// reads its row's 32-byte block as two 16-byte loads that are 512 contiguous
// bytes per warp (row-group tile layout, sc_common.cuh).  The quantised
// activations of the CTA's K slice sit in shared memory and every lane reads
// the same 32 bytes per block (a broadcast).  Partial sums are reduced over
// the 4 warps through shared memory and over the K-split CTAs of a thread
// block cluster through distributed shared memory -- no atomics, no global
// scratch, deterministic.
#include <cooperative_groups.h>

#include "sc_kernels.cuh"

namespace cg = cooperative_groups;

namespace sc {

constexpr int kSmallWarps = 4;
constexpr int kUnroll = 4;

__device__ __forceinline__ int dot32(const int4 w0, const int4 w1, const int4 x0,
                                     const int4 x1) {
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

__device__ __forceinline__ int4 ldg_stream(const int8_t *p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// kDumpDots: instead of the scaled sum, write the raw int32 block dots
// (dots[(n * m + col) * nb + b]) -- the same integer path, exposed so tests
// can check the block dots bit for bit.
template <int MT, bool kDumpDots>
__global__ void __launch_bounds__(kSmallWarps * 32)
    q8_gemm_small_kernel(const int8_t *__restrict__ qs,
                         const __half *__restrict__ scl, int64_t nb,
                         const int8_t *__restrict__ xq,
                         const float *__restrict__ dx, int64_t k_pad,
                         int64_t m_pad, int64_t m,
                         const float *__restrict__ bias, float *__restrict__ y,
                         int64_t n_rows, int y_time_major, int64_t ldy,
                         int ks, int32_t *__restrict__ dots) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rg = blockIdx.x;               // 32-row group
  const int split = blockIdx.y;                // K split = cluster rank
  const int64_t col0 = (int64_t)blockIdx.z * MT;
  const int64_t g = rg >> 2;                   // 128-row tile group
  const int sub = (int)(rg & 3);               // 32-row subgroup in the tile
  const int r = sub * 32 + lane;               // row inside the tile
  const int64_t b0 = nb * split / ks, b1 = nb * (split + 1) / ks;
  const int nbl = (int)(b1 - b0);

  // Shared: xq slice [MT][nbl*32] bytes, dx slice [nbl][MT], partials.
  int8_t *xs = (int8_t *)smem;
  float *dxs = (float *)(smem + (size_t)MT * nbl * 32);
  float *part = dxs + (size_t)nbl * MT;        // [kSmallWarps][MT][32]

  for (int i = threadIdx.x; i < MT * nbl * 2; i += blockDim.x) {
    int mm = i / (nbl * 2), c16 = i % (nbl * 2);
    int64_t col = col0 + mm;
    int4 v = make_int4(0, 0, 0, 0);
    if (col < m_pad) v = *(const int4 *)(xq + col * k_pad + b0 * 32 + c16 * 16);
    *(int4 *)(xs + (size_t)mm * nbl * 32 + c16 * 16) = v;
  }
  for (int i = threadIdx.x; i < nbl * MT; i += blockDim.x) {
    int bb = i / MT, mm = i % MT;
    int64_t col = col0 + mm;
    dxs[i] = col < m_pad ? dx[(b0 + bb) * m_pad + col] : 0.0f;
  }
  __syncthreads();

  float acc[MT];
#pragma unroll
  for (int j = 0; j < MT; j++) acc[j] = 0.0f;

  const int8_t *tile0 = qs + (g * nb) * SC_TILE_BYTES + r * 16;
  const __half *sc0 = scl + (g * nb) * SC_GROUP_ROWS + r;

  // Blocks of this warp: b0 + warp, b0 + warp + 4, ...  Loads for kUnroll
  // blocks are issued before their math so each lane keeps 128 bytes in
  // flight.
  for (int bb = warp; bb < nbl; bb += kSmallWarps * kUnroll) {
    int4 w0[kUnroll], w1[kUnroll];
    float dw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      int bu = bb + u * kSmallWarps;
      if (bu < nbl) {
        const int8_t *t = tile0 + (b0 + bu) * SC_TILE_BYTES;
        w0[u] = ldg_stream(t);
        w1[u] = ldg_stream(t + 2048);
        dw[u] = __half2float(sc0[(b0 + bu) * SC_GROUP_ROWS]);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      int bu = bb + u * kSmallWarps;
      if (bu < nbl) {
#pragma unroll
        for (int j = 0; j < MT; j++) {
          const int4 *xp = (const int4 *)(xs + (size_t)j * nbl * 32 + bu * 32);
          int d = dot32(w0[u], w1[u], xp[0], xp[1]);
          if constexpr (kDumpDots) {
            int64_t n = g * SC_GROUP_ROWS + r, col = col0 + j;
            if (n < n_rows && col < m) dots[(n * m + col) * nb + b0 + bu] = d;
          } else {
            float s = dw[u] * dxs[bu * MT + j];
            acc[j] = fmaf(s, (float)d, acc[j]);
          }
        }
      }
    }
  }
  if constexpr (!kDumpDots) {
    // Reduce the 4 warps' partials.
#pragma unroll
    for (int j = 0; j < MT; j++) part[(warp * MT + j) * 32 + lane] = acc[j];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < MT; j++) {
        float v = part[j * 32 + lane];
#pragma unroll
        for (int w = 1; w < kSmallWarps; w++) v += part[(w * MT + j) * 32 + lane];
        part[j * 32 + lane] = v;
      }
    }
    // Reduce over the cluster's K splits (rank 0 collects).
    if (ks > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      if (split == 0 && warp == 0) {
        for (int q = 1; q < ks; q++) {
          float *rp = cluster.map_shared_rank(part, q);
#pragma unroll
          for (int j = 0; j < MT; j++) part[j * 32 + lane] += rp[j * 32 + lane];
        }
      }
      cluster.sync();
    } else {
      __syncthreads();
    }
    if (split != 0 || warp != 0) return;
    const int64_t n = g * SC_GROUP_ROWS + r;
    if (n >= n_rows) return;
    const float bn = bias ? bias[n] : 0.0f;
#pragma unroll
    for (int j = 0; j < MT; j++) {
      int64_t col = col0 + j;
      if (col < m) {
        float v = part[j * 32 + lane] + bn;
        if (y_time_major)
          y[col * ldy + n] = v;
        else
          y[n * ldy + col] = v;
      }
    }
  }
}

static int pick_ks(int64_t row_groups, int64_t nb, int64_t mtiles, int sm_count) {
  // Aim for about two CTAs per SM with at least 8 K blocks per CTA (two per
  // warp); the split is a cluster dimension, so at most 8.
  int ks = 1;
  while (ks < 8 && row_groups * mtiles * ks < 2 * sm_count && nb / (ks * 2) >= 8) ks *= 2;
  return ks;
}

template <int MT, bool kDump>
static int launch_small(const SmallGemmArgs &a, int ks, cudaStream_t st) {
  const Q8Weights *w = a.w;
  int64_t row_groups = w->rows_pad / 32;
  int64_t mtiles = ceil_div(a.m, MT);
  int64_t nbl_max = ceil_div(w->nb, ks);
  size_t smem = (size_t)MT * nbl_max * 32 + (size_t)nbl_max * MT * 4 +
                (size_t)kSmallWarps * MT * 32 * 4;
  auto kern = q8_gemm_small_kernel<MT, kDump>;
  // Raise the dynamic shared-memory limit once per device (not inside every
  // launch, so graph capture sees only the launch itself).
  static size_t smem_set[64] = {};
  int dev = 0;
  SC_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && dev < 64 && smem_set[dev] < smem) {
    SC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)row_groups, (unsigned)ks, (unsigned)mtiles);
  cfg.blockDim = dim3(kSmallWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)ks;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SC_CUDA(cudaLaunchKernelEx(&cfg, kern, (const int8_t *)w->qs, (const __half *)w->sc,
                             w->nb, a.xq, a.dx, a.k_pad, a.m_pad, a.m, a.bias, a.y,
                             w->rows, a.y_time_major, a.ldy, ks, a.dots));
  return kOk;
}

int gemm_small(const SmallGemmArgs &a, int sm_count, cudaStream_t st) {
  int mt = a.m <= 1 ? 1 : a.m <= 2 ? 2 : a.m <= 4 ? 4 : a.m <= 8 ? 8 : 16;
  int64_t mtiles = ceil_div(a.m, mt);
  int ks = pick_ks(a.w->rows_pad / 32, a.w->nb, mtiles, sm_count);
  // Shared memory must hold the K slice of xq for MT columns.
  while (ks < 8 && (size_t)mt * ceil_div(a.w->nb, ks) * 36 > 160 * 1024) ks *= 2;
  if ((size_t)mt * ceil_div(a.w->nb, ks) * 36 > 200 * 1024) {
    set_error("q8_gemm: K=%lld too large for the small-M kernel", (long long)a.w->k);
    return kErrUnsupported;
  }
  if (a.dots) {
    switch (mt) {
      case 1: return launch_small<1, true>(a, ks, st);
      case 2: return launch_small<2, true>(a, ks, st);
      case 4: return launch_small<4, true>(a, ks, st);
      case 8: return launch_small<8, true>(a, ks, st);
      default: return launch_small<16, true>(a, ks, st);
    }
  }
  switch (mt) {
    case 1: return launch_small<1, false>(a, ks, st);
    case 2: return launch_small<2, false>(a, ks, st);
    case 4: return launch_small<4, false>(a, ks, st);
    case 8: return launch_small<8, false>(a, ks, st);
    default: return launch_small<16, false>(a, ks, st);
  }
}

}  // namespace sc
