// q8_gemm_small.cu -- weight-streaming Q8_0 GEMM for small M (frames x
// streams up to a few dozen): the bandwidth-bound streaming-chunk case.
//
// Computes y[col, n] = sum_b dw[n, b] * dx[col, b] * sum_{i<32} w[n, 32b+i] *
// xq[col, 32b+i] (+ bias[n]) -- the arithmetic of sgemm_kernel.rs:156-201 and
// simd_kernel.rs:333-393: exact int8 x int8 block dots (dp4a, int32), one f32
// scale product per (row, column, block), f32 accumulation.
//
// A CTA owns one 128-row tile group and a slice of the K blocks:
//   1. one thread issues two 1-D bulk copies (TMA engine, no multicast) of the
//      slice's weight tiles and scales -- contiguous in the row-group tile
//      layout -- into shared memory, then the CTA lets the next kernel launch
//      (programmatic dependent launch) and waits for the previous one, so
//      the weight stream overlaps the previous kernel's tail;
//   2. the CTA quantises its frames' K slice itself (bit-exact quantize_col,
//      one warp per 32-block), so no separate quantiser launch or global
//      scratch is needed;
//   3. 8 warps (4 row subgroups x 2 block parities) run dp4a block dots from
//      shared memory -- lane = weight row, 16-byte conflict-free reads, the
//      activations a broadcast -- with one f32 FMA per (row, frame, block);
//   4. partial sums are reduced over the warps in shared memory and over the
//      K-split CTAs of the thread-block cluster through distributed shared
//      memory: deterministic, no atomics.
#include <cooperative_groups.h>

#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace cg = cooperative_groups;

namespace sc {

// Build-time tuning knobs (defaults are the measured best).
#ifndef SC_STREAM_KS_MAX
#define SC_STREAM_KS_MAX 8  // largest K split (cluster size)
#endif
#ifndef SC_STREAM_PDL
#define SC_STREAM_PDL 1     // launch with programmatic stream serialization
#endif

constexpr int kStreamThreads = 256;
constexpr int kNblCap = 40;  // K blocks per CTA slice (shared-memory bound)

static __device__ unsigned g_small_status;

struct StreamParams {
  const int8_t *qs;
  const __half *sc;
  int64_t nb, n_rows, k;
  const float *x;       // f32 activations (quantised in-kernel), or nullptr
  int64_t ldx;
  int x_feature_major;
  const int8_t *xq;     // pre-quantised [m_pad][k_pad] when x == nullptr
  const float *dx;      // [nb][m_pad]
  int64_t k_pad, m_pad;
  int64_t m;
  const float *bias;
  float *y;
  int y_time_major;
  int64_t ldy;
  int ks, nbl_max;
  int32_t *dots;
  unsigned *status;
  Epilogue epi;
};

__device__ __forceinline__ int dot32(const int4 w0, const int4 w1, const int4 x0, const int4 x1) {
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

// kDump: write the raw int32 block dots (dots[(n*m + col)*nb + b]) instead of
// y -- the same integer path, exposed so tests can check it bit for bit.
template <int MT, bool kDump>
__global__ void __launch_bounds__(kStreamThreads)
    q8_gemm_stream_kernel(const __grid_constant__ StreamParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t g = blockIdx.x;
  const int split = blockIdx.y;
  const int64_t col0 = (int64_t)blockIdx.z * MT;
  const int64_t b0 = p.nb * split / p.ks, b1 = p.nb * (split + 1) / p.ks;
  const int nbl = (int)(b1 - b0);

  unsigned char *wbuf = smem;                                    // [nbl][4096]
  __half *sbuf = (__half *)(smem + (size_t)p.nbl_max * SC_TILE_BYTES);  // [nbl][128]
  int8_t *xs = (int8_t *)(sbuf + (size_t)p.nbl_max * SC_GROUP_ROWS);   // [MT][nbl*32]
  float *dxs = (float *)(xs + (size_t)MT * p.nbl_max * 32);      // [nbl][MT]
  // partial sums (then the barrier) at the next 16-byte boundary: the scales
  // before them take nbl_max * MT * 4 bytes, not always a multiple of 8
  float *part = (float *)(((uintptr_t)(dxs + (size_t)p.nbl_max * MT) + 15) & ~(uintptr_t)15);  // [8][MT][32]
  uint64_t *bar = (uint64_t *)(part + 8 * MT * 32);

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t wbytes = (uint32_t)nbl * SC_TILE_BYTES, sbytes = (uint32_t)nbl * SC_GROUP_ROWS * 2;
    mbar_arrive_expect_tx(bar, wbytes + sbytes);
    bulk_g2s(wbuf, p.qs + (g * p.nb + b0) * SC_TILE_BYTES, wbytes, bar);
    bulk_g2s(sbuf, p.sc + (g * p.nb + b0) * SC_GROUP_ROWS, sbytes, bar);
  }
  // Weights and scales are never written by a kernel, so they may be fetched
  // before the previous kernel (which may produce x) has finished.
  pdl_launch_dependents();
  pdl_wait();

  // ---- activations of this CTA's frames and K slice -> shared memory ----
  // Each warp first issues the loads of up to 8 (frame, block) pairs, then
  // quantises them, so the loads' latencies overlap instead of adding up.
  if (p.x) {
    constexpr int kPairs = 8;
    const int npairs = MT * nbl;
    for (int base = warp; base < npairs; base += kPairs * (kStreamThreads / 32)) {
      float v[kPairs];
      bool valid[kPairs];
#pragma unroll
      for (int i = 0; i < kPairs; i++) {
        const int pair = base + i * (kStreamThreads / 32);
        const int j = pair / nbl, bb = pair % nbl;
        const int64_t col = col0 + j, kk = (b0 + bb) * 32 + lane;
        valid[i] = pair < npairs && col < p.m && kk < p.k;
        v[i] = 0.0f;
        if (valid[i]) v[i] = p.x_feature_major ? p.x[kk * p.ldx + col] : p.x[col * p.ldx + kk];
      }
#pragma unroll
      for (int i = 0; i < kPairs; i++) {
        const int pair = base + i * (kStreamThreads / 32);
        if (pair >= npairs) break;
        const int j = pair / nbl, bb = pair % nbl;
        float sblk;
        const int8_t q = warp_quantize_block(v[i], valid[i], sblk);
        xs[(size_t)j * nbl * 32 + bb * 32 + lane] = q;
        if (lane == 0) dxs[bb * MT + j] = col0 + j < p.m ? sblk : 0.0f;
      }
    }
  } else {
    for (int i = tid; i < MT * nbl * 2; i += kStreamThreads) {
      const int j = i / (nbl * 2), c16 = i % (nbl * 2);
      const int64_t col = col0 + j;
      int4 v = make_int4(0, 0, 0, 0);
      if (col < p.m_pad) v = *(const int4 *)(p.xq + col * p.k_pad + b0 * 32 + c16 * 16);
      *(int4 *)(xs + (size_t)j * nbl * 32 + c16 * 16) = v;
    }
    for (int i = tid; i < nbl * MT; i += kStreamThreads) {
      const int bb = i / MT, j = i % MT;
      const int64_t col = col0 + j;
      dxs[i] = col < p.m_pad ? p.dx[(b0 + bb) * p.m_pad + col] : 0.0f;
    }
  }
  __syncthreads();
  if (!mbar_wait(bar, 0) && lane == 0) atomicOr(p.status, kStatusWaitTimeout);

  // ---- dp4a block dots ----
  const int rs = warp & 3, kp = warp >> 2;
  const int r = rs * 32 + lane;
  float acc[MT];
#pragma unroll
  for (int j = 0; j < MT; j++) acc[j] = 0.0f;
#pragma unroll 2
  for (int bb = kp; bb < nbl; bb += 2) {
    const unsigned char *t = wbuf + (size_t)bb * SC_TILE_BYTES + r * 16;
    const int4 w0 = *(const int4 *)t, w1 = *(const int4 *)(t + 2048);
    const float dw = __half2float(sbuf[bb * SC_GROUP_ROWS + r]);
#pragma unroll
    for (int j = 0; j < MT; j++) {
      const int4 *xp = (const int4 *)(xs + (size_t)j * nbl * 32 + bb * 32);
      const int d = dot32(w0, w1, xp[0], xp[1]);
      if constexpr (kDump) {
        const int64_t n = g * SC_GROUP_ROWS + r, col = col0 + j;
        if (n < p.n_rows && col < p.m) p.dots[(n * p.m + col) * p.nb + b0 + bb] = d;
      } else {
        acc[j] = fmaf(dw * dxs[bb * MT + j], (float)d, acc[j]);
      }
    }
  }
  if constexpr (!kDump) {
  // ---- reductions: block parities, then the cluster's K splits ----
#pragma unroll
  for (int j = 0; j < MT; j++) part[(warp * MT + j) * 32 + lane] = acc[j];
  __syncthreads();
  if (warp < 4) {
#pragma unroll
    for (int j = 0; j < MT; j++)
      part[(warp * MT + j) * 32 + lane] += part[((warp + 4) * MT + j) * 32 + lane];
  }
  // Reduce-scatter over the cluster's K splits: rank q sums rows
  // [q*128/ks, (q+1)*128/ks) of every split (all remote loads in flight at
  // once) and writes them, so no rank gathers the whole tile serially.
  cg::cluster_group cluster = cg::this_cluster();
  if (p.ks > 1)
    cluster.sync();
  else
    __syncthreads();
  const int rows_per = SC_GROUP_ROWS / p.ks;
  for (int e = tid; e < rows_per * MT; e += kStreamThreads) {
    const int rr = split * rows_per + e / MT, j = e % MT;  // row in tile, frame
    const int idx = ((rr >> 5) * MT + j) * 32 + (rr & 31);
    float v = part[idx];
    if (p.ks > 1) {
      float rv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) rv[q] = (q < p.ks && q != split) ? cluster.map_shared_rank(part, q)[idx] : 0.0f;
      v = 0.0f;
#pragma unroll
      for (int q = 0; q < 8; q++) v += q == split ? part[idx] : rv[q];
    }
    const int64_t n = g * SC_GROUP_ROWS + rr, col = col0 + j;
    if (n < p.n_rows && col < p.m) {
      v += p.bias ? p.bias[n] : 0.0f;
      const int64_t idx = p.y_time_major ? col * p.ldy + n : n * p.ldy + col;
      p.y[idx] = apply_epilogue(p.epi, v, idx);
    }
  }
  if (p.ks > 1) cluster.sync();  // keep this CTA's partials alive for its peers
  }
}

static size_t stream_smem(int mt, int nbl_max) {
  return (size_t)nbl_max * (SC_TILE_BYTES + SC_GROUP_ROWS * 2) + (size_t)mt * nbl_max * 32 +
         (size_t)nbl_max * mt * 4 + 16 + (size_t)8 * mt * 32 * 4 + 16;  // + alignment pad, barrier
}

// Shared-memory limit raised so far per device, per kernel instance.
template <int MT, bool kDump>
static std::atomic<size_t> *stream_smem_limit() {
  static std::atomic<size_t> limit[64];
  return limit;
}

template <int MT, bool kDump>
static int launch_stream(StreamParams &p, int64_t groups, int64_t mtiles, cudaStream_t st) {
  auto kern = q8_gemm_stream_kernel<MT, kDump>;
  const size_t smem = stream_smem(MT, p.nbl_max);
  const int rc = raise_smem_limit((const void *)kern, smem, stream_smem_limit<MT, kDump>());
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)groups, (unsigned)p.ks, (unsigned)mtiles);
  cfg.blockDim = dim3(kStreamThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.ks;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  // no cluster without a K split: the kernel then syncs only its own CTA
  cfg.attrs = p.ks > 1 ? attr : attr + 1;
  cfg.numAttrs = (p.ks > 1 ? 1 : 0) + (SC_STREAM_PDL ? 1 : 0);
  note_launch();
  SC_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
  return kOk;
}

static unsigned *small_status_ptr() {
  static std::atomic<unsigned *> ptr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned *q = ptr[dev].load(std::memory_order_acquire);
  if (!q) {
    void *a = nullptr;
    if (cudaGetSymbolAddress(&a, g_small_status) != cudaSuccess) return nullptr;
    q = (unsigned *)a;
    ptr[dev].store(q, std::memory_order_release);  // every caller stores the same address
  }
  return q;
}

template <int MT>
static int prime_stream() {
  return raise_smem_limit((const void *)q8_gemm_stream_kernel<MT, false>, stream_smem(MT, kNblCap),
                          stream_smem_limit<MT, false>());
}

int small_gemm_prime() {
  if (!small_status_ptr()) {
    set_error("q8_gemm: status word lookup failed");
    return kErrCuda;
  }
  int rc = prime_stream<1>();
  if (!rc) rc = prime_stream<2>();
  if (!rc) rc = prime_stream<4>();
  if (!rc) rc = prime_stream<8>();
  if (!rc) rc = prime_stream<16>();
  return rc;
}

int small_gemm_status(unsigned *out) {
  unsigned v = 0, zero = 0;
  SC_CUDA(cudaMemcpyFromSymbol(&v, g_small_status, sizeof(v)));
  SC_CUDA(cudaMemcpyToSymbol(g_small_status, &zero, sizeof(zero)));
  *out = v;
  return kOk;
}

int gemm_small(const SmallGemmArgs &a, int sm_count, cudaStream_t st) {
  const Q8Weights *w = a.w;
  const int mt = a.m <= 1 ? 1 : a.m <= 2 ? 2 : a.m <= 4 ? 4 : a.m <= 8 ? 8 : 16;
  const int64_t mtiles = ceil_div(a.m, mt);
  const int64_t groups = w->rows_pad / SC_GROUP_ROWS;
  // K split (a cluster dimension, at most 8): smallest power of two that
  // fills the GPU, keeps at least two blocks per CTA and fits shared memory.
  // One or two frames with a K that fits one CTA: no split (measured: the
  // cluster reduction costs more than the extra parallelism buys there).
  int ks = 1;
  const bool no_split = a.m <= 2 && w->nb <= kNblCap;
  while (ks < SC_STREAM_KS_MAX && (ceil_div(w->nb, ks) > kNblCap ||
                    (!no_split && groups * mtiles * ks < sm_count && w->nb / (ks * 2) >= 2)))
    ks *= 2;
  if (ceil_div(w->nb, ks) > kNblCap || ks > 8) {
    set_error("q8_gemm: K=%lld too large for the streaming kernel", (long long)w->k);
    return kErrUnsupported;
  }
  unsigned *status = small_status_ptr();
  if (!status) {
    set_error("q8_gemm: status word lookup failed");
    return kErrCuda;
  }
  StreamParams p{};
  p.qs = w->qs;
  p.sc = w->sc;
  p.nb = w->nb;
  p.n_rows = w->rows;
  p.k = w->k;
  p.x = a.x;
  p.ldx = a.ldx;
  p.x_feature_major = a.x_feature_major;
  p.xq = a.xq;
  p.dx = a.dx;
  p.k_pad = a.k_pad;
  p.m_pad = a.m_pad;
  p.m = a.m;
  p.bias = a.bias;
  p.y = a.y;
  p.y_time_major = a.y_time_major;
  p.ldy = a.ldy;
  p.ks = ks;
  p.nbl_max = (int)ceil_div(w->nb, ks);
  p.dots = a.dots;
  p.status = status;
  p.epi = a.epi;
  if (a.dots) {
    switch (mt) {
      case 1: return launch_stream<1, true>(p, groups, mtiles, st);
      case 2: return launch_stream<2, true>(p, groups, mtiles, st);
      case 4: return launch_stream<4, true>(p, groups, mtiles, st);
      case 8: return launch_stream<8, true>(p, groups, mtiles, st);
      default: return launch_stream<16, true>(p, groups, mtiles, st);
    }
  }
  switch (mt) {
    case 1: return launch_stream<1, false>(p, groups, mtiles, st);
    case 2: return launch_stream<2, false>(p, groups, mtiles, st);
    case 4: return launch_stream<4, false>(p, groups, mtiles, st);
    case 8: return launch_stream<8, false>(p, groups, mtiles, st);
    default: return launch_stream<16, false>(p, groups, mtiles, st);
  }
}

}  // namespace sc
