// q8_gemm_batch.cu -- many independent small-M Q8_0 GEMMs in one streaming
// pass: y_i = W_i x_i (+ bias_i) for i < n, every x_i with the same frame
// count t <= 16.
//
// A single small-M GEMM moves a few MB of weights, which HBM delivers in well
// under a microsecond; one launch's fixed costs (launch, first bytes' latency,
// the K-split reduction, the tail) are several times that.  Independent
// GEMMs -- the attention's Q, K, V and position projections, one projection
// over many adapters, the layer-shape sweep of the benchmark -- need not pay
// them one by one: here one persistent launch streams all their weights back
// to back, so the HBM stream never stops between matrices.
//
// Arithmetic per output as the single-GEMM streaming kernel (q8_gemm_small.cu):
// exact int8 x int8 block dots (dp4a), acc += (dw * dx) * dot with one fused
// multiply-add per block, f32 accumulation (the reference's SIMD dispatch for
// up to 16 frames sums in another f32 order, simd_kernel.rs:333-393; outputs
// agree within the 1e-4 x RMS bar).  Activations are quantised exactly as
// quantize_col (sgemm_kernel.rs:57-90) by a first launch.
//
// Stream kernel, persistent (one CTA per SM): work unit = (GEMM, 128-row
// group), all of K; units are dealt round-robin.  Warp 0: one thread streams
// each stage -- 8 K blocks of the unit's weight tiles and scales, and the
// same 8 blocks' activation codes and scales -- with bulk copies (no
// multicast) into a ring of shared-memory stages.  The weights never
// change, so the first stages' weights go out before the quantiser has
// finished; their activations follow once it has.  Warps 1-8 compute from
// shared memory only:
//   * 1-2 frames: lane = weight row, 4 row quarters x 2 block parities, dp4a
//     against broadcast activation codes; the two parities' partial sums
//     are added in shared memory at the end;
//   * 4-16 frames: warp w owns 16 of the 128 rows and takes every block: one
//     int8 tensor-core MMA (mma.sync m16n8k32, s32 accumulator cleared per
//     block, so every block's dot is exact) per 8 frames, the weight
//     fragments read straight from the row-group tile layout and the
//     activation fragments from the swizzled code rows (both conflict-free
//     4-byte loads).
//
// Activation codes of one GEMM, per group of 8 K blocks (4 KB, one bulk copy
// per stage): frame j's 256 bytes at j * 256, the block-bb half h (16 bytes)
// in 16-byte unit (2 bb + h) ^ (j % 8), so that the eight frames of an MMA
// fragment read eight different bank groups.  Scales: dx[b * 16 + j].
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

constexpr int kBatchKb = 8;      // K blocks per stage
constexpr int kBatchStages = 5;  // 5 x 39 KB in flight per SM
constexpr int kBatchComputeWarps = 8;
constexpr int kBatchThreads = 32 + 32 * kBatchComputeWarps;
constexpr int kBatchActBytes = kBatchFrames * kBatchKb * 32;  // one stage's activation codes
constexpr int kBatchScOff = kBatchKb * SC_TILE_BYTES;                   // weight scales
constexpr int kBatchActOff = kBatchScOff + kBatchKb * SC_GROUP_ROWS * 2;  // activation codes
constexpr int kBatchDxOff = kBatchActOff + kBatchActBytes;               // activation scales
constexpr int kBatchStage = kBatchDxOff + kBatchKb * kBatchFrames * 4;

// byte offset of activation code (frame j, k index kk) within its GEMM's codes
__device__ __forceinline__ int64_t batch_code_offset(int j, int64_t kk) {
  const int64_t b = kk >> 5;
  const int unit = (int)((b & 7) * 2 + ((kk >> 4) & 1));
  return (b >> 3) * kBatchActBytes + j * 256 + ((unit ^ (j & 7)) << 4) + (kk & 15);
}

static __device__ unsigned g_batch_status;

struct BatchParams {
  int n, t, y_time_major, total_units;
  unsigned *status;
  BatchItem items[kMaxBatch];
};

__device__ __forceinline__ int bdot32(const int4 w0, const int4 w1, const int4 x0, const int4 x1) {
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

// Item owning work unit u (the items' units are consecutive).
__device__ __forceinline__ int batch_item(const BatchParams &p, int u) {
  int lo = 0, hi = p.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.items[mid].unit0 <= u) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Activation codes of every item: one warp per (item, frame < t, block).
// Codes and scales of frames t .. 15 are never written: the stream kernel
// computes those frames' columns from whatever the workspace holds and
// never stores them (every output column depends on its own frame only).
__global__ void batch_quantize_kernel(const __grid_constant__ BatchParams p) {
  const int i = blockIdx.y;
  const BatchItem &it = p.items[i];
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (int64_t)p.t * it.nb) return;
  const int j = (int)(wid / it.nb), b = (int)(wid % it.nb);
  const int64_t kk = (int64_t)b * 32 + lane;
  const bool valid = kk < it.k;
  const float v = valid ? (it.x_feature_major ? it.x[kk * it.ldx + j] : it.x[(int64_t)j * it.ldx + kk]) : 0.0f;
  float s;
  const int8_t q = warp_quantize_block(v, valid, s);
  it.xq[batch_code_offset(j, kk)] = q;
  if (lane == 0) it.dx[(int64_t)b * kBatchFrames + j] = s;
  pdl_launch_dependents();
}

// One m16n8k32 int8 MMA: d = a (16 x 32, row) . b (32 x 8, col), from zero.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0));
}

template <int MT>
__global__ void __launch_bounds__(kBatchThreads, 1) q8_gemm_batch_kernel(const __grid_constant__ BatchParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *full = (uint64_t *)(smem + kBatchStages * kBatchStage);
  uint64_t *empty = full + kBatchStages;
  float *part = (float *)(empty + kBatchStages);  // [8 warps][MT][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBatchStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kBatchComputeWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  bool ok = true;
  if (warp == 0) {
    // ---- producer: weights never change, so they stream before the
    // activation codes' kernel has finished ----
    if (lane == 0) {
      // stage s's activations: codes and scales of blocks b0 .. b0 + nblk
      auto acts = [&](int s, const BatchItem &it, int b0, int nblk) {
        unsigned char *st = smem + s * kBatchStage;
        bulk_g2s(st + kBatchActOff, it.xq + (int64_t)(b0 / kBatchKb) * kBatchActBytes, kBatchActBytes, &full[s]);
        bulk_g2s(st + kBatchDxOff, it.dx + (int64_t)b0 * kBatchFrames, nblk * kBatchFrames * 4, &full[s]);
      };
      // the first ring's worth of stages, whose activations wait for the quantiser
      int held_item[kBatchStages], held_b0[kBatchStages], held_n[kBatchStages];
      bool acts_ready = false;
      auto release_held = [&](int n_held) {
        pdl_wait();  // the activation codes are written
        for (int h = 0; h < n_held; h++) acts(h, p.items[held_item[h]], held_b0[h], held_n[h]);
        acts_ready = true;
      };
      int gs = 0;
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
        const int ii = batch_item(p, u);
        const BatchItem &it = p.items[ii];
        const int64_t g = u - it.unit0;
        for (int b0 = 0; b0 < it.nb; b0 += kBatchKb, gs++) {
          const int s = gs % kBatchStages, nblk = it.nb - b0 < kBatchKb ? it.nb - b0 : kBatchKb;
          if (!acts_ready && gs == kBatchStages) release_held(kBatchStages);
          if (!mbar_wait(&empty[s], ((uint32_t)(gs / kBatchStages) & 1u) ^ 1u)) { ok = false; break; }
          unsigned char *st = smem + s * kBatchStage;
          mbar_arrive_expect_tx(&full[s],
                                nblk * (SC_TILE_BYTES + SC_GROUP_ROWS * 2 + kBatchFrames * 4) + kBatchActBytes);
          bulk_g2s(st, it.qs + (g * it.nb + b0) * SC_TILE_BYTES, nblk * SC_TILE_BYTES, &full[s]);
          bulk_g2s(st + kBatchScOff, it.sc + (g * it.nb + b0) * SC_GROUP_ROWS, nblk * SC_GROUP_ROWS * 2, &full[s]);
          if (acts_ready) {
            acts(s, it, b0, nblk);
          } else {
            held_item[gs] = ii;
            held_b0[gs] = b0;
            held_n[gs] = nblk;
          }
        }
      }
      if (!acts_ready) release_held(gs < kBatchStages ? gs : kBatchStages);
      // the last copies have landed before the CTA can exit
      for (int q = gs - kBatchStages; q < gs; q++)
        if (q >= 0) mbar_wait(&full[q % kBatchStages], (uint32_t)(q / kBatchStages) & 1u);
    }
    __syncwarp();
  } else if constexpr (MT >= 4) {
    // ---- tensor-core path: warp cw owns rows 16 cw .. 16 cw + 15 of the row
    // group; thread (g = lane / 4, q = lane % 4) holds rows 16 cw + g and
    // 16 cw + g + 8 at frames 2 q, 2 q + 1 (+ 8 per further 8-frame tile) ----
    constexpr int NT = MT / 8 > 0 ? MT / 8 : 1;  // 8-frame tiles (MT 4 uses one; columns of frames >= t are not stored)
    const int cw = warp - 1, g = lane >> 2, q = lane & 3;
    const int r0 = 16 * cw + g;
    int gs = 0;
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
      const BatchItem &it = p.items[batch_item(p, u)];
      const int64_t gr = u - it.unit0;
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[nt][e] = 0.0f;
      for (int b0 = 0; b0 < it.nb; b0 += kBatchKb, gs++) {
        const int s = gs % kBatchStages, nblk = it.nb - b0 < kBatchKb ? it.nb - b0 : kBatchKb;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)(gs / kBatchStages) & 1u))) { ok = false; break; }
        const unsigned char *st = smem + s * kBatchStage;
        const __half *scs = (const __half *)(st + kBatchScOff);
        const unsigned char *sa = st + kBatchActOff;
        const float *sdx = (const float *)(st + kBatchDxOff);
        for (int bb = 0; bb < nblk; bb++) {
          uint32_t xb[NT][2];
          float dxv[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            // frame 8 nt + g (frame % 8 == g): block bb's halves in units (2 bb + h) ^ g
            const unsigned char *xr = sa + (8 * nt + g) * 256 + 4 * q;
            xb[nt][0] = *(const uint32_t *)(xr + (((2 * bb) ^ g) << 4));
            xb[nt][1] = *(const uint32_t *)(xr + (((2 * bb + 1) ^ g) << 4));
            dxv[nt][0] = sdx[bb * kBatchFrames + 8 * nt + 2 * q];
            dxv[nt][1] = sdx[bb * kBatchFrames + 8 * nt + 2 * q + 1];
          }
          const unsigned char *tw = st + bb * SC_TILE_BYTES;
          uint32_t a[4];
          a[0] = *(const uint32_t *)(tw + r0 * 16 + 4 * q);
          a[1] = *(const uint32_t *)(tw + (r0 + 8) * 16 + 4 * q);
          a[2] = *(const uint32_t *)(tw + 2048 + r0 * 16 + 4 * q);
          a[3] = *(const uint32_t *)(tw + 2048 + (r0 + 8) * 16 + 4 * q);
          const float dw0 = __half2float(scs[bb * SC_GROUP_ROWS + r0]);
          const float dw1 = __half2float(scs[bb * SC_GROUP_ROWS + r0 + 8]);
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            int d[4];
            mma_s8(d, a, xb[nt]);
            acc[nt][0] = fmaf(dw0 * dxv[nt][0], (float)d[0], acc[nt][0]);
            acc[nt][1] = fmaf(dw0 * dxv[nt][1], (float)d[1], acc[nt][1]);
            acc[nt][2] = fmaf(dw1 * dxv[nt][0], (float)d[2], acc[nt][2]);
            acc[nt][3] = fmaf(dw1 * dxv[nt][1], (float)d[3], acc[nt][3]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      if (!ok) break;
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int64_t n = gr * SC_GROUP_ROWS + r0 + (e >> 1) * 8;
          const int fr = 8 * nt + 2 * q + (e & 1);
          if (fr < p.t && n < it.rows)
            it.y[p.y_time_major ? (int64_t)fr * it.ldy + n : n * it.ldy + fr] =
                acc[nt][e] + (it.bias ? it.bias[n] : 0.0f);
        }
    }
  } else {
    const int cw = warp - 1, rs = cw & 3, kp = cw >> 2;
    const int r = rs * 32 + lane;
    int gs = 0;
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
      const BatchItem &it = p.items[batch_item(p, u)];
      const int64_t g = u - it.unit0;
      float acc[MT];
#pragma unroll
      for (int j = 0; j < MT; j++) acc[j] = 0.0f;
      for (int b0 = 0; b0 < it.nb; b0 += kBatchKb, gs++) {
        const int s = gs % kBatchStages, nblk = it.nb - b0 < kBatchKb ? it.nb - b0 : kBatchKb;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)(gs / kBatchStages) & 1u))) { ok = false; break; }
        const unsigned char *st = smem + s * kBatchStage;
        const __half *scs = (const __half *)(st + kBatchScOff);
        const unsigned char *sa = st + kBatchActOff;
        const float *sdx = (const float *)(st + kBatchDxOff);
        for (int bb = kp; bb < nblk; bb += 2) {
          const unsigned char *tw = st + bb * SC_TILE_BYTES + r * 16;
          const int4 w0 = *(const int4 *)tw, w1 = *(const int4 *)(tw + 2048);
          const float dw = __half2float(scs[bb * SC_GROUP_ROWS + r]);
#pragma unroll
          for (int j = 0; j < MT; j++) {
            const unsigned char *xr = sa + j * 256;
            const int d = bdot32(w0, w1, *(const int4 *)(xr + (((2 * bb) ^ j) << 4)),
                                 *(const int4 *)(xr + (((2 * bb + 1) ^ j) << 4)));
            acc[j] = fmaf(dw * sdx[bb * kBatchFrames + j], (float)d, acc[j]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      if (!ok) break;
      // the two block parities' partial sums, then y (+ bias)
#pragma unroll
      for (int j = 0; j < MT; j++) part[(cw * MT + j) * 32 + lane] = acc[j];
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kBatchComputeWarps) : "memory");
      if (kp == 0) {
        const int64_t n = g * SC_GROUP_ROWS + r;
        if (n < it.rows) {
          const float bn = it.bias ? it.bias[n] : 0.0f;
#pragma unroll
          for (int j = 0; j < MT; j++)
            if (j < p.t) {
              const float v = part[(cw * MT + j) * 32 + lane] + part[((cw + 4) * MT + j) * 32 + lane] + bn;
              it.y[p.y_time_major ? (int64_t)j * it.ldy + n : n * it.ldy + j] = v;
            }
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kBatchComputeWarps) : "memory");
    }
  }
  if (!ok) atomicOr(p.status, kStatusWaitTimeout);
}

static unsigned *batch_status_ptr() {
  static std::atomic<unsigned *> ptr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned *q = ptr[dev].load(std::memory_order_acquire);
  if (!q) {
    void *a = nullptr;
    if (cudaGetSymbolAddress(&a, g_batch_status) != cudaSuccess) return nullptr;
    q = (unsigned *)a;
    ptr[dev].store(q, std::memory_order_release);
  }
  return q;
}

template <int MT>
static std::atomic<size_t> *batch_smem_limit() {
  static std::atomic<size_t> limit[64];
  return limit;
}

constexpr size_t kBatchSmem = (size_t)kBatchStages * kBatchStage + 16 * kBatchStages +
                              (size_t)kBatchComputeWarps * 2 * 32 * 4;

template <int MT>
static int launch_batch(const BatchParams &p, int sm_count, cudaStream_t st) {
  auto kern = q8_gemm_batch_kernel<MT>;
  const int rc = raise_smem_limit((const void *)kern, kBatchSmem, batch_smem_limit<MT>());
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.total_units < sm_count ? p.total_units : sm_count), 1, 1);
  cfg.blockDim = dim3(kBatchThreads, 1, 1);
  cfg.dynamicSmemBytes = kBatchSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  SC_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
  return kOk;
}

int batch_gemm_status(unsigned *out) {
  unsigned v = 0, zero = 0;
  SC_CUDA(cudaMemcpyFromSymbol(&v, g_batch_status, sizeof(v)));
  SC_CUDA(cudaMemcpyToSymbol(g_batch_status, &zero, sizeof(zero)));
  *out = v;
  return kOk;
}

// per GEMM: its activation codes in whole 8-block groups, then its scales
static size_t batch_code_bytes(int64_t nb) { return (size_t)ceil_div(nb, kBatchKb) * kBatchActBytes; }
static size_t batch_dx_bytes(int64_t nb) { return ((size_t)kBatchFrames * nb * 4 + 255) / 256 * 256; }

size_t batch_ws_bytes(const BatchItem *items, int n) {
  size_t bytes = 0;
  for (int i = 0; i < n; i++) bytes += batch_code_bytes(items[i].nb) + batch_dx_bytes(items[i].nb);
  return bytes;
}

int gemm_batch(BatchItem *items, int n, int t, int y_time_major, void *ws, size_t ws_bytes, int sm_count,
               cudaStream_t st) {
  if (n <= 0 || n > kMaxBatch || t <= 0 || t > kBatchFrames) {
    set_error("q8_gemm_batch: 1..%d GEMMs of 1..%d frames", kMaxBatch, kBatchFrames);
    return kErrInvalid;
  }
  if (ws_bytes < batch_ws_bytes(items, n) || ((uintptr_t)ws & 255)) {
    set_error("q8_gemm_batch: workspace needs %zu bytes at 256-byte alignment", batch_ws_bytes(items, n));
    return kErrInvalid;
  }
  BatchParams p{};
  p.n = n;
  p.t = t;
  p.y_time_major = y_time_major;
  p.status = batch_status_ptr();
  if (!p.status) {
    set_error("q8_gemm_batch: status word lookup failed");
    return kErrCuda;
  }
  char *w = (char *)ws;
  int units = 0, nb_max = 0;
  for (int i = 0; i < n; i++) {
    BatchItem it = items[i];
    it.xq = (int8_t *)w;
    w += batch_code_bytes(it.nb);
    it.dx = (float *)w;
    w += batch_dx_bytes(it.nb);
    it.unit0 = units;
    units += it.groups;
    nb_max = it.nb > nb_max ? it.nb : nb_max;
    p.items[i] = it;
  }
  p.total_units = units;
  dim3 qgrid((unsigned)ceil_div((int64_t)t * nb_max * 32, 256), (unsigned)n);
  batch_quantize_kernel<<<qgrid, 256, 0, st>>>(p);
  note_launch();
  SC_CUDA(cudaGetLastError());
  const int mt = t <= 1 ? 1 : t <= 2 ? 2 : t <= 4 ? 4 : t <= 8 ? 8 : 16;
  switch (mt) {
    case 1: return launch_batch<1>(p, sm_count, st);
    case 2: return launch_batch<2>(p, sm_count, st);
    case 4: return launch_batch<4>(p, sm_count, st);
    case 8: return launch_batch<8>(p, sm_count, st);
    default: return launch_batch<16>(p, sm_count, st);
  }
}

}  // namespace sc
