// q8_gemm_tc.cu -- large-M Q8_0 GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in tensor memory).
//
// Same arithmetic as the reference (sgemm_kernel.rs:156-201): for every 32-wide
// K block the exact int32 dot of int8 weights and int8 activation codes, scaled
// by dw[n, b] * dx[col, b] and accumulated in f32.  Because each K block has
// its own pair of scales, the int32 accumulator cannot run across blocks:
// every tcgen05.mma covers exactly one block (M = 128 weight rows, N = FT
// frames, K = 32) into a fresh TMEM buffer, and drain warps read it back
// (tcgen05.ld), scale it and add it to f32 accumulators in registers while the
// tensor core already computes the next block into the other buffer.
//
// CTA roles (warp-specialised, one CTA per 128-row group x FT-frame tile):
//   warp 0       producer: 1-D bulk copies (TMA engine, no multicast) into a
//                ring of shared-memory stages of kTcKb K blocks each: the
//                blocks' weight tiles (the row-group tile layout is already
//                the no-swizzle K-major UMMA operand layout), activation
//                tiles, weight scales and activation scales, one copy each;
//   warp 1       allocates TMEM and issues one tcgen05.mma per block (single
//                thread) into a rotating TMEM accumulator, committing to the
//                accumulator's "full" barrier, and to the stage's "empty"
//                barrier after the stage's last block;
//   warps 2..    drain warpgroups: each thread owns one weight row (TMEM lane)
//                and 32 frame columns; per block it reads the accumulator
//                (tcgen05.ld), releases it, and applies the block's scales in
//                packed f32x2 arithmetic in the reference scalar oracle's
//                order; the int32 -> f32 conversion is an exact integer add.
// Every mbarrier wait is bounded; a wait that gives up sets a status bit and
// the kernel runs to its end without waiting again, so it cannot hang.
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

// K blocks per shared-memory stage: one bulk copy per operand moves
// kTcKb consecutive blocks (weight tiles, activation tiles and both scale
// rows are contiguous in their layouts), so a stage costs four copies for
// kTcKb blocks.  Bulk copies issued by one thread complete one after
// another, so each (copy kind, stage phase) pair has its own producer lane.
#ifndef SC_TC_KB
#define SC_TC_KB 4
#endif
#ifndef SC_TC_STAGES
#define SC_TC_STAGES 4
#endif
#ifndef SC_TC_PHASES
#define SC_TC_PHASES 2
#endif
constexpr int kTcKb = SC_TC_KB;
constexpr int kTcStages = SC_TC_STAGES;
constexpr int kTcPhases = SC_TC_PHASES;
static_assert(kTcStages >= kTcPhases, "every producer phase needs a stage in flight");
// TMEM accumulators (FT columns each): the MMA of a block may start once
// the drain has read the accumulator it reuses.  128-frame tiles take all
// 512 columns (one CTA per SM); 64-frame tiles take 256, so two CTAs share
// an SM (their drains run independently, and twice as many tiles per wave
// even out the last wave of a grid of a few hundred tiles).
template <int FT>
constexpr int tc_acc_bufs() { return FT == 64 ? 4 : (512 / FT < 8 ? 512 / FT : 8); }
template <int FT>
constexpr int tc_ctas_per_sm() { return FT == 64 ? 2 : 1; }

static __device__ unsigned g_tc_status;

struct TcParams {
  const int8_t *qs;      // weight tiles
  const __half *sc;      // weight scales [g][b][128]
  int64_t nb, n_rows;
  const int8_t *xq;      // activation tiles [t_pad/FT][nb][2][FT][16]
  const float *dx;       // activation scales [nb][t_pad]
  int64_t t, t_pad;
  const float *bias;
  float *y;
  int y_time_major;
  int64_t ldy;
  unsigned *status;
  Epilogue epi;
  QOut qout;
  float neg_zero;  // -0.0f, opaque to the compiler (see the drain)
};

// ---- tcgen05 wrappers -----------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, no swizzle, K-major canonical layout:
// core matrices of 8 rows x 16 bytes, `lbo` bytes between the two 16-byte
// K halves, `sbo` bytes between consecutive 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(const void *smem, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_u32(smem);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;               // base offset 0, layout type 0 = no swizzle
}

// Instruction descriptor: kind::i8, D = s32, A = B = signed int8, both
// K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int FT, int DWG>
struct TcSmem {
  static constexpr int kA = SC_TILE_BYTES * kTcKb;      // kTcKb tiles of 128 x 32 int8
  static constexpr int kB = FT * 32 * kTcKb;            // kTcKb tiles of FT x 32 int8
  static constexpr int kS = SC_GROUP_ROWS * 2 * kTcKb;  // f16 weight scales [kTcKb][128]
  static constexpr int kD = FT * 4 * kTcKb;             // f32 activation scales [kTcKb][FT]
  static constexpr int kStage = kA + kB + kS + kD;      // all multiples of 16
  static constexpr int kAcc = tc_acc_bufs<FT>();
  static constexpr int kBars = 8 * (2 * kTcStages + 2 * kAcc) + 16;
  static constexpr int kBytes = kTcStages * kStage + kBars;
};

// Packed f32x2 arithmetic (two lanes of f32 per 64-bit register pair).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int FT, int DWG>
__global__ void __launch_bounds__(64 + 128 * DWG, tc_ctas_per_sm<FT>()) q8_gemm_tc_kernel(const __grid_constant__ TcParams p) {
  using L = TcSmem<FT, DWG>;
  static_assert(FT == 32 * DWG, "each drain warpgroup owns 32 frame columns");
  constexpr int kAcc = L::kAcc;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t *full = (uint64_t *)(smem + kTcStages * L::kStage);
  uint64_t *empty = full + kTcStages;
  uint64_t *tfull = empty + kTcStages;
  uint64_t *tempty = tfull + kAcc;
  uint32_t *tmem_slot = (uint32_t *)(tempty + kAcc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g = blockIdx.x, ft = blockIdx.y;
  const int nb = (int)p.nb;
  const int n_stages = (nb + kTcKb - 1) / kTcKb;
  constexpr uint32_t kTmemCols = FT * kAcc < 32 ? 32 : FT * kAcc;

  // All inputs are read after the previous kernel on the stream completes;
  // TMEM is allocated after that too, so a CTA never holds tensor memory
  // while it waits on another grid.
  pdl_launch_dependents();
  pdl_wait();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mbar_init(&full[s], 4);             // one arrive.expect_tx per copy lane
      mbar_init(&empty[s], 1 + 4 * DWG);  // MMA commit + one arrival per drain warp
    }
    for (int b = 0; b < kAcc; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4 * DWG);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  bool ok = true;
  if (warp == 0) {
    if (lane < 4 * kTcPhases) {
      const int cp = lane & 3, phase = lane >> 2;  // copy kind, stage phase
      for (int si = phase; si < n_stages && ok; si += kTcPhases) {
        const int s = si % kTcStages;
        if (!mbar_wait(&empty[s], ((uint32_t)(si / kTcStages) & 1u) ^ 1u)) { ok = false; break; }
        const int b0 = si * kTcKb, nblk = nb - b0 < kTcKb ? nb - b0 : kTcKb;
        unsigned char *st = smem + s * L::kStage;
        // each copy lane arrives with its own byte count before its copy, so
        // the stage completes only when all four have arrived and landed
        if (cp == 0) {
          mbar_arrive_expect_tx(&full[s], nblk * SC_TILE_BYTES);
          bulk_g2s(st, p.qs + (g * p.nb + b0) * SC_TILE_BYTES, nblk * SC_TILE_BYTES, &full[s]);
        } else if (cp == 1) {
          mbar_arrive_expect_tx(&full[s], nblk * FT * 32);
          bulk_g2s(st + L::kA, p.xq + (ft * p.nb + b0) * (int64_t)(FT * 32), nblk * FT * 32, &full[s]);
        } else if (cp == 2) {
          mbar_arrive_expect_tx(&full[s], nblk * SC_GROUP_ROWS * 2);
          bulk_g2s(st + L::kA + L::kB, p.sc + (g * p.nb + b0) * SC_GROUP_ROWS, nblk * SC_GROUP_ROWS * 2, &full[s]);
        } else {
          mbar_arrive_expect_tx(&full[s], nblk * FT * 4);
          bulk_g2s(st + L::kA + L::kB + L::kS, p.dx + (ft * p.nb + b0) * (int64_t)FT, nblk * FT * 4, &full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_i8(FT);
      int b = 0;
      for (int si = 0; si < n_stages && ok; si++) {
        const int s = si % kTcStages;
        if (!mbar_wait(&full[s], (uint32_t)(si / kTcStages) & 1u)) { ok = false; break; }
        const int nblk = nb - si * kTcKb < kTcKb ? nb - si * kTcKb : kTcKb;
        const unsigned char *st = smem + s * L::kStage;
        for (int i = 0; i < nblk; i++, b++) {
          const int buf = b % kAcc;
          if (!mbar_wait(&tempty[buf], ((uint32_t)(b / kAcc) & 1u) ^ 1u)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = umma_desc(st + i * SC_TILE_BYTES, 2048, 128);
          const uint64_t bd = umma_desc(st + L::kA + i * FT * 32, FT * 16, 128);
          tc_mma_i8(tmem_base + (uint32_t)(buf * FT), ad, bd, idesc, 0u);
          tc_commit(&tfull[buf]);
        }
        tc_commit(&empty[s]);  // the stage's tiles are free once its MMAs complete
      }
    }
    __syncwarp();
  } else {
    // ---- drain warpgroups: 32 frame columns per thread ----
    const int dw_idx = warp - 2;
    const int wg = dw_idx >> 2;         // column slice
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int col_base = wg * 32;
    // int32 -> f32 without I2F: for |d| < 2^22, the float with bit pattern
    // d + 0x4B400000 is exactly 1.5 * 2^23 + d (block dots are below 2^20).
    const uint64_t neg_magic = pack2(-12582912.0f, -12582912.0f);
    // fma(s, dot, -0) is the rounded product s * dot (an exact zero keeps its
    // sign: +0 + -0 = +0, -0 + -0 = -0); -0 arrives as a kernel parameter so
    // the code generator cannot turn the fma back into a multiply and fuse
    // it into the following add.
    const uint64_t nz2 = pack2(p.neg_zero, p.neg_zero);
    uint64_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; j++) acc[j] = 0ull;
    int b = 0;
    for (int si = 0; si < n_stages && ok; si++) {
      const int s = si % kTcStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)(si / kTcStages) & 1u))) { ok = false; break; }
      const int nblk = nb - si * kTcKb < kTcKb ? nb - si * kTcKb : kTcKb;
      const unsigned char *st = smem + s * L::kStage;
      for (int i = 0; i < nblk; i++, b++) {
        const int buf = b % kAcc;
        // warp-uniform wait: tcgen05.ld below needs the whole warp
        if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (uint32_t)(b / kAcc) & 1u))) { ok = false; break; }
        tc_fence_after();
        uint32_t r[32];
        tc_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * FT + col_base), r);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        const float dwv = __half2float(((const __half *)(st + L::kA + L::kB))[i * SC_GROUP_ROWS + row]);
        const uint64_t dw2 = pack2(dwv, dwv);
        const uint64_t *dx2 = (const uint64_t *)(st + L::kA + L::kB + L::kS) + (i * FT + col_base) / 2;
        // acc += (dw * dx) * dot with the three roundings of the reference's
        // scalar oracle (sgemm_kernel.rs:185-196), so each output is bit-equal
        // to q8_gemm_scalar's, in packed f32x2 arithmetic.
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const uint64_t s2 = fmul2(dw2, dx2[j]);  // dw * dx per column
          const uint64_t f2 = fadd2(pack2(__uint_as_float(r[2 * j] + 0x4B400000u),
                                          __uint_as_float(r[2 * j + 1] + 0x4B400000u)),
                                    neg_magic);   // exact block dots as f32
          acc[j] = fadd2(acc[j], ffma2(s2, f2, nz2));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // ---- epilogue: y (+ bias); or the next GEMM's codes, one block of 32
    // output features per warp (the warp's lanes are 32 consecutive rows) ----
    const int64_t n = g * SC_GROUP_ROWS + row;
    if (p.qout.xq) {
      const float bn = p.bias ? p.bias[n] : 0.0f;
      float v[32], a[32];
#pragma unroll
      for (int j = 0; j < 32; j++) {
        v[j] = apply_epilogue(p.epi, __fadd_rn((j & 1) ? hi_of(acc[j >> 1]) : lo_of(acc[j >> 1]), bn), 0);
        a[j] = fabsf(v[j]);
      }
      // block amax of every column over the warp's 32 rows: a butterfly that
      // leaves column col_of(lane) in a[0] of this lane (max ignores order;
      // fmaxf skips NaN like quantize_col's amax)
#pragma unroll
      for (int cnt = 32, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < cnt / 2; i++) {
          const float send = up ? a[i] : a[i + cnt / 2];
          const float keep = up ? a[i + cnt / 2] : a[i];
          a[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
      }
      int mycol = 0;  // column whose amax this lane holds
#pragma unroll
      for (int cnt = 32, off = 16; cnt > 1; cnt >>= 1, off >>= 1)
        if (lane & off) mycol += cnt / 2;
      const float amax = a[0];
      const float sblk = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
      const float inv = __fdiv_rn(1.0f, sblk);
      const int64_t fbase = ft * FT + col_base;  // frames of this thread's columns (< t_pad)
      p.qout.dx[qout_dx_index(p.qout, fbase + mycol, n >> 5)] = sblk;
      // codes: row n is element n % 32 of block n / 32 of the next GEMM's K
      int8_t *dst = p.qout.xq + ((int64_t)ft * p.qout.nb + (n >> 5)) * (FT * 32) + ((n & 31) >> 4) * (FT * 16) +
                    (int64_t)col_base * 16 + (n & 15);
#pragma unroll
      for (int j = 0; j < 32; j++) {
        int src = 0;  // lane holding column j: bit-reverse of the butterfly's split order
#pragma unroll
        for (int cnt = 32, off = 16, jj = j; cnt > 1; cnt >>= 1, off >>= 1)
          if (jj >= cnt / 2) { src |= off; jj -= cnt / 2; }
        const float ij = __shfl_sync(0xffffffffu, inv, src);
        const float aj = __shfl_sync(0xffffffffu, amax, src);
        dst[j * 16] = aj != 0.0f ? rust_round_i8(__fmul_rn(v[j], ij)) : (int8_t)0;
        if (p.y && fbase + j < p.t) p.y[p.y_time_major ? (fbase + j) * p.ldy + n : n * p.ldy + fbase + j] = v[j];
      }
    } else if (n < p.n_rows) {
      const float bn = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int64_t f = ft * FT + col_base + j;
        const float v = (j & 1) ? hi_of(acc[j >> 1]) : lo_of(acc[j >> 1]);
        if (f < p.t) {
          const int64_t idx = p.y_time_major ? f * p.ldy + n : n * p.ldy + f;
          p.y[idx] = apply_epilogue(p.epi, __fadd_rn(v, bn), idx);
        }
      }
    }
  }
  if (!ok) atomicOr(p.status, kStatusWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

static unsigned *tc_status_ptr() {
  static std::atomic<unsigned *> ptr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned *q = ptr[dev].load(std::memory_order_acquire);
  if (!q) {
    void *a = nullptr;
    if (cudaGetSymbolAddress(&a, g_tc_status) != cudaSuccess) return nullptr;
    q = (unsigned *)a;
    ptr[dev].store(q, std::memory_order_release);  // every caller stores the same address
  }
  return q;
}

int tc_gemm_status(unsigned *out) {
  unsigned v = 0, zero = 0;
  SC_CUDA(cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(v)));
  SC_CUDA(cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(zero)));
  *out = v;
  return kOk;
}

// Shared-memory limit raised so far per device, per kernel instance.
template <int FT, int DWG>
static std::atomic<size_t> *tc_smem_limit() {
  static std::atomic<size_t> limit[64];
  return limit;
}

template <int FT, int DWG>
static int prime_tc() {
  return raise_smem_limit((const void *)q8_gemm_tc_kernel<FT, DWG>, TcSmem<FT, DWG>::kBytes,
                          tc_smem_limit<FT, DWG>());
}

int tc_gemm_prime() {
  if (!tc_status_ptr()) {
    set_error("q8_gemm_tc: status word lookup failed");
    return kErrCuda;
  }
  int rc = prime_tc<32, 1>();
  if (!rc) rc = prime_tc<64, 2>();
  if (!rc) rc = prime_tc<128, 4>();
  return rc;
}

template <int FT, int DWG>
static int launch_tc(const TcParams &p, int64_t groups, cudaStream_t st) {
  using L = TcSmem<FT, DWG>;
  auto kern = q8_gemm_tc_kernel<FT, DWG>;
  const int rc = raise_smem_limit((const void *)kern, L::kBytes, tc_smem_limit<FT, DWG>());
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)groups, (unsigned)(p.t_pad / FT), 1);
  cfg.blockDim = dim3(64 + 128 * DWG, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
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

// Frame tile of a GEMM over t frames: 64-frame tiles (two CTAs per SM) up
// to 1024 frames, where a grid of 128-frame tiles would leave most of its
// last wave idle; 128 above (measured at 896 / 1792 frames over the four
// layer shapes: 193 vs 227 us / 305 vs 308 us).
int tc_frame_tile(int64_t t) { return t <= 32 ? 32 : t <= 1024 ? 64 : 128; }

int gemm_tc(const TcGemmArgs &a, cudaStream_t st) {
  const Q8Weights *w = a.w;
  TcParams p{};
  p.qs = w->qs;
  p.sc = w->sc;
  p.nb = w->nb;
  p.n_rows = w->rows;
  p.xq = a.xq;
  p.dx = a.dx;
  p.t = a.t;
  p.t_pad = a.t_pad;
  p.bias = a.bias;
  p.y = a.y;
  p.y_time_major = a.y_time_major;
  p.ldy = a.ldy;
  p.status = tc_status_ptr();
  p.epi = a.epi;
  p.qout = a.qout;
  p.neg_zero = -0.0f;
  if (p.qout.xq && (w->rows % SC_GROUP_ROWS || p.epi.op == kEpiResidual || p.qout.t_pad != a.t_pad ||
                    p.qout.ft != tc_frame_tile(a.t) || p.qout.nb * 32 != w->rows)) {
    set_error("q8_gemm_tc: quantised output needs rows %% 128 == 0, no residual and the same frame tiling");
    return kErrInvalid;
  }
  if (!p.status) {
    set_error("q8_gemm_tc: status word lookup failed");
    return kErrCuda;
  }
  const int ft = tc_frame_tile(a.t);
  if (a.t_pad % ft != 0) {
    set_error("q8_gemm_tc: t_pad %lld is not a multiple of the frame tile %d", (long long)a.t_pad, ft);
    return kErrInvalid;
  }
  const int64_t groups = w->rows_pad / SC_GROUP_ROWS;
  switch (ft) {
    case 32: return launch_tc<32, 1>(p, groups, st);
    case 64: return launch_tc<64, 2>(p, groups, st);
    default: return launch_tc<128, 4>(p, groups, st);
  }
}

}  // namespace sc
