// q8_gemm_tc.cu -- large-M Q8_0 GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::f16 with f32 accumulators in tensor memory), persistent.
//
// Same arithmetic as the reference (sgemm_kernel.rs:156-201): for every 32-wide
// K block the exact dot of the int8 weight codes and int8 activation codes,
// scaled by dw[n, b] * dx[col, b] and accumulated in f32 with three roundings
// (acc + (dw * dx) * dot).  Because each K block has its own pair of scales,
// the dot cannot be accumulated across blocks: every block is its own MMA
// into a TMEM accumulator, and drain warps read it back (tcgen05.ld), scale it
// and add it to f32 accumulators in registers while the tensor core computes
// the next blocks into the other accumulators.
//
// The codes are held as f16 (every int8 value is an f16 integer): a block's
// dot is two K = 16 MMAs of kind::f16 into an f32 accumulator.  Every product
// is an integer of magnitude <= 127^2 and every partial sum stays below 2^24,
// so the f32 accumulator holds the exact integer dot, and the drain needs no
// int -> f32 conversion: three f32 operations per output and block.
//
// Persistent CTAs (one per SM, all 512 TMEM columns): CTA c computes tiles
// c, c + grid, ... of 128 weight rows x FT frames; the operand and scale
// rings and the TMEM accumulator ring run on across tiles, so the next
// tile's copies and MMAs overlap the current tile's epilogue.
//
// CTA roles (warp-specialised):
//   warp 0       producer: one thread issues 1-D bulk copies (TMA engine, no
//                multicast): per operand slot the f16 weight tiles and the
//                f16 activation tiles of kTcKb blocks, per scale chunk the
//                weight and activation scales of kTcScB blocks;
//   warp 1       allocates TMEM; one thread issues two MMAs per block into a
//                rotating accumulator and commits to its "full" barrier, and
//                to the operand slot's "empty" barrier after its last block;
//   warps 2..17  drain: 4 warpgroups, each thread one weight row (its TMEM
//                lane) and FT/4 frame columns; then the tile's epilogue.
// Every mbarrier wait is bounded; a wait that gives up sets a status bit and
// that role stops waiting, so the kernel cannot hang.
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

// Grid: one CTA per SM, each looping over tiles (0), or one CTA per tile (1).
#ifndef SC_TC_GRID_TILES
#define SC_TC_GRID_TILES 0
#endif
constexpr int kTcKb = 4;        // K blocks per operand copy (one ring slot)
constexpr int kTcScB = 8;       // K blocks per scale chunk
constexpr int kTcDrainWarps = 16;
constexpr int kTcThreads = 64 + 32 * kTcDrainWarps;

static __device__ unsigned g_tc_status;

// Shared memory of one CTA:
//   operand ring  kOps slots of kTcKb consecutive K blocks of one tile:
//                 f16 weight tiles [kTcKb][4][128][8] and f16 activation
//                 tiles [kTcKb][4][FT][8], one bulk copy each; a slot is
//                 refilled as soon as the MMAs of its blocks complete;
//   scale ring    kScs slots of kTcScB consecutive K blocks of one tile:
//                 f16 weight scales [kTcScB][128] and f32 activation scales
//                 [kTcScB][FT]; a slot is refilled once every drain warp has
//                 scaled its blocks;
//   transpose     per drain warp 8 frames x 32 rows of f32, through which the
//                 epilogue turns a thread's row of outputs into 16-byte
//                 stores of four rows.
// The copy engine's time per bulk copy hardly depends on its size up to
// 32 KB, so copies are few and large.
template <int FT>
struct TcCfg {
  static constexpr int kCols = FT / 4;                  // frame columns per drain thread
  static constexpr int kAcc = 512 / FT;                 // TMEM accumulators of FT columns
  static constexpr int kPairs = kAcc / 2;               // signalled in pairs (one commit per two blocks)
  static constexpr int kA = kTcKb * 8192;               // f16 weight tiles of a slot
  static constexpr int kOp = kA + kTcKb * FT * 64;      // + f16 activation tiles
  static constexpr int kScW = kTcScB * SC_GROUP_ROWS * 2;
  static constexpr int kSc = kScW + kTcScB * FT * 4;
  static constexpr int kScs = 2;
  static constexpr int kTr = kTcDrainWarps * 8 * 32 * 4;
  static constexpr int kOps = (220 * 1024 - kScs * kSc - kTr) / kOp;
  static constexpr int kBars = 8 * (2 * kOps + 2 * kScs + 2 * kPairs + 1);
  static constexpr int kMisc = 16 + 4 * (kOps + kScs);  // TMEM slot, fail flag, last round per slot
  static constexpr int kBytes = kOps * kOp + kScs * kSc + kTr + kBars + kMisc;
  static_assert(kOps >= 2, "the operand ring needs two slots");
  static_assert(kBytes <= 227 * 1024, "shared memory");
  static_assert(2 * kBytes > 228 * 1024, "one CTA per SM: it takes all 512 TMEM columns");
};

// Epilogue store modes (uniform per launch).
enum : int {
  kStoreDirect = 0,  // each thread stores its outputs (any layout)
  kStoreVec = 1,     // time-major y, 16-byte stores of four rows
};

struct TcParams {
  const __half *qh;      // f16 weight tiles [G][nb][4][128][8]
  const __half *sc;      // weight scales [G][nb][128]
  int64_t nb, n_rows;
  const __half *xq;      // f16 activation tiles [t_pad/FT][nb][4][FT][8]
  const float *dx;       // activation scales [t_pad/FT][nb][FT]
  int64_t t, t_pad, n_ft, n_tiles;
  const float *bias;
  float *y;
  int y_time_major;
  int64_t ldy;
  unsigned *status;
  Epilogue epi;
  QOut qout;
  int store;       // kStoreDirect / kStoreVec (y, no codes)
  float neg_zero;  // -0.0f, opaque to the compiler (see the drain)
};

// ---- tcgen05 wrappers -----------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, no swizzle, K-major canonical layout:
// core matrices of 8 rows x 16 bytes, `lbo` bytes between the two 16-byte
// K chunks of a row's 32 bytes, `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(const void *smem, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_u32(smem);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;               // base offset 0, layout type 0 = no swizzle
}

// Instruction descriptor: kind::f16, D = f32, A = B = f16, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tc_ld<32>(uint32_t taddr, uint32_t (&r)[32]) {
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
template <>
__device__ __forceinline__ void tc_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tc_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Waits for this thread's tcgen05.ld results; the registers pass through the
// statement, so no use of them can be scheduled before the wait.
template <int N>
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tc_wait_ld<32>(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])::"memory");
}
template <>
__device__ __forceinline__ void tc_wait_ld<8>(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7])::"memory");
}
template <>
__device__ __forceinline__ void tc_wait_ld<16>(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])::"memory");
}

// A barrier wait by lane 0 for the whole warp (one shared-memory poll
// instead of 32); __syncwarp orders the lanes' later reads after it.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity) ? 1u : 0u;
  __syncwarp();
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}


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

// acc += (dw * dx) * dot over one block of the thread's C columns, with the
// three roundings of the reference's scalar oracle (sgemm_kernel.rs:185-196);
// r holds the block's exact integer dots as f32.  fma(s, dot, -0) is the
// rounded product s * dot (an exact zero keeps its sign: +0 + -0 = +0,
// -0 + -0 = -0); -0 arrives as a kernel parameter (nz2) so the code
// generator cannot turn the fma back into a multiply and fuse it into the
// following add.
// The thread's columns are drained in two halves of H = C / 2 (acc pairs
// OFF .. OFF + H/2 - 1), so one half's accumulator load is in flight while
// the other half is scaled.
template <int H, int OFF, int NACC>
__device__ __forceinline__ void drain_half(uint64_t (&acc)[NACC], const uint32_t (&r)[H], uint64_t dw2,
                                           const uint64_t *dx2, uint64_t nz2) {
#pragma unroll
  for (int jj = 0; jj < H / 2; jj++) {
    const uint64_t s2 = fmul2(dw2, dx2[jj]);  // dw * dx per column
    const uint64_t f2 = (uint64_t)r[2 * jj] | ((uint64_t)r[2 * jj + 1] << 32);
    acc[OFF + jj] = fadd2(acc[OFF + jj], ffma2(s2, f2, nz2));
  }
}

// Tile t of the work list is row group t / n_ft, frame tile t % n_ft: the
// tiles in flight at once share their row groups' weights in L2.  A CTA's
// blocks are numbered gb = 0, 1, ... over its tiles in order; operand slots
// (go), scale chunks (gc) and accumulator pairs (gp) are numbered the same
// way by every role.  Accumulators are used in pairs: pair slot ps = gp %
// kPairs holds a tile's blocks 2i and 2i + 1 in accumulators 2 ps and 2 ps +
// 1, signalled by one commit (a tcgen05.commit costs the issuing thread
// several times an MMA) and released by the drain once both are loaded.
template <int FT>
__global__ void __launch_bounds__(kTcThreads, 1) q8_gemm_tc_kernel(const __grid_constant__ TcParams p) {
  using L = TcCfg<FT>;
  constexpr int C = L::kCols, kPairs = L::kPairs, kOps = L::kOps, kScs = L::kScs;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char *ops = smem;                          // operand ring
  unsigned char *scs = smem + kOps * L::kOp;          // scale ring
  float *trs = (float *)(scs + kScs * L::kSc);        // transpose buffers
  uint64_t *op_full = (uint64_t *)((unsigned char *)trs + L::kTr);
  uint64_t *op_empty = op_full + kOps;
  uint64_t *sc_full = op_empty + kOps;
  uint64_t *sc_empty = sc_full + kScs;
  uint64_t *tfull = sc_empty + kScs;
  uint64_t *tempty = tfull + kPairs;
  uint64_t *mma_done = tempty + kPairs;
  uint32_t *misc = (uint32_t *)(mma_done + 1);  // [0] TMEM base, [1] fail flag
  int *last_round = (int *)(misc + 4);          // [kOps + kScs]: last fill of each slot

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = (int)p.nb;
  const int opt = (nb + kTcKb - 1) / kTcKb;    // operand slots per tile

  // All inputs are read after the previous kernel on the stream completes;
  // TMEM is allocated after that too, so a CTA never holds tensor memory
  // while it waits on another grid.
  pdl_launch_dependents();
  pdl_wait();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kOps; s++) {
      mbar_init(&op_full[s], 1);   // the producer's arrival; the copies' bytes
      mbar_init(&op_empty[s], 1);  // the commit after the slot's last MMA
    }
    for (int s = 0; s < kScs; s++) {
      mbar_init(&sc_full[s], 1);
      mbar_init(&sc_empty[s], kTcDrainWarps);  // every drain warp
    }
    for (int s = 0; s < kOps + kScs; s++) last_round[s] = -1;
    for (int b = 0; b < kPairs; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kTcDrainWarps);
    }
    mbar_init(mma_done, 1);
    misc[1] = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(misc)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  bool ok = true;
  if (warp == 0) {
    // ---- producer: one thread issues every copy (lanes of one warp that
    // wait on different barriers would serialise) ----
    if (lane == 0) {
      int go = 0, gc = 0;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        const int64_t g = tile / p.n_ft, ft = tile % p.n_ft;
        for (int j = 0; j < opt && ok; j++, go++) {
          const int k0 = j * kTcKb;
          if (k0 % kTcScB == 0) {  // the scale chunk that starts here
            const int s = gc % kScs, nblk = nb - k0 < kTcScB ? nb - k0 : kTcScB;
            if (!mbar_wait(&sc_empty[s], ((uint32_t)(gc / kScs) & 1u) ^ 1u)) { ok = false; break; }
            unsigned char *dst = scs + s * L::kSc;
            last_round[kOps + s] = gc / kScs;
            mbar_arrive_expect_tx(&sc_full[s], nblk * (SC_GROUP_ROWS * 2 + FT * 4));
            bulk_g2s(dst, p.sc + (g * p.nb + k0) * SC_GROUP_ROWS, nblk * SC_GROUP_ROWS * 2, &sc_full[s]);
            bulk_g2s(dst + L::kScW, p.dx + (ft * p.nb + k0) * (int64_t)FT, nblk * FT * 4, &sc_full[s]);
            gc++;
          }
          const int s = go % kOps, nblk = nb - k0 < kTcKb ? nb - k0 : kTcKb;
          if (!mbar_wait(&op_empty[s], ((uint32_t)(go / kOps) & 1u) ^ 1u)) { ok = false; break; }
          unsigned char *dst = ops + s * L::kOp;
          last_round[s] = go / kOps;
          mbar_arrive_expect_tx(&op_full[s], nblk * (8192 + FT * 64));
          bulk_g2s(dst, p.qh + (g * p.nb + k0) * 4096, nblk * 8192, &op_full[s]);
          bulk_g2s(dst + L::kA, p.xq + (ft * p.nb + k0) * (int64_t)(FT * 32), nblk * FT * 64, &op_full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(FT);
      // descriptors of slot 0's first block; a block's and a K half's are
      // these plus their byte offset / 16 (the start-address field, bits
      // 0-13, holds shared-memory addresses below 256 KB without carrying)
      const uint64_t a0 = umma_desc(ops, 2048, 128), b0 = umma_desc(ops + L::kA, FT * 16, 128);
      int go = 0, gp = 0;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        uint64_t as = 0, bs = 0;
        for (int k = 0; k < nb; k++) {
          const int s = go % kOps, i = k % kTcKb, ps = gp % kPairs;
          if (i == 0) {  // the operand slot of blocks k .. k + kTcKb - 1
            if (!mbar_wait(&op_full[s], (uint32_t)(go / kOps) & 1u)) { ok = false; break; }
            as = a0 + (uint64_t)((s * L::kOp) >> 4);
            bs = b0 + (uint64_t)((s * L::kOp) >> 4);
          }
          if ((k & 1) == 0) {  // a new accumulator pair
            if (!mbar_wait(&tempty[ps], ((uint32_t)(gp / kPairs) & 1u) ^ 1u)) { ok = false; break; }
            tc_fence_after();
          }
          const uint32_t d = tmem_base + (uint32_t)((2 * ps + (k & 1)) * FT);
          const uint64_t ai = as + (uint64_t)((i * 8192) >> 4), bi = bs + (uint64_t)((i * FT * 64) >> 4);
          tc_mma_f16(d, ai, bi, idesc, 0u);                                            // K 0-15
          tc_mma_f16(d, ai + (4096 >> 4), bi + (uint64_t)((FT * 32) >> 4), idesc, 1u);  // K 16-31
          if ((k & 1) || k + 1 == nb) {
            tc_commit(&tfull[ps]);
            gp++;
          }
          if (i == kTcKb - 1 || k + 1 == nb) {
            tc_commit(&op_empty[s]);  // the slot is free once its MMAs complete
            go++;
          }
        }
      }
      // every MMA this thread issued completes before TMEM is released
      tc_commit(mma_done);
      if (!mbar_wait(mma_done, 0)) ok = false;
    }
    __syncwarp();
  } else {
    // ---- drain: C frame columns per thread ----
    const int dwi = warp - 2;
    const int cg = dwi >> 2;       // column slice
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int col_base = cg * C;
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col_base;
    const uint64_t nz2 = pack2(p.neg_zero, p.neg_zero);
    float *tr = trs + dwi * 8 * 32;  // this warp's transpose buffer [8 frames][32 rows]
    int gp = 0, gc = 0;
    for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
      const int64_t g = tile / p.n_ft, ft = tile % p.n_ft;
      uint64_t acc[C / 2];
#pragma unroll
      for (int j = 0; j < C / 2; j++) acc[j] = 0ull;
      // The tile's blocks, each drained in two halves of the thread's
      // columns: while one half is scaled the other half's accumulator load
      // is in flight, and an accumulator pair is released as soon as both
      // blocks' loads have landed.  rA holds the next block's first half.
      constexpr int H = C / 2;
      uint32_t rA[H], rB[H];
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[gp % kPairs], (uint32_t)(gp / kPairs) & 1u))) { ok = false; break; }
      tc_fence_after();
      tc_ld<H>(taddr + (uint32_t)(2 * (gp % kPairs) * FT), rA);
      for (int k = 0; k < nb; k++) {
        const int kc = k % kTcScB, ss = gc % kScs;  // block kc of scale chunk gc
        if (kc == 0 && !__all_sync(0xffffffffu, mbar_wait(&sc_full[ss], (uint32_t)(gc / kScs) & 1u))) { ok = false; break; }
        const unsigned char *sc = scs + ss * L::kSc;
        const float dwv = __half2float(((const __half *)sc)[kc * SC_GROUP_ROWS + row]);
        const uint64_t dw2 = pack2(dwv, dwv);
        const uint64_t *dx2 = (const uint64_t *)(sc + L::kScW) + (kc * FT + col_base) / 2;
        const int ps = gp % kPairs;
        const uint32_t tb = taddr + (uint32_t)((2 * ps + (k & 1)) * FT);
        tc_wait_ld<H>(rA);
        tc_ld<H>(tb + H, rB);
        drain_half<H, 0>(acc, rA, dw2, dx2, nz2);
        tc_wait_ld<H>(rB);
        const bool pair_end = (k & 1) || k + 1 == nb;
        if (pair_end) {  // both of the pair's accumulators are loaded
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[ps]);
          gp++;
        }
        if (k + 1 < nb) {
          if (pair_end) {
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[gp % kPairs], (uint32_t)(gp / kPairs) & 1u))) { ok = false; break; }
            tc_fence_after();
          }
          tc_ld<H>(taddr + (uint32_t)((2 * (gp % kPairs) + ((k + 1) & 1)) * FT), rA);
        }
        drain_half<H, H / 2>(acc, rB, dw2, dx2 + H / 2, nz2);
        if (kc == kTcScB - 1 || k + 1 == nb) {  // the chunk's scales are used
          __syncwarp();
          if (lane == 0) mbar_arrive(&sc_empty[ss]);
          gc++;
        }
      }
      if (!ok) break;
      // ---- epilogue: u = acc + bias (then SiLU / ReLU) per row; then y,
      // with the residual, or the next GEMM's codes ----
      const int64_t n = g * SC_GROUP_ROWS + row;
      const int64_t fbase = ft * FT + col_base;  // frames of this thread's columns (< t_pad)
      const float bn = p.bias && n < p.n_rows ? p.bias[n] : 0.0f;
      float v[C];
#pragma unroll
      for (int j = 0; j < C; j++) {
        const float u = __fadd_rn((j & 1) ? hi_of(acc[j >> 1]) : lo_of(acc[j >> 1]), bn);
        v[j] = p.epi.op == kEpiResidual ? u : apply_epilogue(p.epi, u, 0);
      }
      if (p.qout.xq) {
        float a[C];
#pragma unroll
        for (int j = 0; j < C; j++) a[j] = fabsf(v[j]);
        // block amax of every column over the warp's 32 rows: a butterfly
        // that halves the columns a lane holds at each step (offsets 16, 8,
        // ...), leaving column col_of(lane) in a[0]; with fewer than 32
        // columns, the lanes that then share a column combine theirs.  max
        // ignores order; fmaxf skips NaN like quantize_col's amax.
#pragma unroll
        for (int cnt = C, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
          const bool up = (lane & off) != 0;
#pragma unroll
          for (int i = 0; i < cnt / 2; i++) {
            const float send = up ? a[i] : a[i + cnt / 2];
            const float keep = up ? a[i + cnt / 2] : a[i];
            a[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, off));
          }
        }
        constexpr int kShare = 32 / C;  // lanes per column after the butterfly
#pragma unroll
        for (int off = kShare / 2; off > 0; off >>= 1) a[0] = fmaxf(a[0], __shfl_xor_sync(0xffffffffu, a[0], off));
        int mycol = 0;  // column whose amax this lane holds
#pragma unroll
        for (int cnt = C, off = 16; cnt > 1; cnt >>= 1, off >>= 1)
          if (lane & off) mycol += cnt / 2;
        const float amax = a[0];
        const float sblk = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
        const float inv = __fdiv_rn(1.0f, sblk);
        if ((lane & (kShare - 1)) == 0) p.qout.dx[qout_dx_index(p.qout, fbase + mycol, n >> 5)] = sblk;
        // codes: row n is element n % 32 of block n / 32 of the next GEMM's K
        __half *dst = p.qout.xq + qout_code_index(p.qout, fbase, n);
#pragma unroll
        for (int j = 0; j < C; j++) {
          int src = 0;  // a lane holding column j: the inverse of the butterfly's split order
#pragma unroll
          for (int cnt = C, off = 16, jj = j; cnt > 1; cnt >>= 1, off >>= 1)
            if (jj >= cnt / 2) { src |= off; jj -= cnt / 2; }
          const float ij = __shfl_sync(0xffffffffu, inv, src);
          const float aj = __shfl_sync(0xffffffffu, amax, src);
          dst[j * 8] = code_half(aj != 0.0f ? rust_round_i8(__fmul_rn(v[j], ij)) : (int8_t)0);
          if (p.y && fbase + j < p.t) p.y[p.y_time_major ? (fbase + j) * p.ldy + n : n * p.ldy + fbase + j] = v[j];
        }
      } else if (p.store == kStoreVec) {
        // time-major y in 16-byte stores of four rows: per 8 frames, the
        // warp's 32 x 8 outputs pass through its transpose buffer; lane l
        // then holds items l and l + 32 (frame item / 8, rows 4 (item % 8)
        // .. + 3 of the warp)
        const int64_t n0 = g * SC_GROUP_ROWS + quarter * 32;
        const bool res = p.epi.op == kEpiResidual;
#pragma unroll
        for (int c8 = 0; c8 < C / 8; c8++) {
#pragma unroll
          for (int e = 0; e < 8; e++) tr[e * 32 + lane] = v[8 * c8 + e];
          __syncwarp();
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int item = lane + 32 * h, e = item >> 3, r4 = (item & 7) * 4;
            const int64_t f = fbase + 8 * c8 + e, nn = n0 + r4;
            float4 u4 = *reinterpret_cast<const float4 *>(tr + e * 32 + r4);
            if (f < p.t && nn < p.n_rows) {
              float *yp = p.y + f * p.ldy + nn;
              if (res) {  // y = res + alpha * u, elementwise (res may be y itself)
                const float4 r = *reinterpret_cast<const float4 *>(p.epi.res + f * p.ldy + nn);
                const float al = p.epi.alpha;
                u4 = make_float4(__fadd_rn(r.x, __fmul_rn(al, u4.x)), __fadd_rn(r.y, __fmul_rn(al, u4.y)),
                                 __fadd_rn(r.z, __fmul_rn(al, u4.z)), __fadd_rn(r.w, __fmul_rn(al, u4.w)));
              }
              *reinterpret_cast<float4 *>(yp) = u4;
            }
          }
          __syncwarp();
        }
      } else if (n < p.n_rows) {
#pragma unroll
        for (int j = 0; j < C; j++) {
          const int64_t f = fbase + j;
          if (f < p.t) {
            const int64_t idx = p.y_time_major ? f * p.ldy + n : n * p.ldy + f;
            p.y[idx] = p.epi.op == kEpiResidual ? __fadd_rn(p.epi.res[idx], __fmul_rn(p.epi.alpha, v[j])) : v[j];
          }
        }
      }
    }
    // no TMEM load of this thread is outstanding (a role that gave up may
    // have left one) before the kernel ends
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  }
  if (!ok) {
    atomicOr(p.status, kStatusWaitTimeout);
    atomicOr(&misc[1], 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (misc[1] && threadIdx.x == 0) {
    // a role gave up: wait (bounded) for bulk copies that may still be
    // landing in this CTA's shared memory before it exits
    for (int s = 0; s < kOps + kScs; s++)
      if (last_round[s] >= 0) mbar_wait(s < kOps ? &op_full[s] : &sc_full[s - kOps], (uint32_t)last_round[s] & 1u);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
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
template <int FT>
static std::atomic<size_t> *tc_smem_limit() {
  static std::atomic<size_t> limit[64];
  return limit;
}

template <int FT>
static int prime_tc() {
  return raise_smem_limit((const void *)q8_gemm_tc_kernel<FT>, TcCfg<FT>::kBytes, tc_smem_limit<FT>());
}

int tc_gemm_prime() {
  if (!tc_status_ptr()) {
    set_error("q8_gemm_tc: status word lookup failed");
    return kErrCuda;
  }
  int rc = prime_tc<64>();
  if (!rc) rc = prime_tc<128>();
  return rc;
}

template <int FT>
static int launch_tc(const TcParams &p, int sm_count, cudaStream_t st) {
  using L = TcCfg<FT>;
  auto kern = q8_gemm_tc_kernel<FT>;
  const int rc = raise_smem_limit((const void *)kern, L::kBytes, tc_smem_limit<FT>());
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(SC_TC_GRID_TILES || p.n_tiles < sm_count ? p.n_tiles : sm_count), 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
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

// Frame tile of a GEMM over t frames (also the tile of its code layout):
// 128-frame tiles, 64 for batches that a 128-frame tile would mostly pad
// (measured in the 256-stream encoder step, two 896-frame halves in flight:
// 19.6 ms per step with 128-frame tiles, 21.6 ms with 64).
#ifndef SC_TC_FT64_MAX
#define SC_TC_FT64_MAX 64
#endif
int tc_frame_tile(int64_t t) { return t <= SC_TC_FT64_MAX ? 64 : 128; }

int gemm_tc(const TcGemmArgs &a, cudaStream_t st) {
  const Q8Weights *w = a.w;
  if (!w->qh) {
    set_error("q8_gemm_tc: weights have no f16 tiles");
    return kErrInvalid;
  }
  TcParams p{};
  p.qh = w->qh;
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
  // time-major y whose frame rows start 16-byte aligned: vector stores
  p.store = !p.qout.xq && p.y && p.y_time_major && p.ldy % 4 == 0 && p.n_rows % 4 == 0 &&
                    ((uintptr_t)p.y & 15) == 0 && (p.epi.op != kEpiResidual || ((uintptr_t)p.epi.res & 15) == 0)
                ? kStoreVec
                : kStoreDirect;
  const int ft = tc_frame_tile(a.t);
  if (p.qout.xq && (w->rows % SC_GROUP_ROWS || p.epi.op == kEpiResidual || p.qout.t_pad != a.t_pad ||
                    p.qout.ft != ft || p.qout.nb * 32 != w->rows)) {
    set_error("q8_gemm_tc: quantised output needs rows %% 128 == 0, no residual and the same frame tiling");
    return kErrInvalid;
  }
  if (!p.status) {
    set_error("q8_gemm_tc: status word lookup failed");
    return kErrCuda;
  }
  if (a.t_pad % ft != 0) {
    set_error("q8_gemm_tc: t_pad %lld is not a multiple of the frame tile %d", (long long)a.t_pad, ft);
    return kErrInvalid;
  }
  p.n_ft = a.t_pad / ft;
  p.n_tiles = (w->rows_pad / SC_GROUP_ROWS) * p.n_ft;
  if (p.n_tiles == 0) return kOk;
  int dev, sms;
  const int rc = current_device(&dev, &sms);
  if (rc) return rc;
  return ft == 64 ? launch_tc<64>(p, sms, st) : launch_tc<128>(p, sms, st);
}

}  // namespace sc

