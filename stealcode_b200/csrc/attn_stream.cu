// attn_stream.cu -- fused cache-aware streaming rel-pos self-attention.
//
// Restates the attention section of block_new (streaming.rs:492-589) and the
// reference GPU operator AttnStreamKernel (gpu/kernels.rs:1137-1156,
// shaders/attn_stream.wgsl):
//
//   score[q, kk, h] = scale * sum_i (q[i] + u[i]) k[kk, i]
//                             + (q[i] + v[i]) pos_p[qq - fr + pos_off, i]
//   out[q, h]       = softmax over the query's band  .  V
//
// with the chunk-aligned band [sat(q/chunk - left_chunks)*chunk,
// min((q/chunk + 1)*chunk, k_hi)).  One CTA per (head, stream), one thread
// per head-dim element.  Every value is rounded exactly as the reference's
// CPU kernels round it, so the output is bit-equal to score_dot + softmax_v
// (simd_kernel.rs:930-1104):
//   A. scores: a half-warp owns a tile of KT keys x CQ queries; its lane l is
//      the reference's SIMD lane l (dims l, l+16, ...) and keeps one
//      accumulator per (query, key) with the reference's two chained FMAs
//      acc = fma(q+u, k, fma(q+v, p, acc)); the 16 lane accumulators are
//      then summed in lane order and scaled.  Each K row is read once per
//      CTA, pos rows about twice (neighbouring tiles share a diagonal).
//   C. band mask + softmax per query: max, exp, the sum taken sequentially
//      over the band, inv = 1/sum, weights e*inv.
//   D. P.V with one thread per dim: acc = fma(w, v, acc) over the band in
//      order, V rows streamed once.
// In ring mode the K/V of the chunk's new frames come from the projection
// output and are written into the stream's HBM ring (slot = frame % cap);
// older band frames are read from the ring.
#include "sc_device.cuh"
#include "sc_kernels.cuh"

namespace sc {

__device__ __forceinline__ void band_of(int64_t qq, int64_t chunk, int64_t left_chunks,
                                        int64_t k_hi, int64_t &kmin, int64_t &kmax) {
  int64_t qc = qq / chunk;
  kmin = (qc > left_chunks ? qc - left_chunks : 0) * chunk;
  int64_t hi = (qc + 1) * chunk;
  kmax = hi < k_hi ? hi : k_hi;
}

// Ring slot of band key 0: frame k_lo plus the step graph's frame shift.
__device__ __forceinline__ int band_slot0(const AttnParams &p) {
  if (p.cap <= 0) return 0;
  const int64_t sh = p.frame_shift ? *p.frame_shift : 0;
  return (int)((p.k_lo + sh) % p.cap);
}

#ifndef SC_ATTN_PREFETCH
#define SC_ATTN_PREFETCH 1
#endif
constexpr int kLanes = 16;        // the reference's SIMD width for score_dot
constexpr int kRedStride = 17;    // padded row of the lane-sum buffer

template <int CQ>
struct AttnTile {
  static constexpr int KT = 64 / CQ;  // keys per half-warp tile
};

template <int HD, int CQ>
__host__ __device__ constexpr size_t attn_smem_floats(int band) {
  return (size_t)CQ * band + 2 * (size_t)CQ * HD + (size_t)(HD / kLanes) * CQ * AttnTile<CQ>::KT * kRedStride;
}

// HD = head_dim (one thread per dim); CQ = queries padded (8 or 16).
template <int HD, int CQ>
__global__ void __launch_bounds__(HD) attn_stream_kernel(const AttnParams p) {
  constexpr int NW = HD / 32;
  constexpr int NHW = HD / kLanes;  // half-warps
  constexpr int KT = AttnTile<CQ>::KT;
  constexpr int NCH = HD / kLanes;  // 16-dim chunks per head row
  constexpr int NPV = CQ + KT - 1;  // pos rows one tile touches
  extern __shared__ __align__(16) float sm[];
  const int band = (int)(p.k_hi - p.k_lo);
  float *s_qk = sm;                   // [CQ][band]  scores, then weights
  float *s_qu = sm + CQ * band;       // [CQ][HD]    q + u
  float *s_qv = s_qu + CQ * HD;       // [CQ][HD]    q + v
  float *s_red = s_qv + CQ * HD;      // [NHW][CQ*KT][kRedStride]
  const int h = blockIdx.x;
  const int64_t z = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int hoff = h * HD;
  const int c = p.c;

  // Band key kk is frame k_lo + kk: from the projection output when
  // kk >= kk_new, else from ring slot (k_lo + kk) % cap (band <= cap, so one
  // wrap at most).  Int32 index math, no 64-bit modulo in the loops.
  const int kk_new = (int)(p.new_lo - p.k_lo);
  const int slot0 = band_slot0(p);
  const int cap = (int)p.cap;
  auto ring_row = [&](float *ring, int kk) -> float * {
    int slot = slot0 + kk;
    slot = slot >= cap ? slot - cap : slot;
    return ring + (z * cap + slot) * (int64_t)p.d + hoff;
  };
  auto key_row = [&](float *ring, const float *nw, int kk) -> const float * {
    if (kk >= kk_new) return nw + (z * p.rows_new + (kk - kk_new)) * p.ld_new + hoff;
    return ring_row(ring, kk);
  };
  const int kk_s = (int)(p.s - p.k_lo);  // keys >= kk_s are this chunk's new frames

  for (int j = 0; j < CQ; j++) {
    float qd = j < c ? p.q[(z * c + j) * p.ldq + hoff + t] : 0.0f;
    s_qu[j * HD + t] = j < c ? __fadd_rn(qd, p.u[hoff + t]) : 0.0f;
    s_qv[j * HD + t] = j < c ? __fadd_rn(qd, p.v[hoff + t]) : 0.0f;
  }
  __syncthreads();

  // ---- A: scores, half-warp tiles of KT keys x CQ queries ----
  {
    const int hw = t / kLanes, l = t % kLanes;
    float *red = s_red + hw * (CQ * KT * kRedStride);
    // pos row of (query j, key kt0 + b) is prow0 - kt0 + j - b
    const int64_t prow0 = p.s + p.pos_off - p.k_lo - p.pr_lo;
    // Every half-warp takes the same number of rounds (the __syncwarp()s
    // below need both halves of the warp); a tile past the band computes
    // on clamped rows and stores nothing.
    for (int base = 0; base < band; base += NHW * KT) {
      const int kt0 = base + hw * KT;
      float acc[CQ][KT];
#pragma unroll
      for (int j = 0; j < CQ; j++)
#pragma unroll
        for (int b = 0; b < KT; b++) acc[j][b] = 0.0f;
      const float *krow[KT];
      float *kdst[KT];
#pragma unroll
      for (int b = 0; b < KT; b++) {
        const int kk = kt0 + b < band ? kt0 + b : band - 1;
        krow[b] = key_row(p.k_ring, p.k_new, kk);
        kdst[b] = (p.k_ring && kt0 + b >= kk_s && kt0 + b < band) ? ring_row(p.k_ring, kk) : nullptr;
      }
      const float *prow[NPV];
#pragma unroll
      for (int m = 0; m < NPV; m++) {
        int64_t pi = prow0 - kt0 - (KT - 1) + m;  // masked pairs may fall outside
        pi = pi < 0 ? 0 : (pi >= p.np ? p.np - 1 : pi);
        prow[m] = p.pos_p + (p.pr_lo + pi) * (int64_t)p.d + hoff;
      }
      // operands of chunk ch + 1 are loaded while chunk ch computes
      float kv[KT], pv[NPV];
#pragma unroll
      for (int b = 0; b < KT; b++) kv[b] = krow[b][l];
#pragma unroll
      for (int m = 0; m < NPV; m++) pv[m] = prow[m][l];
#pragma unroll 1
      for (int ch = 0; ch < NCH; ch++) {
        const int i = ch * kLanes + l;
#if SC_ATTN_PREFETCH
        const int in = ch + 1 < NCH ? i + kLanes : i;
        float kn[KT], pn[NPV];
#pragma unroll
        for (int b = 0; b < KT; b++) kn[b] = krow[b][in];
#pragma unroll
        for (int m = 0; m < NPV; m++) pn[m] = prow[m][in];
#else
#pragma unroll
        for (int b = 0; b < KT; b++) kv[b] = krow[b][i];
#pragma unroll
        for (int m = 0; m < NPV; m++) pv[m] = prow[m][i];
#endif
#pragma unroll
        for (int b = 0; b < KT; b++)
          if (kdst[b]) kdst[b][i] = kv[b];
#pragma unroll
        for (int j = 0; j < CQ; j++) {
          const float qu = s_qu[j * HD + i], qv = s_qv[j * HD + i];
#pragma unroll
          for (int b = 0; b < KT; b++) {
            const float inner = __fmaf_rn(qv, pv[j - b + KT - 1], acc[j][b]);
            acc[j][b] = __fmaf_rn(qu, kv[b], inner);
          }
        }
#if SC_ATTN_PREFETCH
#pragma unroll
        for (int b = 0; b < KT; b++) kv[b] = kn[b];
#pragma unroll
        for (int m = 0; m < NPV; m++) pv[m] = pn[m];
#endif
      }
#pragma unroll
      for (int j = 0; j < CQ; j++)
#pragma unroll
        for (int b = 0; b < KT; b++) red[(j * KT + b) * kRedStride + l] = acc[j][b];
      __syncwarp();
      for (int pr = l; pr < CQ * KT; pr += kLanes) {
        const int j = pr / KT, b = pr % KT;
        float sum = red[pr * kRedStride];
#pragma unroll
        for (int q = 1; q < kLanes; q++) sum = __fadd_rn(sum, red[pr * kRedStride + q]);
        if (j < c && kt0 + b < band) s_qk[j * band + kt0 + b] = __fmul_rn(sum, p.scale);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  // ---- C: band mask + softmax per query (simd_kernel.rs:1010-1104) ----
  for (int j = warp; j < c; j += NW) {
    int64_t qq = p.s + j, kmin, kmax;
    band_of(qq, p.chunk, p.left_chunks, p.k_hi, kmin, kmax);
    int k0 = (int)(kmin - p.k_lo), k1 = (int)(kmax - p.k_lo);
    float mx = -INFINITY;
    for (int kk = k0 + lane; kk < k1; kk += 32) mx = fmaxf(mx, s_qk[j * band + kk]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int kk = k0 + lane; kk < k1; kk += 32) s_qk[j * band + kk] = exp_rn(__fsub_rn(s_qk[j * band + kk], mx));
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      float sum = 0.0f;
      for (int kk = k0; kk < k1; kk++) sum = __fadd_rn(sum, s_qk[j * band + kk]);
      inv = __fdiv_rn(1.0f, sum);
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int kk = k0 + lane; kk < k1; kk += 32) s_qk[j * band + kk] = __fmul_rn(s_qk[j * band + kk], inv);
  }
  __syncthreads();
  // ---- D: P.V, one thread per head dim ----
  {
    int k0s[CQ], k1s[CQ];
#pragma unroll
    for (int j = 0; j < CQ; j++) {
      int64_t kmin = 0, kmax = 0;
      if (j < c) band_of(p.s + j, p.chunk, p.left_chunks, p.k_hi, kmin, kmax);
      k0s[j] = j < c ? (int)(kmin - p.k_lo) : 0;
      k1s[j] = j < c ? (int)(kmax - p.k_lo) : 0;
    }
    float acc[CQ];
#pragma unroll
    for (int j = 0; j < CQ; j++) acc[j] = 0.0f;
#pragma unroll 4
    for (int kk = 0; kk < band; kk++) {
      float vv = key_row(p.v_ring, p.v_new, kk)[t];
      if (p.v_ring && kk >= kk_s) ring_row(p.v_ring, kk)[t] = vv;
#pragma unroll
      for (int j = 0; j < CQ; j++)
        if (kk >= k0s[j] && kk < k1s[j]) acc[j] = __fmaf_rn(s_qk[j * band + kk], vv, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < CQ; j++)
      if (j < c) p.out[(z * c + j) * p.ldo + hoff + t] = acc[j];
  }
}

// ---------------------------------------------------------------------------
// Staged variant (the path every band that fits in shared memory takes):
// the same arithmetic in the same order, with the head's K band, its pos
// rows and q+u / q+v staged once in shared memory in a lane-major order --
// element i = 16*ch + l of a row sits at (ch/4)*64 + 4l + ch%4 -- so that
// SIMD lane l reads four consecutive chunks of a row with one 16-byte load.
// A warp takes KT keys, each half-warp a group of 4 queries.  After the
// scores, the V band replaces K in shared memory (cp.async, overlapped with
// the softmax) and P.V runs from there with the weights outside each
// query's band set to zero (fma(0, v, acc) == acc, so the sum over the band
// in order is unchanged).
constexpr int kStageKT = 8;

__device__ __forceinline__ int lane_major(int i) { return (i >> 6) * 64 + (i & 15) * 4 + ((i >> 4) & 3); }

__device__ __forceinline__ float f4c(const float4 &v, int c) {
  return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__host__ __device__ constexpr int stage_band_pad(int band) { return (band + 3) & ~3; }

template <int HD, int CQ>
__host__ __device__ constexpr size_t attn_stage_smem_floats(int band, int np) {
  return (size_t)band * HD + (size_t)np * HD + 2 * (size_t)CQ * HD + (size_t)CQ * stage_band_pad(band) +
         (size_t)(HD / 16) * 4 * kStageKT * kRedStride;
}

// Rows in natural order (the sc_attn_stream* API); the encoder's lane-major
// rows take attn_lm_kernel below.
template <int HD, int CQ>
__global__ void __launch_bounds__(HD, 2) attn_stage_kernel(const AttnParams p) {
  constexpr int NW = HD / 32;
  constexpr int NQG = CQ / 4;        // query groups of 4
  constexpr int KT = kStageKT;
  constexpr int NPV = 4 + KT - 1;    // pos rows of one (group, tile)
  constexpr int NHALF = HD / 64;     // 4-chunk slices per row
  extern __shared__ __align__(16) float sm[];
  const int band = (int)(p.k_hi - p.k_lo), np = p.np, bp = stage_band_pad(band);
  float *s_k = sm;                   // [band][HD] K lane-major, later V natural
  float *s_p = s_k + band * HD;      // [np][HD]   pos rows lane-major
  float *s_qu = s_p + np * HD;       // [CQ][HD]   q + u lane-major
  float *s_qv = s_qu + CQ * HD;      // [CQ][HD]   q + v lane-major
  float *s_w = s_qv + CQ * HD;       // [CQ][bp]   scores, then weights
  float *s_red = s_w + CQ * bp;      // [2*NW][4*KT][kRedStride]
  const int h = blockIdx.x;
  const int64_t z = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int hoff = h * HD;
  const int c = p.c;
  const int64_t zq = p.zrows > 0 ? p.zrows : c, zn = p.zrows > 0 ? p.zrows : p.rows_new;
  const int kk_new = (int)(p.new_lo - p.k_lo);
  const int slot0 = band_slot0(p);
  const int cap = (int)p.cap;
  auto ring_row = [&](float *ring, int kk) -> float * {
    int slot = slot0 + kk;
    slot = slot >= cap ? slot - cap : slot;
    return ring + (z * cap + slot) * (int64_t)p.d + hoff;
  };
  auto key_row = [&](float *ring, const float *nw, int kk) -> const float * {
    if (kk >= kk_new) return nw + (z * zn + p.r0 + (kk - kk_new)) * p.ld_new + hoff;
    return ring_row(ring, kk);
  };
  const int kk_s = (int)(p.s - p.k_lo);

  // ---- stage K, pos rows (async copies, all in flight at once), q; the
  // new K rows also go to the ring.  Natural rows are copied element by
  // element into their lane-major slots. ----
  {
    const int dt = lane_major(t);
    for (int kk = 0; kk < band; kk++) cp_async4(s_k + kk * HD + dt, key_row(p.k_ring, p.k_new, kk) + t);
    const float *prow = p.pos_p + p.pr_lo * (int64_t)p.d + hoff + t;
    for (int r = 0; r < np; r++) cp_async4(s_p + r * HD + dt, prow + (int64_t)r * p.d);
  }
  if (p.k_ring)
    for (int kk = max(kk_s, 0) + warp; kk < band; kk += NW) {
      const float *src = key_row(p.k_ring, p.k_new, kk);
      float *dst = ring_row(p.k_ring, kk);
      for (int e4 = lane; e4 < HD / 4; e4 += 32)
        *reinterpret_cast<float4 *>(dst + e4 * 4) = *reinterpret_cast<const float4 *>(src + e4 * 4);
    }
  {
    const int dt = lane_major(t);
    for (int j = 0; j < CQ; j++) {
      const float qd = j < c ? p.q[(z * zq + p.r0 + j) * p.ldq + hoff + t] : 0.0f;
      s_qu[j * HD + dt] = j < c ? __fadd_rn(qd, p.u[hoff + t]) : 0.0f;
      s_qv[j * HD + dt] = j < c ? __fadd_rn(qd, p.v[hoff + t]) : 0.0f;
    }
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- A: scores (score_dot order) ----
  {
    const int hw2 = lane >> 4, l = lane & 15;
    float *red = s_red + (warp * 2 + hw2) * (4 * KT * kRedStride);
    // pos row of (query j, key kk) is prow0 + j - kk
    const int prow0 = (int)(p.s + p.pos_off - p.k_lo - p.pr_lo);
    for (int kt0 = warp * KT; kt0 < band; kt0 += NW * KT) {
      for (int qg = hw2; qg < NQG; qg += 2) {
        float acc[4][KT];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
          for (int b = 0; b < KT; b++) acc[j][b] = 0.0f;
        int koff[KT], poff[NPV];
#pragma unroll
        for (int b = 0; b < KT; b++) koff[b] = min(kt0 + b, band - 1) * HD + l * 4;
#pragma unroll
        for (int m = 0; m < NPV; m++) {
          int pi = prow0 - kt0 + 4 * qg - (KT - 1) + m;  // masked pairs may fall outside
          pi = pi < 0 ? 0 : (pi >= np ? np - 1 : pi);
          poff[m] = pi * HD + l * 4;
        }
        const int qoff = 4 * qg * HD + l * 4;
#pragma unroll
        for (int hh = 0; hh < NHALF; hh++) {
          float4 kv[KT], pv[NPV], qu[4], qv[4];
#pragma unroll
          for (int b = 0; b < KT; b++) kv[b] = *reinterpret_cast<const float4 *>(s_k + koff[b] + hh * 64);
#pragma unroll
          for (int m = 0; m < NPV; m++) pv[m] = *reinterpret_cast<const float4 *>(s_p + poff[m] + hh * 64);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            qu[j] = *reinterpret_cast<const float4 *>(s_qu + qoff + j * HD + hh * 64);
            qv[j] = *reinterpret_cast<const float4 *>(s_qv + qoff + j * HD + hh * 64);
          }
#pragma unroll
          for (int cc = 0; cc < 4; cc++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
              for (int b = 0; b < KT; b++) {
                const float inner = __fmaf_rn(f4c(qv[j], cc), f4c(pv[j - b + KT - 1], cc), acc[j][b]);
                acc[j][b] = __fmaf_rn(f4c(qu[j], cc), f4c(kv[b], cc), inner);
              }
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
          for (int b = 0; b < KT; b++) red[(j * KT + b) * kRedStride + l] = acc[j][b];
        __syncwarp();
        for (int pr = l; pr < 4 * KT; pr += kLanes) {
          const int j = 4 * qg + pr / KT, b = pr % KT;
          float sum = red[pr * kRedStride];
#pragma unroll
          for (int q = 1; q < kLanes; q++) sum = __fadd_rn(sum, red[pr * kRedStride + q]);
          if (j < c && kt0 + b < band) s_w[j * bp + kt0 + b] = __fmul_rn(sum, p.scale);
        }
        __syncwarp();
      }
    }
  }
  __syncthreads();
  // ---- V band into shared memory (natural order), overlapped with C ----
  for (int kk = warp; kk < band; kk += NW) {
    const float *src = key_row(p.v_ring, p.v_new, kk);
    for (int e4 = lane; e4 < HD / 4; e4 += 32) cp_async16(s_k + kk * HD + e4 * 4, src + e4 * 4);
    if (p.v_ring && kk >= kk_s) {
      float *dst = ring_row(p.v_ring, kk);
      for (int e4 = lane; e4 < HD / 4; e4 += 32)
        *reinterpret_cast<float4 *>(dst + e4 * 4) = *reinterpret_cast<const float4 *>(src + e4 * 4);
    }
  }
  // ---- C: band mask + softmax per query (simd_kernel.rs:1010-1104) ----
  for (int j = warp; j < CQ; j += NW) {
    float *row = s_w + j * bp;
    if (j >= c) {
      for (int kk = lane; kk < bp; kk += 32) row[kk] = 0.0f;
      continue;
    }
    int64_t kmin, kmax;
    band_of(p.s + j, p.chunk, p.left_chunks, p.k_hi, kmin, kmax);
    const int k0 = (int)(kmin - p.k_lo), k1 = (int)(kmax - p.k_lo);
    float mx = -INFINITY;
    for (int kk = k0 + lane; kk < k1; kk += 32) mx = fmaxf(mx, row[kk]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int kk = lane; kk < bp; kk += 32)
      row[kk] = (kk >= k0 && kk < k1) ? exp_rn(__fsub_rn(row[kk], mx)) : 0.0f;
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      float sum = 0.0f;
      for (int kk = k0; kk < k1; kk++) sum = __fadd_rn(sum, row[kk]);
      inv = __fdiv_rn(1.0f, sum);
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int kk = lane; kk < bp; kk += 32) row[kk] = __fmul_rn(row[kk], inv);
  }
  cp_async_wait_all();
  __syncthreads();
  // ---- D: P.V over the band in order, one thread per head dim ----
  {
    float acc[CQ];
#pragma unroll
    for (int j = 0; j < CQ; j++) acc[j] = 0.0f;
    for (int kk0 = 0; kk0 < bp; kk0 += 4) {
      float4 w[CQ];
#pragma unroll
      for (int j = 0; j < CQ; j++) w[j] = *reinterpret_cast<const float4 *>(s_w + j * bp + kk0);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int kk = kk0 + e;
        if (kk >= band) break;
        const float vv = s_k[kk * HD + t];
#pragma unroll
        for (int j = 0; j < CQ; j++) acc[j] = __fmaf_rn(f4c(w[j], e), vv, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < CQ; j++)
      if (j < c) {
        if (p.out) p.out[(z * zq + p.r0 + j) * p.ldo + hoff + t] = acc[j];
        if (p.qout.xq) {  // the warp's 32 dims are one block of the out-proj input
          float sblk;
          const int8_t q = warp_quantize_block(acc[j], true, sblk);
          p.qout.xq[qout_code_index(p.qout, z * zq + p.r0 + j, hoff + t)] = code_half(q);
          if (lane == 0) p.qout.dx[qout_dx_index(p.qout, z * zq + p.r0 + j, (hoff + t) >> 5)] = sblk;
        }
      }
  }
}

// ---- lane-major kernel (the encoder's layout) ------------------------------
// The same arithmetic as the kernels above, laid out for occupancy: four
// CTAs per SM (at most 128 registers a thread, about 51 KB of shared memory
// at band 77) and uniform control flow.
//   A. a warp takes one tile of kLmKT = 4 keys for two groups of 4 queries
//      (one per half-warp): 16 accumulators per lane, pos rows read through
//      L1 from one precomputed row offset each.  K tiles sit kLmTile floats
//      apart (4 rows + 32 spare), and the 16 lane sums of the tile's pairs
//      go through the tile itself once its K rows are dead: half-warp hw's
//      pair pr, lane x at hw*272 + pr*17 + x, conflict-free for the stores
//      (one pair, 16 lanes) and the ordered reads (16 pairs, one lane), and
//      every address an immediate offset.
//   C. per query: max and exp over the band on the warp's lanes, then the
//      warp's two queries' sequential sums on two lanes at once.
//   D. P.V over the keys any query of the call attends to ([k0 of the
//      first query, k1 of the last)), 4 keys per step, a uniform tail.
__device__ __forceinline__ void band_of32(int qq, int chunk, int left_chunks, int k_hi, int &kmin, int &kmax) {
  const int qc = qq / chunk;
  kmin = (qc > left_chunks ? qc - left_chunks : 0) * chunk;
  const int hi = (qc + 1) * chunk;
  kmax = hi < k_hi ? hi : k_hi;
}

constexpr int kLmKT = 4;
constexpr int kLmRed = 2 * 16 * 17;  // lane-sum scratch of one warp's tile

template <int HD>
__host__ __device__ constexpr int lm_tile_floats() {
  return kLmKT * HD + 32 > kLmRed ? kLmKT * HD + 32 : kLmRed;
}

__host__ __device__ constexpr int lm_wstride(int band) {
  // a multiple of 4 (16-byte weight loads) with an odd number of 16-byte
  // units, so that the rows of queries j and j + 4 sit in different banks
  return ((band + 3) & ~3) | 4;
}

template <int HD, int CQ>
__host__ __device__ constexpr size_t attn_lm_smem_floats(int band) {
  return (size_t)((band + kLmKT - 1) / kLmKT) * lm_tile_floats<HD>() + 2 * (size_t)CQ * HD +
         (size_t)CQ * lm_wstride(band) + (CQ == 8 ? 0 : (size_t)(HD / 32) * kLmRed);
}

template <int HD, int CQ>
__global__ void __launch_bounds__(HD, 4) attn_lm_kernel(const AttnParams p) {
  constexpr int NW = HD / 32;
  constexpr int KT = kLmKT;
  constexpr int NQG = CQ / 4;          // query groups of 4; a warp takes two
  constexpr int NPV = 4 + KT - 1;      // pos rows of one (group, tile)
  constexpr int NHALF = HD / 64;       // 16-byte slices of a lane's dims
  constexpr int TS = lm_tile_floats<HD>();
  // the tile holds the lane sums when one warp owns the tile
  constexpr bool kRedInK = NQG == 2;
  extern __shared__ __align__(16) float sm[];
  const int band = (int)(p.k_hi - p.k_lo), nt = (band + KT - 1) / KT, bw = lm_wstride(band);
  float *s_k = sm;                     // [nt][TS]: row kk at (kk/4)*TS + (kk%4)*HD; K lane-major, later V natural
  float *s_qu = s_k + nt * TS;         // [CQ][HD] q + u lane-major
  float *s_qv = s_qu + CQ * HD;        // [CQ][HD] q + v lane-major
  float *s_w = s_qv + CQ * HD;         // [CQ][bw] scores, then weights
  float *s_red = s_w + CQ * bw;        // [NW][kLmRed] when two warps share a tile
  auto srow = [&](int kk) { return s_k + (kk >> 2) * TS + (kk & 3) * HD; };
  const int h = blockIdx.x;
  const int64_t z = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int hoff = h * HD;
  const int c = p.c;
  const int64_t zq = p.zrows > 0 ? p.zrows : c, zn = p.zrows > 0 ? p.zrows : p.rows_new;
  // Frame numbers fit in 32 bits (attn_prepare checks k_hi).  The values
  // below come straight from the parameters where they are used, so that
  // none of them stays live through the score tiles.
#define LM_S32 ((int)p.s)
#define LM_KLO ((int)p.k_lo)
  // Band row kk into the tile layout, a warp per row and 16 bytes a lane: the
  // call's new frames (kk >= kk_new) from the projection output, also
  // written to the ring (slot = frame % cap), older frames from the ring.
  auto stage_rows = [&](float *ring, const float *nw) {
    const int kk_new = (int)p.new_lo - LM_KLO, cap = (int)p.cap;
    const int slot0 = band_slot0(p);
    const int64_t new_row0 = z * zn + p.r0;  // projection row of frame new_lo
    const bool lane_on = HD / 4 >= 32 || lane < HD / 4;
    float *rz = ring ? ring + z * cap * (int64_t)p.d + hoff + lane * 4 : nullptr;
    int slot = slot0 + warp;
    slot = slot >= cap ? slot - cap : slot;
    for (int kk = warp; kk < band; kk += NW) {
      if (kk >= kk_new) {
        const float *src = nw + (new_row0 + (kk - kk_new)) * p.ld_new + hoff + lane * 4;
        if (lane_on) cp_async16(srow(kk) + lane * 4, src);
      } else if (lane_on) {
        cp_async16(srow(kk) + lane * 4, rz + slot * p.d);
      }
      slot += NW;
      slot = slot >= cap ? slot - cap : slot;
    }
  };
  // The call's new rows, landed in shared memory, into the ring (slot =
  // frame % cap): stores only, so no load latency in the staging loop.
  auto ring_rows = [&](float *ring) {
    if (!ring) return;
    const int kk_new = (int)p.new_lo - LM_KLO, cap = (int)p.cap;
    float *rz = ring + z * cap * (int64_t)p.d + hoff + lane * 4;
    const int slot0 = band_slot0(p);
    for (int kk = kk_new + warp; kk < band; kk += NW) {
      int slot = slot0 + kk;
      slot = slot >= cap ? slot - cap : slot;
      if (HD / 4 >= 32 || lane < HD / 4)
        *reinterpret_cast<float4 *>(rz + slot * p.d) = *reinterpret_cast<const float4 *>(srow(kk) + lane * 4);
    }
  };

  // ---- stage: K band, q + u and q + v; then the new K rows into the ring ----
  stage_rows(p.k_ring, p.k_new);
  {
    const float uu = p.u[hoff + t], vv = p.v[hoff + t];
    const float *qrow = p.q + (z * zq + p.r0) * p.ldq + hoff + t;
#pragma unroll
    for (int j = 0; j < CQ; j++) {
      const float qd = j < c ? qrow[(int64_t)j * p.ldq] : 0.0f;
      s_qu[j * HD + t] = j < c ? __fadd_rn(qd, uu) : 0.0f;
      s_qv[j * HD + t] = j < c ? __fadd_rn(qd, vv) : 0.0f;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (p.k_ring) {  // before the score tiles reuse the K rows as scratch
    ring_rows(p.k_ring);
    __syncthreads();
  }

  // ---- A: scores (score_dot order) ----
  {
    const int hw = lane >> 4, l = lane & 15;
    // pos row of (query j, key kk) is prow0 + j - kk
    const int prow0 = LM_S32 + (int)(p.pos_off - p.pr_lo) - LM_KLO;
    const float *pbase = p.pos_p + p.pr_lo * (int64_t)p.d + hoff + l * 4;
    const int nunits = nt * (NQG / 2);
    for (int u = warp; u < nunits; u += NW) {
      const int tile = u / (NQG / 2), qg = (u % (NQG / 2)) * 2 + hw, kt0 = tile * KT;
      float acc[4][KT];
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int b = 0; b < KT; b++) acc[j][b] = 0.0f;
      int poff[NPV];
#pragma unroll
      for (int m = 0; m < NPV; m++) {
        const int pi = prow0 - kt0 + 4 * qg - (KT - 1) + m;  // masked pairs may fall outside
        poff[m] = (pi < 0 ? 0 : (pi >= p.np ? p.np - 1 : pi)) * p.d;
      }
      const float *kb = s_k + tile * TS + l * 4;
      const float *qub = s_qu + 4 * qg * HD + l * 4, *qvb = s_qv + 4 * qg * HD + l * 4;
#pragma unroll
      for (int hh = 0; hh < NHALF; hh++) {
        float4 kv[KT], pv[NPV], qu[4], qv[4];
#pragma unroll
        for (int b = 0; b < KT; b++) kv[b] = *reinterpret_cast<const float4 *>(kb + b * HD + hh * 64);
#pragma unroll
        for (int m = 0; m < NPV; m++) pv[m] = __ldg(reinterpret_cast<const float4 *>(pbase + poff[m] + hh * 64));
#pragma unroll
        for (int j = 0; j < 4; j++) {
          qu[j] = *reinterpret_cast<const float4 *>(qub + j * HD + hh * 64);
          qv[j] = *reinterpret_cast<const float4 *>(qvb + j * HD + hh * 64);
        }
#pragma unroll
        for (int cc = 0; cc < 4; cc++)
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int b = 0; b < KT; b++) {
              const float inner = __fmaf_rn(f4c(qv[j], cc), f4c(pv[j - b + KT - 1], cc), acc[j][b]);
              acc[j][b] = __fmaf_rn(f4c(qu[j], cc), f4c(kv[b], cc), inner);
            }
      }
      // the 16 lane sums of each of the half-warp's 16 pairs
      float *red = (kRedInK ? s_k + tile * TS : s_red + warp * kLmRed) + hw * 272;
      __syncwarp();  // both half-warps are done with the tile's K rows
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int b = 0; b < KT; b++) red[(j * KT + b) * 17 + l] = acc[j][b];
      __syncwarp();
      {
        const float *rr = red + l * 17;  // pair pr = l
        float sum = rr[0];
#pragma unroll
        for (int x = 1; x < kLanes; x++) sum = __fadd_rn(sum, rr[x]);
        const int j = 4 * qg + l / KT, kk = kt0 + l % KT;
        if (j < c && kk < band) s_w[j * bw + kk] = __fmul_rn(sum, p.scale);
      }
      __syncwarp();  // the scratch is read before the warp's next tile
    }
  }
  __syncthreads();
  // ---- V band into shared memory (natural order), overlapped with C ----
  stage_rows(p.v_ring, p.v_new);
  // ---- C: band mask + softmax per query (simd_kernel.rs:1010-1104) ----
  {
    constexpr int QPW = (CQ + NW - 1) / NW;  // queries per warp
#pragma unroll
    for (int i = 0; i < QPW; i++) {
      const int j = warp + i * NW;
      if (j >= CQ) continue;
      float *row = s_w + j * bw;
      if (j >= c) {
        for (int kk = lane; kk < bw; kk += 32) row[kk] = 0.0f;
        continue;
      }
      int k0, k1;
      band_of32(LM_S32 + j, (int)p.chunk, (int)p.left_chunks, (int)p.k_hi, k0, k1);
      k0 -= LM_KLO;
      k1 -= LM_KLO;
      float mx = -INFINITY;
      for (int kk = k0 + lane; kk < k1; kk += 32) mx = fmaxf(mx, row[kk]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      for (int kk = lane; kk < bw; kk += 32) row[kk] = (kk >= k0 && kk < k1) ? exp_rn(__fsub_rn(row[kk], mx)) : 0.0f;
    }
    __syncwarp();
    // lane i sums the warp's i-th query over its band in order, the warp's
    // lanes side by side (rows j and j + NW sit in different banks)
    float mine = 0.0f;
    {
      const int j = warp + lane * NW;
      if (lane < QPW && j < c) {
        int k0, k1;
        band_of32(LM_S32 + j, (int)p.chunk, (int)p.left_chunks, (int)p.k_hi, k0, k1);
        const float *row = s_w + j * bw - LM_KLO;
        float sum = 0.0f;
        for (int kk = k0; kk < k1; kk++) sum = __fadd_rn(sum, row[kk]);
        mine = __fdiv_rn(1.0f, sum);
      }
    }
#pragma unroll
    for (int i = 0; i < QPW; i++) {
      const int j = warp + i * NW;
      const float inv = __shfl_sync(0xffffffffu, mine, i);
      if (j >= c) continue;
      float *row = s_w + j * bw;
      for (int kk = lane; kk < bw; kk += 32) row[kk] = __fmul_rn(row[kk], inv);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  ring_rows(p.v_ring);
  // ---- D: P.V over the keys the call attends to, one thread per head dim ----
  {
    int kmin, kmax, kmin2, kmax2;
    band_of32(LM_S32, (int)p.chunk, (int)p.left_chunks, (int)p.k_hi, kmin, kmax);
    band_of32(LM_S32 + c - 1, (int)p.chunk, (int)p.left_chunks, (int)p.k_hi, kmin2, kmax2);
    const int ka = (kmin - LM_KLO) & ~3, kb = kmax2 - LM_KLO;
    float acc[CQ];
#pragma unroll
    for (int j = 0; j < CQ; j++) acc[j] = 0.0f;
    int kk = ka;
    for (; kk + 4 <= kb; kk += 4) {
      float4 w[CQ];
#pragma unroll
      for (int j = 0; j < CQ; j++) w[j] = *reinterpret_cast<const float4 *>(s_w + j * bw + kk);
      float vv[4];
      const float *vt = s_k + (kk >> 2) * TS + t;
#pragma unroll
      for (int e = 0; e < 4; e++) vv[e] = vt[e * HD];
#pragma unroll
      for (int e = 0; e < 4; e++)
#pragma unroll
        for (int j = 0; j < CQ; j++) acc[j] = __fmaf_rn(f4c(w[j], e), vv[e], acc[j]);
    }
    for (; kk < kb; kk++) {
      const float vv = srow(kk)[t];
#pragma unroll
      for (int j = 0; j < CQ; j++) acc[j] = __fmaf_rn(s_w[j * bw + kk], vv, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < CQ; j++)
      if (j < c) {
        if (p.out) p.out[(z * zq + p.r0 + j) * p.ldo + hoff + t] = acc[j];
        if (p.qout.xq) {  // the warp's 32 dims are one block of the out-proj input
          float sblk;
          const int8_t q = warp_quantize_block(acc[j], true, sblk);
          p.qout.xq[qout_code_index(p.qout, z * zq + p.r0 + j, hoff + t)] = code_half(q);
          if (lane == 0) p.qout.dx[qout_dx_index(p.qout, z * zq + p.r0 + j, (hoff + t) >> 5)] = sblk;
        }
      }
  }
}

#undef LM_S32
#undef LM_KLO

// Validates the band and pos rows the chunk touches, fills pr_lo/np.
int attn_prepare(AttnParams &p, int64_t n_pos) {
  if (p.c <= 0 || p.c > 16 || p.d <= 0 || p.n_heads <= 0 || p.d % p.n_heads != 0) {
    set_error("attn_stream: bad shape c=%d d=%d n_heads=%d (c must be 1..16)", p.c, p.d, p.n_heads);
    return kErrInvalid;
  }
  int hd = p.d / p.n_heads;
  if (hd != 128 && hd != 64) {
    set_error("attn_stream: head_dim %d unsupported (64 or 128)", hd);
    return kErrUnsupported;
  }
  if (p.chunk <= 0 || p.left_chunks < 0 || p.s < 0 || p.k_lo < 0 || p.k_hi <= p.k_lo ||
      p.k_hi - p.k_lo > 256 || p.k_hi + p.chunk >= ((int64_t)1 << 30) || p.left_chunks >= ((int64_t)1 << 30)) {
    set_error("attn_stream: bad band [%lld, %lld) chunk %lld (band must be 1..256)",
              (long long)p.k_lo, (long long)p.k_hi, (long long)p.chunk);
    return kErrInvalid;
  }
  int64_t lo = INT64_MAX, hi = INT64_MIN;
  for (int j = 0; j < p.c; j++) {
    int64_t qq = p.s + j;
    int64_t qc = qq / p.chunk;
    int64_t kmin = (qc > p.left_chunks ? qc - p.left_chunks : 0) * p.chunk;
    int64_t kmax = (qc + 1) * p.chunk < p.k_hi ? (qc + 1) * p.chunk : p.k_hi;
    if (kmin < p.k_lo || kmax <= kmin || qq >= p.k_hi) {
      set_error("attn_stream: query %lld band [%lld, %lld) outside [k_lo=%lld, k_hi=%lld)",
                (long long)qq, (long long)kmin, (long long)kmax, (long long)p.k_lo,
                (long long)p.k_hi);
      return kErrInvalid;
    }
    int64_t a = qq + p.pos_off - (kmax - 1), b = qq + p.pos_off - kmin;
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if (lo < 0 || hi >= n_pos) {
    set_error("attn_stream: pos rows [%lld, %lld] outside pos_p [0, %lld)", (long long)lo,
              (long long)hi, (long long)n_pos);
    return kErrInvalid;
  }
  if (p.k_ring) {
    if (p.cap < p.k_hi - p.k_lo || p.new_lo != p.s || p.rows_new != p.k_hi - p.s) {
      set_error("attn_stream: ring cap %lld smaller than band %lld or new frames inconsistent",
                (long long)p.cap, (long long)(p.k_hi - p.k_lo));
      return kErrInvalid;
    }
  }
  p.pr_lo = lo;
  p.np = (int)(hi - lo + 1);
  return kOk;
}

// The staged kernel needs 16-byte aligned rows and its shared-memory
// footprint within the 227 KB a CTA may use.
template <int HD, int CQ>
static bool stage_fits(const AttnParams &p) {
  const int band = (int)(p.k_hi - p.k_lo);
  auto al = [](const void *q) { return ((uintptr_t)q & 15) == 0; };
  const bool aligned = al(p.q) && al(p.k_new) && al(p.v_new) && al(p.pos_p) && p.d % 4 == 0 && p.ldq % 4 == 0 &&
                       p.ld_new % 4 == 0 && (!p.k_ring || (al(p.k_ring) && al(p.v_ring)));
  return aligned && (p.lane_major || attn_stage_smem_floats<HD, CQ>(band, p.np) * sizeof(float) <= 227 * 1024);
}

template <int HD, int CQ>
static int launch_stage(const AttnParams &p, int64_t n_streams, cudaStream_t st) {
  const int band = (int)(p.k_hi - p.k_lo);
  const size_t smem = attn_stage_smem_floats<HD, CQ>(band, p.np) * sizeof(float);
  auto kern = attn_stage_kernel<HD, CQ>;
  static std::atomic<size_t> smem_limit[64];
  const int rc = raise_smem_limit((const void *)kern, smem, smem_limit);
  if (rc) return rc;
  kern<<<dim3((unsigned)p.n_heads, (unsigned)n_streams), HD, smem, st>>>(p);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

template <int HD, int CQ>
static int launch_lane_major(const AttnParams &p, int64_t n_streams, cudaStream_t st) {
  const int band = (int)(p.k_hi - p.k_lo);
  const size_t smem = attn_lm_smem_floats<HD, CQ>(band) * sizeof(float);
  if (smem > 227 * 1024) {
    set_error("attn_stream: band %d needs %zu bytes of shared memory", band, smem);
    return kErrUnsupported;
  }
  auto kern = attn_lm_kernel<HD, CQ>;
  static std::atomic<size_t> smem_limit[64];
  const int rc = raise_smem_limit((const void *)kern, smem, smem_limit);
  if (rc) return rc;
  kern<<<dim3((unsigned)p.n_heads, (unsigned)n_streams), HD, smem, st>>>(p);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

template <int HD, int CQ>
static int launch_attn_t(const AttnParams &p, int64_t n_streams, cudaStream_t st) {
  if (p.lane_major && stage_fits<HD, CQ>(p)) return launch_lane_major<HD, CQ>(p, n_streams, st);
  if (!p.lane_major && stage_fits<HD, CQ>(p)) return launch_stage<HD, CQ>(p, n_streams, st);
  if (p.lane_major || p.qout.xq || p.zrows) {
    set_error("attn_stream: lane-major rows / quantised output / row sub-ranges need the staged kernel (band %lld too large or "
              "rows unaligned)",
              (long long)(p.k_hi - p.k_lo));
    return kErrUnsupported;
  }
  int band = (int)(p.k_hi - p.k_lo);
  size_t smem = attn_smem_floats<HD, CQ>(band) * sizeof(float);
  auto kern = attn_stream_kernel<HD, CQ>;
  static std::atomic<size_t> smem_limit[64];
  const int rc = raise_smem_limit((const void *)kern, smem, smem_limit);
  if (rc) return rc;
  kern<<<dim3((unsigned)p.n_heads, (unsigned)n_streams), HD, smem, st>>>(p);
  note_launch();
  SC_CUDA(cudaGetLastError());
  return kOk;
}

int launch_attn(const AttnParams &p, int64_t n_streams, cudaStream_t st) {
  int hd = p.d / p.n_heads;
  if (n_streams <= 0 || n_streams > 65535) {
    set_error("attn_stream: n_streams %lld out of range", (long long)n_streams);
    return kErrInvalid;
  }
  if (hd == 128) return p.c <= 8 ? launch_attn_t<128, 8>(p, n_streams, st)
                                  : launch_attn_t<128, 16>(p, n_streams, st);
  return p.c <= 8 ? launch_attn_t<64, 8>(p, n_streams, st) : launch_attn_t<64, 16>(p, n_streams, st);
}

}  // namespace sc
