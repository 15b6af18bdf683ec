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
#include "sc_kernels.cuh"

namespace sc {

__device__ __forceinline__ void band_of(int64_t qq, int64_t chunk, int64_t left_chunks,
                                        int64_t k_hi, int64_t &kmin, int64_t &kmax) {
  int64_t qc = qq / chunk;
  kmin = (qc > left_chunks ? qc - left_chunks : 0) * chunk;
  int64_t hi = (qc + 1) * chunk;
  kmax = hi < k_hi ? hi : k_hi;
}

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

  auto key_row = [&](const float *ring, const float *nw, int64_t fr) -> const float * {
    if (fr >= p.new_lo) return nw + (z * p.rows_new + (fr - p.new_lo)) * p.ld_new + hoff;
    return ring + (z * p.cap + fr % p.cap) * (int64_t)p.d + hoff;
  };

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
        const int64_t fr = p.k_lo + (kt0 + b < band ? kt0 + b : band - 1);
        krow[b] = key_row(p.k_ring, p.k_new, fr);
        kdst[b] = (p.k_ring && fr >= p.s && kt0 + b < band)
                      ? p.k_ring + (z * p.cap + fr % p.cap) * (int64_t)p.d + hoff
                      : nullptr;
      }
      const float *prow[NPV];
#pragma unroll
      for (int m = 0; m < NPV; m++) {
        int64_t pi = prow0 - kt0 - (KT - 1) + m;  // masked pairs may fall outside
        pi = pi < 0 ? 0 : (pi >= p.np ? p.np - 1 : pi);
        prow[m] = p.pos_p + (p.pr_lo + pi) * (int64_t)p.d + hoff;
      }
#pragma unroll 1
      for (int ch = 0; ch < NCH; ch++) {
        const int i = ch * kLanes + l;
        float kv[KT], pv[NPV];
#pragma unroll
        for (int b = 0; b < KT; b++) kv[b] = krow[b][i];
#pragma unroll
        for (int m = 0; m < NPV; m++) pv[m] = prow[m][i];
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
    for (int kk = 0; kk < band; kk++) {
      int64_t fr = p.k_lo + kk;
      float vv = key_row(p.v_ring, p.v_new, fr)[t];
      if (p.v_ring && fr >= p.s) p.v_ring[(z * p.cap + fr % p.cap) * (int64_t)p.d + hoff + t] = vv;
#pragma unroll
      for (int j = 0; j < CQ; j++)
        if (kk >= k0s[j] && kk < k1s[j]) acc[j] = __fmaf_rn(s_qk[j * band + kk], vv, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < CQ; j++)
      if (j < c) p.out[(z * c + j) * p.ldo + hoff + t] = acc[j];
  }
}

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
      p.k_hi - p.k_lo > 256) {
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

template <int HD, int CQ>
static int launch_attn_t(const AttnParams &p, int64_t n_streams, cudaStream_t st) {
  int band = (int)(p.k_hi - p.k_lo);
  size_t smem = attn_smem_floats<HD, CQ>(band) * sizeof(float);
  auto kern = attn_stream_kernel<HD, CQ>;
  static size_t smem_set[64] = {};
  int dev = 0;
  SC_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && dev < 64 && smem_set[dev] < smem) {
    SC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[dev] = smem;
  }
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
