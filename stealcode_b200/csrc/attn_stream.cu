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
// per head-dim element.  Each K, V and pos row of the head is read exactly
// once per CTA and used by all the chunk's queries:
//   A. QK^T: warps take band rows; each lane holds HD/32 dims of every
//      query's (q + u); one multi-value butterfly reduces all queries'
//      partials;
//   B. pos term R[q, p] = (q + v) . pos_p[p] over the pos rows the chunk
//      touches (the Toeplitz structure: c + band - 1 rows, not c * band);
//   C. band mask + softmax per query (exp, max, 1/sum as the reference);
//   D. P.V with one thread per dim, V rows streamed once.
// In ring mode the K/V of the chunk's new frames come from the projection
// output and are written into the stream's HBM ring (slot = frame % cap);
// older band frames are read from the ring.
#include "sc_kernels.cuh"

namespace sc {

// Reduce NV per-lane values over the warp in log2(NV) exchange steps (each
// step halves the values a lane carries), then plain xor steps.  Afterwards
// the lane holds the full sum of value index multi_idx(lane).
template <int NV>
__device__ __forceinline__ float multi_reduce(float (&v)[NV], int lane) {
#pragma unroll
  for (int cnt = NV, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
    const int half = cnt >> 1;
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; i++) {
      float send = up ? v[i] : v[i + half];
      float keep = up ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  float r = v[0];
  constexpr int steps = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
#pragma unroll
  for (int off = 16 >> steps; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
  return r;
}

template <int NV>
__device__ __forceinline__ int multi_idx(int lane) {
  int idx = 0;
#pragma unroll
  for (int cnt = NV, off = 16; cnt > 1; cnt >>= 1, off >>= 1)
    if (lane & off) idx += cnt >> 1;
  return idx;
}

__device__ __forceinline__ void band_of(int64_t qq, int64_t chunk, int64_t left_chunks,
                                        int64_t k_hi, int64_t &kmin, int64_t &kmax) {
  int64_t qc = qq / chunk;
  kmin = (qc > left_chunks ? qc - left_chunks : 0) * chunk;
  int64_t hi = (qc + 1) * chunk;
  kmax = hi < k_hi ? hi : k_hi;
}

// HD = head_dim (one thread per dim, HD/32 warps); CQ = queries padded.
template <int HD, int CQ>
__global__ void __launch_bounds__(HD) attn_stream_kernel(const AttnParams p) {
  constexpr int NW = HD / 32;
  constexpr int VPL = HD / 32;  // dims per lane in phases A/B
  extern __shared__ __align__(16) float sm[];
  const int band = (int)(p.k_hi - p.k_lo);
  float *s_qk = sm;                      // [CQ][band]  scores, then probabilities
  float *s_r = sm + CQ * band;           // [CQ][np]
  const int h = blockIdx.x;
  const int64_t z = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int hoff = h * HD;
  const int c = p.c;

  auto key_row = [&](const float *ring, const float *nw, int64_t fr) -> const float * {
    if (fr >= p.new_lo) return nw + (z * p.rows_new + (fr - p.new_lo)) * p.ld_new + hoff;
    return ring + (z * p.cap + fr % p.cap) * (int64_t)p.d + hoff;
  };

  // ---- A: QK^T over the band ----
  {
    float qa[CQ][VPL];
#pragma unroll
    for (int j = 0; j < CQ; j++)
#pragma unroll
      for (int e = 0; e < VPL; e++) {
        int dim = lane * VPL + e;
        qa[j][e] = j < c ? p.q[(z * c + j) * p.ldq + hoff + dim] + p.u[hoff + dim] : 0.0f;
      }
    for (int kk = warp; kk < band; kk += NW) {
      int64_t fr = p.k_lo + kk;
      const float *kr = key_row(p.k_ring, p.k_new, fr);
      float kv[VPL];
#pragma unroll
      for (int e = 0; e < VPL; e++) kv[e] = kr[lane * VPL + e];
      if (p.k_ring && fr >= p.s) {
        float *dst = p.k_ring + (z * p.cap + fr % p.cap) * (int64_t)p.d + hoff;
#pragma unroll
        for (int e = 0; e < VPL; e++) dst[lane * VPL + e] = kv[e];
      }
      float part[CQ];
#pragma unroll
      for (int j = 0; j < CQ; j++) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < VPL; e++) a = fmaf(qa[j][e], kv[e], a);
        part[j] = a;
      }
      float r = multi_reduce<CQ>(part, lane);
      int idx = multi_idx<CQ>(lane);
      constexpr int lowmask = (32 / CQ) - 1;
      if ((lane & lowmask) == 0 && idx < c) s_qk[idx * band + kk] = r;
    }
  }
  // ---- B: pos term over the touched pos rows ----
  {
    float qb[CQ][VPL];
#pragma unroll
    for (int j = 0; j < CQ; j++)
#pragma unroll
      for (int e = 0; e < VPL; e++) {
        int dim = lane * VPL + e;
        qb[j][e] = j < c ? p.q[(z * c + j) * p.ldq + hoff + dim] + p.v[hoff + dim] : 0.0f;
      }
    for (int pi = warp; pi < p.np; pi += NW) {
      const float *pr = p.pos_p + (p.pr_lo + pi) * (int64_t)p.d + hoff;
      float pv[VPL];
#pragma unroll
      for (int e = 0; e < VPL; e++) pv[e] = pr[lane * VPL + e];
      float part[CQ];
#pragma unroll
      for (int j = 0; j < CQ; j++) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < VPL; e++) a = fmaf(qb[j][e], pv[e], a);
        part[j] = a;
      }
      float r = multi_reduce<CQ>(part, lane);
      int idx = multi_idx<CQ>(lane);
      constexpr int lowmask = (32 / CQ) - 1;
      if ((lane & lowmask) == 0 && idx < c) s_r[idx * p.np + pi] = r;
    }
  }
  __syncthreads();
  // ---- C: band mask + softmax per query ----
  for (int j = warp; j < c; j += NW) {
    int64_t qq = p.s + j, kmin, kmax;
    band_of(qq, p.chunk, p.left_chunks, p.k_hi, kmin, kmax);
    int k0 = (int)(kmin - p.k_lo), k1 = (int)(kmax - p.k_lo);
    float mx = -INFINITY;
    for (int kk = k0 + lane; kk < k1; kk += 32) {
      int pi = (int)(qq + p.pos_off - (p.k_lo + kk) - p.pr_lo);
      float sc = (s_qk[j * band + kk] + s_r[j * p.np + pi]) * p.scale;
      s_qk[j * band + kk] = sc;
      mx = fmaxf(mx, sc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int kk = k0 + lane; kk < k1; kk += 32) {
      float e = expf(s_qk[j * band + kk] - mx);
      s_qk[j * band + kk] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float inv = 1.0f / sum;
    for (int kk = k0 + lane; kk < k1; kk += 32) s_qk[j * band + kk] *= inv;
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
        if (kk >= k0s[j] && kk < k1s[j]) acc[j] = fmaf(s_qk[j * band + kk], vv, acc[j]);
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
  size_t smem = (size_t)CQ * (band + p.np) * sizeof(float);
  auto kern = attn_stream_kernel<HD, CQ>;
  static size_t smem_set[64] = {};
  int dev = 0;
  SC_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && dev < 64 && smem_set[dev] < smem) {
    SC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[dev] = smem;
  }
  kern<<<dim3((unsigned)p.n_heads, (unsigned)n_streams), HD, smem, st>>>(p);
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
