// sc_device.cuh -- device-side helpers shared by the kernels: the bit-exact
// per-block activation quantiser, mbarrier + bulk-copy (TMA, no multicast)
// wrappers with bounded waits, and programmatic-dependent-launch controls.
#pragma once

#include <stdint.h>

#include "sc_common.cuh"

namespace sc {

// ---- activation quantisation (quantize_col, sgemm_kernel.rs:57-90) -------
// Rust `(v).round() as i8`: round half away from zero, saturate, NaN -> 0.
__device__ __forceinline__ int8_t rust_round_i8(float v) {
  float r = roundf(v);
  if (r != r) return 0;
  r = fminf(fmaxf(r, -128.0f), 127.0f);
  return (int8_t)(int)r;
}

// An int8 code as the f16 operand of the tensor-core GEMM (exact).
__device__ __forceinline__ __half code_half(int8_t q) { return __short2half_rn((short)q); }

// One 32-wide block held one element per lane (valid = inside k).  Returns
// the lane's code and the block scale s (same in every lane): amax ignores
// NaN like `if v > maxv`, an all-zero block gets s = 1 and zero codes, s =
// amax / 127 and inv = 1 / s with IEEE division, q = round(x * inv).
__device__ __forceinline__ int8_t warp_quantize_block(float v, bool valid, float &s_out) {
  float amax = valid ? fabsf(v) : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (amax != amax) amax = 0.0f;
  const float s = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
  int8_t q = 0;
  if (amax != 0.0f && valid) q = rust_round_i8(__fmul_rn(v, __fdiv_rn(1.0f, s)));
  s_out = s;
  return q;
}

// ---- shared-memory barriers and bulk copies -------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async proxy (bulk copies, MMA).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after about two seconds of SM clock and returns
// false, so a lost arrival cannot hang the GPU.
constexpr long long kWaitCycles = 4000000000LL;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- programmatic dependent launch ---------------------------------------
// Everything before pdl_wait() may overlap the previous kernel on the stream
// (only reads of data that kernel does not write); pdl_launch_dependents()
// lets the next kernel start its own prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Status bits a kernel ORs into its status word when a bounded wait gives up.
enum : unsigned { kStatusWaitTimeout = 1u };

}  // namespace sc
