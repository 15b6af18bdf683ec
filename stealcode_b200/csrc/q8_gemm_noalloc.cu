// q8_gemm_noalloc.cu -- sc_q8_gemm_noalloc: the Q8_0 GEMM for callers that
// must not allocate device memory.
//
// sc_q8_gemm needs scratch for the quantised activations: either a caller
// workspace or a library workspace grown with cudaMalloc on first use.  Some
// hosts cannot do either:
//   * a plugin called from inside someone else's CUDA-graph capture, where a
//     cudaMalloc would break the capture;
//   * a real-time audio callback, which must not block, and cudaMalloc or
//     cudaFree may synchronise the whole device;
//   * an engine that owns all device memory and forbids libraries from
//     touching the allocator, but has no API for handing out workspaces.
// This entry point keeps its scratch in a fixed file-scope device array
// instead.  The array exists once per GPU that loads the library and lives
// until the process exits.
#include <mutex>

#include "sc_kernels.cuh"
#include "../../include/stealcode_b200.h"

namespace sc {

const Q8Weights *q8w_weights(const sc_q8w *w);

// The scratch: quantised activations [t_pad][k_pad] int8, then their block
// scales [nblocks][t_pad] f32 -- the same layout as a sc_q8_gemm workspace.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
static void *g_noalloc_ptr[64];
static std::mutex g_noalloc_mu;

// The first call on a device also does every GEMM path's own one-time set-up
// (status words, shared-memory limits), so later calls of any frame count
// make no such host calls.
static int noalloc_scratch(int dev, void **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    int rc = small_gemm_prime();
    if (!rc) rc = mid_gemm_prime();
    if (!rc) rc = tc_gemm_prime();
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}

}  // namespace sc

using namespace sc;

extern "C" int sc_q8_gemm_noalloc(const sc_q8w *w, const float *x, int64_t t, int32_t x_layout,
                                  int64_t ldx, const float *bias, float *y, int32_t y_layout,
                                  int64_t ldy, void *stream) {
  if (!w) {
    set_error("q8_gemm_noalloc: null weights");
    return kErrInvalid;
  }
  const Q8Weights *W = q8w_weights(w);
  if (t < 0) {
    set_error("q8_gemm_noalloc: invalid argument (t=%lld)", (long long)t);
    return kErrInvalid;
  }
  if (t == 0) return kOk;
  size_t need = gemm_ws_bytes(t, W->k);
  if (need > (size_t)SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES) {
    set_error("q8_gemm_noalloc: t=%lld frames of k=%lld need %zu bytes of scratch, more than the "
              "fixed %u-byte array; split the frames over several calls or use sc_q8_gemm",
              (long long)t, (long long)W->k, need, (unsigned)SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES);
    return kErrInvalid;
  }
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  void *scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  // Every scratch byte the kernels read is written earlier in this same call
  // (the quantiser fills all t_pad rows, padding rows with zero codes), so
  // nothing is cleared; leftovers of the previous call are never read.
  return gemm_impl(W, x, t, x_layout, ldx, bias, y, y_layout, ldy, scratch,
                   (size_t)SC_Q8_GEMM_NOALLOC_SCRATCH_BYTES, nullptr, (cudaStream_t)stream,
                   Epilogue{});
}
