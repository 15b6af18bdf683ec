// sc_common.cuh -- shared definitions for the stealcode_b200 CUDA library.
//
// Repacked Q8_0 weight layout ("row-group tiles"), used by every GEMM kernel:
//   * rows are padded to a multiple of SC_GROUP_ROWS (128), K to a multiple of
//     32 (one Q8_0 block);
//   * quants: int8 tiles of [128 rows x 32 k] (4 KiB), tile (g, b) at byte
//     (g * nb + b) * 4096; inside a tile, byte i of row r sits at
//     (i / 16) * 2048 + r * 16 + (i % 16).  A warp that maps lanes to rows
//     reads 512 contiguous bytes per 16-byte load, and the tile is the
//     no-swizzle K-major canonical layout of a tcgen05 shared-memory operand
//     (core matrix = 8 rows x 16 bytes; 128 bytes between row octets, 2048
//     bytes between the two 16-byte K halves);
//   * scales: f16 [G][nb][128]: the scale of row g*128 + r, block b at
//     (g * nb + b) * 128 + r (256 contiguous bytes per tile).
// Padding rows and padding K positions hold zero quants and zero scales.
//   * f16 quants for the tensor-core path (every int8 value is an f16
//     integer): tile (g, b) of 128 rows x 32 k at element (g * nb + b) * 4096;
//     inside it, element k of row r at ((k % 32) / 8) * 1024 + r * 8 + k % 8
//     (four 8-wide K chunks, each the no-swizzle K-major core-matrix layout
//     of 128 rows x 16 bytes).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SC_GROUP_ROWS 128
#define SC_TILE_BYTES (SC_GROUP_ROWS * 32)

namespace sc {

struct Q8Weights {
  int64_t rows;       // N (output features)
  int64_t k;          // K (input features)
  int64_t rows_pad;   // N rounded up to 128
  int64_t nb;         // K blocks of 32
  int8_t *qs;         // device, rows_pad * nb * 32 bytes
  __half *sc;         // device, rows_pad * nb halves
  __half *qh;         // device, the quants as f16 tiles for the tensor-core path (rows_pad * nb * 32 halves)
  int device;
};

// Error codes shared with include/stealcode_b200.h.
enum : int {
  kOk = 0,
  kErrInvalid = -1,
  kErrAlloc = -2,
  kErrCuda = -3,
  kErrTimeout = -4,
  kErrUnsupported = -5,
  kErrState = -6,
};

void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
// Counts one kernel launch issued by this library (sc_launch_count).
void note_launch();
// Adds n (may be negative) to the launch count: a step graph's launches are
// counted when it replays, not when it is captured.
void note_launches(long long n);
// cudaMalloc for every device allocation of this library; fails with
// cudaErrorMemoryAllocation, without allocating, once the bytes allocated
// since sc_debug_set_device_alloc_cap would exceed that cap.
cudaError_t dev_malloc(void **p, size_t bytes);

#define SC_CUDA(call)                                       \
  do {                                                      \
    cudaError_t _e = (call);                                \
    if (_e != cudaSuccess) return sc::cuda_fail(_e, #call); \
  } while (0)

__host__ __device__ static inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

#ifdef __CUDACC__
// exp(x) rounded once to f32 from a double-precision exp: the correctly
// rounded value (a double-rounding miss needs the exact value within 2^-29
// of a float midpoint).  glibc's expf, which Rust's f32::exp calls on
// Linux, is one ulp off this for about 6 inputs in 10^4.
__device__ __forceinline__ float exp_rn(float x) { return (float)exp((double)x); }

// SiLU exactly as the reference writes it: v * (1 + exp(-v)).recip()
// (simd_kernel.rs:817-839), with IEEE rounding at every step.
__device__ __forceinline__ float silu_ref(float v) {
  return __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-v))));
}
#endif

}  // namespace sc
