// sc_api.cu -- the C ABI of libstealcode_cuda.so (declared in
// include/stealcode_b200.h).  Every entry point validates its arguments,
// returns 0 or a negative error code and never aborts; sc_last_error() gives
// the message of the calling thread's last failure.
#include <atomic>
#include <mutex>
#include <new>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "sc_kernels.cuh"
#include "../../include/stealcode_b200.h"

namespace sc {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what) {
  set_error("CUDA error %d (%s) in %s", (int)e, cudaGetErrorString(e), what);
  return kErrCuda;
}

// ---- per-device state: SM count and a default workspace ----------------
struct DeviceState {
  std::atomic<int> sm_count{0};
  void *ws = nullptr;
  size_t ws_bytes = 0;
  void *stage = nullptr;  // host-twin staging for x and y (grow-only)
  size_t stage_bytes = 0;
  std::mutex mu;
  std::mutex stage_mu;
};
static DeviceState g_dev[64];

static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void note_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Allocation cap for failure-path tests (sc_debug_set_device_alloc_cap):
// -1 = none; else the bytes the library may still allocate.
static std::atomic<long long> g_alloc_left{-1};

cudaError_t dev_malloc(void **p, size_t bytes) {
  *p = nullptr;
  long long left = g_alloc_left.load(std::memory_order_relaxed);
  while (left >= 0) {
    if ((long long)bytes > left) return cudaErrorMemoryAllocation;
    if (g_alloc_left.compare_exchange_weak(left, left - (long long)bytes, std::memory_order_relaxed)) break;
  }
  return cudaMalloc(p, bytes);
}

int current_device(int *dev, int *sm_count) {
  SC_CUDA(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= 64) {
    set_error("device ordinal %d out of range", *dev);
    return kErrInvalid;
  }
  DeviceState &ds = g_dev[*dev];
  int n = ds.sm_count.load(std::memory_order_relaxed);
  if (n == 0) {
    SC_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, *dev));
    ds.sm_count.store(n, std::memory_order_relaxed);
  }
  if (sm_count) *sm_count = n;
  return kOk;
}

int raise_smem_limit(const void *kern, size_t bytes, std::atomic<size_t> *limit) {
  if (bytes <= 48 * 1024) return kOk;
  int dev = 0;
  SC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return kErrInvalid;
  }
  if (limit[dev].load(std::memory_order_acquire) >= bytes) return kOk;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (limit[dev].load(std::memory_order_relaxed) >= bytes) return kOk;
  SC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  limit[dev].store(bytes, std::memory_order_release);
  return kOk;
}

// Workspace of a GEMM call: quantised activations [m_pad][k_pad] int8 then
// their scales [nb][m_pad] f32.
size_t gemm_ws_bytes(int64_t m, int64_t k) {
  int64_t nb = ceil_div(k, 32), m_pad = ceil_div(m, 128) * 128;
  size_t a = (size_t)m_pad * nb * 32 * 2;  // codes: int8, or f16 for the tensor-core path
  a = (a + 255) / 256 * 256;
  return a + (size_t)nb * m_pad * 4 + 256;
}

static int default_ws(size_t bytes, void **out) {
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  DeviceState &ds = g_dev[dev];
  std::lock_guard<std::mutex> lk(ds.mu);
  if (ds.ws_bytes < bytes) {
    if (ds.ws) {
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
      cudaFree(ds.ws);
      ds.ws = nullptr;
      ds.ws_bytes = 0;
    }
    size_t nbytes = bytes < ((size_t)64 << 20) ? ((size_t)64 << 20) : bytes;
    cudaError_t e = dev_malloc(&ds.ws, nbytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("workspace cudaMalloc(%zu) failed: %s", nbytes, cudaGetErrorString(e));
      return kErrAlloc;
    }
    ds.ws_bytes = nbytes;
  }
  *out = ds.ws;
  return kOk;
}

static bool layout_ok(int32_t l) { return l == SC_LAYOUT_FEATURE_MAJOR || l == SC_LAYOUT_TIME_MAJOR; }

// Frames up to which the weight-streaming kernel runs (the reference's SIMD
// dispatch covers up to 16 frames); up to kMidMaxFrames the mid-size dp4a
// kernel in q8_gemm_scalar's order; above it the tensor-core kernel.
constexpr int64_t kSmallMaxFrames = 16;
constexpr int64_t kMidMaxFrames = 128;

// Quantise + GEMM on device pointers.
int gemm_impl(const Q8Weights *w, const float *x, int64_t t, int32_t x_layout, int64_t ldx,
              const float *bias, float *y, int32_t y_layout, int64_t ldy, void *ws,
              size_t ws_bytes, int32_t *dots, cudaStream_t st, Epilogue epi, bool force_tc) {
  if (!w || !x || (!y && !dots) || t < 0 || !layout_ok(x_layout) || !layout_ok(y_layout)) {
    set_error("q8_gemm: invalid argument");
    return kErrInvalid;
  }
  if (t == 0 || w->rows == 0 || w->k == 0) return kOk;  // zero dims: no-op, like q8_gemm
  if (ldx <= 0) ldx = x_layout == SC_LAYOUT_TIME_MAJOR ? w->k : t;
  if (ldy <= 0) ldy = y_layout == SC_LAYOUT_TIME_MAJOR ? w->rows : t;
  if ((x_layout == SC_LAYOUT_TIME_MAJOR && ldx < w->k) || (x_layout == SC_LAYOUT_FEATURE_MAJOR && ldx < t) ||
      (y_layout == SC_LAYOUT_TIME_MAJOR && ldy < w->rows) || (y_layout == SC_LAYOUT_FEATURE_MAJOR && ldy < t)) {
    set_error("q8_gemm: leading dimension too small");
    return kErrInvalid;
  }
  int dev, sms;
  int rc = current_device(&dev, &sms);
  if (rc) return rc;
  if (dev != w->device) {
    set_error("q8_gemm: weights live on device %d, current device is %d", w->device, dev);
    return kErrInvalid;
  }
  size_t need = gemm_ws_bytes(t, w->k);
  if (ws && (ws_bytes < need || ((uintptr_t)ws & 255))) {
    set_error("q8_gemm: workspace needs %zu bytes at 256-byte alignment", need);
    return kErrInvalid;
  }
  if (t > kSmallMaxFrames && t <= kMidMaxFrames && !force_tc && !dots) {
    // Mid-size path: plain [m_pad][k_pad] codes, then the dp4a kernel.
    if (!ws) {
      rc = default_ws(need, &ws);
      if (rc) return rc;
    }
    const int64_t m_pad = ceil_div(t, 128) * 128, k_pad = w->nb * 32;
    int8_t *xq = (int8_t *)ws;
    float *dx = (float *)((char *)ws + ((size_t)m_pad * k_pad + 255) / 256 * 256);
    rc = quantize_act(x, t, w->k, ldx, x_layout == SC_LAYOUT_FEATURE_MAJOR, m_pad, xq, dx, st, 0);
    if (rc) return rc;
    MidGemmArgs ma{w, xq, dx, t, m_pad, k_pad, bias, y, y_layout == SC_LAYOUT_TIME_MAJOR, ldy, epi};
    return gemm_mid(ma, st);
  }
  if ((t > kSmallMaxFrames || force_tc) && !dots) {
    // Tensor-core path: quantise into the tiled operand layout, then tcgen05.
    if (!ws) {
      rc = default_ws(need, &ws);
      if (rc) return rc;
    }
    const int ft = tc_frame_tile(t);
    const int64_t t_pad = ceil_div(t, ft) * ft, k_pad = w->nb * 32;
    __half *xq = (__half *)ws;
    float *dx = (float *)((char *)ws + ((size_t)t_pad * k_pad * 2 + 255) / 256 * 256);
    rc = quantize_act(x, t, w->k, ldx, x_layout == SC_LAYOUT_FEATURE_MAJOR, t_pad, xq, dx, st, ft);
    if (rc) return rc;
    TcGemmArgs ta{w, xq, dx, t, t_pad, bias, y, y_layout == SC_LAYOUT_TIME_MAJOR, ldy, epi};
    return gemm_tc(ta, st);
  }
  // The streaming kernel quantises the activations itself.
  SmallGemmArgs a{w, x, ldx, x_layout == SC_LAYOUT_FEATURE_MAJOR, nullptr, nullptr, 0, 0, t, bias, y,
                  y_layout == SC_LAYOUT_TIME_MAJOR, ldy, dots, epi};
  return gemm_small(a, sms, st);
}

}  // namespace sc

using namespace sc;

struct sc_q8w {
  Q8Weights w;
};

namespace sc {
const Q8Weights *q8w_weights(const sc_q8w *w) { return &w->w; }
}  // namespace sc

extern "C" {

long long sc_launch_count(void) { return sc::g_launches.load(std::memory_order_relaxed); }

int sc_debug_set_device_alloc_cap(int64_t bytes) {
  sc::g_alloc_left.store(bytes < 0 ? -1 : bytes, std::memory_order_relaxed);
  return kOk;
}

const char *sc_last_error(void) { return g_err; }

int sc_abi_version(void) { return SC_ABI_VERSION; }

int sc_q8_repack_device(const uint8_t *blocks_dev, int64_t rows, int64_t k, int64_t block_bytes,
                        int64_t qoff, void *stream, sc_q8w **out) {
  if (!out || !blocks_dev || rows <= 0 || k <= 0) {
    set_error("q8_repack: invalid argument (rows=%lld k=%lld)", (long long)rows, (long long)k);
    return kErrInvalid;
  }
  *out = nullptr;
  if (block_bytes != 34 || qoff != 2) {
    set_error("q8_repack: only 34-byte [f16 d][32 x i8] blocks (GGUF dtype 8) map to the f16-scale "
              "device layout; got block_bytes=%lld qoff=%lld", (long long)block_bytes, (long long)qoff);
    return kErrUnsupported;
  }
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  sc_q8w *h = new (std::nothrow) sc_q8w();
  if (!h) { set_error("q8_repack: host allocation failed"); return kErrAlloc; }
  Q8Weights &w = h->w;
  w.rows = rows;
  w.k = k;
  w.nb = ceil_div(k, 32);
  w.rows_pad = ceil_div(rows, SC_GROUP_ROWS) * SC_GROUP_ROWS;
  w.device = dev;
  size_t qbytes = (size_t)w.rows_pad * w.nb * 32, sbytes = (size_t)w.rows_pad * w.nb * 2;
  if (dev_malloc((void **)&w.qs, qbytes) != cudaSuccess || dev_malloc((void **)&w.sc, sbytes) != cudaSuccess ||
      dev_malloc((void **)&w.qh, 2 * qbytes) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w.qs);
    cudaFree(w.sc);
    delete h;
    set_error("q8_repack: cudaMalloc of %zu bytes failed", 3 * qbytes + sbytes);
    return kErrAlloc;
  }
  rc = repack_q8_device(blocks_dev, rows, k, block_bytes, qoff, &w, (cudaStream_t)stream);
  if (rc) {
    cudaFree(w.qs);
    cudaFree(w.sc);
    cudaFree(w.qh);
    delete h;
    return rc;
  }
  *out = h;
  return kOk;
}

int sc_q8_repack(const uint8_t *blocks, int64_t rows, int64_t k, int64_t block_bytes, int64_t qoff,
                 sc_q8w **out) {
  if (!out || !blocks || rows <= 0 || k <= 0 || block_bytes <= 0) {
    set_error("q8_repack: invalid argument");
    return kErrInvalid;
  }
  *out = nullptr;
  if (block_bytes != 34 || qoff != 2) {
    set_error("q8_repack: only 34-byte [f16 d][32 x i8] blocks (GGUF dtype 8) map to the f16-scale "
              "device layout; got block_bytes=%lld qoff=%lld", (long long)block_bytes, (long long)qoff);
    return kErrUnsupported;
  }
  size_t bytes = (size_t)rows * ceil_div(k, 32) * block_bytes;
  uint8_t *raw = nullptr;
  if (dev_malloc((void **)&raw, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("q8_repack: staging cudaMalloc(%zu) failed", bytes);
    return kErrAlloc;
  }
  cudaError_t e = cudaMemcpy(raw, blocks, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(raw);
    return cuda_fail(e, "cudaMemcpy(raw blocks)");
  }
  int rc = sc_q8_repack_device(raw, rows, k, block_bytes, qoff, nullptr, out);
  e = cudaDeviceSynchronize();
  cudaFree(raw);
  if (rc) return rc;
  if (e != cudaSuccess) {
    sc_q8w_free(*out);
    *out = nullptr;
    return cuda_fail(e, "repack");
  }
  return kOk;
}

int sc_q8w_free(sc_q8w *w) {
  if (!w) return kOk;
  cudaFree(w->w.qs);
  cudaFree(w->w.sc);
  cudaFree(w->w.qh);
  delete w;
  return kOk;
}

int sc_q8w_shape(const sc_q8w *w, int64_t *rows, int64_t *k) {
  if (!w) { set_error("q8w_shape: null handle"); return kErrInvalid; }
  if (rows) *rows = w->w.rows;
  if (k) *k = w->w.k;
  return kOk;
}

int sc_q8w_device_layout(const sc_q8w *w, const int8_t **quants, const uint16_t **scales,
                         int64_t *rows_pad, int64_t *nblocks) {
  if (!w) { set_error("q8w_device_layout: null handle"); return kErrInvalid; }
  if (quants) *quants = w->w.qs;
  if (scales) *scales = (const uint16_t *)w->w.sc;
  if (rows_pad) *rows_pad = w->w.rows_pad;
  if (nblocks) *nblocks = w->w.nb;
  return kOk;
}

int sc_device_status(uint32_t *flags) {
  if (!flags) { set_error("device_status: null pointer"); return kErrInvalid; }
  unsigned v = 0, v2 = 0, v3 = 0;
  int rc = small_gemm_status(&v);
  if (!rc) rc = tc_gemm_status(&v2);
  if (!rc) rc = batch_gemm_status(&v3);
  if (rc) return rc;
  *flags = v | v2 | v3;
  return kOk;
}

int64_t sc_q8_gemm_workspace_bytes(int64_t t, int64_t k) {
  if (t <= 0 || k <= 0) return 0;
  return (int64_t)gemm_ws_bytes(t, k);
}

int sc_q8_gemm(const sc_q8w *w, const float *x, int64_t t, int32_t x_layout, int64_t ldx,
               const float *bias, float *y, int32_t y_layout, int64_t ldy, void *workspace,
               int64_t workspace_bytes, void *stream) {
  if (!w) { set_error("q8_gemm: null weights"); return kErrInvalid; }
  return gemm_impl(&w->w, x, t, x_layout, ldx, bias, y, y_layout, ldy, workspace,
                   (size_t)(workspace_bytes < 0 ? 0 : workspace_bytes), nullptr, (cudaStream_t)stream, Epilogue{});
}

int sc_q8_block_dots(const sc_q8w *w, const float *x, int64_t t, int32_t x_layout, int64_t ldx,
                     int32_t *dots, void *stream) {
  if (!w || !dots) { set_error("q8_block_dots: invalid argument"); return kErrInvalid; }
  return gemm_impl(&w->w, x, t, x_layout, ldx, nullptr, nullptr, SC_LAYOUT_TIME_MAJOR, 0, nullptr, 0,
                   dots, (cudaStream_t)stream, Epilogue{});
}

int sc_q8_quantize(const float *x, int64_t m, int64_t k, int32_t x_layout, int64_t ldx, int8_t *xq,
                   float *dx, void *stream) {
  if (!x || !xq || !dx || m <= 0 || k <= 0 || !layout_ok(x_layout)) {
    set_error("q8_quantize: invalid argument");
    return kErrInvalid;
  }
  if (ldx <= 0) ldx = x_layout == SC_LAYOUT_TIME_MAJOR ? k : m;
  // xq rows are k_pad = 32*nblocks bytes; dx is [nblocks][m].
  return quantize_act(x, m, k, ldx, x_layout == SC_LAYOUT_FEATURE_MAJOR, m, xq, dx, (cudaStream_t)stream);
}

int sc_q8mat_gemm_t(const sc_q8w *w, const float *x_host, int64_t t, float *y_host) {
  if (!w || !x_host || !y_host || t < 0) { set_error("q8mat_gemm_t: invalid argument"); return kErrInvalid; }
  if (t == 0) return kOk;
  const Q8Weights &W = w->w;
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  DeviceState &ds = g_dev[dev];
  std::lock_guard<std::mutex> lk(ds.stage_mu);
  size_t xb = ((size_t)W.k * t * 4 + 255) / 256 * 256, yb = (size_t)W.rows * t * 4;
  if (ds.stage_bytes < xb + yb) {
    if (ds.stage) {
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
      cudaFree(ds.stage);
      ds.stage = nullptr;
      ds.stage_bytes = 0;
    }
    if (dev_malloc((void **)&ds.stage, xb + yb) != cudaSuccess) {
      cudaGetLastError();
      set_error("q8mat_gemm_t: staging cudaMalloc(%zu) failed", xb + yb);
      return kErrAlloc;
    }
    ds.stage_bytes = xb + yb;
  }
  float *xd = (float *)ds.stage, *yd = (float *)((char *)ds.stage + xb);
  cudaError_t e = cudaMemcpyAsync(xd, x_host, (size_t)W.k * t * 4, cudaMemcpyHostToDevice, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(x)");
  rc = gemm_impl(&W, xd, t, SC_LAYOUT_FEATURE_MAJOR, t, nullptr, yd, SC_LAYOUT_FEATURE_MAJOR, t, nullptr, 0,
                 nullptr, 0, Epilogue{});
  if (rc) return rc;
  e = cudaMemcpyAsync(y_host, yd, yb, cudaMemcpyDeviceToHost, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(y)");
  e = cudaStreamSynchronize(0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  return kOk;
}

int sc_q8_gemm_q(const sc_q8w *w, const int8_t *xq, const float *dx, int64_t t, int64_t t_pad,
                 const float *bias, float *y, int32_t y_layout, int64_t ldy, void *stream) {
  if (!w || !xq || !dx || !y || t < 0 || t_pad < t || !layout_ok(y_layout) ||
      ((uintptr_t)xq & 15)) {
    set_error("q8_gemm_q: invalid argument (xq must be 16-byte aligned, t_pad >= t)");
    return kErrInvalid;
  }
  if (t == 0) return kOk;
  const Q8Weights &W = w->w;
  if (ldy <= 0) ldy = y_layout == SC_LAYOUT_TIME_MAJOR ? W.rows : t;
  if ((y_layout == SC_LAYOUT_TIME_MAJOR && ldy < W.rows) || (y_layout == SC_LAYOUT_FEATURE_MAJOR && ldy < t)) {
    set_error("q8_gemm_q: leading dimension too small");
    return kErrInvalid;
  }
  int dev, sms;
  int rc = current_device(&dev, &sms);
  if (rc) return rc;
  SmallGemmArgs a{&W, nullptr, 0, 0, xq, dx, W.nb * 32, t_pad, t, bias, y, y_layout == SC_LAYOUT_TIME_MAJOR, ldy,
                  nullptr, Epilogue{}};
  return gemm_small(a, sms, (cudaStream_t)stream);
}

static int batch_items(const sc_q8w *const *w, const float *const *x, const float *const *bias, float *const *y,
                       int32_t n, int64_t t, int32_t x_layout, int32_t y_layout, std::vector<BatchItem> &items) {
  if (!w || n <= 0 || n > kMaxBatch || t < 0 || t > kBatchFrames || !layout_ok(x_layout) || !layout_ok(y_layout)) {
    set_error("q8_gemm_batch: 1..%d GEMMs of 0..%d frames and valid layouts", kMaxBatch, kBatchFrames);
    return kErrInvalid;
  }
  int dev;
  int rc = current_device(&dev, nullptr);
  if (rc) return rc;
  items.resize(n);
  for (int i = 0; i < n; i++) {
    if (!w[i] || (x && !x[i]) || (y && !y[i])) {
      set_error("q8_gemm_batch: null weights, input or output %d", i);
      return kErrInvalid;
    }
    const Q8Weights &W = w[i]->w;
    if (W.device != dev) {
      set_error("q8_gemm_batch: weights %d live on device %d, current device is %d", i, W.device, dev);
      return kErrInvalid;
    }
    BatchItem it{};
    it.qs = W.qs;
    it.sc = W.sc;
    it.x = x ? x[i] : nullptr;
    it.bias = bias ? bias[i] : nullptr;
    it.y = y ? y[i] : nullptr;
    it.ldx = x_layout == SC_LAYOUT_TIME_MAJOR ? W.k : t;
    it.ldy = y_layout == SC_LAYOUT_TIME_MAJOR ? W.rows : t;
    it.nb = (int32_t)W.nb;
    it.rows = (int32_t)W.rows;
    it.groups = (int32_t)(W.rows_pad / SC_GROUP_ROWS);
    it.k = (int32_t)W.k;
    it.x_feature_major = x_layout == SC_LAYOUT_FEATURE_MAJOR;
    items[i] = it;
  }
  return kOk;
}

int64_t sc_q8_gemm_batch_workspace_bytes(const sc_q8w *const *w, int32_t n) {
  std::vector<BatchItem> items;
  if (batch_items(w, nullptr, nullptr, nullptr, n, 1, SC_LAYOUT_TIME_MAJOR, SC_LAYOUT_TIME_MAJOR, items)) return -1;
  return (int64_t)batch_ws_bytes(items.data(), n);
}

int sc_q8_gemm_batch(const sc_q8w *const *w, const float *const *x, const float *const *bias, float *const *y,
                     int32_t n, int64_t t, int32_t x_layout, int32_t y_layout, void *workspace,
                     int64_t workspace_bytes, void *stream) {
  std::vector<BatchItem> items;
  if (!x || !y) {
    set_error("q8_gemm_batch: invalid argument");
    return kErrInvalid;
  }
  int rc = batch_items(w, x, bias, y, n, t, x_layout, y_layout, items);
  if (rc) return rc;
  if (t == 0) return kOk;
  const size_t need = batch_ws_bytes(items.data(), n);
  if (!workspace) {
    rc = default_ws(need, &workspace);
    if (rc) return rc;
    workspace_bytes = (int64_t)need;
  }
  int dev, sms;
  rc = current_device(&dev, &sms);
  if (rc) return rc;
  return gemm_batch(items.data(), n, (int)t, y_layout == SC_LAYOUT_TIME_MAJOR, workspace, (size_t)workspace_bytes,
                    sms, (cudaStream_t)stream);
}

int sc_q8_gemm_host(size_t m, size_t k, size_t n, const uint8_t *w, size_t padded_row, size_t block_bytes,
                    size_t qoff, const float *x, float *y) {
  if (m == 0 || k == 0 || n == 0) return kOk;  // sgemm_kernel.rs:110-112
  if (!w || !x || !y || block_bytes == 0 || padded_row != ((k + 31) / 32) * block_bytes) {
    set_error("q8_gemm_host: invalid argument (padded_row must be ceil(k/32)*block_bytes)");
    return kErrInvalid;
  }
  sc_q8w *h = nullptr;
  int rc = sc_q8_repack(w, (int64_t)m, (int64_t)k, (int64_t)block_bytes, (int64_t)qoff, &h);
  if (rc) return rc;
  rc = sc_q8mat_gemm_t(h, x, (int64_t)n, y);
  sc_q8w_free(h);
  return rc;
}

static int attn_common(AttnParams &p, int64_t n_pos, int64_t n_streams, cudaStream_t st) {
  int rc = attn_prepare(p, n_pos);
  if (rc) return rc;
  return launch_attn(p, n_streams, st);
}

int sc_attn_stream(const float *q, const float *kv, const float *vv, const float *pos_p, int64_t n_pos,
                   const float *q_bias, const float *v_bias, int64_t c, int64_t d, int64_t n_heads,
                   float scale, int64_t s, int64_t k_lo, int64_t band, int64_t chunk,
                   int64_t left_chunks, int64_t k_hi, int64_t pos_off, float *out, void *stream) {
  if (!q || !kv || !vv || !pos_p || !q_bias || !v_bias || !out || band != k_hi - k_lo) {
    set_error("attn_stream: invalid argument (band must equal k_hi - k_lo)");
    return kErrInvalid;
  }
  AttnParams p{};
  p.q = q; p.ldq = d;
  p.k_new = kv; p.v_new = vv; p.ld_new = d; p.rows_new = band; p.new_lo = k_lo;
  p.k_ring = nullptr; p.v_ring = nullptr; p.cap = 1;
  p.pos_p = pos_p; p.u = q_bias; p.v = v_bias; p.out = out; p.ldo = d;
  p.c = (int)c; p.d = (int)d; p.n_heads = (int)n_heads; p.scale = scale;
  p.s = s; p.k_lo = k_lo; p.k_hi = k_hi; p.chunk = chunk; p.left_chunks = left_chunks; p.pos_off = pos_off;
  return attn_common(p, n_pos, 1, (cudaStream_t)stream);
}

int sc_attn_stream_host(const float *q, const float *kv, const float *vv, const float *pos_p, int64_t n_pos,
                        const float *q_bias, const float *v_bias, int64_t c, int64_t d, int64_t n_heads,
                        float scale, int64_t s, int64_t k_lo, int64_t band, int64_t chunk,
                        int64_t left_chunks, int64_t k_hi, int64_t pos_off, float *out) {
  if (!q || !kv || !vv || !pos_p || !q_bias || !v_bias || !out || c <= 0 || d <= 0 || band <= 0 || n_pos <= 0) {
    set_error("attn_stream_host: invalid argument");
    return kErrInvalid;
  }
  size_t qb = (size_t)c * d * 4, kb = (size_t)band * d * 4, pb = (size_t)n_pos * d * 4, db = (size_t)d * 4;
  size_t total = qb * 2 + kb * 2 + pb + db * 2;
  char *buf = nullptr;
  if (dev_malloc((void **)&buf, total + 7 * 256) != cudaSuccess) {
    cudaGetLastError();
    set_error("attn_stream_host: cudaMalloc failed");
    return kErrAlloc;
  }
  size_t off = 0;
  auto take = [&](size_t b) { char *r = buf + off; off += (b + 255) / 256 * 256; return (float *)r; };
  float *qd = take(qb), *kd = take(kb), *vd = take(kb), *pd = take(pb), *ud = take(db), *bd = take(db),
        *od = take(qb);
  int rc = kOk;
  cudaError_t e = cudaSuccess;
  if ((e = cudaMemcpy(qd, q, qb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(kd, kv, kb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(vd, vv, kb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(pd, pos_p, pb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(ud, q_bias, db, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(bd, v_bias, db, cudaMemcpyHostToDevice)) != cudaSuccess)
    rc = cuda_fail(e, "cudaMemcpy(attn inputs)");
  if (!rc) rc = sc_attn_stream(qd, kd, vd, pd, n_pos, ud, bd, c, d, n_heads, scale, s, k_lo, band, chunk,
                               left_chunks, k_hi, pos_off, od, nullptr);
  if (!rc && (e = cudaMemcpy(out, od, qb, cudaMemcpyDeviceToHost)) != cudaSuccess)
    rc = cuda_fail(e, "cudaMemcpy(out)");
  cudaFree(buf);
  return rc;
}

int sc_attn_stream_ring(const float *q, int64_t ldq, const float *k_new, const float *v_new, int64_t ld_new,
                        float *k_ring, float *v_ring, int64_t cap, int64_t n_streams, const float *pos_p,
                        int64_t n_pos, const float *q_bias, const float *v_bias, int64_t c, int64_t d,
                        int64_t n_heads, float scale, int64_t s, int64_t k_lo, int64_t chunk,
                        int64_t left_chunks, int64_t k_hi, int64_t pos_off, float *out, int64_t ldo,
                        void *stream) {
  if (!q || !k_new || !v_new || !k_ring || !v_ring || !pos_p || !q_bias || !v_bias || !out || cap <= 0 ||
      n_streams <= 0 || k_hi != s + c) {
    set_error("attn_stream_ring: invalid argument (k_hi must equal s + c)");
    return kErrInvalid;
  }
  AttnParams p{};
  p.q = q; p.ldq = ldq > 0 ? ldq : d;
  p.k_new = k_new; p.v_new = v_new; p.ld_new = ld_new > 0 ? ld_new : d; p.rows_new = c; p.new_lo = s;
  p.k_ring = k_ring; p.v_ring = v_ring; p.cap = cap;
  p.pos_p = pos_p; p.u = q_bias; p.v = v_bias; p.out = out; p.ldo = ldo > 0 ? ldo : d;
  p.c = (int)c; p.d = (int)d; p.n_heads = (int)n_heads; p.scale = scale;
  p.s = s; p.k_lo = k_lo; p.k_hi = k_hi; p.chunk = chunk; p.left_chunks = left_chunks; p.pos_off = pos_off;
  return attn_common(p, n_pos, n_streams, (cudaStream_t)stream);
}

}  // extern "C"
