// unltd_gemv_noalloc: the decode GEMV for callers that cannot allocate GPU
// memory.
//
// The ordinary entry points keep their per-call scratch (the x image the prep
// kernel builds) in memory owned by a unltd_ctx, which cudaMalloc'ed it and
// grows it with cudaMalloc when a larger dim_in arrives. Some callers cannot
// do that: code running inside an allocator or a memory pool that must not
// re-enter it, hosts that pre-reserve all device memory and forbid further
// cudaMalloc, or code that may not trigger the implicit device
// synchronisation cudaMalloc/cudaFree can cause. This variant takes its
// scratch from a fixed array compiled into the library instead, so a call
// allocates nothing (no cudaMalloc, no cudaFree, no torch allocation).
//
// Limits and sharing:
//  * kNoallocScratchBytes (64 KiB) of device memory is reserved on every GPU
//    that loads the library, for the life of the process;
//  * the x image must fit in it: dim_in <= 16384 in every mode (F32X needs
//    848 bytes per 256 inputs, Q8K_EXACT 336 or 528); larger dim_in is
//    rejected with UNLTD_ERR_UNSUPPORTED before anything is launched;
//  * all calls on a device share that one array and it keeps the last call's
//    contents: two calls whose kernels overlap on the GPU (different streams
//    without ordering between them) race on it and give wrong results.
//    Order them on one stream, or with events.
//  * the first call on each device does the set-up below (symbol address and
//    kernel attributes) with that device current; make that first call
//    before any stream capture begins. A set-up that failed is retried by the
//    next call.
//  * a kernel that gives up on a bounded pipeline wait records the timeout in
//    the error word of the weight's context (allocated when that context was
//    created): once the stream passed here has finished, unltd_ctx_synchronize
//    on that context returns UNLTD_ERR_TIMEOUT.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = 64 * 1024;
constexpr size_t kNoallocMaxDimIn = 16384;

// The scratch. Its name in host code is only a handle for the runtime; the
// device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
struct DeviceSetup {
  bool done = false;
  uint8_t *scratch = nullptr;
  int num_sms = 0;
};
std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

// With `device` current: the symbol's device address and the kernels'
// shared-memory attributes. Marks the device done only when every step
// succeeded, so a failure (for example a first call made during stream
// capture) is retried by the next call.
cudaError_t setup_device(int device, DeviceSetup &s) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  e = unltd::gemv_prewarm(device);
  if (e != cudaSuccess) return e;
  s.scratch = static_cast<uint8_t *>(p);
  s.num_sms = sms;
  s.done = true;
  return cudaSuccess;
}

}  // namespace

extern "C" int32_t unltd_gemv_noalloc(unltd_weight w, const float *x_dev, float *y_dev, int32_t mode,
                                      void *stream) {
  using namespace unltd;
  if (!w || !x_dev || !y_dev) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_noalloc: NULL argument");
  if (mode != MODE_F32X && mode != MODE_Q8K)
    return set_error(UNLTD_ERR_INVALID_ARG, "gemv_noalloc: unknown mode " + std::to_string(mode));
  if (w->dtype != Q4K && w->dtype != Q6K && w->dtype != Q8_0)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_noalloc: only Q4_K, Q6_K and Q8_0 weights");
  if (mode == MODE_Q8K && w->dtype == Q8_0)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_noalloc: Q8_0 has no Q8_K dot (use MODE_F32X)");
  if (w->dim_in > kNoallocMaxDimIn)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_noalloc: dim_in " + std::to_string(w->dim_in) +
                                                " exceeds the fixed scratch limit of 16384");
  const int nspans = w->dtype == Q8_0 ? (int)((w->nb + 7) / 8) : (int)w->nb;
  const size_t img = (size_t)nspans * img_stride(w->dtype, mode);
  if (img > kNoallocScratchBytes)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_noalloc: x image does not fit the fixed scratch");

  const int device = w->ctx->device;
  if (device < 0 || device >= kMaxDevices) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_noalloc: device id");
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_error(e, "gemv_noalloc: current device");
  if (prev != device) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_error(e, "gemv_noalloc: select the weight's device");
  }
  int32_t rc = UNLTD_OK;
  DeviceSetup s;
  {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DeviceSetup &g = g_setup[device];
    if (!g.done) e = setup_device(device, g);
    s = g;
  }
  if (!s.done) {
    rc = cuda_error(e, "gemv_noalloc: set-up (cudaGetSymbolAddress, kernel attributes)");
  } else {
    // A context on the stack: no allocation; it carries the stream, points the
    // image scratch at the fixed array (never freed or grown: scratch_fixed)
    // and records timeouts in the weight's context error word.
    unltd_ctx_s c;
    c.device = device;
    c.num_sms = s.num_sms;
    c.stream = static_cast<cudaStream_t>(stream);
    c.own_stream = c.stream;
    c.scratch = s.scratch;
    c.scratch_bytes = kNoallocScratchBytes;
    c.scratch_fixed = true;
    c.err = w->ctx->err;
    GemvArgs a{w, x_dev, y_dev, mode, nullptr, nullptr, nullptr};
    rc = gemv_launch(&c, a);
  }
  if (prev >= 0 && prev != device) {
    e = cudaSetDevice(prev);
    if (e != cudaSuccess && rc == UNLTD_OK) rc = cuda_error(e, "gemv_noalloc: restore the caller's device");
  }
  return rc;
}
