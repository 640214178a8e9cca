// dr_loss_backward_noalloc: forward + MSE + analytic backward with no device
// allocation at all.
//
// Who needs it: callers that must not call cudaMalloc/cudaFree on their hot
// path. cudaMalloc synchronizes the device and may block for milliseconds, so
// real-time and latency-bounded loops (an interactive fitter stepping once per
// frame, a serving loop with a deadline) cannot afford it; hosts that own all
// device memory through a fixed budget or their own allocator (plugin hosts,
// memory-capped multi-tenant processes) forbid it outright. The regular entry
// points allocate their scratch lazily in the dr_ctx; this one takes it from a
// fixed array compiled into the library instead.
//
// The scratch lives in one file-scope __device__ array, kNoAllocScratchBytes
// (about 3.3 MB) per GPU that loads the library, held until process exit. Host
// code must not pass the array's name to a kernel: in host code it is only a
// stand-in, not a device address. The first call on each device (with that
// device current) resolves the real address with cudaGetSymbolAddress and
// caches it; make that first call before any stream capture. Later calls made
// outside a capture resolve it again (a cheap lookup), so a device reset,
// which reloads the module and may move the array, never leaves a stale
// address behind; a call inside a capture uses the cached one. Every call
// shares the array, so calls whose work overlaps on the GPU (different
// streams, or different host threads without ordering) race and must be
// serialized by the caller.

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/diffrast_cuda.h"
#include "dr_device.cuh"
#include "dr_internal.h"

using namespace dr;

namespace {

constexpr size_t kRecBytes = sizeof(TriRec) * (size_t)DR_NOALLOC_MAX_TRIANGLES;
constexpr size_t kPartialBytes = sizeof(double) * (size_t)DR_NOALLOC_MAX_TILES;
constexpr size_t kCounterBytes = sizeof(unsigned) * (size_t)DR_NOALLOC_MAX_BATCH;
constexpr size_t kNoAllocScratchBytes = kRecBytes + kPartialBytes + kCounterBytes;

// 256-byte alignment keeps every sub-buffer (records, partials, counters)
// aligned for vector access.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
std::atomic<unsigned char*> g_scratch_ptr[kMaxDevices];

dr_status noalloc_fail(dr_status s, const char* msg) {
  set_last_error(msg);  // reported by dr_last_error()
  return s;
}

// The device address of the scratch array on the current device. Set up on
// the first call per device (with that device current); refreshed on every
// call whose stream is not being captured, so the cache never outlives the
// module it came from. Inside a capture the cached address is used, and a
// capture before any set-up is an error.
dr_status scratch_for_current_device(cudaStream_t stream, unsigned char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(DR_NO_DEVICE, "dr_loss_backward_noalloc: no usable current CUDA device");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    cap = cudaStreamCaptureStatusActive;  // unknown: do not touch the runtime's state
  }
  unsigned char* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (cap != cudaStreamCaptureStatusNone) {
    if (!p)
      return noalloc_fail(DR_INVALID_ARGUMENT,
                          "dr_loss_backward_noalloc: the first call on a device must come "
                          "before any stream capture");
    *out = p;
    return DR_OK;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  if (e != cudaSuccess || !addr) {
    cudaGetLastError();
    return noalloc_fail(DR_LAUNCH, "dr_loss_backward_noalloc: cudaGetSymbolAddress failed");
  }
  p = static_cast<unsigned char*>(addr);
  g_scratch_ptr[dev].store(p, std::memory_order_release);
  *out = p;
  return DR_OK;
}

}  // namespace

extern "C" {

dr_status dr_loss_backward_noalloc(const float* params, const float* background, int B, int T,
                                   int H, int W, float sigma, const float* targets, int layout,
                                   float* grads, float* losses, dr_stream_t stream) {
  if (B < 0 || T < 0 || H <= 0 || W <= 0)
    return noalloc_fail(DR_INVALID_ARGUMENT, "dr_loss_backward_noalloc: bad sizes");
  if (!std::isfinite(sigma) || sigma <= 0.0f)
    return noalloc_fail(DR_INVALID_ARGUMENT,
                        "dr_loss_backward_noalloc: sigma must be positive and finite");
  if (layout != DR_LAYOUT_BHWC && layout != DR_LAYOUT_BCHW)
    return noalloc_fail(DR_INVALID_ARGUMENT, "dr_loss_backward_noalloc: unknown layout");
  if (B == 0) return DR_OK;
  if (!targets || (T > 0 && (!params || !grads)))
    return noalloc_fail(DR_INVALID_ARGUMENT, "dr_loss_backward_noalloc: null pointer");
  const long long tiles_x = (W + 15) / 16, tiles_y = (H + 15) / 16;
  if (H > 32768 || W > 32768 || (long long)B * T > DR_NOALLOC_MAX_TRIANGLES ||
      B > DR_NOALLOC_MAX_BATCH || (long long)B * tiles_x * tiles_y > DR_NOALLOC_MAX_TILES)
    return noalloc_fail(DR_TOO_LARGE,
                        "dr_loss_backward_noalloc: the call exceeds the static scratch "
                        "(B*T <= DR_NOALLOC_MAX_TRIANGLES, B <= DR_NOALLOC_MAX_BATCH, "
                        "B*tiles <= DR_NOALLOC_MAX_TILES); use dr_loss_backward");

  cudaStream_t s = (cudaStream_t)stream;
  unsigned char* base = nullptr;
  dr_status st = scratch_for_current_device(s, &base);
  if (st) return st;
  TriRec* recs = reinterpret_cast<TriRec*>(base);
  double* partials = reinterpret_cast<double*>(base + kRecBytes);
  unsigned* counters = reinterpret_cast<unsigned*>(base + kRecBytes + kPartialBytes);

  // The array keeps the previous call's contents: the tile counters must
  // start at zero, and grads are accumulated into.
  if (cudaMemsetAsync(counters, 0, sizeof(unsigned) * (size_t)B, s) != cudaSuccess ||
      (T > 0 && cudaMemsetAsync(grads, 0, sizeof(float) * (size_t)B * T * kParams, s) !=
                    cudaSuccess)) {
    cudaGetLastError();
    return noalloc_fail(DR_LAUNCH, "dr_loss_backward_noalloc: cudaMemsetAsync failed");
  }
  if (launch_setup(params, B * T, W, H, sigma, 1, recs, s) != cudaSuccess) {
    cudaGetLastError();
    return noalloc_fail(DR_LAUNCH, "dr_loss_backward_noalloc: set-up kernel launch failed");
  }

  RasterArgs a;
  memset(&a, 0, sizeof(a));
  a.recs = recs;
  a.B = B;
  a.T = T;
  a.H = H;
  a.W = W;
  a.tiles_x = (int)tiles_x;
  a.tile_row0 = 0;
  a.tile_row_step = 1;
  a.sigma_eff = std::fmax(sigma, 1e-8f);
  a.inv_sigma = (float)(1.0 / (double)a.sigma_eff);
  a.precision = 0;
  if (background) {
    a.bg3[0] = background[0];
    a.bg3[1] = background[1];
    a.bg3[2] = background[2];
  }
  a.layout = layout;
  a.other = targets;
  a.grad_scale = 2.0f / (float)((long long)H * W * 3);
  a.grads = grads;
  a.loss_partials = partials;
  a.loss_counters = counters;
  a.losses = losses;
  a.n_values = (double)H * (double)W * 3.0;
  if (launch_raster(kModeLoss, a, (int)(tiles_x * tiles_y), s) != cudaSuccess) {
    cudaGetLastError();
    return noalloc_fail(DR_LAUNCH, "dr_loss_backward_noalloc: raster kernel launch failed");
  }
  return DR_OK;
}

}  // extern "C"
