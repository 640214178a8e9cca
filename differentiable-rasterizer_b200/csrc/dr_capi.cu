// C ABI of libdiffrast_cuda.so (declared in include/diffrast_cuda.h).
//
// Host side of the B200 rasterizer: argument checks that mirror the reference's
// (diffrast-py/src/lib.rs:162-195, 256-273, 344-361; diffrast-gpu/src/lib.rs:914-929),
// a per-context scratch pool with hit/miss counters (BufferPool, lib.rs:130-188),
// the launch sequence of each entry point, and the on-device fit loop.

#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/diffrast_cuda.h"
#include "dr_device.cuh"
#include "dr_internal.h"

using namespace dr;

namespace {

thread_local std::string g_last_error;

dr_status fail(dr_status s, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

dr_status cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(DR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
  }
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
    return fail(DR_NO_DEVICE, "%s: %s", what, cudaGetErrorString(e));
  return fail(DR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

#define DR_CUDA(call, what)                       \
  do {                                            \
    cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Limits: 16-bit-safe tile math and the CUDA grid's y dimension.
constexpr int kMaxSide = 32768;
constexpr int kMaxBatch = 65535;
constexpr long long kMaxTris = 1 << 24;
constexpr int kTileSide = 16;
// GpuRasterizer::POLL_TIMEOUT (diffrast-gpu/src/lib.rs:229): the bound on every
// host wait for device work.
constexpr double kPollTimeoutS = 60.0;

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// One named, grow-only device buffer. A request that fits is a pool hit.
struct Slot {
  void* ptr = nullptr;
  size_t cap = 0;
};

}  // namespace

namespace dr {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace dr

struct dr_ctx {
  int device = 0;
  std::mutex mu;
  int bg_on_device = 0;
  int precision = 0;
  int split_blocks = 0;  // dr_set_triangle_split: 0 automatic, 1 never, k exactly
  int reduce_mode = DR_REDUCE_WORKGROUP;  // dr_set_reduce_mode (both values: one reduction)
  int deterministic = 0;                  // dr_set_deterministic
  uint64_t hits = 0, misses = 0;
  Slot recs, partials, counters, bgbuf, split;
  Slot det_fx, det_nf;  // deterministic mode: fixed-point sums and non-finite flags
  // fit state
  Slot fit_params, fit_m, fit_v, fit_grads, fit_losses, fit_state, fit_best, fit_target;
  cudaStream_t capture_stream = nullptr;
  cudaGraphExec_t fit_exec = nullptr;
  std::vector<unsigned char> fit_key;
  // dr_loss_backward_host: device copies of the caller's host buffers, and the
  // streams and events of its upload / compute / download pipeline.
  Slot io_params, io_targets, io_grads, io_losses;
  cudaStream_t io_copy = nullptr, io_comp[2] = {nullptr, nullptr};
  cudaEvent_t io_ev[DR_HOST_CHUNKS_MAX + 1] = {};

  ~dr_ctx() {}
};

namespace {

dr_status ensure(dr_ctx* c, Slot& s, size_t bytes, bool zero) {
  if (bytes == 0) bytes = 16;
  if (s.cap >= bytes) {
    c->hits++;
    return DR_OK;
  }
  c->misses++;
  if (s.ptr) {
    cudaDeviceSynchronize();  // the old buffer may still be in use by queued work
    cudaFree(s.ptr);
    s.ptr = nullptr;
    s.cap = 0;
  }
  size_t want = bytes + bytes / 4;  // headroom for slowly growing shapes
  cudaError_t e = cudaMalloc(&s.ptr, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    e = cudaMalloc(&s.ptr, bytes);
    want = bytes;
  }
  if (e != cudaSuccess) {
    s.ptr = nullptr;
    return cuda_fail(e, "cudaMalloc(scratch)");
  }
  s.cap = want;
  if (zero) {
    e = cudaMemset(s.ptr, 0, want);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(scratch)");
  }
  return DR_OK;
}

// Every scratch buffer a context owns.
std::vector<Slot*> slots(dr_ctx* c) {
  return {&c->recs,       &c->partials,   &c->counters,  &c->bgbuf,      &c->split,
          &c->det_fx,     &c->det_nf,     &c->fit_params, &c->fit_m,     &c->fit_grads,
          &c->fit_v,      &c->fit_losses, &c->fit_state,  &c->fit_best,  &c->fit_target,
          &c->io_params,  &c->io_targets, &c->io_grads,   &c->io_losses};
}

uint64_t pool_bytes(dr_ctx* c) {
  uint64_t b = 0;
  for (Slot* s : slots(c)) b += s->cap;
  return b;
}

void free_slot(Slot& s) {
  if (s.ptr) cudaFree(s.ptr);
  s.ptr = nullptr;
  s.cap = 0;
}

bool finite_positive(float s) { return std::isfinite(s) && s > 0.0f; }

// Shape/argument checks shared by the batched entry points. Mirrors
// diffrast-py/src/lib.rs:162-195 (sigma, zero sizes) and the GPU crate's
// TooLarge conditions.
dr_status check_common(dr_ctx* ctx, const float* params, int B, int T, int H, int W, float sigma,
                       int layout) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (B < 0 || T < 0) return fail(DR_INVALID_ARGUMENT, "negative batch or triangle count");
  if (H <= 0 || W <= 0) return fail(DR_INVALID_ARGUMENT, "height and width must be non-zero");
  if (!finite_positive(sigma)) return fail(DR_INVALID_ARGUMENT, "sigma must be positive and finite");
  if (layout != DR_LAYOUT_BHWC && layout != DR_LAYOUT_BCHW)
    return fail(DR_INVALID_ARGUMENT, "unknown layout %d", layout);
  if (H > kMaxSide || W > kMaxSide)
    return fail(DR_TOO_LARGE, "canvas %dx%d exceeds the %d-pixel limit per side", W, H, kMaxSide);
  if (B > kMaxBatch) return fail(DR_TOO_LARGE, "batch %d exceeds %d", B, kMaxBatch);
  if ((long long)T > kMaxTris) return fail(DR_TOO_LARGE, "%d triangles exceeds %lld", T, kMaxTris);
  if ((long long)B * T > (1LL << 28))
    return fail(DR_TOO_LARGE, "%lld triangles in one batch exceeds %lld", (long long)B * T,
                1LL << 28);
  if (B > 0 && T > 0 && !params) return fail(DR_INVALID_ARGUMENT, "null params");
  return DR_OK;
}

// The raster arguments every launch shares: sizes, sigma, precision, layout
// and the loss normalisation (no background, records or buffers).
void base_args(const dr_ctx* ctx, int B, int T, int H, int W, float sigma, int layout,
               RasterArgs& a) {
  memset(&a, 0, sizeof(a));
  a.B = B;
  a.T = T;
  a.H = H;
  a.W = W;
  a.tiles_x = (W + kTileSide - 1) / kTileSide;
  a.tile_row0 = 0;
  a.tile_row_step = 1;
  a.sigma_eff = std::fmax(sigma, 1e-8f);  // raster.rs:75 sigma.max(1e-8)
  a.inv_sigma = (float)(1.0 / (double)a.sigma_eff);
  a.precision = ctx->precision;
  a.layout = layout;
  a.n_values = (double)H * (double)W * 3.0;
  a.grad_scale = 2.0f / (float)((long long)H * W * 3);  // grad.rs:112
}

// Builds the shared part of the raster arguments and runs the set-up kernel.
dr_status prepare(dr_ctx* ctx, const float* params, const float* background, int bg_per_scene,
                  int B, int T, int H, int W, float sigma, int layout, int tape, RasterArgs& a,
                  cudaStream_t s) {
  base_args(ctx, B, T, H, W, sigma, layout, a);
  a.bg_per_scene = bg_per_scene ? 1 : 0;
  if (!background) {
    a.bg3[0] = a.bg3[1] = a.bg3[2] = 0.0f;
  } else if (ctx->bg_on_device) {
    a.bg_dev = background;
  } else if (!bg_per_scene) {
    a.bg3[0] = background[0];
    a.bg3[1] = background[1];
    a.bg3[2] = background[2];
  } else {
    dr_status st = ensure(ctx, ctx->bgbuf, sizeof(float) * 3 * (size_t)std::max(B, 1), false);
    if (st) return st;
    DR_CUDA(cudaMemcpyAsync(ctx->bgbuf.ptr, background, sizeof(float) * 3 * (size_t)B,
                            cudaMemcpyHostToDevice, s),
            "copy backgrounds");
    a.bg_dev = (const float*)ctx->bgbuf.ptr;
  }
  // The records, then their pixel boxes packed (the tile masks read these).
  size_t rec_bytes = tri_rec_bytes() * (size_t)B * (size_t)T;
  dr_status st = ensure(ctx, ctx->recs, rec_bytes + sizeof(int4) * (size_t)B * T, false);
  if (st) return st;
  a.recs = (const TriRec*)ctx->recs.ptr;
  int4* boxes = (int4*)((unsigned char*)ctx->recs.ptr + rec_bytes);
  a.boxes = boxes;
  DR_CUDA(launch_setup(params, B * T, W, H, sigma, tape, (TriRec*)ctx->recs.ptr, s, boxes),
          "set-up kernel");
  return DR_OK;
}

dr_status loss_scratch(dr_ctx* ctx, RasterArgs& a, int n_tiles) {
  dr_status st = ensure(ctx, ctx->partials, sizeof(double) * (size_t)a.B * n_tiles, false);
  if (st) return st;
  st = ensure(ctx, ctx->counters, sizeof(unsigned) * (size_t)a.B, true);
  if (st) return st;
  a.loss_partials = (double*)ctx->partials.ptr;
  a.loss_counters = (unsigned*)ctx->counters.ptr;
  return DR_OK;
}

// Deterministic mode's scratch for n_tris (scene, triangle) pairs, cleared on
// the stream (the finalize leaves it clear too; this also covers a call that
// failed half way). Sets the launch's fixed-point pointers; off: leaves them null.
dr_status det_scratch(dr_ctx* ctx, RasterArgs& a, size_t n_tris, cudaStream_t s) {
  if (!ctx->deterministic || n_tris == 0) return DR_OK;
  dr_status st = ensure(ctx, ctx->det_fx, n_tris * kParams * sizeof(long long), true);
  if (st) return st;
  st = ensure(ctx, ctx->det_nf, n_tris * sizeof(int), true);
  if (st) return st;
  DR_CUDA(cudaMemsetAsync(ctx->det_fx.ptr, 0, n_tris * kParams * sizeof(long long), s),
          "clear fixed-point sums");
  DR_CUDA(cudaMemsetAsync(ctx->det_nf.ptr, 0, n_tris * sizeof(int), s), "clear flags");
  a.grads_fx = (long long*)ctx->det_fx.ptr;
  a.grads_nf = (int*)ctx->det_nf.ptr;
  return DR_OK;
}

// Bytes of the pixel tape's flag header (one int per scene and region,
// rounded up to 16 bytes) and of the whole tape.
size_t tape_header_bytes(int B, int H, int W) {
  const int tiles_x = (W + kTileSide - 1) / kTileSide, tiles_y = (H + kTileSide - 1) / kTileSide;
  const size_t n = (size_t)B * tape_regions(tiles_x, tiles_y) * sizeof(int);
  return (n + 15) / 16 * 16;
}

dr_status backward_common(dr_ctx* ctx, int mode, const float* params, const float* background,
                          int bg_per_scene, int B, int T, int H, int W, float sigma,
                          const float* other, int layout, int shard, int n_shards, float* grads,
                          float* losses, double* loss_sums, float* image, cudaStream_t s,
                          const void* tape = nullptr) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (B > 0 && (!other || (T > 0 && !grads)))
    return fail(DR_INVALID_ARGUMENT, "null target/gradient or grads pointer");
  if (n_shards < 1 || shard < 0 || shard >= n_shards)
    return fail(DR_INVALID_ARGUMENT, "shard %d of %d is out of range", shard, n_shards);
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  if (T > 0)
    DR_CUDA(cudaMemsetAsync(grads, 0, sizeof(float) * (size_t)B * T * kParams, s), "zero grads");
  RasterArgs a;
  st = prepare(ctx, params, background, bg_per_scene, B, T, H, W, sigma, layout, 1, a, s);
  if (st) return st;
  int tiles_y = (H + kTileSide - 1) / kTileSide;
  a.tile_row0 = shard;
  a.tile_row_step = n_shards;
  int rows = tiles_y > shard ? (tiles_y - shard + n_shards - 1) / n_shards : 0;
  int n_tiles = a.tiles_x * rows;
  a.other = other;
  a.grads = grads;
  a.image = image;
  a.losses = losses;
  a.loss_sums = loss_sums;
  if (tape && n_shards == 1) {
    a.tape_flags = (int*)tape;
    a.tape = (float4*)((unsigned char*)tape + tape_header_bytes(B, H, W));
  }
  if (mode == kModeLoss) {
    if (n_tiles == 0) {
      if (losses) DR_CUDA(cudaMemsetAsync(losses, 0, sizeof(float) * B, s), "zero losses");
      if (loss_sums) DR_CUDA(cudaMemsetAsync(loss_sums, 0, sizeof(double) * B, s), "zero sums");
      return DR_OK;
    }
    st = loss_scratch(ctx, a, n_tiles);
    if (st) return st;
  }
  // Too few tiles to fill the GPU: split each pixel's chain into triangle
  // blocks (all tile rows only).
  const int k = n_shards > 1 ? 1
                : ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(B, T, n_tiles);
  if ((st = det_scratch(ctx, a, (size_t)B * T, s))) return st;
  if (k > 1) {
    st = ensure(ctx, ctx->split, raster_split_bytes(B, k, H, W), false);
    if (st) return st;
    DR_CUDA(launch_raster_split(mode, a, n_tiles, k, (float4*)ctx->split.ptr, s),
            "split raster kernels");
  } else {
    DR_CUDA(launch_raster(mode, a, n_tiles, s), "raster kernel");
  }
  if (a.grads_fx)
    DR_CUDA(launch_det_finalize(a.grads_fx, a.grads_nf, grads, (long long)B * T * kParams, s),
            "deterministic finalize");
  return DR_OK;
}

}  // namespace

extern "C" {

const char* dr_last_error(void) { return g_last_error.c_str(); }

const char* dr_status_string(dr_status s) {
  switch (s) {
    case DR_OK: return "ok";
    case DR_INVALID_ARGUMENT: return "invalid argument";
    case DR_TOO_LARGE: return "too large";
    case DR_NO_DEVICE: return "no CUDA device";
    case DR_TIMEOUT: return "timeout";
    case DR_LAUNCH: return "CUDA launch/runtime error";
    case DR_COMM: return "collective failed";
    case DR_OUT_OF_MEMORY: return "out of device memory";
    case DR_INTERNAL: return "internal error";
  }
  return "unknown status";
}

int dr_params_per_triangle(void) { return kParams; }
const char* dr_version(void) { return "0.1.0"; }

int dr_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

dr_status dr_device_name(int device, char* buf, size_t len) {
  if (!buf || len == 0) return fail(DR_INVALID_ARGUMENT, "null buffer");
  int n = dr_device_count();
  if (device < 0 || device >= n) return fail(DR_NO_DEVICE, "no CUDA device %d (have %d)", device, n);
  cudaDeviceProp p;
  DR_CUDA(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
  snprintf(buf, len, "%s", p.name);
  return DR_OK;
}

dr_status dr_ctx_create(int device, dr_ctx** out) {
  if (!out) return fail(DR_INVALID_ARGUMENT, "null output pointer");
  *out = nullptr;
  int n = dr_device_count();
  if (n == 0) return fail(DR_NO_DEVICE, "no CUDA device is visible");
  if (device < 0 || device >= n) return fail(DR_NO_DEVICE, "no CUDA device %d (have %d)", device, n);
  DeviceGuard g(device);
  cudaError_t e = cudaFree(nullptr);  // establish the primary context
  if (e != cudaSuccess) return cuda_fail(e, "CUDA context initialisation");
  dr_ctx* c = new dr_ctx();
  c->device = device;
  *out = c;
  return DR_OK;
}

dr_status dr_ctx_destroy(dr_ctx* c) {
  if (!c) return DR_OK;
  {
    DeviceGuard g(c->device);
    cudaDeviceSynchronize();
    for (Slot* s : slots(c)) free_slot(*s);
    if (c->fit_exec) cudaGraphExecDestroy(c->fit_exec);
    if (c->capture_stream) cudaStreamDestroy(c->capture_stream);
    for (cudaStream_t st : {c->io_copy, c->io_comp[0], c->io_comp[1]})
      if (st) cudaStreamDestroy(st);
    for (cudaEvent_t ev : c->io_ev)
      if (ev) cudaEventDestroy(ev);
  }
  delete c;
  return DR_OK;
}

dr_status dr_set_background_location(dr_ctx* ctx, int on_device) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  ctx->bg_on_device = on_device ? 1 : 0;
  return DR_OK;
}

dr_status dr_set_triangle_split(dr_ctx* ctx, int blocks) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (blocks < 0 || blocks > 65535)
    return fail(DR_INVALID_ARGUMENT, "triangle blocks must be in [0, 65535], got %d", blocks);
  std::lock_guard<std::mutex> lock(ctx->mu);
  ctx->split_blocks = blocks;
  if (ctx->fit_exec) {
    cudaGraphExecDestroy(ctx->fit_exec);
    ctx->fit_exec = nullptr;
    ctx->fit_key.clear();
  }
  return DR_OK;
}

dr_status dr_set_precision(dr_ctx* ctx, int precision) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (precision < DR_PRECISION_REFERENCE || precision > DR_PRECISION_FAST)
    return fail(DR_INVALID_ARGUMENT, "unknown precision mode %d", precision);
  std::lock_guard<std::mutex> lock(ctx->mu);
  ctx->precision = precision;
  if (ctx->fit_exec) {
    cudaGraphExecDestroy(ctx->fit_exec);
    ctx->fit_exec = nullptr;
    ctx->fit_key.clear();
  }
  return DR_OK;
}

dr_status dr_query_path(dr_ctx* ctx, int B, int T, int H, int W, int* path) {
  if (!ctx || !path) return fail(DR_INVALID_ARGUMENT, "null pointer");
  if (B < 0 || T < 0 || H <= 0 || W <= 0) return fail(DR_INVALID_ARGUMENT, "bad sizes");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  const int tiles_x = (W + kTileSide - 1) / kTileSide, tiles_y = (H + kTileSide - 1) / kTileSide;
  const int k = ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(B, T, tiles_x * tiles_y);
  *path = raster_path(B, T, tiles_x, tiles_y, k);
  return DR_OK;
}

dr_status dr_render(dr_ctx* ctx, const float* params, const float* background, int bg_per_scene,
                    int B, int T, int H, int W, float sigma, int layout, float* image,
                    dr_stream_t stream) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (B > 0 && !image) return fail(DR_INVALID_ARGUMENT, "null image pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  RasterArgs a;
  st = prepare(ctx, params, background, bg_per_scene, B, T, H, W, sigma, layout, 0, a, s);
  if (st) return st;
  a.image = image;
  int n_tiles = a.tiles_x * ((H + kTileSide - 1) / kTileSide);
  DR_CUDA(launch_raster(kModeRender, a, n_tiles, s), "raster kernel");
  return DR_OK;
}

dr_status dr_loss_backward(dr_ctx* ctx, const float* params, const float* background,
                           int bg_per_scene, int B, int T, int H, int W, float sigma,
                           const float* targets, int layout, float* grads, float* losses,
                           float* image, dr_stream_t stream) {
  return backward_common(ctx, kModeLoss, params, background, bg_per_scene, B, T, H, W, sigma,
                         targets, layout, 0, 1, grads, losses, nullptr, image,
                         (cudaStream_t)stream);
}

dr_status dr_grad_backward(dr_ctx* ctx, const float* params, const float* background,
                           int bg_per_scene, int B, int T, int H, int W, float sigma,
                           const float* grad_images, int layout, float* grads,
                           dr_stream_t stream) {
  return backward_common(ctx, kModeGrad, params, background, bg_per_scene, B, T, H, W, sigma,
                         grad_images, layout, 0, 1, grads, nullptr, nullptr, nullptr,
                         (cudaStream_t)stream);
}

uint64_t dr_pixel_tape_bytes(int B, int H, int W) {
  if (B < 0 || H <= 0 || W <= 0) return 0;
  return tape_header_bytes(B, H, W) + (uint64_t)B * H * W * sizeof(float4);
}

dr_status dr_render_taped(dr_ctx* ctx, const float* params, const float* background,
                          int bg_per_scene, int B, int T, int H, int W, float sigma, int layout,
                          float* image, void* tape, dr_stream_t stream) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (B > 0 && (!image || !tape)) return fail(DR_INVALID_ARGUMENT, "null image or tape pointer");
  if (((uintptr_t)tape & 15u) != 0) return fail(DR_INVALID_ARGUMENT, "tape must be 16-byte aligned");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  RasterArgs a;
  st = prepare(ctx, params, background, bg_per_scene, B, T, H, W, sigma, layout, 0, a, s);
  if (st) return st;
  a.image = image;
  const int tiles_y = (H + kTileSide - 1) / kTileSide;
  const int n_tiles = a.tiles_x * tiles_y;
  if (raster_path(B, T, a.tiles_x, tiles_y, 1) == 1) {
    a.tape_flags = (int*)tape;
    a.tape = (float4*)((unsigned char*)tape + tape_header_bytes(B, H, W));
  } else {  // only the region kernel keeps a tape: flag every region
    DR_CUDA(cudaMemsetAsync(tape, 1, tape_header_bytes(B, H, W), s), "flag the tape unused");
  }
  DR_CUDA(launch_raster(kModeRender, a, n_tiles, s), "raster kernel");
  return DR_OK;
}

dr_status dr_grad_backward_taped(dr_ctx* ctx, const float* params, const float* background,
                                 int bg_per_scene, int B, int T, int H, int W, float sigma,
                                 const float* grad_images, int layout, const void* tape,
                                 float* grads, dr_stream_t stream) {
  if (B > 0 && !tape) return fail(DR_INVALID_ARGUMENT, "null tape pointer");
  if (((uintptr_t)tape & 15u) != 0) return fail(DR_INVALID_ARGUMENT, "tape must be 16-byte aligned");
  return backward_common(ctx, kModeGrad, params, background, bg_per_scene, B, T, H, W, sigma,
                         grad_images, layout, 0, 1, grads, nullptr, nullptr, nullptr,
                         (cudaStream_t)stream, tape);
}

dr_status dr_loss_backward_sharded(dr_ctx* ctx, const float* params, const float* background,
                                   int bg_per_scene, int B, int T, int H, int W, float sigma,
                                   const float* targets, int layout, int shard, int n_shards,
                                   float* grads, double* loss_sums, dr_stream_t stream) {
  return backward_common(ctx, kModeLoss, params, background, bg_per_scene, B, T, H, W, sigma,
                         targets, layout, shard, n_shards, grads, nullptr, loss_sums, nullptr,
                         (cudaStream_t)stream);
}

dr_status dr_triangle_block_forward(dr_ctx* ctx, const float* params, const float* background,
                                    int bg_per_scene, int B, int T, int H, int W, float sigma,
                                    int n_blocks, int block, float* state, dr_stream_t stream) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, DR_LAYOUT_BHWC);
  if (st) return st;
  if (n_blocks < 1 || n_blocks > 65535 || block < 0 || block >= n_blocks)
    return fail(DR_INVALID_ARGUMENT, "block %d of %d is out of range", block, n_blocks);
  if (B > 0 && !state) return fail(DR_INVALID_ARGUMENT, "null state pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  RasterArgs a;
  st = prepare(ctx, params, background, bg_per_scene, B, T, H, W, sigma, DR_LAYOUT_BHWC, 1, a, s);
  if (st) return st;
  const int n_tiles = a.tiles_x * ((H + kTileSide - 1) / kTileSide);
  DR_CUDA(launch_triangle_block(0, kModeLoss, a, n_tiles, n_blocks, block, (float4*)state, s),
          "triangle-block forward");
  return DR_OK;
}

dr_status dr_triangle_block_backward(dr_ctx* ctx, const float* params, const float* background,
                                     int bg_per_scene, int B, int T, int H, int W, float sigma,
                                     int n_blocks, int block, const float* state,
                                     const float* other, int layout, int grad_input, float* grads,
                                     float* losses, float* image, dr_stream_t stream) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (n_blocks < 1 || n_blocks > 65535 || block < 0 || block >= n_blocks)
    return fail(DR_INVALID_ARGUMENT, "block %d of %d is out of range", block, n_blocks);
  if (grad_input != 0 && grad_input != 1)
    return fail(DR_INVALID_ARGUMENT, "grad_input must be 0 (target) or 1 (image gradient)");
  if (B > 0 && (!state || !other || (T > 0 && !grads)))
    return fail(DR_INVALID_ARGUMENT, "null state, target/gradient or grads pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (T > 0)
    DR_CUDA(cudaMemsetAsync(grads, 0, sizeof(float) * (size_t)B * T * kParams, s), "zero grads");
  RasterArgs a;
  st = prepare(ctx, params, background, bg_per_scene, B, T, H, W, sigma, layout, 1, a, s);
  if (st) return st;
  const int n_tiles = a.tiles_x * ((H + kTileSide - 1) / kTileSide);
  const int mode = grad_input ? kModeGrad : kModeLoss;
  a.other = other;
  a.grads = grads;
  a.image = image;
  a.losses = losses;
  if (mode == kModeLoss) {
    st = loss_scratch(ctx, a, n_tiles);
    if (st) return st;
  }
  DR_CUDA(launch_triangle_block(1, mode, a, n_tiles, n_blocks, block,
                                (float4*)const_cast<float*>(state), s),
          "triangle-block backward");
  return DR_OK;
}

int dr_host_chunks(int B, int* lo, int* hi) {
  if (B <= 0 || !lo || !hi) return 0;
  const double cut[DR_HOST_CHUNKS_MAX - 1] = {0.0625, 0.25, 0.5, 0.75};
  int n = 0, prev = 0;
  for (int i = 0; i < DR_HOST_CHUNKS_MAX; ++i) {
    const int c = i + 1 < DR_HOST_CHUNKS_MAX ? (int)(B * cut[i] + 0.5) : B;
    if (c > prev) {
      lo[n] = prev;
      hi[n] = c;
      ++n;
      prev = c;
    }
  }
  return n;
}

dr_status dr_loss_backward_host(dr_ctx* ctx, const float* params, const float* background,
                                int bg_per_scene, int B, int T, int H, int W, float sigma,
                                const float* targets, int layout, float* grads, float* losses,
                                dr_stream_t stream) {
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (B > 0 && (!targets || !losses || (T > 0 && !grads)))
    return fail(DR_INVALID_ARGUMENT, "null target, losses or grads pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  const size_t per_p = (size_t)T * kParams, per_t = (size_t)H * W * 3;
  const int tiles = ((W + kTileSide - 1) / kTileSide) * ((H + kTileSide - 1) / kTileSide);
  int lo[DR_HOST_CHUNKS_MAX], hi[DR_HOST_CHUNKS_MAX], k[DR_HOST_CHUNKS_MAX];
  size_t split_at[DR_HOST_CHUNKS_MAX + 1] = {0};
  const int nc = dr_host_chunks(B, lo, hi);
  for (int c = 0; c < nc; ++c) {
    const int n = hi[c] - lo[c];
    k[c] = ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(n, T, tiles);
    split_at[c + 1] = split_at[c] + (k[c] > 1 ? raster_split_bytes(n, k[c], H, W) : 0);
  }
  const bool per_scene = background && bg_per_scene;
  if ((st = ensure(ctx, ctx->io_params, sizeof(float) * per_p * B, false))) return st;
  if ((st = ensure(ctx, ctx->io_targets, sizeof(float) * per_t * B, false))) return st;
  if ((st = ensure(ctx, ctx->io_grads, sizeof(float) * per_p * B, false))) return st;
  if ((st = ensure(ctx, ctx->io_losses, sizeof(float) * (size_t)B, false))) return st;
  if ((st = ensure(ctx, ctx->recs, (tri_rec_bytes() + sizeof(int4)) * (size_t)B * T, false)))
    return st;
  if ((st = ensure(ctx, ctx->partials, sizeof(double) * (size_t)B * tiles, false))) return st;
  if ((st = ensure(ctx, ctx->counters, sizeof(unsigned) * (size_t)B, true))) return st;
  if (split_at[nc] && (st = ensure(ctx, ctx->split, split_at[nc], false))) return st;
  if (per_scene && (st = ensure(ctx, ctx->bgbuf, sizeof(float) * 3 * (size_t)B, false)))
    return st;
  if (ctx->deterministic && T > 0) {
    if ((st = ensure(ctx, ctx->det_fx, per_p * B * sizeof(long long), true))) return st;
    if ((st = ensure(ctx, ctx->det_nf, (size_t)T * B * sizeof(int), true))) return st;
  }
  if (!ctx->io_copy) {
    // Created once per context; on a failure nothing half-made is kept.
    cudaStream_t q[3] = {};
    cudaError_t e = cudaSuccess;
    for (cudaStream_t& x : q)
      if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking);
    for (cudaEvent_t& ev : ctx->io_ev)
      if (e == cudaSuccess && !ev) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      for (cudaStream_t x : q)
        if (x) cudaStreamDestroy(x);
      return cuda_fail(e, "creating the host pipeline's streams and events");
    }
    ctx->io_copy = q[0];
    ctx->io_comp[0] = q[1];
    ctx->io_comp[1] = q[2];
  }
  float* P = (float*)ctx->io_params.ptr;
  float* Tg = (float*)ctx->io_targets.ptr;
  float* G = (float*)ctx->io_grads.ptr;
  float* L = (float*)ctx->io_losses.ptr;
  TriRec* R = (TriRec*)ctx->recs.ptr;
  cudaError_t err = cudaSuccess;
  const char* where = "";
  auto chk = [&](cudaError_t e, const char* what) {
    if (err == cudaSuccess && e != cudaSuccess) {
      err = e;
      where = what;
    }
  };
  // After the caller's stream's work.
  cudaEvent_t after = ctx->io_ev[DR_HOST_CHUNKS_MAX];
  chk(cudaEventRecord(after, (cudaStream_t)stream), "ordering after the caller's stream");
  for (cudaStream_t q : {ctx->io_copy, ctx->io_comp[0], ctx->io_comp[1]})
    chk(cudaStreamWaitEvent(q, after, 0), "ordering after the caller's stream");
  if (per_scene)
    chk(cudaMemcpyAsync(ctx->bgbuf.ptr, background, sizeof(float) * 3 * (size_t)B,
                        cudaMemcpyHostToDevice, ctx->io_copy),
        "uploading backgrounds");
  const bool det = ctx->deterministic && T > 0;
  if (det) {  // cleared ahead of the uploads, which every chunk waits for
    chk(cudaMemsetAsync(ctx->det_fx.ptr, 0, per_p * B * sizeof(long long), ctx->io_copy),
        "clearing fixed-point sums");
    chk(cudaMemsetAsync(ctx->det_nf.ptr, 0, (size_t)T * B * sizeof(int), ctx->io_copy),
        "clearing flags");
  }
  // Every upload is queued first: a download into pageable memory blocks the
  // host thread, and must not hold back later chunks' uploads.
  for (int c = 0; c < nc; ++c) {
    const size_t l = lo[c], n = hi[c] - lo[c];
    chk(cudaMemcpyAsync(P + l * per_p, params + l * per_p, sizeof(float) * n * per_p,
                        cudaMemcpyHostToDevice, ctx->io_copy),
        "uploading parameters");
    chk(cudaMemcpyAsync(Tg + l * per_t, targets + l * per_t, sizeof(float) * n * per_t,
                        cudaMemcpyHostToDevice, ctx->io_copy),
        "uploading targets");
    chk(cudaEventRecord(ctx->io_ev[c], ctx->io_copy), "recording an upload");
  }
  for (int c = 0; c < nc && err == cudaSuccess; ++c) {
    const size_t l = lo[c];
    const int n = hi[c] - lo[c];
    cudaStream_t q = ctx->io_comp[c & 1];
    chk(cudaStreamWaitEvent(q, ctx->io_ev[c], 0), "waiting for an upload");
    if (T > 0)
      chk(cudaMemsetAsync(G + l * per_p, 0, sizeof(float) * n * per_p, q), "zeroing gradients");
    RasterArgs a;
    base_args(ctx, n, T, H, W, sigma, layout, a);
    if (per_scene) {
      a.bg_dev = (const float*)ctx->bgbuf.ptr + 3 * l;
      a.bg_per_scene = 1;
    } else if (background) {
      a.bg3[0] = background[0];
      a.bg3[1] = background[1];
      a.bg3[2] = background[2];
    }
    a.recs = R + l * T;
    int4* boxes = (int4*)(R + (size_t)B * T) + l * T;  // packed boxes after all records
    a.boxes = boxes;
    chk(launch_setup(P + l * per_p, n * T, W, H, sigma, 1, R + l * T, q, boxes),
        "set-up kernel");
    a.other = Tg + l * per_t;
    a.grads = G + l * per_p;
    a.losses = L + l;
    a.loss_partials = (double*)ctx->partials.ptr + l * tiles;
    a.loss_counters = (unsigned*)ctx->counters.ptr + l;
    if (det) {
      a.grads_fx = (long long*)ctx->det_fx.ptr + l * per_p;
      a.grads_nf = (int*)ctx->det_nf.ptr + l * T;
    }
    if (k[c] > 1)
      chk(launch_raster_split(kModeLoss, a, tiles, k[c],
                              (float4*)((char*)ctx->split.ptr + split_at[c]), q),
          "split raster kernels");
    else
      chk(launch_raster(kModeLoss, a, tiles, q), "raster kernel");
    if (det)
      chk(launch_det_finalize(a.grads_fx, a.grads_nf, G + l * per_p, (long long)n * per_p, q),
          "deterministic finalize");
    if (T > 0)
      chk(cudaMemcpyAsync(grads + l * per_p, G + l * per_p, sizeof(float) * n * per_p,
                          cudaMemcpyDeviceToHost, q),
          "downloading gradients");
    chk(cudaMemcpyAsync(losses + l, L + l, sizeof(float) * n, cudaMemcpyDeviceToHost, q),
        "downloading losses");
  }
  // The host buffers stay in use until every stream is done, errors included.
  // Each wait is bounded (POLL_TIMEOUT, diffrast-gpu/src/lib.rs:223-229); on a
  // timeout the copies may still be running, and dr_ctx_destroy waits for them.
  for (cudaStream_t q : {ctx->io_comp[0], ctx->io_comp[1], ctx->io_copy}) {
    if (err != cudaSuccess) {
      chk(cudaStreamSynchronize(q), "host pipeline");
      continue;
    }
    const dr_status ws = dr_stream_wait(q, kPollTimeoutS);
    if (ws == DR_TIMEOUT) return ws;
    if (ws != DR_OK) chk(cudaStreamSynchronize(q), "host pipeline");
  }
  if (err != cudaSuccess) return cuda_fail(err, where);
  return DR_OK;
}

dr_status dr_backward(dr_ctx* ctx, const float* params, const float* background, int T, int H,
                      int W, float sigma, const float* target, int layout, int mode, float* grads,
                      float* loss, float* image, dr_stream_t stream) {
  if (mode != DR_BACKWARD_TAPED && mode != DR_BACKWARD_RECOMPUTE)
    return fail(DR_INVALID_ARGUMENT, "unknown backward mode %d", mode);
  return backward_common(ctx, kModeLoss, params, background, 0, 1, T, H, W, sigma, target, layout,
                         0, 1, grads, loss, nullptr, image, (cudaStream_t)stream);
}

dr_status dr_set_reduce_mode(dr_ctx* ctx, int mode) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (mode != DR_REDUCE_DIRECT && mode != DR_REDUCE_WORKGROUP)
    return fail(DR_INVALID_ARGUMENT, "unknown reduce mode %d", mode);
  std::lock_guard<std::mutex> lock(ctx->mu);
  ctx->reduce_mode = mode;
  return DR_OK;
}

dr_status dr_get_reduce_mode(dr_ctx* ctx, int* mode) {
  if (!ctx || !mode) return fail(DR_INVALID_ARGUMENT, "null pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  *mode = ctx->reduce_mode;
  return DR_OK;
}

dr_status dr_set_deterministic(dr_ctx* ctx, int on) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (on != 0 && on != 1) return fail(DR_INVALID_ARGUMENT, "deterministic must be 0 or 1, got %d", on);
  std::lock_guard<std::mutex> lock(ctx->mu);
  ctx->deterministic = on;
  if (ctx->fit_exec) {
    cudaGraphExecDestroy(ctx->fit_exec);
    ctx->fit_exec = nullptr;
    ctx->fit_key.clear();
  }
  return DR_OK;
}

dr_status dr_get_deterministic(dr_ctx* ctx, int* on) {
  if (!ctx || !on) return fail(DR_INVALID_ARGUMENT, "null pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  *on = ctx->deterministic;
  return DR_OK;
}

dr_status dr_loss_backward_timed(dr_ctx* ctx, const float* params, const float* background,
                                 int bg_per_scene, int B, int T, int H, int W, float sigma,
                                 const float* targets, int layout, float* grads, float* losses,
                                 dr_backward_timings* timings, dr_stream_t stream) {
  if (!timings) return fail(DR_INVALID_ARGUMENT, "null timings pointer");
  memset(timings, 0, sizeof(*timings));
  dr_status st = check_common(ctx, params, B, T, H, W, sigma, layout);
  if (st) return st;
  if (B > 0 && (!targets || !losses || (T > 0 && !grads)))
    return fail(DR_INVALID_ARGUMENT, "null target, losses or grads pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t np = (size_t)B * T * kParams, nt = (size_t)B * H * W * 3;
  const int tiles = ((W + kTileSide - 1) / kTileSide) * ((H + kTileSide - 1) / kTileSide);
  const int k = ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(B, T, tiles);
  // alloc: the pool grows on the host clock (cudaMalloc is not stream work).
  const auto a0 = std::chrono::steady_clock::now();
  if ((st = ensure(ctx, ctx->io_params, sizeof(float) * np, false))) return st;
  if ((st = ensure(ctx, ctx->io_targets, sizeof(float) * nt, false))) return st;
  if ((st = ensure(ctx, ctx->io_grads, sizeof(float) * np, false))) return st;
  if ((st = ensure(ctx, ctx->io_losses, sizeof(float) * (size_t)B, false))) return st;
  if ((st = ensure(ctx, ctx->recs, (tri_rec_bytes() + sizeof(int4)) * (size_t)B * T, false)))
    return st;
  if ((st = ensure(ctx, ctx->partials, sizeof(double) * (size_t)B * tiles, false))) return st;
  if ((st = ensure(ctx, ctx->counters, sizeof(unsigned) * (size_t)B, true))) return st;
  if (k > 1 && (st = ensure(ctx, ctx->split, raster_split_bytes(B, k, H, W), false))) return st;
  if (background && bg_per_scene &&
      (st = ensure(ctx, ctx->bgbuf, sizeof(float) * 3 * (size_t)B, false)))
    return st;
  if (ctx->deterministic && T > 0) {
    if ((st = ensure(ctx, ctx->det_fx, np * sizeof(long long), true))) return st;
    if ((st = ensure(ctx, ctx->det_nf, (size_t)B * T * sizeof(int), true))) return st;
  }
  timings->alloc_ms =
      (float)std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - a0)
          .count();
  cudaEvent_t ev[4] = {};
  cudaError_t err = cudaSuccess;
  const char* where = "";
  auto chk = [&](cudaError_t e, const char* what) {
    if (err == cudaSuccess && e != cudaSuccess) {
      err = e;
      where = what;
    }
  };
  for (cudaEvent_t& e : ev) chk(cudaEventCreate(&e), "creating timing events");
  float* P = (float*)ctx->io_params.ptr;
  float* Tg = (float*)ctx->io_targets.ptr;
  float* G = (float*)ctx->io_grads.ptr;
  float* L = (float*)ctx->io_losses.ptr;
  RasterArgs a;
  base_args(ctx, B, T, H, W, sigma, layout, a);
  if (err == cudaSuccess) {
    chk(cudaEventRecord(ev[0], s), "recording an event");
    // pack: uploads and the set-up kernel.
    if (T > 0)
      chk(cudaMemcpyAsync(P, params, sizeof(float) * np, cudaMemcpyHostToDevice, s),
          "uploading parameters");
    chk(cudaMemcpyAsync(Tg, targets, sizeof(float) * nt, cudaMemcpyHostToDevice, s),
        "uploading targets");
    if (background && bg_per_scene) {
      chk(cudaMemcpyAsync(ctx->bgbuf.ptr, background, sizeof(float) * 3 * (size_t)B,
                          cudaMemcpyHostToDevice, s),
          "uploading backgrounds");
      a.bg_dev = (const float*)ctx->bgbuf.ptr;
      a.bg_per_scene = 1;
    } else if (background) {
      a.bg3[0] = background[0];
      a.bg3[1] = background[1];
      a.bg3[2] = background[2];
    }
    a.recs = (const TriRec*)ctx->recs.ptr;
    int4* boxes = (int4*)((unsigned char*)ctx->recs.ptr + tri_rec_bytes() * (size_t)B * T);
    a.boxes = boxes;
    chk(launch_setup(P, B * T, W, H, sigma, 1, (TriRec*)ctx->recs.ptr, s, boxes),
        "set-up kernel");
    chk(cudaEventRecord(ev[1], s), "recording an event");
    // dispatch: the fused kernel.
    if (T > 0) chk(cudaMemsetAsync(G, 0, sizeof(float) * np, s), "zeroing gradients");
    a.other = Tg;
    a.grads = G;
    a.losses = L;
    a.loss_partials = (double*)ctx->partials.ptr;
    a.loss_counters = (unsigned*)ctx->counters.ptr;
    if (err == cudaSuccess && det_scratch(ctx, a, (size_t)B * T, s) != DR_OK)
      chk(cudaErrorUnknown, "clearing the deterministic sums");
    if (k > 1)
      chk(launch_raster_split(kModeLoss, a, tiles, k, (float4*)ctx->split.ptr, s),
          "split raster kernels");
    else
      chk(launch_raster(kModeLoss, a, tiles, s), "raster kernel");
    if (a.grads_fx)
      chk(launch_det_finalize(a.grads_fx, a.grads_nf, G, (long long)B * T * kParams, s),
          "deterministic finalize");
    chk(cudaEventRecord(ev[2], s), "recording an event");
    // readback.
    if (T > 0)
      chk(cudaMemcpyAsync(grads, G, sizeof(float) * np, cudaMemcpyDeviceToHost, s),
          "downloading gradients");
    chk(cudaMemcpyAsync(losses, L, sizeof(float) * B, cudaMemcpyDeviceToHost, s),
        "downloading losses");
    chk(cudaEventRecord(ev[3], s), "recording an event");
  }
  dr_status ws = DR_OK;
  if (err == cudaSuccess) {
    ws = dr_stream_wait(stream, kPollTimeoutS);
    if (ws == DR_OK) {
      chk(cudaEventElapsedTime(&timings->pack_ms, ev[0], ev[1]), "reading timing events");
      chk(cudaEventElapsedTime(&timings->dispatch_ms, ev[1], ev[2]), "reading timing events");
      chk(cudaEventElapsedTime(&timings->readback_ms, ev[2], ev[3]), "reading timing events");
    }
  } else {
    cudaStreamSynchronize(s);  // nothing of ours may still read the caller's buffers
  }
  for (cudaEvent_t e : ev)
    if (e) cudaEventDestroy(e);
  if (ws != DR_OK) return ws;
  if (err != cudaSuccess) return cuda_fail(err, where);
  timings->loss_ms = 0.0f;
  return DR_OK;
}

uint64_t dr_tape_bytes(uint64_t n_tris, uint64_t width, uint64_t height) {
  return n_tris * width * height * 3 * 4;
}

uint64_t dr_scratch_bytes(dr_ctx* ctx, int B, int T, int H, int W) {
  if (!ctx || B < 0 || T < 0 || H <= 0 || W <= 0) return 0;
  const int tiles = ((W + kTileSide - 1) / kTileSide) * ((H + kTileSide - 1) / kTileSide);
  int k = 1;
  {
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    k = ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(B, T, tiles);
  }
  uint64_t b = (uint64_t)(tri_rec_bytes() + sizeof(int4)) * B * T +
               sizeof(double) * (uint64_t)B * tiles +
               sizeof(unsigned) * (uint64_t)B;
  if (k > 1) b += raster_split_bytes(B, k, H, W);
  return b;
}

int dr_is_discrete(int device) {
  int n = dr_device_count();
  if (device < 0 || device >= n) return -1;
  int integrated = 0;
  if (cudaDeviceGetAttribute(&integrated, cudaDevAttrIntegrated, device) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return integrated ? 0 : 1;
}

dr_status dr_device_alloc(dr_ctx* ctx, size_t bytes, void** out) {
  if (!ctx || !out) return fail(DR_INVALID_ARGUMENT, "null pointer");
  *out = nullptr;
  DeviceGuard g(ctx->device);
  DR_CUDA(cudaMalloc(out, bytes ? bytes : 1), "cudaMalloc");
  return DR_OK;
}

dr_status dr_device_free(dr_ctx* ctx, void* ptr) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (!ptr) return DR_OK;
  DeviceGuard g(ctx->device);
  DR_CUDA(cudaFree(ptr), "cudaFree");
  return DR_OK;
}

dr_status dr_memcpy(dr_ctx* ctx, void* dst, const void* src, size_t bytes, dr_stream_t stream) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (bytes == 0) return DR_OK;
  if (!dst || !src) return fail(DR_INVALID_ARGUMENT, "null pointer");
  DeviceGuard g(ctx->device);
  DR_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream), "copy");
  return DR_OK;
}

dr_status dr_mse_loss(dr_ctx* ctx, const float* images, const float* targets, int B,
                      int64_t n_per_image, float* losses, dr_stream_t stream) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (B < 0 || n_per_image < 0) return fail(DR_INVALID_ARGUMENT, "negative size");
  if (B > 0 && (!images || !targets || !losses)) return fail(DR_INVALID_ARGUMENT, "null pointer");
  if (B > 2147483647) return fail(DR_TOO_LARGE, "batch too large");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  if (B == 0) return DR_OK;
  const int nb = B < 65535 ? B : 65535;  // batches beyond this run in slices
  dr_status st = ensure(ctx, ctx->partials,
                        sizeof(double) * (size_t)nb * mse_partials_per_image(n_per_image), false);
  if (st) return st;
  st = ensure(ctx, ctx->counters, sizeof(unsigned) * (size_t)nb, true);
  if (st) return st;
  DR_CUDA(launch_mse(images, targets, B, (long long)n_per_image, losses,
                     (double*)ctx->partials.ptr, (unsigned*)ctx->counters.ptr,
                     (cudaStream_t)stream),
          "mse kernel");
  return DR_OK;
}

dr_status dr_adam_step(dr_ctx* ctx, float* params, float* m, float* v, const float* grads,
                       int64_t n, float lr_pos, float lr_color, float lr_alpha, uint32_t step,
                       float beta1, float beta2, float eps, int project, dr_stream_t stream) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  if (n < 0) return fail(DR_INVALID_ARGUMENT, "negative length");
  if (n > 0 && (!params || !m || !v || !grads)) return fail(DR_INVALID_ARGUMENT, "null pointer");
  if (step == 0) return fail(DR_INVALID_ARGUMENT, "Adam step count starts at 1");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  AdamArgs a;
  memset(&a, 0, sizeof(a));
  a.params = params;
  a.m = m;
  a.v = v;
  a.grads = grads;
  a.n = n;
  a.lr_pos = lr_pos;
  a.lr_color = lr_color;
  a.lr_alpha = lr_alpha;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.one_minus_beta1 = 1.0f - beta1;
  a.one_minus_beta2 = 1.0f - beta2;
  a.eps = eps;
  // optim.rs:309-310: 1 - beta.powi(t), f32 square-and-multiply.
  auto powi = [](float base, int e) {
    float r = 1.0f;
    for (;;) {
      if (e & 1) r *= base;
      e /= 2;
      if (e == 0) break;
      base *= base;
    }
    return r;
  };
  a.bc1 = 1.0f - powi(beta1, (int)step);
  a.bc2 = 1.0f - powi(beta2, (int)step);
  a.project = project;
  DR_CUDA(launch_adam(a, (cudaStream_t)stream), "adam kernel");
  return DR_OK;
}

dr_status dr_pool_stats_get(dr_ctx* ctx, dr_pool_stats* out) {
  if (!ctx || !out) return fail(DR_INVALID_ARGUMENT, "null pointer");
  std::lock_guard<std::mutex> lock(ctx->mu);
  out->hits = ctx->hits;
  out->misses = ctx->misses;
  out->bytes = pool_bytes(ctx);
  return DR_OK;
}

dr_status dr_clear_pool(dr_ctx* ctx) {
  if (!ctx) return fail(DR_INVALID_ARGUMENT, "null context");
  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  for (Slot* s : slots(ctx)) free_slot(*s);
  if (ctx->fit_exec) {
    cudaGraphExecDestroy(ctx->fit_exec);
    ctx->fit_exec = nullptr;
    ctx->fit_key.clear();
  }
  return DR_OK;
}

dr_status dr_stream_wait(dr_stream_t stream, double timeout_s) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery((cudaStream_t)stream);
    if (e == cudaSuccess) return DR_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, "stream");
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s)
      return fail(DR_TIMEOUT, "the GPU did not finish within %.1f s", timeout_s);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// ---------------------------------------------------------------------------
// dr_fit: the whole Fitter loop on the device, captured once into a graph.
// ---------------------------------------------------------------------------

static int validate_fit(const dr_fit_config* c, int T) {  // fit.rs:98-117
  if (T == 0) return 1;
  if (!(std::isfinite(c->sigma_start) && std::isfinite(c->sigma_end)) || c->sigma_start <= 0.0f ||
      c->sigma_end <= 0.0f)
    return 2;
  if (c->sigma_start < c->sigma_end) return 3;
  for (float lr : {c->lr_pos, c->lr_color, c->lr_alpha})
    if (!std::isfinite(lr) || lr <= 0.0f) return 4;
  return 0;
}

static float sigma_at(const dr_fit_config* c, int64_t i) {  // fit.rs:343-349
  if (c->iters <= 1) return c->sigma_end;
  float t = (float)i / (float)(c->iters - 1);
  return c->sigma_start * powf(c->sigma_end / c->sigma_start, t);
}

dr_status dr_fit(dr_ctx* ctx, const float* target, int H, int W, const float* init_params,
                 const float* background, int T, const dr_fit_config* cfg, float* best_params,
                 float* final_params, float* losses, dr_fit_report* report, dr_stream_t stream) {
  if (!ctx || !cfg || !report) return fail(DR_INVALID_ARGUMENT, "null pointer");
  memset(report, 0, sizeof(*report));
  report->best_loss = INFINITY;
  int ce = validate_fit(cfg, T);
  if (ce) {
    report->config_error = ce;
    static const char* names[] = {"", "NoTriangles", "NonPositiveSigma", "SigmaNotDecreasing",
                                  "NonPositiveLearningRate"};
    return fail(DR_INVALID_ARGUMENT, "invalid fit config: %s", names[ce]);
  }
  if (cfg->iters < 0) return fail(DR_INVALID_ARGUMENT, "negative iteration count");
  dr_status st = check_common(ctx, init_params, 1, T, H, W, cfg->sigma_end, DR_LAYOUT_BHWC);
  if (st) return st;
  if (!target || !init_params || !best_params || !final_params || (cfg->iters > 0 && !losses))
    return fail(DR_INVALID_ARGUMENT, "null pointer");
  if (cfg->iters > (1 << 24)) return fail(DR_TOO_LARGE, "too many iterations");

  std::lock_guard<std::mutex> lock(ctx->mu);
  DeviceGuard g(ctx->device);
  cudaStream_t s = (cudaStream_t)stream;
  const size_t np = (size_t)T * kParams;
  const int iters = (int)cfg->iters;
  float bg[3] = {0.f, 0.f, 0.f};
  if (background) memcpy(bg, background, sizeof(bg));

  if ((st = ensure(ctx, ctx->fit_params, np * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_m, np * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_v, np * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_grads, np * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_losses, (size_t)std::max(iters, 1) * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_state, sizeof(FitState), true))) return st;
  if ((st = ensure(ctx, ctx->fit_best, np * 4, false))) return st;
  if ((st = ensure(ctx, ctx->fit_target, (size_t)H * W * 3 * 4, false))) return st;
  const bool det = ctx->deterministic != 0;
  if (det && (st = ensure(ctx, ctx->det_fx, np * sizeof(long long), true))) return st;
  if (det && (st = ensure(ctx, ctx->det_nf, (size_t)T * sizeof(int), true))) return st;
  int tiles = ((W + kTileSide - 1) / kTileSide) * ((H + kTileSide - 1) / kTileSide);
  const int split_k = ctx->split_blocks ? ctx->split_blocks : raster_split_blocks(1, T, tiles);
  if (split_k > 1 && (st = ensure(ctx, ctx->split, raster_split_bytes(1, split_k, H, W), false)))
    return st;
  if ((st = ensure(ctx, ctx->recs, tri_rec_bytes() * (size_t)T, false))) return st;
  if ((st = ensure(ctx, ctx->partials, sizeof(double) * (size_t)tiles, false))) return st;
  if ((st = ensure(ctx, ctx->counters, sizeof(unsigned), true))) return st;

  float* P = (float*)ctx->fit_params.ptr;
  float* M = (float*)ctx->fit_m.ptr;
  float* V = (float*)ctx->fit_v.ptr;
  float* Gr = (float*)ctx->fit_grads.ptr;
  float* L = (float*)ctx->fit_losses.ptr;
  FitState* S = (FitState*)ctx->fit_state.ptr;
  float* Best = (float*)ctx->fit_best.ptr;
  float* Tgt = (float*)ctx->fit_target.ptr;

  // The graph reads and writes only this context's buffers: the caller's
  // target and initial scene are copied in before it runs and the results
  // copied out after, so a caller that hands over fresh tensors each call
  // (new allocations, new addresses) reuses the same graph. It bakes the
  // buffers' addresses, the sizes and the config: reuse it when all match.
  std::vector<unsigned char> key;
  auto push = [&](const void* p, size_t n) {
    const unsigned char* b = (const unsigned char*)p;
    key.insert(key.end(), b, b + n);
  };
  const void* ptrs[] = {Tgt,           Best,          P, M, V, Gr, L, S, ctx->recs.ptr,
                        ctx->partials.ptr, ctx->counters.ptr, ctx->split.ptr,
                        det ? ctx->det_fx.ptr : nullptr, det ? ctx->det_nf.ptr : nullptr};
  push(ptrs, sizeof(ptrs));
  push(cfg, sizeof(*cfg));
  int dims[3] = {H, W, T};
  push(dims, sizeof(dims));
  push(bg, sizeof(bg));

  if (!ctx->fit_exec || key != ctx->fit_key) {
    if (ctx->fit_exec) {
      cudaGraphExecDestroy(ctx->fit_exec);
      ctx->fit_exec = nullptr;
    }
    if (!ctx->capture_stream)
      DR_CUDA(cudaStreamCreateWithFlags(&ctx->capture_stream, cudaStreamNonBlocking),
              "capture stream");
    cudaStream_t cs = ctx->capture_stream;
    DR_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t err = cudaSuccess;
    auto chk = [&](cudaError_t e) {
      if (err == cudaSuccess && e != cudaSuccess) err = e;
    };
    chk(cudaMemcpyAsync(Best, P, np * 4, cudaMemcpyDeviceToDevice, cs));
    if (det) {  // each iteration's finalize leaves them clear for the next
      chk(cudaMemsetAsync(ctx->det_fx.ptr, 0, np * sizeof(long long), cs));
      chk(cudaMemsetAsync(ctx->det_nf.ptr, 0, (size_t)T * sizeof(int), cs));
    }
    chk(cudaMemsetAsync(M, 0, np * 4, cs));
    chk(cudaMemsetAsync(V, 0, np * 4, cs));
    chk(launch_fit_init(S, cs));
    // Iteration 0's gradients and records; each iteration's Adam kernel then
    // clears the gradients and writes the next iteration's records.
    chk(cudaMemsetAsync(Gr, 0, np * 4, cs));
    chk(launch_setup(P, T, W, H, sigma_at(cfg, 0), 1, (TriRec*)ctx->recs.ptr, cs));
    for (int i = 0; i < iters; ++i) {
      float sigma = sigma_at(cfg, i);
      RasterArgs a;
      memset(&a, 0, sizeof(a));
      a.recs = (const TriRec*)ctx->recs.ptr;
      a.B = 1;
      a.T = T;
      a.H = H;
      a.W = W;
      a.tiles_x = (W + kTileSide - 1) / kTileSide;
      a.tile_row0 = 0;
      a.tile_row_step = 1;
      a.sigma_eff = std::fmax(sigma, 1e-8f);
      a.inv_sigma = (float)(1.0 / (double)a.sigma_eff);
      a.precision = ctx->precision;
      a.bg3[0] = bg[0];
      a.bg3[1] = bg[1];
      a.bg3[2] = bg[2];
      a.layout = kLayoutBHWC;
      a.other = Tgt;
      a.grad_scale = 2.0f / (float)((long long)H * W * 3);
      a.grads = Gr;
      a.loss_partials = (double*)ctx->partials.ptr;
      a.loss_counters = (unsigned*)ctx->counters.ptr;
      a.losses = &S->loss;
      a.n_values = (double)H * (double)W * 3.0;
      a.skip_flag = &S->stopped;
      a.fit = S;
      a.fit_losses = L;
      a.fit_patience = cfg->patience;
      a.fit_min_delta = cfg->min_delta;
      a.fit_iter = i;
      if (det) {
        a.grads_fx = (long long*)ctx->det_fx.ptr;
        a.grads_nf = (int*)ctx->det_nf.ptr;
      }
      if (split_k > 1)
        chk(launch_raster_split(kModeLoss, a, tiles, split_k, (float4*)ctx->split.ptr, cs));
      else
        chk(launch_raster(kModeLoss, a, tiles, cs));
      if (det) chk(launch_det_finalize(a.grads_fx, a.grads_nf, Gr, (long long)np, cs));
      AdamArgs ad;
      memset(&ad, 0, sizeof(ad));
      ad.params = P;
      ad.m = M;
      ad.v = V;
      ad.grads = Gr;
      ad.n = (long long)np;
      ad.lr_pos = cfg->lr_pos;
      ad.lr_color = cfg->lr_color;
      ad.lr_alpha = cfg->lr_alpha;
      ad.beta1 = 0.9f;
      ad.beta2 = 0.999f;
      ad.one_minus_beta1 = 1.0f - 0.9f;
      ad.one_minus_beta2 = 1.0f - 0.999f;
      ad.eps = 1e-8f;
      // Adam::t equals i + 1 at iteration i: it steps every iteration until
      // the fit stops, and nothing runs after that.
      float b1 = 1.0f, b2 = 1.0f, base1 = 0.9f, base2 = 0.999f;
      for (int e = i + 1;;) {
        if (e & 1) {
          b1 *= base1;
          b2 *= base2;
        }
        e /= 2;
        if (e == 0) break;
        base1 *= base1;
        base2 *= base2;
      }
      ad.bc1 = 1.0f - b1;
      ad.bc2 = 1.0f - b2;
      ad.project = 1;
      ad.run_flag = &S->run_adam;
      ad.copy_flag = &S->copy_best;
      ad.copy_dst = Best;
      const bool last = i + 1 == iters;
      chk(launch_fit_adam_setup(ad, Gr, T, W, H, last ? sigma : sigma_at(cfg, i + 1),
                                last ? nullptr : (TriRec*)ctx->recs.ptr, cs));
    }
    cudaGraph_t graph = nullptr;
    cudaError_t e_end = cudaStreamEndCapture(cs, &graph);
    if (err != cudaSuccess || e_end != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return cuda_fail(err != cudaSuccess ? err : e_end, "capturing the fit loop");
    }
    cudaError_t ei = cudaGraphInstantiate(&ctx->fit_exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) {
      ctx->fit_exec = nullptr;
      return cuda_fail(ei, "instantiating the fit graph");
    }
    ctx->fit_key = key;
  }
  DR_CUDA(cudaMemcpyAsync(Tgt, target, (size_t)H * W * 3 * 4, cudaMemcpyDeviceToDevice, s),
          "copy the target in");
  DR_CUDA(cudaMemcpyAsync(P, init_params, np * 4, cudaMemcpyDeviceToDevice, s),
          "copy the initial scene in");
  DR_CUDA(cudaGraphLaunch(ctx->fit_exec, s), "launching the fit graph");
  DR_CUDA(cudaMemcpyAsync(best_params, Best, np * 4, cudaMemcpyDeviceToDevice, s),
          "copy the best scene out");
  DR_CUDA(cudaMemcpyAsync(final_params, P, np * 4, cudaMemcpyDeviceToDevice, s),
          "copy the final scene out");
  // Bounded wait first (POLL_TIMEOUT semantics), then the blocking reads.
  st = dr_stream_wait(stream, 600.0);
  if (st) return st;
  FitState hs;
  DR_CUDA(cudaMemcpy(&hs, S, sizeof(hs), cudaMemcpyDeviceToHost), "read fit state");
  if (hs.count > 0)
    DR_CUDA(cudaMemcpy(losses, L, sizeof(float) * (size_t)hs.count, cudaMemcpyDeviceToHost),
            "read losses");
  report->n_losses = hs.count;
  report->best_iter = hs.best_iter;
  report->best_loss = hs.best_loss;
  report->stop_reason = hs.stopped ? hs.stop_reason : DR_STOP_COMPLETED;
  return DR_OK;
}

}  // extern "C"
