/*
 * diffrast_cuda.h - C ABI of libdiffrast_cuda.so, the sm_100a (B200) soft-triangle
 * rasterizer: batched forward compositing, per-image MSE, analytic backward and a
 * fused Adam step, for VivianSobers/Differentiable-Rasterizer's hot path.
 *
 * This is the drop-in boundary. Every entry point takes plain pointers and sizes;
 * there are no torch or Rust types in the signatures. Data pointers are DEVICE
 * memory owned by the caller unless a parameter says "host". Work is enqueued on
 * `stream` (a cudaStream_t; NULL is the legacy default stream) and returns before
 * it completes, except where a function says it synchronizes.
 *
 * Layouts (identical to the reference's, diffrast-py/src/lib.rs:10-13):
 *   params  (B, T, 10) f32, per triangle [x0, y0, x1, y1, x2, y2, r, g, b, a],
 *           vertices in normalized image space (scene.rs:78-92)
 *   images  (B, H, W, 3) f32 linear RGB (DR_LAYOUT_BHWC, canvas.rs:6-11) or
 *           (B, 3, H, W) (DR_LAYOUT_BCHW, what torch_layer.rasterize returns)
 *   background  3 floats shared by the batch, or (B, 3) when bg_per_scene != 0
 *           (forward_batch.wgsl:18-20); host or device memory both accepted
 *           (see dr_set_background_location)
 *
 * Errors: every function returns a dr_status. A non-OK status leaves a message
 * for the calling thread in dr_last_error(). Statuses map one to one onto the
 * reference's GpuError (crates/diffrast-gpu/src/lib.rs:42-72) and its panics.
 * There is no CPU fallback: a missing or failing device is an error.
 *
 * Threading: a context may be used from several threads, but the calls it
 * serves share its scratch memory, so they must be ordered on ONE stream (or use
 * one context per stream).
 */
#ifndef DIFFRAST_CUDA_H
#define DIFFRAST_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DR_N_PARAMS 10 /* scene.rs:21 Triangle::N_PARAMS */

#if defined(__GNUC__)
#define DR_API __attribute__((visibility("default")))
#else
#define DR_API
#endif

typedef struct dr_ctx dr_ctx;
typedef void* dr_stream_t; /* a cudaStream_t */

/* GpuError (diffrast-gpu/src/lib.rs:42-72) plus the argument panics. */
typedef enum dr_status {
  DR_OK = 0,
  DR_INVALID_ARGUMENT = 1, /* size / shape mismatch, bad sigma (ValueError, asserts) */
  DR_TOO_LARGE = 2,        /* GpuError::TooLarge (incl. ragged batch, no triangles) */
  DR_NO_DEVICE = 3,        /* GpuError::NoAdapter */
  DR_TIMEOUT = 4,          /* GpuError::Timeout (bounded host wait expired) */
  DR_LAUNCH = 5,           /* a CUDA launch or runtime error (GpuError::DeviceRequest) */
  DR_COMM = 6,             /* a collective failed (multi-GPU paths) */
  DR_OUT_OF_MEMORY = 7,    /* device allocation failed */
  DR_INTERNAL = 8
} dr_status;

typedef enum dr_layout { DR_LAYOUT_BHWC = 0, DR_LAYOUT_BCHW = 1 } dr_layout;

/* --- context ------------------------------------------------------------ */

/* Creates a context on CUDA device `device`. Replaces GpuRasterizer::new
 * (diffrast-gpu/src/lib.rs:232-319): there are no pipelines to compile; the
 * context owns only scratch memory and its reuse pool. */
DR_API dr_status dr_ctx_create(int device, dr_ctx** out);

/* Waits for the context's device work and frees its scratch. Replaces dropping
 * the GpuRasterizer / diffrast_rs.shutdown_gpu (diffrast-py/src/lib.rs:435-444). */
DR_API dr_status dr_ctx_destroy(dr_ctx* ctx);

/* Thread-local message for the last non-OK status on this thread. */
DR_API const char* dr_last_error(void);
DR_API const char* dr_status_string(dr_status s);

/* Parameters per triangle (diffrast-py/src/lib.rs:453-456). */
DR_API int dr_params_per_triangle(void);
DR_API const char* dr_version(void);

/* Device name into buf (GpuRasterizer::adapter_info, lib.rs:374-376;
 * diffrast_rs.gpu_adapter, diffrast-py/src/lib.rs:447-450). */
DR_API dr_status dr_device_name(int device, char* buf, size_t len);
/* Number of visible CUDA devices (0 when none). */
DR_API int dr_device_count(void);

/* Where `background` pointers live: 0 = host memory (default), 1 = device. */
DR_API dr_status dr_set_background_location(dr_ctx* ctx, int on_device);

/* Arithmetic of soft-edge pixels (the band where 0 < coverage < 1).
 *   DR_PRECISION_REFERENCE (default): the nearest edge's distance, the sigmoid
 *     and the gradient direction follow the reference's f32 operations and
 *     rounding (raster.rs:124-134, grad.rs:231-270). Within ~1e-5 of an edge
 *     the reference's f32 gradient direction carries cancellation error of
 *     ~1e-7/dist; this mode reproduces it, so results match the reference.
 *   DR_PRECISION_STRICT: every edge with the reference's exact arithmetic
 *     (IEEE division and sqrt throughout); slowest, for bisecting parity.
 *   DR_PRECISION_FAST: closed-form shortcuts and approximate reciprocals;
 *     closer to the exact (f64) gradient than the reference itself, but not
 *     bit-compatible with its f32 rounding near edges.
 * No reference counterpart (the reference has one precision). */
typedef enum dr_precision {
  DR_PRECISION_REFERENCE = 0,
  DR_PRECISION_STRICT = 1,
  DR_PRECISION_FAST = 2
} dr_precision;
DR_API dr_status dr_set_precision(dr_ctx* ctx, int precision);

/* Triangle-block split of loss/gradient calls (dr_loss_backward,
 * dr_grad_backward, dr_fit). When a call's scenes x 16x16 tiles are too few to
 * fill the GPU (a small image, one scene), each pixel's compositing chain is
 * cut into blocks of consecutive triangles. The blocks run as separate CTAs and
 * their compositing maps are combined per pixel. 0 = choose automatically
 * (default), 1 = never split, k >= 2 = exactly k blocks (at most 65535; calls
 * sharded by tile rows never split). Results agree with the unsplit path to
 * rounding. No reference counterpart. */
DR_API dr_status dr_set_triangle_split(dr_ctx* ctx, int blocks);

/* Which kernel dr_loss_backward / dr_grad_backward take for a batch of B
 * scenes of T triangles at H x W on this context's device (its triangle-split
 * setting included): DR_PATH_TILE (one CTA per scene and 16x16 tile, lists in
 * fixed windows of 128 triangles), DR_PATH_REGION (T <= 128 and at least one
 * wave of CTAs: one CTA per 32x16 region, the list binned once for its 16 warp
 * blocks), DR_PATH_SPLIT (too few tiles to fill the GPU: the triangle-block
 * split) or DR_PATH_TILE_GATHER (the tile kernel for 128 < T <= 8192, its
 * lists gathered from a per-tile mask of the triangles whose boxes meet the
 * tile). For tests and profiling; results agree to rounding whichever path
 * runs. No reference counterpart (the reference has one WGSL pipeline per
 * call). */
typedef enum dr_path {
  DR_PATH_TILE = 0,
  DR_PATH_REGION = 1,
  DR_PATH_SPLIT = 2,
  DR_PATH_TILE_GATHER = 3
} dr_path;
DR_API dr_status dr_query_path(dr_ctx* ctx, int B, int T, int H, int W, int* path);

/* --- hot path ------------------------------------------------------------ */

/* Forward render of a batch into `image` (layout as given).
 * Replaces GpuRasterizer::render_many (diffrast-gpu/src/lib.rs:615-633) and
 * diffrast_rs.render_batch (diffrast-py/src/lib.rs:172-231); semantics of
 * raster::render (crates/diffrast/src/raster.rs:37-68). B == 0 is a no-op. */
DR_API dr_status dr_render(dr_ctx* ctx, const float* params, const float* background, int bg_per_scene,
                    int B, int T, int H, int W, float sigma, int layout, float* image,
                    dr_stream_t stream);

/* Forward + per-image MSE + analytic backward against targets, in one pass.
 * grads (B,T,10) is overwritten; losses (B,) (may be NULL) receives
 * mse(render, target) as canvas.rs:45-59 computes it (f64 sum); image (may be
 * NULL) receives the render. Replaces GpuRasterizer::backward_many
 * (diffrast-gpu/src/lib.rs:639-816) and diffrast_rs.fused_loss_backward
 * (diffrast-py/src/lib.rs:331-412); semantics of grad::backward_batch
 * (crates/diffrast/src/grad.rs:192-207). */
DR_API dr_status dr_loss_backward(dr_ctx* ctx, const float* params, const float* background,
                           int bg_per_scene, int B, int T, int H, int W, float sigma,
                           const float* targets, int layout, float* grads, float* losses,
                           float* image, dr_stream_t stream);

/* dr_loss_backward on HOST buffers: params, background, targets, grads and
 * losses are all host memory (pinned memory, e.g. cudaHostAlloc'd, moves at
 * full PCIe rate; pageable memory works, through the driver's staging). The
 * batch is cut into scene chunks (dr_host_chunks). Every chunk's upload is
 * queued on a copy stream first; each chunk's set-up, raster launch and
 * download then run on one of two compute streams as soon as its upload
 * lands, so uploads, kernels and downloads overlap. The call returns when
 * grads and losses are in host memory (the work is ordered after `stream`).
 * Same results as dr_loss_backward. Replaces the host-array path of
 * diffrast_rs.fused_loss_backward (diffrast-py/src/lib.rs:331-412: numpy in,
 * numpy out) and GpuRasterizer::backward_many's upload / readback
 * (diffrast-gpu/src/lib.rs:639-816). */
DR_API dr_status dr_loss_backward_host(dr_ctx* ctx, const float* params,
                                       const float* background, int bg_per_scene, int B, int T,
                                       int H, int W, float sigma, const float* targets,
                                       int layout, float* grads, float* losses,
                                       dr_stream_t stream);

/* The scene chunks dr_loss_backward_host cuts a batch of B into: chunk c is
 * scenes [lo[c], hi[c]). Cuts fall at 1/16, 1/4, 1/2 and 3/4 of the batch: the
 * first chunk, whose upload overlaps nothing, is small, and the others are
 * large enough for their kernels to keep up with the uploads. 32 scenes go as
 * 2, 6, 8, 8, 8. lo and hi hold DR_HOST_CHUNKS_MAX entries. Returns the number
 * of chunks (0 for B <= 0). */
#define DR_HOST_CHUNKS_MAX 5
DR_API int dr_host_chunks(int B, int* lo, int* hi);

/* Backward from an upstream image gradient dL/d(image) (same layout rules).
 * grads (B,T,10) is overwritten. Replaces GpuRasterizer::backward_many_from_grad
 * (diffrast-gpu/src/lib.rs:828-910) and diffrast_rs.backward_batch
 * (diffrast-py/src/lib.rs:243-324). */
DR_API dr_status dr_grad_backward(dr_ctx* ctx, const float* params, const float* background,
                           int bg_per_scene, int B, int T, int H, int W, float sigma,
                           const float* grad_images, int layout, float* grads,
                           dr_stream_t stream);

/* The taped pair of render_with_tape + backward_from_grad (grad.rs:56-106;
 * BackwardMode::Taped, diffrast-gpu/src/lib.rs:211-220) in a compact form:
 * instead of every triangle's coverage (T x H x W x 12 bytes, tape_bytes),
 * the tape holds one 16-byte word per pixel, the forward's running product of
 * (1 - w) (mantissa, exponent and its last zero and NaN layers), plus a flag
 * word per (scene, 32x16 region). dr_render_taped renders exactly as
 * dr_render and fills the tape; dr_grad_backward_taped, given the same
 * params, sizes, sigma and background, returns exactly what dr_grad_backward
 * returns, reading the products back instead of running the forward walk
 * again. Where the tape cannot stand in (a region holding a NaN-alpha
 * triangle, which render() paints and the backward drops; shapes that do not
 * take the region kernel) the backward recomputes. The
 * tape is caller-owned device memory of dr_pixel_tape_bytes(B, H, W) bytes,
 * 16-byte aligned. No reference counterpart for the compact form. */
DR_API uint64_t dr_pixel_tape_bytes(int B, int H, int W);
DR_API dr_status dr_render_taped(dr_ctx* ctx, const float* params, const float* background,
                                 int bg_per_scene, int B, int T, int H, int W, float sigma,
                                 int layout, float* image, void* tape, dr_stream_t stream);
DR_API dr_status dr_grad_backward_taped(dr_ctx* ctx, const float* params,
                                        const float* background, int bg_per_scene, int B, int T,
                                        int H, int W, float sigma, const float* grad_images,
                                        int layout, const void* tape, float* grads,
                                        dr_stream_t stream);

/* Row-sharded dr_loss_backward for one large scene split across devices: this
 * call covers the 16-pixel tile rows r with r % n_shards == shard. grads
 * receives this shard's partial gradient (overwritten); loss_sums (B,) f64
 * receives this shard's sum of squared error (divide the all-reduced sum by
 * H*W*3 for the MSE). No reference counterpart: the reference has no
 * multi-device path; the sum over shards equals dr_loss_backward. */
DR_API dr_status dr_loss_backward_sharded(dr_ctx* ctx, const float* params, const float* background,
                                   int bg_per_scene, int B, int T, int H, int W, float sigma,
                                   const float* targets, int layout, int shard, int n_shards,
                                   float* grads, double* loss_sums, dr_stream_t stream);

/* One scene batch sharded by triangle blocks across devices (or run block by
 * block on one): the triangles are cut into n_blocks consecutive blocks of
 * ceil(T / n_blocks), and each caller owns block `block`. No reference
 * counterpart: the reference has no multi-device path.
 *
 * dr_triangle_block_forward composites the block over black for every pixel.
 * It writes the block's running product into slice `block` of `state`, a device
 * buffer of n_blocks * B * H * W * DR_TRIANGLE_BLOCK_STATE_BYTES bytes, block-major
 * (each slice contiguous, so ranks can all-gather their slices).
 *
 * dr_triangle_block_backward needs every slice of `state` and only reads it.
 * It combines the blocks' per-pixel maps into the final image (optional
 * `image`, layout as `other`) and the per-scene loss (`losses`, when
 * grad_input == 0). It then runs block `block`'s gradient pass: `grads`
 * (B, T, 10) is overwritten, nonzero only on the block's triangles. `other`
 * is the target (grad_input == 0, MSE as
 * dr_loss_backward) or the upstream image gradient (grad_input == 1, as
 * dr_grad_backward). The sum of `grads` over all blocks equals dr_loss_backward
 * to rounding. */
#define DR_TRIANGLE_BLOCK_STATE_BYTES 32
DR_API dr_status dr_triangle_block_forward(dr_ctx* ctx, const float* params,
                                           const float* background, int bg_per_scene, int B,
                                           int T, int H, int W, float sigma, int n_blocks,
                                           int block, float* state, dr_stream_t stream);
DR_API dr_status dr_triangle_block_backward(dr_ctx* ctx, const float* params,
                                            const float* background, int bg_per_scene, int B,
                                            int T, int H, int W, float sigma, int n_blocks,
                                            int block, const float* state, const float* other,
                                            int layout, int grad_input, float* grads,
                                            float* losses, float* image, dr_stream_t stream);

/* Per-image MSE of two (B, n) arrays with an f64 sum.
 * Replaces GpuRasterizer::encode_loss / loss_batch.wgsl (diffrast-gpu/src/lib.rs:1004-1031)
 * and Canvas::mse (crates/diffrast/src/canvas.rs:45-59). */
DR_API dr_status dr_mse_loss(dr_ctx* ctx, const float* images, const float* targets, int B,
                      int64_t n_per_image, float* losses, dr_stream_t stream);

/* One Adam step (optim.rs:40-60) over n params with the per-parameter rate
 * pattern of fit.rs:388-396 (index % 10: 0-5 lr_pos, 6-8 lr_color, 9 lr_alpha),
 * then fit.rs:399-424 `project` when project != 0. `step` is the 1-based step
 * count t used for bias correction (Adam::t after its increment). m and v are
 * the caller's moment buffers. Bit-identical to the reference's f32 arithmetic. */
DR_API dr_status dr_adam_step(dr_ctx* ctx, float* params, float* m, float* v, const float* grads,
                       int64_t n, float lr_pos, float lr_color, float lr_alpha, uint32_t step,
                       float beta1, float beta2, float eps, int project, dr_stream_t stream);

/* FitConfig (crates/diffrast/src/fit.rs:49-89) minus triangles/seed, which
 * come with the initial scene. patience < 0 means None. */
typedef struct dr_fit_config {
  int64_t iters;
  float sigma_start, sigma_end;
  float lr_pos, lr_color, lr_alpha;
  int64_t patience;
  float min_delta;
} dr_fit_config;

typedef enum dr_stop_reason {
  DR_STOP_COMPLETED = 0,
  DR_STOP_CONVERGED = 1,
  DR_STOP_DIVERGED = 2
} dr_stop_reason;

/* FitReport (fit.rs:128-140). */
typedef struct dr_fit_report {
  int64_t n_losses;
  int64_t best_iter;
  float best_loss;
  int stop_reason;
  int config_error; /* 0, or ConfigError 1..4 (fit.rs:27-32 order) */
} dr_fit_report;

/* The whole fit loop on the device (fit.rs:166-181, Fitter::step fit.rs:243-288):
 * per iteration sigma_at (fit.rs:343-349), fused forward+MSE+backward, the
 * Diverged / best / patience bookkeeping, Adam and projection, all without a
 * host round trip; synchronizes once at the end. target (H,W,3) and
 * init_params (T,10) are device memory; background is 3 host floats (the
 * seeded scene's background, fit.rs:357). best_params / final_params (T,10)
 * are device outputs; losses is a HOST array of at least iters floats.
 * An invalid config returns DR_INVALID_ARGUMENT with report->config_error set. */
DR_API dr_status dr_fit(dr_ctx* ctx, const float* target, int H, int W, const float* init_params,
                 const float* background, int T, const dr_fit_config* cfg, float* best_params,
                 float* final_params, float* losses, dr_fit_report* report, dr_stream_t stream);

/* dr_loss_backward with no device allocation: no context, no cudaMalloc, no
 * cudaFree. No counterpart in the reference. For callers that must not
 * allocate on their hot path: cudaMalloc synchronizes the device and can stall
 * for milliseconds (fatal to frame- or deadline-bound loops), and some hosts
 * hand out device memory only from their own fixed budget. Scratch comes from
 * one static array compiled into the library (about 3.3 MB on every GPU that
 * loads it, held until exit), so a call is limited to B*T <=
 * DR_NOALLOC_MAX_TRIANGLES, B <= DR_NOALLOC_MAX_BATCH and
 * B * ceil(H/16) * ceil(W/16) <= DR_NOALLOC_MAX_TILES (DR_TOO_LARGE beyond).
 * Runs on the current device and `stream`; background is 3 host floats (or
 * NULL for black), shared by the batch; precision is the default. The first
 * call on each device sets up the array's address: make it before any stream
 * capture. Later calls outside a capture look the address up again, so the
 * entry point stays valid after a device reset. All calls share the array, so
 * calls that could overlap on the GPU race: serialize them. Outputs as
 * dr_loss_backward (grads overwritten, losses may be NULL). */
#define DR_NOALLOC_MAX_TRIANGLES 16384
#define DR_NOALLOC_MAX_BATCH 1024
#define DR_NOALLOC_MAX_TILES 65536
DR_API dr_status dr_loss_backward_noalloc(const float* params, const float* background, int B,
                                          int T, int H, int W, float sigma, const float* targets,
                                          int layout, float* grads, float* losses,
                                          dr_stream_t stream);

/* --- the rest of GpuRasterizer's surface ---------------------------------- */

/* BackwardMode (diffrast-gpu/src/lib.rs:211-220): how the reference's
 * single-scene backward recovers the canvas beneath each triangle, from a
 * stored tape (Taped) or by re-walking the triangles (Recompute). This
 * library's backward keeps no tape and needs no O(T^2) re-walk (it takes the
 * attenuation from two prefix products), so both values run the same kernel and
 * give the same results; both are accepted so that callers keep working. */
typedef enum dr_backward_mode { DR_BACKWARD_TAPED = 0, DR_BACKWARD_RECOMPUTE = 1 } dr_backward_mode;

/* One scene's forward + MSE + backward with an explicit mode. Replaces
 * GpuRasterizer::backward / backward_with (diffrast-gpu/src/lib.rs:503-604).
 * params (T,10), target (H,W,3) or (3,H,W) per layout, grads (T,10), loss (1
 * float, may be NULL) and image (may be NULL) are device memory; background as
 * for dr_loss_backward (3 floats). Same results as dr_loss_backward with B = 1.
 * Any mode other than the two above is DR_INVALID_ARGUMENT. */
DR_API dr_status dr_backward(dr_ctx* ctx, const float* params, const float* background, int T,
                             int H, int W, float sigma, const float* target, int layout, int mode,
                             float* grads, float* loss, float* image, dr_stream_t stream);

/* ReduceMode (diffrast-gpu/src/lib.rs:76-84): how the batched backward sums
 * gradients, per contributing pixel (Direct) or per workgroup (Workgroup, the
 * reference's default). This library always reduces each warp's 32 pixels with
 * shuffles, each CTA's warps in shared memory, and issues one global atomic per
 * (triangle, parameter, CTA); both values select that reduction, so results do
 * not depend on the value. The setting is kept per context (default
 * DR_REDUCE_WORKGROUP) and read back by dr_get_reduce_mode. */
typedef enum dr_reduce_mode { DR_REDUCE_DIRECT = 0, DR_REDUCE_WORKGROUP = 1 } dr_reduce_mode;
DR_API dr_status dr_set_reduce_mode(dr_ctx* ctx, int mode);
DR_API dr_status dr_get_reduce_mode(dr_ctx* ctx, int* mode);

/* Deterministic gradients (default off): with on = 1, every gradient call on
 * this context (dr_loss_backward, dr_grad_backward, dr_backward,
 * dr_loss_backward_sharded, dr_loss_backward_host, dr_loss_backward_timed and
 * dr_fit) sums its per-warp contributions in 64-bit fixed point (2^-36
 * resolution) instead of float atomics, so repeated calls, and repeated fits,
 * give bit-identical gradients whatever the order the GPU adds them in. The
 * sums are converted to f32 once at the end. A warp total of magnitude 2^20 or
 * more, infinite or NaN makes that gradient NaN or an infinity (NaN when the
 * signs disagree), as the float sum would. Costs one extra kernel per call and
 * 10 KB more shared memory per CTA. dr_loss_backward_noalloc and the
 * triangle-block entry points keep float atomics. No reference counterpart
 * (the reference's sums are order-dependent too). */
DR_API dr_status dr_set_deterministic(dr_ctx* ctx, int on);
DR_API dr_status dr_get_deterministic(dr_ctx* ctx, int* on);

/* BackwardTimings (diffrast-gpu/src/lib.rs:96-114): where the time of one
 * host-buffer loss + backward call went, in milliseconds.
 *   pack_ms      uploads of params, backgrounds and targets, plus the set-up
 *                kernel that packs the triangle records (CUDA events)
 *   alloc_ms     growing the context's scratch pool (host clock; 0 when every
 *                buffer was a pool hit)
 *   dispatch_ms  the fused forward + MSE + backward kernel (CUDA events)
 *   readback_ms  downloads of gradients and losses (CUDA events)
 *   loss_ms      0: the per-image MSE is reduced inside the dispatch, where the
 *                reference reduced it on the host afterwards
 * total = the sum of the five. */
typedef struct dr_backward_timings {
  float pack_ms, alloc_ms, dispatch_ms, readback_ms, loss_ms;
} dr_backward_timings;

/* dr_loss_backward on HOST buffers (params (B,T,10), targets, grads (B,T,10),
 * losses (B,)), run phase by phase on `stream` with events between the phases,
 * filling *timings. Replaces GpuRasterizer::backward_many_timed
 * (diffrast-gpu/src/lib.rs:656-663, 676-816). Like the reference's timed form,
 * the phases do not overlap, so it is slower than dr_loss_backward_host; the
 * breakdown is a diagnostic. Returns after the results are in host memory, or
 * DR_TIMEOUT after 60 s (the reference's POLL_TIMEOUT); after a timeout the
 * host buffers stay in use until the device finishes (dr_ctx_destroy waits). */
DR_API dr_status dr_loss_backward_timed(dr_ctx* ctx, const float* params,
                                        const float* background, int bg_per_scene, int B, int T,
                                        int H, int W, float sigma, const float* targets,
                                        int layout, float* grads, float* losses,
                                        dr_backward_timings* timings, dr_stream_t stream);

/* GpuRasterizer::tape_bytes (diffrast-gpu/src/lib.rs:391-393): the bytes the
 * reference's taped mode stores for T triangles at width x height,
 * T * width * height * 3 * 4. This library stores no tape (DR_BACKWARD_TAPED
 * allocates none of it); the device scratch its calls do use is
 * dr_scratch_bytes. */
DR_API uint64_t dr_tape_bytes(uint64_t n_tris, uint64_t width, uint64_t height);

/* Device scratch a context holds for a loss or gradient call of B scenes of T
 * triangles at H x W (triangle records and their packed boxes, loss partials
 * and counters, and the triangle-split state when the call is too small to
 * fill the GPU). No reference counterpart. Returns 0 for invalid sizes. */
DR_API uint64_t dr_scratch_bytes(dr_ctx* ctx, int B, int T, int H, int W);

/* GpuRasterizer::is_discrete (diffrast-gpu/src/lib.rs:379-388): 1 for a
 * discrete GPU, 0 for one integrated with the host, -1 for no such device. */
DR_API int dr_is_discrete(int device);

/* --- device memory for bindings without a CUDA runtime -------------------- */

/* For callers that bind only this library (the Rust shim, ctypes): device
 * buffers on the context's device, and copies between any two of host and
 * device memory (the direction follows from the pointers, unified addressing).
 * dr_memcpy is ordered on `stream`; a copy into or out of pageable host memory
 * completes before it returns. No reference counterpart (wgpu owned all
 * buffers). */
DR_API dr_status dr_device_alloc(dr_ctx* ctx, size_t bytes, void** out);
DR_API dr_status dr_device_free(dr_ctx* ctx, void* ptr);
DR_API dr_status dr_memcpy(dr_ctx* ctx, void* dst, const void* src, size_t bytes,
                           dr_stream_t stream);

/* --- pool / sync ---------------------------------------------------------- */

/* PoolStats (diffrast-gpu/src/lib.rs:153-158): scratch reuse counters. */
typedef struct dr_pool_stats {
  uint64_t hits, misses, bytes;
} dr_pool_stats;

DR_API dr_status dr_pool_stats_get(dr_ctx* ctx, dr_pool_stats* out); /* lib.rs:346-349 */
DR_API dr_status dr_clear_pool(dr_ctx* ctx);                           /* lib.rs:352-356 */

/* Bounded wait for `stream`: polls and returns DR_TIMEOUT after timeout_s
 * seconds (GpuRasterizer::POLL_TIMEOUT, diffrast-gpu/src/lib.rs:223-229). */
DR_API dr_status dr_stream_wait(dr_stream_t stream, double timeout_s);

#ifdef __cplusplus
}
#endif

#endif /* DIFFRAST_CUDA_H */
