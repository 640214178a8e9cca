// Internal interface between the C ABI (dr_capi.cu) and the kernels
// (dr_kernels.cu). Not installed; callers use include/diffrast_cuda.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dr {

struct TriRec;

enum RasterMode { kModeRender = 0, kModeLoss = 1, kModeGrad = 2,
                  // Triangle-block split (launch_raster_split): per (tile, block) forward
                  // over black, then per (tile, block) the combine of every block's
                  // forward state and the block's gradient pass, for the loss or for an
                  // upstream image gradient.
                  kModeSplitFwd = 3, kModeSplitBwd = 4, kModeSplitBwdGrad = 5 };
enum Layout { kLayoutBHWC = 0, kLayoutBCHW = 1 };

struct FitState;

struct RasterArgs {
  const TriRec* recs;  // B*T records from the set-up kernel
  // Optional: the records' pixel boxes again, 16 bytes each, packed (empty
  // for triangles that cannot paint): the tile masks read these.
  const int4* boxes;
  int B, T, H, W;
  int tiles_x;
  int tile_row0, tile_row_step;  // tile rows covered: row0 + i * step
  int tile_rows;                 // number of covered tile rows (set by launch_raster)
  float sigma_eff;               // max(sigma, 1e-8) (raster.rs:75)
  float inv_sigma;               // 1 / sigma_eff
  int precision;                 // 0 reference rounding, 1 strict, 2 fast (band arithmetic)
  float bg3[3];                  // shared background when bg_dev is null
  const float* bg_dev;           // device background: 3 floats, or B*3 when bg_per_scene
  int bg_per_scene;
  int layout;                 // Layout of image / other
  float* image;               // optional rendered output
  const float* other;         // target (kModeLoss) or upstream gradient (kModeGrad)
  float grad_scale;           // 2/N as f32 (grad.rs:112)
  float* grads;               // (B,T,10), accumulated into (zeroed by the caller)
  double* loss_partials;      // B * tiles-in-launch scratch
  unsigned* loss_counters;    // B counters, zero between launches
  float* losses;              // optional (B,) mean squared error
  double* loss_sums;          // optional (B,) sum of squared error
  double n_values;            // H*W*3
  const int* skip_flag;       // optional: nonzero -> the kernel does nothing
  int split_k;                // triangle blocks of a split launch (else 0)
  int split_base;             // first block of this launch (grid z adds to it)
  float4* split_state;        // per (block, scene, pixel): 2 float4 of forward state
  // Deterministic gradient sums (dr_set_deterministic), else null: (B,T,10)
  // fixed-point sums and one non-finite flag word per (scene, triangle), both
  // zero on entry; launch_det_finalize turns them into `grads`.
  long long* grads_fx;
  int* grads_nf;
  // Pixel tape (dr_render_taped / dr_grad_backward_taped), else null: per pixel
  // of the batch the forward's running product (m, e, z0, zn), and per (scene,
  // region) a flag, nonzero where the tape cannot stand in for the forward.
  float4* tape;
  int* tape_flags;
  // dr_fit only (B = 1): the CTA that completes the loss also runs Fitter::step's
  // bookkeeping for iteration fit_iter (fit.rs:243-288).
  FitState* fit;
  float* fit_losses;
  long long fit_patience;     // < 0: none
  float fit_min_delta;
  int fit_iter;
  // Tile kernel launch order: nonzero -> tiles in rings around the canvas
  // centre, else central rows first (set per launch by the tile launcher).
  int tile_rings;
};

struct AdamArgs {
  float* params;
  float* m;
  float* v;
  const float* grads;
  long long n;
  float lr_pos, lr_color, lr_alpha;
  float beta1, beta2, one_minus_beta1, one_minus_beta2, eps;
  float bc1, bc2;  // 1 - beta^t in f32 (optim.rs:309-310)
  int project;     // fit.rs:399-424 after the update
  const int* skip_flag;  // optional: nonzero -> no-op
  const int* run_flag;   // optional: zero -> no update (copy still happens)
  const int* copy_flag;  // optional: nonzero -> copy_dst <- params first
  float* copy_dst;
};

struct FitState {
  float loss;       // written by the raster kernel each iteration
  float best_loss;
  int count;        // losses recorded
  int since;        // iterations since the last improvement
  int best_iter;
  int stopped;
  int stop_reason;  // 0 Completed, 1 Converged, 2 Diverged
  int run_adam;
  int copy_best;
  int pad[3];
};

size_t raster_smem_bytes();
// Sets the calling thread's dr_last_error() message.
void set_last_error(const char* msg);
cudaError_t launch_fit_init(FitState* st, cudaStream_t s);
// One fit iteration's Adam step (skipped unless the fit state says run) and
// the next iteration's set-up at next_sigma, one thread per triangle; also
// clears the gradients for the next raster launch. recs null: no set-up.
cudaError_t launch_fit_adam_setup(const AdamArgs& a, float* grads, int T, int W, int H,
                                  float next_sigma, TriRec* recs, cudaStream_t s);
size_t tri_rec_bytes();
// boxes (optional): each record's pixel box again, packed, for the tile masks.
cudaError_t launch_setup(const float* params, int BT, int W, int H, float sigma,
                         int tape_semantics, TriRec* recs, cudaStream_t s,
                         int4* boxes = nullptr);
cudaError_t launch_raster(int mode, const RasterArgs& a, int n_tiles, cudaStream_t s);
// Deterministic gradient sums: grads[i] from the fixed-point sum fx[i] and the
// non-finite flags nf[i / 10], n = B * T * 10 values; fx and nf are left zero
// for the next launch.
cudaError_t launch_det_finalize(long long* fx, int* nf, float* grads, long long n, cudaStream_t s);
// Regions per scene of the region kernel (the pixel tape's flags per scene).
long long tape_regions(int tiles_x, int tile_rows);
// Which kernel a launch over B scenes of tiles_x x tile_rows tiles takes:
// 0 the tile kernel, 1 the region kernel, 2 the triangle-block split (split_k > 1).
int raster_path(int B, int T, int tiles_x, int tile_rows, int split_k);
// Triangle blocks for a loss/grad launch over all tile rows of B scenes: 1 when
// the plain launch fills the GPU, else up to 8 (at least 32 triangles each).
int raster_split_blocks(int B, int T, int n_tiles);
// Bytes of split state a launch with k blocks needs (2 float4 per scene, block
// and pixel).
inline size_t raster_split_bytes(int B, int k, int H, int W) {
  return (size_t)B * k * H * W * 2 * sizeof(float4);
}
// kModeLoss / kModeGrad as two launches over k triangle blocks: forward per
// (tile, block) over black into the split state; then per (tile, block) the
// per-pixel combine of the blocks' affine maps (final colour, loss, canvas
// entering the block, attenuation from the blocks above) and the block's
// gradient pass. All tile rows (row0 0, step 1).
cudaError_t launch_raster_split(int mode, const RasterArgs& a, int n_tiles, int k, float4* split,
                                cudaStream_t s);
// One GPU's share of a scene batch sharded by triangle blocks: phase 0 runs
// block `block`'s forward over all pixels into its slice of `state`
// (n_blocks x B x H x W x 32 bytes); phase 1, with every slice present, runs
// the combine (final colour, loss) and the block's gradient pass.
cudaError_t launch_triangle_block(int phase, int mode, const RasterArgs& a, int n_tiles,
                                  int n_blocks, int block, float4* state, cudaStream_t s);
// Per-image MSE scratch: B * mse_partials_per_image(n) doubles and B counters
// (zero between launches; the kernel leaves them zero).
size_t mse_partials_per_image(long long n);
cudaError_t launch_mse(const float* img, const float* tgt, int B, long long n, float* losses,
                       double* partials, unsigned* counters, cudaStream_t s);
cudaError_t launch_adam(const AdamArgs& a, cudaStream_t s);

}  // namespace dr
