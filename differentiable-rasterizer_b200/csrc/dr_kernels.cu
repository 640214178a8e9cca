// sm_100a kernels for the soft-triangle rasterizer hot path.
//
//   dr_setup_kernel    one thread per (scene, triangle): TriRec (box cull,
//                      edge data, clamped alpha, fast-path line equations)
//   dr_raster_kernel   one CTA per (scene, 16x16 tile): order-preserving
//                      per-tile triangle lists staged in shared memory, then
//                      forward compositing, MSE, and the analytic backward
//   dr_mse_kernel      per-image MSE with an f64 sum (canvas.rs:45-59)
//   dr_adam_kernel     Adam::step + project, elementwise (optim.rs, fit.rs)
//
// The backward runs in *forward* triangle order. The reference walks the
// triangles front to back with g <- g * (1 - w) and needs the canvas beneath
// each triangle (grad.rs:13-19, 124-128); un-compositing by dividing by
// (1 - w) is unstable, and a per-pixel tape is large. Here the scalar
// attenuation reaching layer k, A_k = prod_{j>k} (1 - w_j), is obtained as
// the ratio of two prefix products P_L / P_k computed in two passes, with the
// products renormalised by 2^64 to stay in range and exact zeros / NaNs of
// (1 - w) treated as barriers (everything beneath an opaque layer gets exactly
// zero, beneath a NaN layer NaN, as the reference's running product does).
// Every per-layer gradient term is then available in the same pass that
// recomposites the canvas, so no tape and no O(T^2) re-walk is needed.

#include <atomic>
#include <cstdint>
#include <cstdio>

#include "dr_device.cuh"
#include "dr_math.cuh"
#include "dr_internal.h"

namespace dr {

constexpr int kTile = 16;
constexpr int kBlockW = 8, kBlockH = 4;                  // one warp's pixel block, a pixel per lane
constexpr int kWarps = (kTile / kBlockW) * (kTile / kBlockH);
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 128;                              // triangles binned per round (<= kThreads)
constexpr int kBlocksPerTile = kWarps;                    // 2 columns x 4 rows of warp blocks
constexpr int kRegionCols = 2;                           // region kernel: 2 tiles wide
static_assert(kBlocksPerTile == 8, "tile block codes are stored as one 64-bit word");
constexpr float kRenorm = 18446744073709551616.0f;        // 2^64
constexpr float kRenormInv = 5.42101086242752217e-20f;    // 2^-64

// ---------------------------------------------------------------------------
// Set-up
// ---------------------------------------------------------------------------

// Rust `f as usize` on a value already clamped to >= 0, saturating, then
// compared against the canvas size: only min(value, n) matters except for the
// `+ 1` wrap at usize::MAX.
__device__ __forceinline__ long long box_lo(float f, int n) {
  if (!(f > 0.0f)) return 0;
  if (f >= (float)n) return n;
  return (long long)f;
}
__device__ __forceinline__ long long box_hi(float f, int n) {
  if (!(f > 0.0f)) return 1 < n ? 1 : n;
  if (f >= 18446744073709551616.0f) return 0;  // usize::MAX + 1 wraps to 0
  if (f >= (float)n) return n;
  long long v = (long long)f + 1;
  return v < n ? v : n;
}

// The record of triangle i (one scene-major index over the batch).
__device__ __forceinline__ TriRec make_record(const float* __restrict__ params, int i, int W, int H,
                                              float sigma, int tape_semantics) {
  const float* p = params + (size_t)i * kParams;
  float v[6];
#pragma unroll
  for (int j = 0; j < 6; ++j) v[j] = p[j];
  float col[3] = {p[6], p[7], p[8]};
  float raw_alpha = p[9];

  TriRec r;
  for (int k = 0; k < 3; ++k) {
    r.ed[k].ax = v[2 * k];
    r.ed[k].ay = v[2 * k + 1];
  }
  for (int j = 0; j < 3; ++j) r.color[j] = col[j];
  float alpha = rclamp(raw_alpha, 0.0f, 1.0f);
  r.alpha = alpha;
  int flags = 0;
  if (raw_alpha > 0.0f && raw_alpha < 1.0f) flags |= kAlphaActive;

  // pixel_bounds (raster.rs:144-168), f32 exactly as written there.
  bool finite = true;
  float lo_x = __int_as_float(0x7f800000), lo_y = lo_x;
  float hi_x = -lo_x, hi_y = -lo_x;
  for (int k = 0; k < 3; ++k) {
    float x = v[2 * k], y = v[2 * k + 1];
    if (!isfinite(x) || !isfinite(y)) finite = false;
    lo_x = fminf(lo_x, x);
    hi_x = fmaxf(hi_x, x);
    lo_y = fminf(lo_y, y);
    hi_y = fmaxf(hi_y, y);
  }
  float pad = __fmul_rn(6.0f, sigma);
  long long bx0 = box_lo(fmaxf(floorf(__fmul_rn(__fsub_rn(lo_x, pad), (float)W)), 0.0f), W);
  long long by0 = box_lo(fmaxf(floorf(__fmul_rn(__fsub_rn(lo_y, pad), (float)H)), 0.0f), H);
  long long bx1 = box_hi(fmaxf(ceilf(__fmul_rn(__fadd_rn(hi_x, pad), (float)W)), 0.0f), W);
  long long by1 = box_hi(fmaxf(ceilf(__fmul_rn(__fadd_rn(hi_y, pad), (float)H)), 0.0f), H);
  bool has_box = finite && bx0 < bx1 && by0 < by1;
  r.bbox[0] = (int)bx0;
  r.bbox[1] = (int)by0;
  r.bbox[2] = (int)bx1;
  r.bbox[3] = (int)by1;

  // render() skips only `alpha <= 0` (raster.rs:49), so a NaN alpha paints
  // NaN; render_with_tape() keeps only `alpha > 0` (grad.rs:62), so the tape
  // path (every backward) drops a NaN-alpha triangle entirely.
  bool alpha_ok = tape_semantics ? (alpha > 0.0f) : !(alpha <= 0.0f);
  // w = alpha * cov <= alpha: an alpha at or below MIN_WEIGHT never paints.
  if (alpha <= kMinWeight) alpha_ok = false;
  if (has_box && alpha_ok) flags |= kLive;
  if (!(flags & kLive)) r.bbox[0] = r.bbox[1] = r.bbox[2] = r.bbox[3] = 0;  // meets no tile

  // Edge vectors and squared lengths with the reference's rounding.
  for (int k = 0; k < 3; ++k) {
    int a = k, b = (k + 1) % 3;
    float ex = __fsub_rn(v[2 * b], v[2 * a]);
    float ey = __fsub_rn(v[2 * b + 1], v[2 * a + 1]);
    r.ed[k].ex = ex;
    r.ed[k].ey = ey;
    r.len2[k] = __fadd_rn(__fmul_rn(ex, ex), __fmul_rn(ey, ey));
  }

  // Edge-line equations for the conservative fast paths, in double. Valid
  // only for a clearly non-degenerate triangle with a finite alpha.
  double ex0 = (double)v[2] - v[0], ey0 = (double)v[3] - v[1];
  double ex2 = (double)v[4] - v[0], ey2 = (double)v[5] - v[1];
  double area2 = ex0 * ey2 - ey0 * ex2;
  double maxl2 = 0.0, maxabs = 0.0;
  for (int k = 0; k < 3; ++k) {
    double l2 = (double)r.ed[k].ex * r.ed[k].ex + (double)r.ed[k].ey * r.ed[k].ey;
    maxl2 = fmax(maxl2, l2);
    maxabs = fmax(maxabs, fmax(fabs((double)v[2 * k]), fabs((double)v[2 * k + 1])));
  }
  bool fast = has_box && isfinite(alpha) && fabs(area2) > 1e-6 * maxl2 && maxl2 > 1e-14;
  double s = area2 >= 0.0 ? 1.0 : -1.0;
  for (int k = 0; k < 3; ++k) {
    int a = k, b = (k + 1) % 3;
    double ex = (double)v[2 * b] - v[2 * a], ey = (double)v[2 * b + 1] - v[2 * a + 1];
    double len = sqrt(ex * ex + ey * ey);
    if (!(len > 0.0)) {
      fast = false;
      len = 1.0;
    }
    double nx = s * -ey / len, ny = s * ex / len;
    r.ed[k].nx = (float)nx;
    r.ed[k].ny = (float)ny;
    r.ed[k].c = (float)(-(nx * v[2 * a] + ny * v[2 * a + 1]));
  }
  // Slack for evaluating n.p + c in f32 and for the reference's own f32
  // distance rounding: a few ulps of the largest magnitude involved.
  r.margin = (float)(4e-6 * (2.0 + maxabs));
  // Pixels more than rej outside an edge line have w = alpha * cov below
  // MIN_WEIGHT (cov <= exp(-dist/sigma) and alpha e^{-x} <= 1e-6 for
  // x >= ln(alpha * 1e6); 0.2 of slack); pixels more than acc inside every
  // edge line have exp(-x) below half an ulp of 1 (x > 16.64), so the
  // reference's sigmoid rounds to exactly 1. Both include the margin.
  const double sig_eff = fmax((double)sigma, 1e-8);
  const double lna = alpha > 0.0f ? log((double)alpha * 1e6) : 0.0;
  r.rej = (float)((fmax(lna, 0.0) + 0.2) * sig_eff) + r.margin;
  r.acc = (float)(16.8 * sig_eff) + r.margin;
  for (int k = 0; k < 3; ++k) r.ed[k].il = r.len2[k] <= 1e-20f ? 0.0f : (float)(1.0 / (double)r.len2[k]);
  r.wind = (float)s;
  if (fast) flags |= kFastOk;
  r.flags = flags;
  return r;
}

// One thread per (scene, triangle). Records are staged in shared memory and
// written as one contiguous run per block: a thread writing its own 160-byte
// record would leave every 16-byte store to a different, partly written sector.
constexpr int kSetupThreads = 128;
__global__ void __launch_bounds__(kSetupThreads) dr_setup_kernel(
    const float* __restrict__ params, int BT, int W, int H, float sigma, int tape_semantics,
    TriRec* __restrict__ recs, int4* __restrict__ boxes) {
  constexpr int kQ = kRecWords / 4;  // float4s per record
  __shared__ float4 stage[kSetupThreads * kQ];
  const int first = blockIdx.x * kSetupThreads;
  const int i = first + (int)threadIdx.x;
  if (i < BT) {
    const TriRec r = make_record(params, i, W, H, sigma, tape_semantics);
    if (boxes) boxes[i] = make_int4(r.bbox[0], r.bbox[1], r.bbox[2], r.bbox[3]);
    const float4* src = reinterpret_cast<const float4*>(&r);
#pragma unroll
    for (int j = 0; j < kQ; ++j) stage[threadIdx.x * kQ + j] = src[j];
  }
  __syncthreads();
  const int n_here = min(kSetupThreads, BT - first);
  float4* dst = reinterpret_cast<float4*>(recs + first);
  for (int k = threadIdx.x; k < n_here * kQ; k += kSetupThreads) dst[k] = stage[k];
}

// ---------------------------------------------------------------------------
// Raster kernel
// ---------------------------------------------------------------------------
//
// A warp owns an 8x4 block of pixels, one pixel per lane. Two kernels share
// the list walks (forward_walk, gradient_walk):
//   tile kernel    one CTA per (scene, 16x16 tile[, triangle block]), 8 warps,
//                  warp w on block w; long lists binned in chunks
//   region kernel  one CTA per (scene, 2x1 tiles) for lists within one chunk;
//                  warps take the region's 16 blocks from a shared counter
// Triangles are binned in order (build_list, build_region_list) and every
// kept entry carries a one-byte code per warp block, decided once at binning
// time from the block's rectangle against the triangle's box and edge lines:
//   kBlkSkip    no pixel of the block can contribute (outside the box, or
//               every pixel more than the triangle's `rej` outside an edge)
//   kBlkBox     the block straddles the box: test each pixel against it
//   kBlkInside  every pixel is more than the triangle's `acc` inside every edge:
//               w == alpha exactly, no geometry
// so whole warps skip or take the cheap path on a uniform branch. Bits 3-5
// of the code mark the edges that can be the nearest edge of a contributing
// pixel of the block (the candidates): an edge whose line stays farther than
// max(rej, acc) from every pixel of the block is farther than that from the
// pixel as a segment too, while a contributing pixel's nearest edge is within
// rej (outside) or acc (inside, where nearest segment = nearest line). Most
// soft-edge blocks have a single candidate, which fixes the nearest edge for
// the whole warp.

constexpr int kBlkSkip = 1, kBlkBox = 2, kBlkInside = 4, kCandShift = 3;
struct Smem {
  TriRec rec[kChunk];
  unsigned char bcode[kChunk][kBlocksPerTile];
  int kidx[kChunk];
  // The image stores of pass 1 and the gradient sums of pass 2 never overlap
  // in time, so they share the space.
  union {
    float acc[kChunk][kParams];
    long long acc64[kChunk][kParams];  // the same sums in fixed point (deterministic mode)
    float4 stage[kWarps][24];          // one warp block's 96 image values (store_block)
  };
  int nf[kChunk];  // deterministic mode: non-finite flags of the list's sums
  int warp_count[kWarps];
  double loss_part[kWarps];
  int is_last;
  // Lists gathered from the tile's mask (scenes of more than kChunk
  // triangles): the mask, one word per 32 triangles, the indices of the next
  // list, and the gather's per-warp totals and position.
  unsigned mask[kThreads];
  int cand[kChunk];
  int wsum[kWarps];
  int mtotal[kWarps];
  int gcount, gwc, gbo;
};

// Region kernel (a list of at most kChunk triangles): one CTA per region of
// 2 x kRows tiles (kRB = 16 kRows warp blocks), one code per warp block of the
// region, warps taking blocks from a shared counter.
template <int kRB>
struct RegionSmem {
  TriRec rec[kChunk];
  unsigned char bcode[kChunk][kRB];
  int kidx[kChunk];
  union {
    float acc[kChunk][kParams];
    long long acc64[kChunk][kParams];  // the same sums in fixed point (deterministic mode)
  };
  int nf[kChunk];  // deterministic mode: non-finite flags of the list's sums
  float4 stage[kWarps][24];  // one warp block's 96 image values (store_block)
  int warp_count[kWarps];
  double loss_part[kRB];
  int next_block;
  int is_last;
};

// Block code of one warp block [bx0,bx1) x [by0,by1) (clipped to the image)
// for one triangle record.
__device__ __forceinline__ int classify_block(const TriRec& r, int bx0, int by0, int bx1, int by1,
                                              int W, int H) {
  if (bx0 >= bx1 || by0 >= by1) return kBlkSkip;
  const int x0 = r.bbox[0], y0 = r.bbox[1], x1 = r.bbox[2], y1 = r.bbox[3];
  if (bx1 <= x0 || bx0 >= x1 || by1 <= y0 || by0 >= y1) return kBlkSkip;
  int code = (x0 <= bx0 && x1 >= bx1 && y0 <= by0 && y1 >= by1) ? 0 : kBlkBox;
  if (r.flags & kFastOk) {
    // Pixel centres of the block span [c - h, c + h] per axis; a linear
    // function's extremes over the rectangle are at l(c) +- (|nx| hx + |ny| hy).
    const float inv_w = 1.0f / (float)W, inv_h = 1.0f / (float)H;
    const float cx = 0.5f * (float)(bx0 + bx1) * inv_w, hx = 0.5f * (float)(bx1 - bx0 - 1) * inv_w;
    const float cy = 0.5f * (float)(by0 + by1) * inv_h, hy = 0.5f * (float)(by1 - by0 - 1) * inv_h;
    const float thr = fmaxf(r.rej, r.acc) + r.margin;
    float lmin_all = __int_as_float(0x7f800000);
    int cand = 0;
#pragma unroll
    for (int e = 0; e < 3; ++e) {
      const float nx = r.ed[e].nx, ny = r.ed[e].ny;
      const float lc = __fmaf_rn(nx, cx, __fmaf_rn(ny, cy, r.ed[e].c));
      const float rad = __fmaf_rn(fabsf(nx), hx, __fmul_rn(fabsf(ny), hy));
      if (__fadd_rn(lc, rad) < -r.rej) return kBlkSkip;
      lmin_all = fminf(lmin_all, __fsub_rn(lc, rad));
      if (!(__fsub_rn(fabsf(lc), rad) > thr)) cand |= 1 << e;
    }
    if (lmin_all > r.acc) return kBlkInside;  // deep inside implies inside the box
    if ((cand & (cand - 1)) && lmin_all > r.margin) {
      // Two or three candidates, every pixel inside every edge line. There the
      // nearest segment is the nearest line (the largest disk around the
      // pixel inside the triangle touches its nearest line within the
      // segment), so an edge whose line lies farther from every pixel than
      // some other edge's line lies from any pixel is never the nearest, not
      // even within rounding: drop it (its cross product has the winding's
      // sign, as for any non-candidate). Near one edge and deep from the
      // others, the block becomes single-edge.
      float lmin[3], umin = __int_as_float(0x7f800000);
#pragma unroll
      for (int e = 0; e < 3; ++e) {
        const float nx = r.ed[e].nx, ny = r.ed[e].ny;
        const float lc = __fmaf_rn(nx, cx, __fmaf_rn(ny, cy, r.ed[e].c));
        const float rad = __fmaf_rn(fabsf(nx), hx, __fmul_rn(fabsf(ny), hy));
        lmin[e] = __fsub_rn(lc, rad);
        umin = fminf(umin, __fadd_rn(lc, rad));
      }
      const float lim = __fadd_rn(umin, __fmul_rn(2.0f, r.margin));
#pragma unroll
      for (int e = 0; e < 3; ++e)
        if (lmin[e] > lim) cand &= ~(1 << e);
    }
    code |= cand << kCandShift;
  } else {
    code |= 7 << kCandShift;
  }
  return code;
}

// Bin one list of at most kChunk triangles against the tile, in order: thread
// i < kChunk offers triangle k (valid false: none); the kept ones land in
// shared memory in thread order with their eight block codes.
__device__ int bin_list(Smem& sm, const TriRec* __restrict__ recs, int k, bool valid, int tx0,
                        int ty0, int W, int H) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  bool keep = false;
  unsigned long long code_all = 0;
  const TriRec* r = recs + k;
  if (valid && (r->flags & kLive)) {
    const TriRec& rr = *r;
    int skipped = 0;
#pragma unroll
    for (int wb = 0; wb < kWarps; ++wb) {
      const int bx0 = tx0 + (wb & 1) * kBlockW, by0 = ty0 + (wb >> 1) * kBlockH;
      const int c = classify_block(rr, bx0, by0, min(bx0 + kBlockW, W), min(by0 + kBlockH, H), W,
                                   H);
      code_all |= (unsigned long long)c << (8 * wb);
      skipped += (c & kBlkSkip) ? 1 : 0;
    }
    keep = skipped < kWarps;
  }
  const unsigned ballot = __ballot_sync(0xffffffffu, keep);
  if (lane == 0) sm.warp_count[warp] = __popc(ballot);
  __syncthreads();
  int base = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int cnt = sm.warp_count[w];
    base += (w < warp) ? cnt : 0;
    total += cnt;
  }
  if (keep) {
    const int slot = base + __popc(ballot & ((1u << lane) - 1u));
    sm.kidx[slot] = k;
    *reinterpret_cast<unsigned long long*>(sm.bcode[slot]) = code_all;
    const float4* src = reinterpret_cast<const float4*>(r);
    float4* dst = reinterpret_cast<float4*>(&sm.rec[slot]);
#pragma unroll
    for (int j = 0; j < kRecWords / 4; ++j) dst[j] = src[j];
  }
  __syncthreads();
  return total;
}

// Bin triangles [c0, c0 + kChunk) of one scene against the tile, in order.
__device__ __forceinline__ int build_list(Smem& sm, const TriRec* __restrict__ recs, int T,
                                          int c0, int tx0, int ty0, int W, int H) {
  const int k = c0 + (int)threadIdx.x;
  return bin_list(sm, recs, k, (int)threadIdx.x < kChunk && k < T, tx0, ty0, W, H);
}

// Tile masks. A scene with more than kChunk triangles would otherwise be
// binned in fixed windows of kChunk triangles, every window tested against
// the tile even when none of its triangles comes near it (most of them, on a
// large canvas). Instead the CTA first marks, 32 triangles to a word, which
// live triangles' pixel boxes meet its tile, then gathers its lists from the
// marked triangles only, kChunk at a time and in triangle order, so the
// composite runs over the same sequence as the fixed windows would give.
// The gather's position (uniform over the CTA) lives in shared memory, not in
// registers that would stay live across the list walks: gwc and gbo are the
// next mask word to gather from and its first unused bit.
struct Range {
  int t0, t1;    // triangles [t0, t1) of the scene, at most kGatherMaxT
  int tx0, ty0;  // the tile's first pixel
  const int4* boxes;  // the scene's packed pixel boxes, or null: the records' own
  __device__ int words() const { return (t1 - t0 + 31) / 32; }
};

// The mask is one word per thread, held whole in shared memory.
constexpr int kGatherMaxT = 32 * kThreads;

// The tile's mask: bit l of word j is set when triangle t0 + 32 j + l is
// live and its pixel box meets the tile (a triangle that is not live has an
// empty box). Warp w fills words w, w + kWarps, ..., one ballot per word, four
// words' 16-byte box loads in flight at a time, and leaves its words' bit count
// in sm.mtotal[w].
__device__ void tile_mask(Smem& sm, const TriRec* __restrict__ recs, const Range& rg, int W,
                          int H) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tx1 = min(rg.tx0 + kTile, W), ty1 = min(rg.ty0 + kTile, H);
  const int end = rg.words();
  int bits = 0;
  for (int j0 = warp; j0 < end; j0 += 4 * kWarps) {
    bool hit[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u * kWarps;
      const int k = rg.t0 + 32 * j + lane;
      hit[u] = false;
      if (j < end && k < rg.t1) {
        const int4 bb = rg.boxes ? rg.boxes[k] : *reinterpret_cast<const int4*>(recs[k].bbox);
        hit[u] = bb.x < tx1 && bb.z > rg.tx0 && bb.y < ty1 && bb.w > rg.ty0;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u * kWarps;
      const unsigned m = __ballot_sync(0xffffffffu, hit[u]);
      if (lane == 0 && j < end) sm.mask[j] = m;
      bits += __popc(m);
    }
  }
  if (lane == 0) sm.mtotal[warp] = bits;
}

// Mark the tile's triangles and set the gather to the first; returns the
// number marked. The caller orders this after every earlier read of the
// gather state.
__device__ __forceinline__ int gather_start(Smem& sm, const TriRec* __restrict__ recs,
                                            const Range& rg, int W, int H) {
  if (threadIdx.x == 0) {
    sm.gwc = 0;
    sm.gbo = 0;
  }
  tile_mask(sm, recs, rg, W, H);
  __syncthreads();
  int total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total += sm.mtotal[w];
  return total;
}

// The next kChunk marked triangles (fewer for the last list), in order, binned
// into shared memory like a window of build_list. Every thread holds one mask
// word: a block-wide prefix sum of the words' bit counts gives each word's
// first slot. Lists are cut at bit granularity, so ceil(marked / kChunk)
// calls take every marked triangle. The caller orders this call after the
// previous one's reads with a barrier.
__device__ int gather_list(Smem& sm, const TriRec* __restrict__ recs, const Range& rg, int W,
                           int H) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = rg.words();
  const int wc = sm.gwc, bo = sm.gbo;
  const int j = wc + (int)threadIdx.x;
  const bool valid = j < nw;
  unsigned m = valid ? sm.mask[j] : 0u;
  if (threadIdx.x == 0) m &= ~0u << bo;  // bits of the first word already used
  const int c = __popc(m);
  int incl = c;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) sm.wsum[warp] = incl;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kWarps; ++w) incl += (w < warp) ? sm.wsum[w] : 0;
  const int excl = incl - c;
  if (valid && excl < kChunk) {
    // This word starts inside the list. The list's last word is the one that
    // fills it or the mask's last word; a word that overfills it gives only
    // its first bits, and the next list resumes after them.
    int slot = excl;
    const int kbase = rg.t0 + 32 * j;
    unsigned mm = m;
    for (; mm && slot < kChunk; mm &= mm - 1) sm.cand[slot++] = kbase + __ffs(mm) - 1;
    if (incl >= kChunk || j + 1 >= nw) {
      sm.gcount = slot;
      sm.gwc = mm ? j : j + 1;
      sm.gbo = mm ? __ffs(mm) - 1 : 0;
    }
  }
  __syncthreads();
  const int n = sm.gcount;
  const int i = (int)threadIdx.x;
  return bin_list(sm, recs, i < n ? sm.cand[i] : 0, i < n, rg.tx0, rg.ty0, W, H);
}

// Pixel origin of warp block `blk` of a region: tiles of 8 blocks in the
// order left-top, right-top[, left-bottom, right-bottom]; each tile's blocks
// as the tile kernel's warps (2 columns x 4 rows). A block on a tile row the
// launch does not cover gets y0 = H: empty.
__device__ __forceinline__ void region_block_origin(const RasterArgs& a, int rx0, int lrow0,
                                                    int blk, int& x0, int& y0) {
  const int t = blk >> 3, wb = blk & 7;
  x0 = rx0 + (t & 1) * kTile + (wb & 1) * kBlockW;
  const int lr = lrow0 + (t >> 1);
  y0 = lr < a.tile_rows ? (a.tile_row0 + lr * a.tile_row_step) * kTile + (wb >> 1) * kBlockH
                        : a.H;
}

// The region's whole list (a.T <= kChunk), in order: two threads per
// triangle, each classifying half of the kRB blocks. Also clears the gradient
// accumulators.
template <int kRB>
__device__ int build_region_list(RegionSmem<kRB>& sm, const RasterArgs& a,
                                 const TriRec* __restrict__ recs, int rx0, int lrow0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = threadIdx.x & 1;
  const int k = (int)threadIdx.x >> 1;
  constexpr int kPer = kRB / 2;
  static_assert((kPer == 8 || kPer == 16) && kThreads / 2 == kChunk,
                "two threads per triangle, 8 or 16 blocks each");
  bool keep_half = false;
  unsigned long long lo = 0x0101010101010101ull, hi = lo;  // all kBlkSkip
  const TriRec* r = recs + k;
  if (k < a.T && (r->flags & kLive)) {
    lo = hi = 0;
#pragma unroll 1
    for (int i = 0; i < kPer; ++i) {
      int x0, y0;
      region_block_origin(a, rx0, lrow0, half * kPer + i, x0, y0);
      const int c =
          classify_block(*r, x0, y0, min(x0 + kBlockW, a.W), min(y0 + kBlockH, a.H), a.W, a.H);
      keep_half |= !(c & kBlkSkip);
      if (i < 8) lo |= (unsigned long long)c << (8 * i);
      else hi |= (unsigned long long)c << (8 * (i - 8));
    }
  }
  // Every lane must take part in the shuffle: it may not sit behind `||`.
  const bool partner_keeps = __shfl_xor_sync(0xffffffffu, keep_half, 1);
  const bool keep = keep_half || partner_keeps;
  const unsigned ballot = __ballot_sync(0xffffffffu, keep && !half);  // one bit per triangle
  if (lane == 0) sm.warp_count[warp] = __popc(ballot);
  if (a.grads_fx) {
    for (int i = threadIdx.x; i < kChunk * kParams; i += kThreads) (&sm.acc64[0][0])[i] = 0;
    for (int i = threadIdx.x; i < kChunk; i += kThreads) sm.nf[i] = 0;
  } else {
    for (int i = threadIdx.x; i < kChunk * kParams; i += kThreads) (&sm.acc[0][0])[i] = 0.0f;
  }
  __syncthreads();
  int base = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int cnt = sm.warp_count[w];
    base += (w < warp) ? cnt : 0;
    total += cnt;
  }
  if (keep) {
    const int slot = base + __popc(ballot & ((1u << (lane & ~1)) - 1u));
    unsigned long long* dst_code = reinterpret_cast<unsigned long long*>(&sm.bcode[slot][half * kPer]);
    dst_code[0] = lo;
    if (kPer == 16) dst_code[1] = hi;
    if (!half) {
      sm.kidx[slot] = k;
      const float4* src = reinterpret_cast<const float4*>(r);
      float4* dst = reinterpret_cast<float4*>(&sm.rec[slot]);
#pragma unroll
      for (int j = 0; j < kRecWords / 4; ++j) dst[j] = src[j];
    }
  }
  __syncthreads();
  return total;
}

struct Consts {
  float sigma_eff, inv_sigma;
  bool det;  // deterministic gradient sums (fixed point)
};

// Precision modes of the soft-edge (band) arithmetic.
//   kPrecRef     default: cheap classification and nearest-edge choice, then
//                the nearest edge's distance, the sigmoid, and the gradient
//                direction with the reference's f32 operations and rounding
//                (raster.rs:124-134, grad.rs:231-270). Near an edge those f32
//                values carry cancellation error of ~1e-7 / dist, which the
//                reference's outputs contain and which this mode reproduces.
//   kPrecStrict  every edge with the reference's exact arithmetic.
//   kPrecFast    exact-math shortcuts (distance = nearest edge line inside,
//                gradient direction = the edge normal) with MUFU reciprocals:
//                closer to the true (f64) gradient, not to the f32 reference.
enum Prec : int { kPrecRef = 0, kPrecStrict = 1, kPrecFast = 2 };

// What one (pixel, triangle) pair contributes. `band` is false when the
// vertex gradient is exactly zero (cov == 1, or dist < 1e-9 as
// grad.rs:252-254). With kGrad, a band pair also carries d(cov)/d(vertex) for
// the two vertices of its nearest edge: (dax, day) for vertex `edge`,
// (dbx, dby) for vertex `edge + 1` (grad.rs:264-268).
struct PairEval {
  float w, cov;
  bool band, hit;
  float dax, day, dbx, dby;
  int edge;
};

// d(cov)/d(vertices) for the nearest edge with the reference's rounding:
// cp = a + t (b - a); u = (pt - cp) / dist; chain = cov (1 - cov) / sigma * sign;
// d[a] = chain * -(1 - t) * u, d[b] = chain * -t * u (grad.rs:256-268).
__device__ __forceinline__ void cov_grad_ref(const TriRec& r, int edge, float t, float dist,
                                             float cov, bool inside, float ptx, float pty,
                                             const Consts& K, PairEval& o) {
  const float ax = r.ed[edge].ax, ay = r.ed[edge].ay;
  const float cpx = __fadd_rn(ax, __fmul_rn(t, r.ed[edge].ex));
  const float cpy = __fadd_rn(ay, __fmul_rn(t, r.ed[edge].ey));
  const float rd = rcp_approx(dist);
  const float ux = div_rn_inv(__fsub_rn(ptx, cpx), dist, rd);
  const float uy = div_rn_inv(__fsub_rn(pty, cpy), dist, rd);
  float chain = div_rn_inv(__fmul_rn(cov, __fsub_rn(1.0f, cov)), K.sigma_eff, K.inv_sigma);
  chain = inside ? chain : -chain;
  const float ka = __fmul_rn(chain, -__fsub_rn(1.0f, t));
  const float kb = __fmul_rn(chain, -t);
  o.dax = __fmul_rn(ka, ux);
  o.day = __fmul_rn(ka, uy);
  o.dbx = __fmul_rn(kb, ux);
  o.dby = __fmul_rn(kb, uy);
  o.edge = edge;
}

// Exact reference arithmetic for one pair (degenerate triangles, NaN alpha,
// near-tie pixels, and every band pair in strict mode): raster.rs:96-106 +
// grad.rs:231-270. Kept out of line: it is rare on the default path, and
// inlining its IEEE divisions at every call site overflows the instruction
// cache of the hot loop.
template <bool kGrad>
__device__ __noinline__ PairEval eval_ref(const TriRec* rp, float ptx, float pty,
                                          float sigma_eff) {
  // Arguments and result by value: a reference to the caller's locals would
  // force them (and every access in the hot loop) into local memory.
  const TriRec& r = *rp;
  PairEval o;
  o.edge = 0;
  o.dax = o.day = o.dbx = o.dby = 0.0f;
  const SdResult g = signed_distance_ref(r.ed, r.len2, ptx, pty);
  o.cov = sigmoid_ref(__fdiv_rn(g.sd, sigma_eff));
  o.w = __fmul_rn(r.alpha, o.cov);
  o.band = !(g.dist < 1e-9f);
  if (kGrad && o.band) {
    const float ax = r.ed[g.edge].ax, ay = r.ed[g.edge].ay;
    const float cpx = __fadd_rn(ax, __fmul_rn(g.t, r.ed[g.edge].ex));
    const float cpy = __fadd_rn(ay, __fmul_rn(g.t, r.ed[g.edge].ey));
    const float ux = __fdiv_rn(__fsub_rn(ptx, cpx), g.dist);
    const float uy = __fdiv_rn(__fsub_rn(pty, cpy), g.dist);
    float chain = __fdiv_rn(__fmul_rn(o.cov, __fsub_rn(1.0f, o.cov)), sigma_eff);
    chain = (g.sd > 0.0f) ? chain : -chain;
    const float ka = __fmul_rn(chain, -__fsub_rn(1.0f, g.t));
    const float kb = __fmul_rn(chain, -g.t);
    o.dax = __fmul_rn(ka, ux);
    o.day = __fmul_rn(ka, uy);
    o.dbx = __fmul_rn(kb, ux);
    o.dby = __fmul_rn(kb, uy);
    o.edge = g.edge;
  }
  o.hit = !(o.w <= kMinWeight);
  return o;
}

// One pair, given the warp block's code. Returns kSkip (no contribution),
// kHit (composites: w > MIN_WEIGHT, `o` filled) or kExact (the caller must
// evaluate it with eval_ref). The arithmetic that decides w uses explicit
// rounding only, so the forward pass and the gradient pass (two
// instantiations) compute bit-identical w.
enum PairStatus : int { kSkip = 0, kHit = 1, kExact = 2 };

template <bool kGrad, int kPrec>
__device__ __forceinline__ int eval_pair(const TriRec& r, int code, int px, int py, float ptx,
                                          float pty, const Consts& K, PairEval& o) {
  if (code & kBlkBox) {
    if (px < r.bbox[0] || px >= r.bbox[2] || py < r.bbox[1] || py >= r.bbox[3]) return kSkip;
  }
  if (code & kBlkInside) {
    o.cov = 1.0f;
    o.w = r.alpha;
    o.band = false;
    return kHit;  // alpha > MIN_WEIGHT is guaranteed by the set-up cull
  }
  if (!(r.flags & kFastOk)) return kExact;
  // Edges that are not candidates lie farther than max(rej, acc) on the inner
  // side of every pixel of the block: they take no part in any decision.
  const int cand = code >> kCandShift;
  const float inf = __int_as_float(0x7f800000);
  const float l0 = (cand & 1) ? __fmaf_rn(r.ed[0].nx, ptx, __fmaf_rn(r.ed[0].ny, pty, r.ed[0].c)) : inf;
  const float l1 = (cand & 2) ? __fmaf_rn(r.ed[1].nx, ptx, __fmaf_rn(r.ed[1].ny, pty, r.ed[1].c)) : inf;
  const float l2 = (cand & 4) ? __fmaf_rn(r.ed[2].nx, ptx, __fmaf_rn(r.ed[2].ny, pty, r.ed[2].c)) : inf;
  const float mn = fminf(fminf(l0, l1), l2);
  if (mn < -r.rej) return kSkip;
  if (mn > r.acc) {
    o.cov = 1.0f;
    o.w = r.alpha;
    o.band = false;
    return kHit;
  }
  if (kPrec == kPrecStrict) return kExact;

  // Within rounding distance of an edge line the inside/outside call, and
  // inside near an angle bisector the choice of nearest edge, could differ
  // from the reference's f32 decision; those rare pixels take the exact path.
  if (fabsf(mn) < r.margin) return kExact;

  // Nearest edge by clamped segment distance (raster.rs:124-134), the same
  // computation inside and outside (inside, the nearest segment distance is
  // the nearest edge-line distance), so no lane diverges on the side.
  const bool inside = mn >= 0.0f;
  int edge = 0;
  float ft = 0.0f, fdx = 0.0f, fdy = 0.0f;
  float bd2 = __int_as_float(0x7f800000), sd2 = bd2, st = 0.0f;
  int sedge = 0;
#pragma unroll
  for (int e = 0; e < 3; ++e) {
    if (!(cand & (1 << e))) continue;
    const float ex = r.ed[e].ex, ey = r.ed[e].ey;
    const float apx = __fsub_rn(ptx, r.ed[e].ax), apy = __fsub_rn(pty, r.ed[e].ay);
    const float te = __saturatef(__fmul_rn(__fmaf_rn(apx, ex, __fmul_rn(apy, ey)), r.ed[e].il));
    const float dx = __fmaf_rn(-te, ex, apx), dy = __fmaf_rn(-te, ey, apy);
    const float d2 = __fmaf_rn(dx, dx, __fmul_rn(dy, dy));
    if (d2 < bd2) {
      sd2 = bd2;
      st = ft;
      sedge = edge;
      bd2 = d2;
      fdx = dx;
      fdy = dy;
      ft = te;
      edge = e;
    } else if (d2 < sd2) {
      sd2 = d2;
      st = te;
      sedge = e;
    }
  }
  const float frs = rsqrt_approx(bd2);
  const float fdist = bd2 > 1e-30f ? __fmul_rn(bd2, frs) : 0.0f;
  // Two edges within rounding distance of each other (an angle bisector
  // inside, a sliver or nearly parallel edges outside) could be ordered
  // differently by the reference's f32 distances, sending this pixel's
  // gradient to another vertex pair: take the exact path. Adjacent edges both
  // clamped to their shared vertex describe the same point: not a tie.
  const bool same_vertex = (sedge == (edge + 1) % 3) ? (ft == 1.0f && st == 0.0f)
                                                     : (ft == 0.0f && st == 1.0f);
  if (!same_vertex && sd2 - bd2 < __fmul_rn(r.margin, __fmaf_rn(2.0f, fdist, r.margin)))
    return kExact;

  if (kPrec == kPrecFast) {
    const float x = __fmul_rn(inside ? fdist : -fdist, K.inv_sigma);
    o.cov = sigmoid_fast(x);
    o.w = __fmul_rn(r.alpha, o.cov);
    o.band = !(fdist < 1e-9f);
    if (kGrad && o.band) {
      const float t = ft, ux = __fmul_rn(fdx, frs), uy = __fmul_rn(fdy, frs);
      const float cov = o.cov;
      const float chain = __fmul_rn(__fmul_rn(cov, __fsub_rn(1.0f, cov)),
                                    inside ? K.inv_sigma : -K.inv_sigma);
      const float ka = __fmul_rn(chain, __fsub_rn(t, 1.0f)), kb = __fmul_rn(chain, -t);
      o.dax = __fmul_rn(ka, ux);
      o.day = __fmul_rn(ka, uy);
      o.dbx = __fmul_rn(kb, ux);
      o.dby = __fmul_rn(kb, uy);
      o.edge = edge;
    }
    return o.w <= kMinWeight ? kSkip : kHit;
  }

  // kPrecRef: the nearest edge's segment distance exactly as
  // point_segment_distance computes it (raster.rs:124-134).
  const float ax = r.ed[edge].ax, ay = r.ed[edge].ay;
  const float ex = r.ed[edge].ex, ey = r.ed[edge].ey, len2 = r.len2[edge];
  const float apx = __fsub_rn(ptx, ax), apy = __fsub_rn(pty, ay);
  float t = 0.0f;
  if (!(len2 <= 1e-20f)) {
    const float dot = __fadd_rn(__fmul_rn(apx, ex), __fmul_rn(apy, ey));
    t = rclamp(div_rn_inv(dot, len2, r.ed[edge].il), 0.0f, 1.0f);
  }
  const float dx = __fsub_rn(apx, __fmul_rn(t, ex));
  const float dy = __fsub_rn(apy, __fmul_rn(t, ey));
  const float dist = sqrt_nr(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)));
  const float sd = inside ? dist : -dist;
  o.cov = sigmoid_rounded(div_rn_inv(sd, K.sigma_eff, K.inv_sigma));
  o.w = __fmul_rn(r.alpha, o.cov);
  o.band = !(dist < 1e-9f);
  if (kGrad && o.band) cov_grad_ref(r, edge, t, dist, o.cov, sd > 0.0f, ptx, pty, K, o);
  return o.w <= kMinWeight ? kSkip : kHit;
}

// One edge's point_segment_distance (raster.rs:124-134) and winding cross
// product (raster.rs:119-122) with the reference's operations and rounding.
struct SegEval {
  float d, t, cross;
};
__device__ __forceinline__ SegEval seg_exact(const TriRec& r, int e, float ptx, float pty) {
  const float ex = r.ed[e].ex, ey = r.ed[e].ey, len2 = r.len2[e];
  const float apx = __fsub_rn(ptx, r.ed[e].ax), apy = __fsub_rn(pty, r.ed[e].ay);
  const float dot = __fadd_rn(__fmul_rn(apx, ex), __fmul_rn(apy, ey));
  SegEval o;
  o.t = len2 <= 1e-20f ? 0.0f : rclamp(div_rn_inv(dot, len2, r.ed[e].il), 0.0f, 1.0f);
  const float dx = __fsub_rn(apx, __fmul_rn(o.t, ex));
  const float dy = __fsub_rn(apy, __fmul_rn(o.t, ey));
  o.d = sqrt_nr(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)));
  o.cross = __fsub_rn(__fmul_rn(ex, apy), __fmul_rn(ey, apx));
  return o;
}

// Soft-edge value of one pair for reference precision, from the candidate
// edges of the pixel's warp block (`cand`, at least one bit). A non-candidate
// edge's line lies more than max(rej, acc) on the inner side of every pixel of
// the block, so:
//  - it is not the reference's nearest edge of any pixel that composites
//    (outside, that edge is nearer than rej; inside, nearer than acc, or
//    cov == 1 exactly), and
//  - its cross product has the sign of the winding, so is_inside
//    (raster.rs:111-122) is decided by the candidates' own cross products.
// Each candidate's distance and cross product are the reference's f32 values,
// and the nearest edge is chosen by the reference's strict `<` in edge order
// (grad.rs:236-242), so ties resolve as the reference resolves them. Pixels
// farther than rej outside, or farther than acc inside every candidate line,
// take the box tests' answers (skip; cov == 1). Degenerate triangles and NaN
// alpha return kExact.
template <bool kGrad>
__device__ __forceinline__ int eval_cand(const TriRec& r, int code, int cand, int px, int py,
                                         float ptx, float pty, const Consts& K, PairEval& o) {
  bool live = true;
  if (code & kBlkBox) {
    live = (px >= r.bbox[0]) & (px < r.bbox[2]) & (py >= r.bbox[1]) & (py < r.bbox[3]);
  }
  if (!(r.flags & kFastOk)) return live ? kExact : kSkip;
  const float inf = __int_as_float(0x7f800000);
  float mn = inf, best = inf, bt = 0.0f;
  float cr[3];
  int edge = 0;
#pragma unroll
  for (int e = 0; e < 3; ++e) {
    cr[e] = r.wind;
    if (!(cand & (1 << e))) continue;
    mn = fminf(mn, __fmaf_rn(r.ed[e].nx, ptx, __fmaf_rn(r.ed[e].ny, pty, r.ed[e].c)));
    const SegEval g = seg_exact(r, e, ptx, pty);
    cr[e] = g.cross;
    if (g.d < best) {
      best = g.d;
      bt = g.t;
      edge = e;
    }
  }
  live = live && !(mn < -r.rej);
  const bool deep = mn > r.acc;
  const bool inside = (cr[0] >= 0.0f && cr[1] >= 0.0f && cr[2] >= 0.0f) ||
                      (cr[0] <= 0.0f && cr[1] <= 0.0f && cr[2] <= 0.0f);
  const float sd = inside ? best : -best;
  const float cov = sigmoid_rounded(div_rn_inv(sd, K.sigma_eff, K.inv_sigma));
  o.cov = deep ? 1.0f : cov;
  o.w = __fmul_rn(r.alpha, o.cov);
  o.band = !deep && !(best < 1e-9f);
  if (kGrad) cov_grad_ref(r, edge, bt, best, o.cov, inside, ptx, pty, K, o);
  return (live && !(o.w <= kMinWeight)) ? kHit : kSkip;
}

// eval_cand for a block whose only candidate is edge E, straight-line: the
// other two cross products have the winding's sign, so is_inside reduces to
// the sign of edge E's cross product against the winding.
template <bool kGrad, int E>
__device__ __forceinline__ int eval_single(const TriRec& r, int code, int px, int py, float ptx,
                                           float pty, const Consts& K, PairEval& o) {
  bool live = true;
  if (code & kBlkBox) {
    live = (px >= r.bbox[0]) & (px < r.bbox[2]) & (py >= r.bbox[1]) & (py < r.bbox[3]);
  }
  const float l = __fmaf_rn(r.ed[E].nx, ptx, __fmaf_rn(r.ed[E].ny, pty, r.ed[E].c));
  live = live && !(l < -r.rej);
  const bool deep = l > r.acc;
  const SegEval g = seg_exact(r, E, ptx, pty);
  const bool inside = r.wind > 0.0f ? g.cross >= 0.0f : g.cross <= 0.0f;
  const float sd = inside ? g.d : -g.d;
  const float cov = sigmoid_rounded(div_rn_inv(sd, K.sigma_eff, K.inv_sigma));
  o.cov = deep ? 1.0f : cov;
  o.w = __fmul_rn(r.alpha, o.cov);
  o.band = !deep && !(g.d < 1e-9f);
  if (kGrad) cov_grad_ref(r, E, g.t, g.d, o.cov, inside, ptx, pty, K, o);
  return (live && !(o.w <= kMinWeight)) ? kHit : kSkip;
}

// Reference-precision soft-edge evaluation, dispatched on the (warp-uniform)
// candidate set.
template <bool kGrad>
__device__ __forceinline__ int eval_ref_prec(const TriRec& r, int code, int cand, int px, int py,
                                             float ptx, float pty, const Consts& K, PairEval& o) {
  if (r.flags & kFastOk) {
    if (cand == 1) return eval_single<kGrad, 0>(r, code, px, py, ptx, pty, K, o);
    if (cand == 2) return eval_single<kGrad, 1>(r, code, px, py, ptx, pty, K, o);
    if (cand == 4) return eval_single<kGrad, 2>(r, code, px, py, ptx, pty, K, o);
  }
  return eval_cand<kGrad>(r, code, cand, px, py, ptx, pty, K, o);
}

// Running product of (1 - w) with 2^64 renormalisation and barrier tracking.
struct Prod {
  float m;
  int e;
  int z0;  // last triangle index with (1 - w) == 0
  int zn;  // last triangle index with (1 - w) NaN
  __device__ void init() {
    m = 1.0f;
    e = 0;
    z0 = -1;
    zn = -1;
  }
  __device__ __forceinline__ void mul(float f, int k) {
    if (f > 0.0f) {  // f = 1 - w lies in [0, 1) or is NaN
      m = __fmul_rn(m, f);
      if (m < kRenormInv) {
        m = __fmul_rn(m, kRenorm);
        e += 1;
      }
    } else {
      if (f == 0.0f) z0 = k;
      else zn = k;
      m = 1.0f;
      e = 0;
    }
  }
};

// A_k = prod over layers above k of (1 - w), from the full product P (after
// the last layer) and the running product Q (through layer k). A barrier
// layer resets Q to 1, so the same ratio yields the product above it.
// The reference attenuates by a running product in the opposite order, so
// the ratio matches it to rounding only and needs no exact division: both
// mantissas lie in [2^-64, 1], where the approximate quotient is within 2 ulp.
__device__ __forceinline__ float attenuation(const Prod& P, const Prod& Q, int k) {
  if (k < P.zn) return __int_as_float(0x7fc00000);
  if (k < P.z0) return 0.0f;
  const float ratio = __fdividef(P.m, Q.m);
  const int de = P.e - Q.e;
  if (de == 0) return ratio;
  if (de == 1) return __fmul_rn(ratio, kRenormInv);
  if (de == 2) return __fmul_rn(__fmul_rn(ratio, kRenormInv), kRenormInv);
  return 0.0f;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Transposed warp reduction of 10 per-lane values: each halving step keeps
// half of the values and trades the other half with the partner lane, so the
// 10 warp totals cost 12 shuffles instead of 50. On return, lane `slot`
// (see reduce10_slot) holds the total of value `slot`'s index.
__device__ __forceinline__ float reduce10(const float (&v)[10], int lane) {
  const unsigned F = 0xffffffffu;
  bool h = lane & 16;
  float a[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const float keep = h ? v[5 + i] : v[i];
    const float send = h ? v[i] : v[5 + i];
    a[i] = keep + __shfl_xor_sync(F, send, 16);
  }
  h = lane & 8;
  float b0, b1, b2;
  {
    const float k0 = h ? a[3] : a[0], s0 = h ? a[0] : a[3];
    const float k1 = h ? a[4] : a[1], s1 = h ? a[1] : a[4];
    const float k2 = h ? 0.0f : a[2], s2 = h ? a[2] : 0.0f;
    b0 = k0 + __shfl_xor_sync(F, s0, 8);
    b1 = k1 + __shfl_xor_sync(F, s1, 8);
    b2 = k2 + __shfl_xor_sync(F, s2, 8);
  }
  h = lane & 4;
  float c0, c1;
  {
    const float k0 = h ? b2 : b0, s0 = h ? b0 : b2;
    const float k1 = h ? 0.0f : b1, s1 = h ? b1 : 0.0f;
    c0 = k0 + __shfl_xor_sync(F, s0, 4);
    c1 = k1 + __shfl_xor_sync(F, s1, 4);
  }
  h = lane & 2;
  const float k = h ? c1 : c0, s = h ? c0 : c1;
  float d = k + __shfl_xor_sync(F, s, 2);
  d += __shfl_xor_sync(F, d, 1);
  return d;
}

// The value index lane `lane` holds after reduce10, or -1.
__device__ __forceinline__ int reduce10_slot(int lane) {
  if (lane & 1) return -1;
  const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
  const int pos = b2 ? (b1 ? -1 : 2) : b1;  // position among the 3 kept after step 2
  if (pos < 0) return -1;
  const int local = b3 ? (pos < 2 ? 3 + pos : -1) : pos;
  return local < 0 ? -1 : 5 * b4 + local;
}

// 4 values (colour and alpha gradients): lane 8*i holds the total of v[i].
__device__ __forceinline__ float reduce4(float v0, float v1, float v2, float v3, int lane) {
  const unsigned F = 0xffffffffu;
  bool h = lane & 16;
  float k0 = h ? v2 : v0, s0 = h ? v0 : v2;
  float k1 = h ? v3 : v1, s1 = h ? v1 : v3;
  k0 += __shfl_xor_sync(F, s0, 16);
  k1 += __shfl_xor_sync(F, s1, 16);
  h = lane & 8;
  float k = h ? k1 : k0;
  const float s = h ? k0 : k1;
  k += __shfl_xor_sync(F, s, 8);
  k += __shfl_xor_sync(F, k, 4);
  k += __shfl_xor_sync(F, k, 2);
  k += __shfl_xor_sync(F, k, 1);
  return k;
}

// 8 values: lanes with (lane & 3) == 0 hold the total of value
// 4 * bit4 + 2 * bit3 + bit2 of the lane index (9 shuffles).
__device__ __forceinline__ float reduce8(const float (&v)[8], int lane) {
  const unsigned F = 0xffffffffu;
  bool h = lane & 16;
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = h ? v[4 + i] : v[i];
    const float send = h ? v[i] : v[4 + i];
    a[i] = keep + __shfl_xor_sync(F, send, 16);
  }
  h = lane & 8;
  float b[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = h ? a[2 + i] : a[i];
    const float send = h ? a[i] : a[2 + i];
    b[i] = keep + __shfl_xor_sync(F, send, 8);
  }
  h = lane & 4;
  float c = (h ? b[1] : b[0]) + __shfl_xor_sync(F, h ? b[0] : b[1], 4);
  c += __shfl_xor_sync(F, c, 2);
  c += __shfl_xor_sync(F, c, 1);
  return c;
}

// Which entry of (a_x, a_y, b_x, b_y, r, g, b, alpha) a lane holds after
// reduce8, as a parameter index for a single-edge entry with edge e
// (a = vertex e, b = vertex e + 1); -1 for lanes that hold no total.
__device__ __forceinline__ int reduce8_param(int lane, int e) {
  if (lane & 3) return -1;
  const int s = lane >> 2;  // 4 * bit4 + 2 * bit3 + bit2
  if (s >= 4) return 6 + (s - 4);
  const int vtx = (s < 2) ? e : (e == 2 ? 0 : e + 1);
  return 2 * vtx + (s & 1);
}

__device__ __forceinline__ size_t pix_index(int layout, int b, int ch, int px, int py, int W,
                                            int H) {
  if (layout == kLayoutBCHW) return (((size_t)b * 3 + ch) * H + py) * W + px;
  return (((size_t)b * H + py) * W + px) * 3 + ch;
}

// Deterministic mode: a list's sums in 64-bit fixed point, 2^-36 resolution,
// so that their value does not depend on the order of the atomic additions
// (integer addition is associative). A warp total of magnitude 2^20 or more,
// infinite or NaN, sets the parameter's bit in a flag word instead (NaN,
// positive, negative: 3 bits per parameter), which the finalize turns into
// NaN or an infinity, as the float sum of such values would be.
constexpr float kDetScale = 68719476736.0f;      // 2^36
constexpr float kDetInv = 1.4551915228366852e-11f;  // 2^-36
constexpr float kDetLimit = 72057594037927936.0f;  // 2^56 = 2^20 * kDetScale
__device__ __forceinline__ int nonfinite_bit(float v, int p) {
  return 1 << (3 * p + (v != v ? 0 : (v > 0.0f ? 1 : 2)));
}
__device__ __forceinline__ void acc_add_fixed(unsigned long long* sum, int* flags, float v, int p) {
  const float s = __fmul_rn(v, kDetScale);
  if (fabsf(s) < kDetLimit)
    atomicAdd(sum, (unsigned long long)__float2ll_rn(s));
  else
    atomicOr(flags, nonfinite_bit(v, p));
}
template <class S>
__device__ __forceinline__ void acc_add(S& sm, int j, int p, float v, bool det) {
  if (!det)
    atomicAdd(&sm.acc[j][p], v);
  else
    acc_add_fixed(reinterpret_cast<unsigned long long*>(&sm.acc64[j][p]), &sm.nf[j], v, p);
}

// Pass 1 over a staged list for one lane's pixel: composites in order
// (raster.rs:63) and keeps the running product of 1 - w. `col` selects the
// warp's block code.
template <int Mode, int kPrec, class S, bool kProd = Mode != kModeRender>
__device__ __forceinline__ void forward_walk(const S& sm, int count, int col, int px, int py,
                                             float ptx, float pty, bool active, const Consts& K,
                                             float& c0, float& c1, float& c2, Prod& P) {
  for (int j = 0; j < count; ++j) {
    const int code = sm.bcode[j][col];
    if (code & kBlkSkip) continue;
    const TriRec& r = sm.rec[j];
    const int k = sm.kidx[j];
    const int cand = code >> kCandShift;
    PairEval pe;
    int st;
    if (code & kBlkInside) {
      pe.w = r.alpha;
      st = kHit;
    } else if (kPrec == kPrecRef) {
      st = eval_ref_prec<false>(r, code, cand, px, py, ptx, pty, K, pe);
    } else {
      st = eval_pair<false, kPrec>(r, code, px, py, ptx, pty, K, pe);
    }
    if (st == kExact) {
      pe = eval_ref<false>(&r, ptx, pty, K.sigma_eff);
      st = pe.hit ? kHit : kSkip;
    }
    if (st != kHit || !active) continue;
    const float w = pe.w, om = __fsub_rn(1.0f, w);
    c0 = __fadd_rn(__fmul_rn(r.color[0], w), __fmul_rn(c0, om));  // raster.rs:63
    c1 = __fadd_rn(__fmul_rn(r.color[1], w), __fmul_rn(c1, om));
    c2 = __fadd_rn(__fmul_rn(r.color[2], w), __fmul_rn(c2, om));
    if (kProd) P.mul(om, k);
  }
}

// Pass 2 over a staged list: recomposites in forward order, and per entry
// reduces the warp's contributions into sm.acc (one shared atomic per value).
template <int kPrec, class S>
__device__ __forceinline__ void gradient_walk(S& sm, int count, int col, int lane, int px, int py,
                                              float ptx, float pty, bool active, const Consts& K,
                                              const Prod& P, Prod& Q, float G0, float G1,
                                              float G2, float& r0, float& r1, float& r2) {
  const int slot10 = reduce10_slot(lane);
  for (int j = 0; j < count; ++j) {
    const int code = sm.bcode[j][col];
    if (code & kBlkSkip) continue;
    const TriRec& r = sm.rec[j];
    const int k = sm.kidx[j];
    const int cand = code >> kCandShift;
    // Single-edge entries accumulate vertex gradients relative to the edge
    // (acc[0..3] = vertex e, vertex e + 1), others by vertex (acc[0..5]).
    const bool single = kPrec == kPrecRef && !(code & kBlkInside) && (cand & (cand - 1)) == 0;
    const int e1 = cand - 1 - (cand >> 2);  // the single candidate: 1, 2, 4 -> 0, 1, 2
    float acc[10];
#pragma unroll
    for (int i = 0; i < 10; ++i) acc[i] = 0.0f;
    bool contrib = false, band = false;
    PairEval pe;
    int st;
    if (code & kBlkInside) {
      pe.w = r.alpha;
      pe.cov = 1.0f;
      pe.band = false;
      st = kHit;
    } else if (kPrec == kPrecRef) {
      st = eval_ref_prec<true>(r, code, cand, px, py, ptx, pty, K, pe);
    } else {
      st = eval_pair<true, kPrec>(r, code, px, py, ptx, pty, K, pe);
    }
    if (st == kExact) {
      pe = eval_ref<true>(&r, ptx, pty, K.sigma_eff);
      st = pe.hit ? kHit : kSkip;
    }
    if (st == kHit && active) {
      contrib = true;
      const float w = pe.w, om = __fsub_rn(1.0f, w);
      Q.mul(om, k);
      const float A = attenuation(P, Q, k);
      const float g0 = __fmul_rn(G0, A), g1 = __fmul_rn(G1, A), g2 = __fmul_rn(G2, A);
      // grad.rs:162-179
      acc[6] = __fmul_rn(g0, w);
      acc[7] = __fmul_rn(g1, w);
      acc[8] = __fmul_rn(g2, w);
      const float e0 = __fsub_rn(r.color[0], r0), e1c = __fsub_rn(r.color[1], r1),
                  e2 = __fsub_rn(r.color[2], r2);
      float d_w = __fmul_rn(g0, e0);
      d_w = __fmaf_rn(g1, e1c, d_w);
      d_w = __fmaf_rn(g2, e2, d_w);
      if (r.flags & kAlphaActive) acc[9] = __fmul_rn(d_w, pe.cov);
      // coverage_with_grad (grad.rs:231-270): nonzero only for band pairs
      // away from the boundary itself (dist >= 1e-9).
      if (pe.band) {
        band = true;
        const float d_cov = __fmul_rn(d_w, r.alpha);
        const float ax = __fmul_rn(d_cov, pe.dax), ay = __fmul_rn(d_cov, pe.day);
        const float bx = __fmul_rn(d_cov, pe.dbx), by = __fmul_rn(d_cov, pe.dby);
        if (single) {
          // With one candidate edge e every compositing pixel's nearest
          // edge is e (eval_cand).
          acc[0] = ax;
          acc[1] = ay;
          acc[2] = bx;
          acc[3] = by;
        } else {
          const int e = pe.edge;
          acc[0] = (e == 0) ? ax : ((e == 2) ? bx : 0.0f);
          acc[1] = (e == 0) ? ay : ((e == 2) ? by : 0.0f);
          acc[2] = (e == 1) ? ax : ((e == 0) ? bx : 0.0f);
          acc[3] = (e == 1) ? ay : ((e == 0) ? by : 0.0f);
          acc[4] = (e == 2) ? ax : ((e == 1) ? bx : 0.0f);
          acc[5] = (e == 2) ? ay : ((e == 1) ? by : 0.0f);
        }
      }
      // The canvas beneath the next layer. It only feeds d_w, so it is kept
      // as dst + w (C - dst), within a few ulps of the reference's
      // C w + dst (1 - w) (raster.rs:63), reusing the differences above.
      r0 = __fmaf_rn(w, e0, r0);
      r1 = __fmaf_rn(w, e1c, r1);
      r2 = __fmaf_rn(w, e2, r2);
    }
    // Per warp: one transposed reduction, then one shared atomic per value.
    const unsigned any = __ballot_sync(0xffffffffu, contrib);
    if (any == 0u) continue;
    if (__any_sync(0xffffffffu, band)) {
      if (single) {
        const float v8[8] = {acc[0], acc[1], acc[2], acc[3], acc[6], acc[7], acc[8], acc[9]};
        const float sum = reduce8(v8, lane);
        const int prm = reduce8_param(lane, e1);
        if (prm >= 0) acc_add(sm, j, prm, sum, K.det);
      } else {
        const float sum = reduce10(acc, lane);
        if (slot10 >= 0) acc_add(sm, j, slot10, sum, K.det);
      }
    } else {
      const float sum = reduce4(acc[6], acc[7], acc[8], acc[9], lane);
      if ((lane & 7) == 0) acc_add(sm, j, 6 + (lane >> 3), sum, K.det);
    }
  }
}

// The canvas a scene starts from: one shared colour or one per scene.
__device__ __forceinline__ void scene_background(const RasterArgs& a, int b, float& c0, float& c1,
                                                 float& c2) {
  c0 = a.bg3[0];
  c1 = a.bg3[1];
  c2 = a.bg3[2];
  if (a.bg_dev) {
    const float* q = a.bg_dev + (a.bg_per_scene ? 3 * b : 0);
    c0 = q[0];
    c1 = q[1];
    c2 = q[2];
  }
}

// G = (2/N)(r - t) (grad.rs:112-114) or the upstream gradient, and the pixel's
// squared error for the loss.
template <int Mode>
__device__ __forceinline__ void top_gradient(const RasterArgs& a, int b, int px, int py,
                                             bool active, float c0, float c1, float c2, float& G0,
                                             float& G1, float& G2, double& sq) {
  G0 = G1 = G2 = 0.0f;
  sq = 0.0;
  if (!active) return;
  const float o0 = a.other[pix_index(a.layout, b, 0, px, py, a.W, a.H)];
  const float o1 = a.other[pix_index(a.layout, b, 1, px, py, a.W, a.H)];
  const float o2 = a.other[pix_index(a.layout, b, 2, px, py, a.W, a.H)];
  if (Mode == kModeLoss) {
    const float d0 = __fsub_rn(c0, o0), d1 = __fsub_rn(c1, o1), d2 = __fsub_rn(c2, o2);
    sq = (double)d0 * d0 + (double)d1 * d1 + (double)d2 * d2;
    G0 = __fmul_rn(a.grad_scale, d0);
    G1 = __fmul_rn(a.grad_scale, d1);
    G2 = __fmul_rn(a.grad_scale, d2);
  } else {
    G0 = o0;
    G1 = o1;
    G2 = o2;
  }
}

__device__ __forceinline__ void store_pixel(const RasterArgs& a, int b, int px, int py, float c0,
                                            float c1, float c2) {
  a.image[pix_index(a.layout, b, 0, px, py, a.W, a.H)] = c0;
  a.image[pix_index(a.layout, b, 1, px, py, a.W, a.H)] = c1;
  a.image[pix_index(a.layout, b, 2, px, py, a.W, a.H)] = c2;
}

// One warp block's image (8 x 4 pixels, a pixel per lane, 3 channels) in
// 16-byte stores: the 96 values go through the warp's shared-memory stage and
// leave as 24 float4 stores, whole 16-byte runs of the image in either layout
// (BHWC: 4 rows of 24 consecutive floats; BCHW: 3 channel planes x 4 rows of
// 8 floats), where scalar stores would write each sector in three passes.
// Needs every lane of the warp (it synchronizes the warp); blocks that cross
// the image border, widths that are not a multiple of 4, or an image pointer
// that is not 16-byte aligned take per-lane scalar stores.
__device__ __forceinline__ void store_block(const RasterArgs& a, int b, int x0, int y0, int lane,
                                            float c0, float c1, float c2, float4* stage) {
  const int px = x0 + (lane & 7), py = y0 + (lane >> 3);
  const bool whole = x0 + kBlockW <= a.W && y0 + kBlockH <= a.H && (a.W & 3) == 0 &&
                     ((uintptr_t)a.image & 15u) == 0;
  if (!whole) {
    if (px < a.W && py < a.H) store_pixel(a, b, px, py, c0, c1, c2);
    return;
  }
  float* st = reinterpret_cast<float*>(stage);
  __syncwarp();  // the previous block's reads of the stage are done
  if (a.layout == kLayoutBCHW) {
    st[lane] = c0;
    st[32 + lane] = c1;
    st[64 + lane] = c2;
  } else {
    st[3 * lane] = c0;  // stride 3 words: 32 distinct banks
    st[3 * lane + 1] = c1;
    st[3 * lane + 2] = c2;
  }
  __syncwarp();
  if (lane < 24) {
    const float4 v = stage[lane];
    float* dst;
    if (a.layout == kLayoutBCHW) {  // lane = channel * 8 + row * 2 + half
      const int ch = lane >> 3, row = (lane >> 1) & 3, half = lane & 1;
      dst = a.image + pix_index(kLayoutBCHW, b, ch, x0 + 4 * half, y0 + row, a.W, a.H);
    } else {  // lane = row * 6 + q: floats 4q..4q+3 of the row's 24
      const int row = lane / 6, q = lane - 6 * row;
      dst = a.image + pix_index(kLayoutBHWC, b, 0, x0, y0 + row, a.W, a.H) + 4 * q;
    }
    *reinterpret_cast<float4*>(dst) = v;
  }
}

// Deterministic mode's flush.
__device__ __forceinline__ void flush_fixed(const long long* acc64, const int* nf, const int* kidx,
                                         int count, long long* fx, int* nfg) {
  for (int i = threadIdx.x; i < count * kParams; i += kThreads) {
    const long long q = acc64[i];
    if (q != 0)
      atomicAdd(reinterpret_cast<unsigned long long*>(&fx[(size_t)kidx[i / kParams] * kParams +
                                                           (i % kParams)]),
                (unsigned long long)q);
  }
  for (int i = threadIdx.x; i < count; i += kThreads)
    if (nf[i]) atomicOr(&nfg[kidx[i]], nf[i]);
}

// One global atomic per nonzero (triangle, parameter) accumulator of a list.
template <bool kDet, class S>
__device__ __forceinline__ void flush_grads(const S& sm, const RasterArgs& a, int b, int count) {
  if (kDet) {  // deterministic mode: fixed-point sums and flag words
    flush_fixed(&sm.acc64[0][0], sm.nf, sm.kidx, count, a.grads_fx + (size_t)b * a.T * kParams,
                a.grads_nf + (size_t)b * a.T);
    return;
  }
  float* g = a.grads + (size_t)b * a.T * kParams;
  for (int i = threadIdx.x; i < count * kParams; i += kThreads) {
    const float v = (&sm.acc[0][0])[i];
    if (v != 0.0f) atomicAdd(&g[(size_t)sm.kidx[i / kParams] * kParams + (i % kParams)], v);
  }
}

// Fitter::step's bookkeeping after iteration `iter`'s loss (fit.rs:243-288):
// record the loss, track the best, stop on divergence or patience, and tell
// the next Adam step whether to run and to copy the best parameters first.
__device__ void fit_control(FitState* st, int iter, float min_delta, long long patience,
                            float* losses) {
  if (st->stopped) {
    st->run_adam = 0;
    st->copy_best = 0;
    return;
  }
  const float loss = st->loss;
  if (!isfinite(loss)) {  // fit.rs:262-265
    st->stopped = 1;
    st->stop_reason = 2;
    st->run_adam = 0;
    st->copy_best = 0;
    return;
  }
  losses[st->count] = loss;
  st->count += 1;
  if (__fadd_rn(loss, min_delta) < st->best_loss) {  // fit.rs:268-275
    st->best_loss = loss;
    st->best_iter = iter;
    st->since = 0;
    st->copy_best = 1;
  } else {
    st->since += 1;
    st->copy_best = 0;
  }
  if (patience >= 0 && (long long)st->since >= patience) {  // fit.rs:278-281
    st->stopped = 1;
    st->stop_reason = 1;
    st->run_adam = 0;
    return;
  }
  st->run_adam = 1;
}

// Per-scene loss: each CTA's f64 partial (slot `slot` of the scene's n_blocks),
// summed in fixed order by the scene's last CTA (canvas.rs:45-59). `part`
// holds this CTA's n_part partials in shared memory; all threads call it after
// the partials are written.
__device__ __forceinline__ void scene_loss(const RasterArgs& a, int b, int slot, int n_blocks,
                                           const double* part, int n_part, double* sm_scratch,
                                           int* is_last) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < n_part; ++w) s += part[w];
    a.loss_partials[(size_t)b * n_blocks + slot] = s;
    __threadfence();
    const unsigned prev = atomicAdd(&a.loss_counters[b], 1u);
    *is_last = (prev == (unsigned)(n_blocks - 1));
  }
  __syncthreads();
  if (*is_last) {
    __threadfence();
    double s = 0.0;
    for (int t = threadIdx.x; t < n_blocks; t += kThreads)
      s += *((volatile double*)&a.loss_partials[(size_t)b * n_blocks + t]);
    s = warp_sum_d(s);
    if (lane == 0) sm_scratch[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      double tot = 0.0;
      for (int w = 0; w < kWarps; ++w) tot += sm_scratch[w];
      if (a.loss_sums) a.loss_sums[b] = tot;
      if (a.losses) a.losses[b] = (float)(tot / a.n_values);  // canvas.rs:58
      a.loss_counters[b] = 0;
      if (a.fit) fit_control(a.fit, a.fit_iter, a.fit_min_delta, a.fit_patience, a.fit_losses);
    }
  }
}

// Split state, block-major so that one block's slice is contiguous (ranks of
// a triangle-sharded scene all-gather their slices): [c0 c1 c2 m] [e z0 zn -]
// per (block, scene, pixel), the block's composite over black and its running
// product from its forward pass.
__device__ __forceinline__ float4* split_pixel(const RasterArgs& a, int k, int b, int px,
                                               int py) {
  return a.split_state + (((size_t)k * a.B + b) * a.H * a.W + (size_t)py * a.W + px) * 2;
}

// Factor a of a block's map x -> a x + c from its forward state: NaN after a
// NaN layer, 0 after an opaque one, else the renormalised running product.
__device__ __forceinline__ float block_factor(const float4& s0, const float4& s1) {
  const int e = __float_as_int(s1.x), z0 = __float_as_int(s1.y), zn = __float_as_int(s1.z);
  return zn >= 0 ? __int_as_float(0x7fc00000) : (z0 >= 0 ? 0.0f : ldexpf(s0.w, -64 * e));
}

// k-th index of 0..n-1 in centre-out order: c, c-1, c+1, c-2, c+2, ...
__device__ __forceinline__ int center_out(int k, int n) {
  const int c = (n - 1) >> 1, j = (k + 1) >> 1;
  const int idx = (k & 1) ? c - j : c + j;
  return idx < 0 ? c + j : idx;
}

// k-th cell of an nx x ny grid in square rings: ring r = max(i, j) holds
// (r, 0..r) then (0..r-1, r); past min(nx, ny) rings, the rest of the longer
// side follows one column (or row) at a time. A bijection onto the grid.
__device__ __forceinline__ void ring_cell(int k, int nx, int ny, int& i, int& j) {
  const int m = min(nx, ny);
  if (k < m * m) {
    int r = (int)sqrtf((float)k);
    while (r * r > k) --r;
    while ((r + 1) * (r + 1) <= k) ++r;
    const int q = k - r * r;
    if (q <= r) {
      i = r;
      j = q;
    } else {
      i = q - r - 1;
      j = r;
    }
  } else if (nx > ny) {
    i = m + (k - m * m) / ny;
    j = (k - m * m) % ny;
  } else {
    j = m + (k - m * m) / nx;
    i = (k - m * m) % nx;
  }
}

// The (scene, tile) a tile-kernel CTA works on. The grid's x-y plane is read
// as one linear index in launch order, scenes fastest and tiles centre-out
// over centre-out column and row indices: the tiles with the most overlapping
// geometry start first and the light border tiles fill the end of the launch,
// which shortens its tail when there are only a few waves of CTAs (a small
// batch, or scenes whose geometry sits in the middle of the canvas). With
// a.tile_rings the tiles come in rings (launches of more than one wave:
// config 5, every vertex in the middle fifth, 3-7 % faster than central rows
// first, config 4 1 % slower); else whole central rows first (a launch of one
// wave, where the order only decides which tiles share an SM: rings made 64^2
// cells up to 10 % slower there). The region kernel keeps rows (1-2 % slower
// in rings).
__device__ __forceinline__ void tile_of_block(const RasterArgs& a, int& b, int& local_tile) {
  const unsigned lin = blockIdx.x + blockIdx.y * gridDim.x;
  b = (int)(lin % (unsigned)a.B);
  const int rank = (int)(lin / (unsigned)a.B);
  int ix = rank % a.tiles_x, iy = rank / a.tiles_x;
  if (a.tile_rings) ring_cell(rank, a.tiles_x, a.tile_rows, ix, iy);
  const int cx = center_out(ix, a.tiles_x);
  const int cy = center_out(iy, a.tile_rows);
  local_tile = cy * a.tiles_x + cx;
}

// Tile kernel: one CTA per (scene, 16x16 tile[, triangle block]), warp w on
// block w; lists longer than kChunk are binned in chunks behind barriers:
// kGather (kChunk < T <= kGatherMaxT) gathers them from the triangles the
// tile's mask marks, in triangle order; otherwise they are fixed windows of
// kChunk triangles. Each form keeps its own straight-line loop: one body with
// both list sources costs the walks 3-15 % more instructions.
template <int Mode, int kPrec, bool kGather = false, bool kDet = false>
__global__ void __launch_bounds__(kThreads, 4) dr_raster_kernel(RasterArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  if (a.skip_flag && *a.skip_flag) return;
  constexpr bool kSplitBwd = Mode == kModeSplitBwd || Mode == kModeSplitBwdGrad;
  constexpr bool kSplit = Mode == kModeSplitFwd || kSplitBwd;
  constexpr bool kLoss = Mode == kModeLoss || Mode == kModeSplitBwd;
  static_assert(!(kGather && kSplit), "split launches bin in windows");

  int b, local_tile;
  tile_of_block(a, b, local_tile);
  const int tile_col = local_tile % a.tiles_x;
  const int tile_row = a.tile_row0 + (local_tile / a.tiles_x) * a.tile_row_step;
  const int tx0 = tile_col * kTile, ty0 = tile_row * kTile;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int px = tx0 + (warp & 1) * kBlockW + (lane & 7);
  const int py = ty0 + (warp >> 1) * kBlockH + (lane >> 3);
  const bool active = px < a.W && py < a.H;
  const float ptx = pixel_center(px, a.W), pty = pixel_center(py, a.H);
  const TriRec* recs = a.recs + (size_t)b * a.T;
  Consts K;
  K.sigma_eff = a.sigma_eff;
  K.inv_sigma = a.inv_sigma;
  K.det = kDet;  // deterministic sums (a.grads_fx set): a separate instantiation
  // Triangles [t0, t1): all of them, or block kb of a split launch.
  const int kb = a.split_base + (int)blockIdx.z;
  const bool lead = !kSplitBwd || blockIdx.z == 0;  // writes the image and the loss
  int t0 = 0, t1 = a.T;
  if (kSplit) {
    const int per = (a.T + a.split_k - 1) / a.split_k;
    t0 = min(a.T, kb * per);
    t1 = min(a.T, t0 + per);
  }
  int n_chunks = (t1 - t0 + kChunk - 1) / kChunk;
  int count = 0;
  Range rg;
  rg.t0 = t0;
  rg.t1 = t1;
  rg.tx0 = tx0;
  rg.ty0 = ty0;
  rg.boxes = a.boxes ? a.boxes + (size_t)b * a.T : nullptr;
  if constexpr (kGather) n_chunks = (gather_start(sm, recs, rg, a.W, a.H) + kChunk - 1) / kChunk;
  Prod P;
  P.init();
  float G0 = 0.0f, G1 = 0.0f, G2 = 0.0f;
  float r0, r1, r2;

  if (!kSplitBwd) {
    // ---- pass 1: forward composite ----------------------------------------
    float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f;  // a block composites over black
    if (!kSplit) scene_background(a, b, c0, c1, c2);
    for (int ci = 0; ci < n_chunks; ++ci) {
      if constexpr (kGather)
        count = gather_list(sm, recs, rg, a.W, a.H);
      else
        count = build_list(sm, recs, t1, t0 + ci * kChunk, tx0, ty0, a.W, a.H);
      forward_walk<Mode, kPrec>(sm, count, warp, px, py, ptx, pty, active, K, c0, c1, c2, P);
    }
    if (Mode == kModeSplitFwd) {
      if (active) {
        float4* sp = split_pixel(a, kb, b, px, py);
        sp[0] = make_float4(c0, c1, c2, P.m);
        sp[1] = make_float4(__int_as_float(P.e), __int_as_float(P.z0), __int_as_float(P.zn), 0.f);
      }
      return;
    }
    if (a.image) store_block(a, b, tx0 + (warp & 1) * kBlockW, ty0 + (warp >> 1) * kBlockH, lane,
                             c0, c1, c2, sm.stage[warp]);
    if (Mode == kModeRender) return;

    // ---- loss and the gradient reaching the top of the stack --------------
    double sq;
    top_gradient<Mode>(a, b, px, py, active, c0, c1, c2, G0, G1, G2, sq);
    if (Mode == kModeLoss) {
      const double ws = warp_sum_d(sq);
      if (lane == 0) sm.loss_part[warp] = ws;
    }
    scene_background(a, b, r0, r1, r2);
  } else {
    // The combine, per pixel from every block's forward state. Block k's
    // layers map the canvas beneath them to a_k x + c_k, a_k the product of
    // their (1 - w) (0 after an opaque layer, NaN after a NaN one, as the
    // reference's running composite propagates them) and c_k their composite
    // over black. The canvas entering block kb is the composition of the maps
    // below it applied to the background, the final colour the composition of
    // all; the gradient reaching block kb is G times the product of a_k over
    // the blocks above, taken from the top down. The CTAs of the launch's
    // first block write the image and the loss.
    r0 = r1 = r2 = 0.0f;
    double sq = 0.0;
    if (active) {
      float d0, d1, d2;
      scene_background(a, b, d0, d1, d2);
      for (int k = 0; k < a.split_k; ++k) {
        const float4* sf = split_pixel(a, k, b, px, py);
        const float4 s0 = sf[0], s1 = sf[1];
        if (k == kb) {
          r0 = d0;
          r1 = d1;
          r2 = d2;
          P.m = s0.w;
          P.e = __float_as_int(s1.x);
          P.z0 = __float_as_int(s1.y);
          P.zn = __float_as_int(s1.z);
        }
        const float f = block_factor(s0, s1);
        d0 = __fadd_rn(__fmul_rn(f, d0), s0.x);
        d1 = __fadd_rn(__fmul_rn(f, d1), s0.y);
        d2 = __fadd_rn(__fmul_rn(f, d2), s0.z);
      }
      if (lead && a.image) store_pixel(a, b, px, py, d0, d1, d2);
      top_gradient<kLoss ? kModeLoss : kModeGrad>(a, b, px, py, true, d0, d1, d2, G0, G1, G2,
                                                   sq);
      float above = 1.0f;
      for (int k = a.split_k - 1; k > kb; --k) {
        const float4* sf = split_pixel(a, k, b, px, py);
        above = __fmul_rn(above, block_factor(sf[0], sf[1]));
      }
      G0 = __fmul_rn(G0, above);
      G1 = __fmul_rn(G1, above);
      G2 = __fmul_rn(G2, above);
    }
    if (kLoss && lead) {
      const double ws = warp_sum_d(sq);
      if (lane == 0) sm.loss_part[warp] = ws;
    }
  }

  // ---- pass 2: recomposite in forward order and accumulate gradients ------
  Prod Q;
  Q.init();
  // A single list from pass 1 is still in shared memory; otherwise the lists
  // are built again, in the same order (gathered from the mask, still held).
  if (kGather && n_chunks > 1) {
    __syncthreads();
    if (threadIdx.x == 0) {
      sm.gwc = 0;
      sm.gbo = 0;
    }
  }
  for (int ci = 0; ci < n_chunks; ++ci) {
    __syncthreads();  // the previous list's flush, or pass 1's image stores in sm.stage
    if (n_chunks > 1 || kSplitBwd) {
      if constexpr (kGather)
        count = gather_list(sm, recs, rg, a.W, a.H);
      else
        count = build_list(sm, recs, t1, t0 + ci * kChunk, tx0, ty0, a.W, a.H);
    }
    if (K.det) {
      for (int i = threadIdx.x; i < count * kParams; i += kThreads) (&sm.acc64[0][0])[i] = 0;
      for (int i = threadIdx.x; i < count; i += kThreads) sm.nf[i] = 0;
    } else {
      for (int i = threadIdx.x; i < count * kParams; i += kThreads) (&sm.acc[0][0])[i] = 0.0f;
    }
    __syncthreads();
    gradient_walk<kPrec>(sm, count, warp, lane, px, py, ptx, pty, active, K, P, Q, G0, G1, G2, r0,
                         r1, r2);
    __syncthreads();
    flush_grads<kDet>(sm, a, b, count);
  }

  if (kLoss && lead)
    scene_loss(a, b, local_tile, a.tiles_x * a.tile_rows, sm.loss_part, kWarps, sm.loss_part,
               &sm.is_last);
}

// Region kernel, for scenes whose whole list fits one chunk (T <= kChunk):
// one CTA per (scene, 2 x kRows tiles), the list binned once for all of the
// region's warp blocks, warps taking blocks from a shared counter. A warp that
// finishes a cheap block takes the next one instead of waiting for the CTA's
// busiest warp; there is no barrier between the list and the final flush.
// kTape: 0 none; 1 (render) also writes each pixel's running product to the
// pixel tape, and per region whether the tape stands in for the forward; 2
// (grad) reads the products back instead of running the forward walk, in
// regions whose flag allows it.
template <int Mode, int kPrec, int kRows, bool kDet = false, int kTape = 0>
__global__ void __launch_bounds__(kThreads, 4) dr_raster_region_kernel(RasterArgs a) {
  constexpr int kRB = kRegionCols * kRows * kBlocksPerTile;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RegionSmem<kRB>& sm = *reinterpret_cast<RegionSmem<kRB>*>(smem_raw);
  if (a.skip_flag && *a.skip_flag) return;

  // 1-D grid over (region, scene), scenes fastest and regions centre-out:
  // central regions carry the most overlapping geometry, and the light edge
  // regions then fill the tail of the launch.
  const int regions_x = (a.tiles_x + kRegionCols - 1) / kRegionCols;
  const int regions_y = (a.tile_rows + kRows - 1) / kRows;
  const int n_regions = regions_x * regions_y;
  const int b = (int)(blockIdx.x % (unsigned)a.B);
  const int rank = (int)(blockIdx.x / (unsigned)a.B);
  const int rx = center_out(rank % regions_x, regions_x);
  const int ry = center_out(rank / regions_x, regions_y);
  const int region = ry * regions_x + rx;
  const int rx0 = rx * kRegionCols * kTile;
  const int lrow0 = ry * kRows;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Consts K;
  K.sigma_eff = a.sigma_eff;
  K.inv_sigma = a.inv_sigma;
  K.det = kDet;  // deterministic sums (a.grads_fx set): a separate instantiation

  if (threadIdx.x == 0) sm.next_block = kWarps;
  const int count = build_region_list(sm, a, a.recs + (size_t)b * a.T, rx0, lrow0);
  const size_t flag_at = (size_t)b * n_regions + region;
  if (kTape == 1) {
    // The forward keeps render()'s semantics (a NaN-alpha triangle paints
    // NaN, raster.rs:49); the backward drops such a triangle (grad.rs:62). A
    // region that holds one has a different running product there: flag it.
    int nan_alpha = 0;
    for (int j = threadIdx.x; j < count; j += kThreads) nan_alpha |= sm.rec[j].alpha != sm.rec[j].alpha;
    nan_alpha = __syncthreads_or(nan_alpha);
    if (threadIdx.x == 0) a.tape_flags[flag_at] = nan_alpha;
  }
  bool from_tape = false;
  if (kTape == 2) from_tape = a.tape_flags[flag_at] == 0 && a.image == nullptr;

  // Blocks are taken at most once each, so no warp runs more than kRB
  // iterations.
  int blk = warp;
  for (int it = 0; it < kRB; ++it) {
    int x0, y0;
    region_block_origin(a, rx0, lrow0, blk, x0, y0);
    const int px = x0 + (lane & 7), py = y0 + (lane >> 3);
    const bool active = px < a.W && py < a.H;
    const float ptx = pixel_center(px, a.W), pty = pixel_center(py, a.H);
    float c0, c1, c2;
    scene_background(a, b, c0, c1, c2);
    Prod P;
    P.init();
    const size_t pix = ((size_t)b * a.H + py) * a.W + px;
    if (kTape == 2 && from_tape) {
      if (active) {
        const float4 t = a.tape[pix];
        P.m = t.x;
        P.e = __float_as_int(t.y);
        P.z0 = __float_as_int(t.z);
        P.zn = __float_as_int(t.w);
      }
    } else {
      forward_walk<Mode, kPrec, RegionSmem<kRB>, Mode != kModeRender || kTape == 1>(
          sm, count, blk, px, py, ptx, pty, active, K, c0, c1, c2, P);
    }
    if (kTape == 1 && active)
      a.tape[pix] = make_float4(P.m, __int_as_float(P.e), __int_as_float(P.z0), __int_as_float(P.zn));
    if (a.image) store_block(a, b, x0, y0, lane, c0, c1, c2, sm.stage[warp]);
    if (Mode != kModeRender) {
      float G0, G1, G2;
      double sq;
      top_gradient<Mode>(a, b, px, py, active, c0, c1, c2, G0, G1, G2, sq);
      if (Mode == kModeLoss) {
        const double ws = warp_sum_d(sq);
        if (lane == 0) sm.loss_part[blk] = ws;
      }
      float r0, r1, r2;
      scene_background(a, b, r0, r1, r2);
      Prod Q;
      Q.init();
      gradient_walk<kPrec>(sm, count, blk, lane, px, py, ptx, pty, active, K, P, Q, G0, G1, G2,
                           r0, r1, r2);
    }
    int next = 0;
    if (lane == 0) next = atomicAdd(&sm.next_block, 1);
    blk = __shfl_sync(0xffffffffu, next, 0);
    if (blk >= kRB) break;
  }

  if (Mode == kModeRender) return;
  __syncthreads();
  flush_grads<kDet>(sm, a, b, count);
  if (Mode == kModeLoss)
    scene_loss(a, b, region, n_regions, sm.loss_part, kRB, sm.loss_part, &sm.is_last);
}

// ---------------------------------------------------------------------------
// MSE (canvas.rs:45-59) and Adam (optim.rs:40-60 + fit.rs:399-424)
// ---------------------------------------------------------------------------

// One block per (chunk of kMseChunk values, image): f32 differences squared
// and summed in f64 (canvas.rs:45-59). Each block writes its partial; the
// image's last block sums the partials in chunk order, so the result does not
// depend on block scheduling.
constexpr int kMseChunk = 8192;
__global__ void dr_mse_kernel(const float* __restrict__ img, const float* __restrict__ tgt,
                              long long n, int vec, double* __restrict__ partials,
                              unsigned* __restrict__ counters, float* __restrict__ losses) {
  __shared__ double part[32];  // one per warp of a block of up to 1024 threads
  __shared__ int is_last;
  const int b = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_warps = (int)(blockDim.x >> 5);
  const long long c0 = (long long)blockIdx.x * kMseChunk;
  const long long c1 = min(c0 + (long long)kMseChunk, n);
  const float* x = img + (size_t)b * n;
  const float* y = tgt + (size_t)b * n;
  double s = 0.0;
  if (vec) {  // n % 4 == 0 and 16-byte aligned images: chunks start on float4s
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* y4 = reinterpret_cast<const float4*>(y);
    for (long long i = c0 / 4 + threadIdx.x; i < c1 / 4; i += blockDim.x) {
      const float4 u = x4[i], w = y4[i];
      const double d0 = (double)__fsub_rn(u.x, w.x), d1 = (double)__fsub_rn(u.y, w.y);
      const double d2 = (double)__fsub_rn(u.z, w.z), d3 = (double)__fsub_rn(u.w, w.w);
      s += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
    }
  } else {
    for (long long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
      const double d = (double)__fsub_rn(x[i], y[i]);
      s += d * d;
    }
  }
  s = warp_sum_d(s);
  if (lane == 0) part[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < n_warps; ++w) t += part[w];
    partials[(size_t)b * gridDim.x + blockIdx.x] = t;
    __threadfence();
    is_last = atomicAdd(&counters[b], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  double t = 0.0;
  for (unsigned i = threadIdx.x; i < gridDim.x; i += blockDim.x)
    t += *((volatile double*)&partials[(size_t)b * gridDim.x + i]);
  t = warp_sum_d(t);
  __syncthreads();  // part[] above has been read
  if (lane == 0) part[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < n_warps; ++w) tot += part[w];
    losses[b] = (float)(tot / (double)n);
    counters[b] = 0;
  }
}

// Adam::step for element i (optim.rs:40-60) with fit.rs's per-parameter rate
// and projection; IEEE division and square root as the reference rounds them.
__device__ __forceinline__ float adam_one(const AdamArgs& a, long long i, float p, float g,
                                          float& m, float& v) {
  const int cls = (int)(i % kParams);
  const float lr = cls < 6 ? a.lr_pos : (cls < 9 ? a.lr_color : a.lr_alpha);
  m = __fadd_rn(__fmul_rn(a.beta1, m), __fmul_rn(a.one_minus_beta1, g));
  v = __fadd_rn(__fmul_rn(a.beta2, v), __fmul_rn(__fmul_rn(a.one_minus_beta2, g), g));
  const float m_hat = __fdiv_rn(m, a.bc1);
  const float v_hat = __fdiv_rn(v, a.bc2);
  p = __fsub_rn(p, __fdiv_rn(__fmul_rn(lr, m_hat), __fadd_rn(__fsqrt_rn(v_hat), a.eps)));
  if (a.project) {
    if (p != p) p = 0.5f;
    if (cls < 6) p = rclamp(p, -0.25f, 1.25f);
    else if (cls < 9) p = rclamp(p, 0.0f, 1.0f);
    else p = rclamp(p, 1e-3f, 0.999f);
  }
  return p;
}

__global__ void dr_adam_kernel(AdamArgs a) {
  if (a.skip_flag && *a.skip_flag) return;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  if (a.copy_flag && *a.copy_flag) a.copy_dst[i] = a.params[i];
  if (a.run_flag && !*a.run_flag) return;
  float m = a.m[i], v = a.v[i];
  const float p = adam_one(a, i, a.params[i], a.grads[i], m, v);
  a.m[i] = m;
  a.v[i] = v;
  a.params[i] = p;
}

// Four consecutive elements per thread with 16-byte loads and stores (n a
// multiple of 4, every array 16-byte aligned); the same per-element update.
__global__ void dr_adam4_kernel(AdamArgs a) {
  if (a.skip_flag && *a.skip_flag) return;
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q * 4 >= a.n) return;
  float4 P = reinterpret_cast<const float4*>(a.params)[q];
  if (a.copy_flag && *a.copy_flag) reinterpret_cast<float4*>(a.copy_dst)[q] = P;
  if (a.run_flag && !*a.run_flag) return;
  const float4 G = reinterpret_cast<const float4*>(a.grads)[q];
  float4 M = reinterpret_cast<const float4*>(a.m)[q];
  float4 V = reinterpret_cast<const float4*>(a.v)[q];
  const long long i = q * 4;
  P.x = adam_one(a, i, P.x, G.x, M.x, V.x);
  P.y = adam_one(a, i + 1, P.y, G.y, M.y, V.y);
  P.z = adam_one(a, i + 2, P.z, G.z, M.z, V.z);
  P.w = adam_one(a, i + 3, P.w, G.w, M.w, V.w);
  reinterpret_cast<float4*>(a.m)[q] = M;
  reinterpret_cast<float4*>(a.v)[q] = V;
  reinterpret_cast<float4*>(a.params)[q] = P;
}

// dr_fit's Adam step (the per-element update of dr_adam_kernel) fused with
// the next iteration's set-up: one thread per triangle updates its 10
// parameters, clears their gradients for the next raster launch and writes
// the triangle's record from the updated parameters. Every load is issued
// before any store (the arrays could alias as far as the compiler knows), so
// the thread waits for memory once rather than once per parameter.
__global__ void __launch_bounds__(kSetupThreads) dr_fit_adam_setup_kernel(
    AdamArgs a, float* __restrict__ grads, int T, int W, int H, float next_sigma,
    TriRec* __restrict__ recs) {
  const int t = blockIdx.x * kSetupThreads + (int)threadIdx.x;
  if (t >= T) return;
  const long long base = (long long)t * kParams;
  float p[kParams], m[kParams], v[kParams], g[kParams];
#pragma unroll
  for (int j = 0; j < kParams; ++j) p[j] = a.params[base + j];
  if (a.copy_flag && *a.copy_flag) {
#pragma unroll
    for (int j = 0; j < kParams; ++j) a.copy_dst[base + j] = p[j];
  }
  if (a.run_flag && !*a.run_flag) return;
#pragma unroll
  for (int j = 0; j < kParams; ++j) {
    m[j] = a.m[base + j];
    v[j] = a.v[base + j];
    g[j] = grads[base + j];
  }
#pragma unroll
  for (int j = 0; j < kParams; ++j) p[j] = adam_one(a, base + j, p[j], g[j], m[j], v[j]);
#pragma unroll
  for (int j = 0; j < kParams; ++j) {
    a.params[base + j] = p[j];
    a.m[base + j] = m[j];
    a.v[base + j] = v[j];
    grads[base + j] = 0.0f;
  }
  if (recs) recs[t] = make_record(p, 0, W, H, next_sigma, 1);
}

// ---------------------------------------------------------------------------
// Fit bookkeeping (Fitter::step, fit.rs:243-288), one thread, no host sync
// ---------------------------------------------------------------------------

__global__ void dr_fit_init_kernel(FitState* st) {
  st->loss = 0.0f;
  st->best_loss = __int_as_float(0x7f800000);
  st->count = 0;
  st->since = 0;
  st->best_iter = 0;
  st->stopped = 0;
  st->stop_reason = 0;
  st->run_adam = 0;
  st->copy_best = 0;
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

size_t raster_smem_bytes() { return sizeof(Smem); }

cudaError_t launch_fit_init(FitState* st, cudaStream_t s) {
  dr_fit_init_kernel<<<1, 1, 0, s>>>(st);
  return cudaGetLastError();
}



cudaError_t launch_fit_adam_setup(const AdamArgs& a, float* grads, int T, int W, int H,
                                  float next_sigma, TriRec* recs, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const int blocks = (T + kSetupThreads - 1) / kSetupThreads;
  dr_fit_adam_setup_kernel<<<blocks, kSetupThreads, 0, s>>>(a, grads, T, W, H, next_sigma, recs);
  return cudaGetLastError();
}

cudaError_t launch_setup(const float* params, int BT, int W, int H, float sigma,
                         int tape_semantics, TriRec* recs, cudaStream_t s, int4* boxes) {
  if (BT == 0) return cudaSuccess;
  const int blocks = (BT + kSetupThreads - 1) / kSetupThreads;
  dr_setup_kernel<<<blocks, kSetupThreads, 0, s>>>(params, BT, W, H, sigma, tape_semantics, recs,
                                                   boxes);
  return cudaGetLastError();
}

static_assert(sizeof(Smem) <= 48 * 1024, "raster smem must fit the default 48 KB limit");
// Four CTAs an SM (the launch bound), each with the 1 KB the system reserves.
static_assert(4 * (sizeof(Smem) + 1024) <= 227 * 1024, "four tile CTAs must fit an SM");

static_assert(sizeof(RegionSmem<32>) <= 48 * 1024, "region smem must fit the default 48 KB limit");

// SMs of the current device (cached per device).
static int device_sms() {
  static std::atomic<int> sms[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  int n = sms[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// The region kernel when the whole list fits one chunk (T <= kChunk) and the
// launch fills at least two waves of its CTAs (4 per SM): a region CTA works
// two tiles, so with fewer CTAs the slowest ones set the time and the tile
// kernel's finer grid, launched in rings, is faster. Measured at 256^2,
// T = 128 (loss + backward): 6 scenes (768 region CTAs) 0.142 ms on the tile
// kernel against 0.171 on the region kernel, 8 scenes (1024) 0.177 against
// 0.187, 11 scenes (1408) 0.232 on both, 12 scenes (1536) 0.251 against 0.247,
// 16 scenes 0.321 against 0.306; at 128^2 with 32 scenes (1024 region CTAs)
// 0.223 against 0.237 (T = 128) and 0.097 against 0.095 (T = 32). Otherwise
// the tile kernel.
// Regions of 2 x 1 tiles: a 2 x 2 region CTA averaged ~150 us at the headline
// size (3.5 waves), and SMs that ran out of CTAs idled for up to 100 us while
// the last ones finished. Halving the unit halves that tail; the list is
// binned twice as often, for about 2 % more work.
constexpr int kRegionRows = 1;
static long long region_ctas(int B, int tiles_x, int tile_rows) {
  return (long long)((tiles_x + kRegionCols - 1) / kRegionCols) *
         ((tile_rows + kRegionRows - 1) / kRegionRows) * B;
}
static bool use_region_kernel(int B, int T, int tiles_x, int tile_rows) {
  return T <= kChunk && region_ctas(B, tiles_x, tile_rows) >= 8LL * device_sms();
}
int raster_path(int B, int T, int tiles_x, int tile_rows, int split_k) {
  if (split_k > 1) return 2;
  if (use_region_kernel(B, T, tiles_x, tile_rows)) return 1;
  return T > kChunk && T <= kGatherMaxT ? 3 : 0;
}
template <int Mode, int kPrec>
static cudaError_t launch_mode(const RasterArgs& a, int n_tiles, cudaStream_t s) {
  constexpr int kRows = kRegionRows;
  constexpr int kRB = kRegionCols * kRows * kBlocksPerTile;
  constexpr bool kGrads = Mode != kModeRender;
  const bool det = kGrads && a.grads_fx != nullptr;
  const long long n_ctas = region_ctas(a.B, a.tiles_x, a.tile_rows);
  if (use_region_kernel(a.B, a.T, a.tiles_x, a.tile_rows)) {
    if (n_ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const unsigned grid = (unsigned)n_ctas;
    if constexpr (Mode == kModeRender || Mode == kModeGrad) {
      if (a.tape) {  // the pixel tape: written by a render, read by a grad call
        constexpr int kTape = Mode == kModeRender ? 1 : 2;
        if (det)
          dr_raster_region_kernel<Mode, kPrec, kRows, kGrads, kTape>
              <<<grid, kThreads, sizeof(RegionSmem<kRB>), s>>>(a);
        else
          dr_raster_region_kernel<Mode, kPrec, kRows, false, kTape>
              <<<grid, kThreads, sizeof(RegionSmem<kRB>), s>>>(a);
        return cudaGetLastError();
      }
    }
    if (det)
      dr_raster_region_kernel<Mode, kPrec, kRows, kGrads>
          <<<grid, kThreads, sizeof(RegionSmem<kRB>), s>>>(a);
    else
      dr_raster_region_kernel<Mode, kPrec, kRows><<<grid, kThreads, sizeof(RegionSmem<kRB>), s>>>(a);
    return cudaGetLastError();
  }
  dim3 grid(n_tiles, a.B);
  const bool gather = a.T > kChunk && a.T <= kGatherMaxT;
  RasterArgs t = a;
  t.tile_rings = (long long)n_tiles * a.B > 4LL * device_sms();  // more than one wave
  if (gather && det)
    dr_raster_kernel<Mode, kPrec, true, kGrads><<<grid, kThreads, sizeof(Smem), s>>>(t);
  else if (gather)
    dr_raster_kernel<Mode, kPrec, true><<<grid, kThreads, sizeof(Smem), s>>>(t);
  else if (det)
    dr_raster_kernel<Mode, kPrec, false, kGrads><<<grid, kThreads, sizeof(Smem), s>>>(t);
  else
    dr_raster_kernel<Mode, kPrec><<<grid, kThreads, sizeof(Smem), s>>>(t);
  return cudaGetLastError();
}

template <int kPrec>
static cudaError_t launch_prec(int mode, const RasterArgs& a, int n_tiles, cudaStream_t s) {
  switch (mode) {
    case kModeRender: return launch_mode<kModeRender, kPrec>(a, n_tiles, s);
    case kModeLoss: return launch_mode<kModeLoss, kPrec>(a, n_tiles, s);
    case kModeGrad: return launch_mode<kModeGrad, kPrec>(a, n_tiles, s);
  }
  return cudaErrorInvalidValue;
}

// n_tiles: the 16x16 tiles per scene the launch covers (a.tiles_x per covered
// tile row). Either kernel uses at most n_tiles loss partials per scene.
int raster_split_blocks(int B, int T, int n_tiles) {
  const long long ctas = (long long)B * n_tiles;
  const int sms = device_sms();
  if (ctas >= 2LL * sms || T < 64) return 1;
  const long long want = (4LL * sms + ctas - 1) / ctas;
  long long k = want < 8 ? want : 8;
  if (k > T / 32) k = T / 32;
  return k < 2 ? 1 : (int)k;
}

// Split backward: per (tile, block) the combine and the block's gradient pass,
// for the loss or for an upstream image gradient.
template <int kPrec>
static cudaError_t launch_split_bwd(int mode, const RasterArgs& a, dim3 grid, cudaStream_t s) {
  const bool det = a.grads_fx != nullptr;
  if (mode == kModeLoss && det)
    dr_raster_kernel<kModeSplitBwd, kPrec, false, true><<<grid, kThreads, sizeof(Smem), s>>>(a);
  else if (mode == kModeLoss)
    dr_raster_kernel<kModeSplitBwd, kPrec><<<grid, kThreads, sizeof(Smem), s>>>(a);
  else if (det)
    dr_raster_kernel<kModeSplitBwdGrad, kPrec, false, true>
        <<<grid, kThreads, sizeof(Smem), s>>>(a);
  else
    dr_raster_kernel<kModeSplitBwdGrad, kPrec><<<grid, kThreads, sizeof(Smem), s>>>(a);
  return cudaGetLastError();
}

template <int kPrec>
static cudaError_t launch_split_prec(int mode, const RasterArgs& a, int n_tiles, cudaStream_t s) {
  RasterArgs f = a;
  f.image = nullptr;  // the backward's first block writes the image
  const dim3 grid(n_tiles, a.B, a.split_k);
  dr_raster_kernel<kModeSplitFwd, kPrec><<<grid, kThreads, sizeof(Smem), s>>>(f);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_split_bwd<kPrec>(mode, a, grid, s);
}

cudaError_t launch_raster_split(int mode, const RasterArgs& args, int n_tiles, int k, float4* split,
                                cudaStream_t s) {
  if (args.B == 0 || n_tiles == 0) return cudaSuccess;
  if (args.tiles_x <= 0 || k < 1 || k > 65535 || !split ||
      (mode != kModeLoss && mode != kModeGrad) || args.tile_row0 != 0 || args.tile_row_step != 1)
    return cudaErrorInvalidValue;
  RasterArgs a = args;
  a.tile_rows = n_tiles / a.tiles_x;
  a.split_k = k;
  a.split_base = 0;
  a.split_state = split;
  switch (a.precision) {
    case kPrecRef: return launch_split_prec<kPrecRef>(mode, a, n_tiles, s);
    case kPrecStrict: return launch_split_prec<kPrecStrict>(mode, a, n_tiles, s);
    case kPrecFast: return launch_split_prec<kPrecFast>(mode, a, n_tiles, s);
  }
  return cudaErrorInvalidValue;
}

template <int kPrec>
static cudaError_t launch_block_prec(int phase, int mode, const RasterArgs& a, int n_tiles,
                                     cudaStream_t s) {
  const dim3 grid(n_tiles, a.B, 1);
  if (phase == 0) {
    RasterArgs f = a;
    f.image = nullptr;
    dr_raster_kernel<kModeSplitFwd, kPrec><<<grid, kThreads, sizeof(Smem), s>>>(f);
    return cudaGetLastError();
  }
  return launch_split_bwd<kPrec>(mode, a, grid, s);
}

cudaError_t launch_triangle_block(int phase, int mode, const RasterArgs& args, int n_tiles,
                                  int n_blocks, int block, float4* state, cudaStream_t s) {
  if (args.B == 0 || n_tiles == 0) return cudaSuccess;
  if (args.tiles_x <= 0 || n_blocks < 1 || block < 0 || block >= n_blocks || !state ||
      (phase == 1 && mode != kModeLoss && mode != kModeGrad) || args.tile_row0 != 0 ||
      args.tile_row_step != 1)
    return cudaErrorInvalidValue;
  RasterArgs a = args;
  a.tile_rows = n_tiles / a.tiles_x;
  a.split_k = n_blocks;
  a.split_base = block;
  a.split_state = state;
  switch (a.precision) {
    case kPrecRef: return launch_block_prec<kPrecRef>(phase, mode, a, n_tiles, s);
    case kPrecStrict: return launch_block_prec<kPrecStrict>(phase, mode, a, n_tiles, s);
    case kPrecFast: return launch_block_prec<kPrecFast>(phase, mode, a, n_tiles, s);
  }
  return cudaErrorInvalidValue;
}

// Deterministic mode's last step, one thread per (scene, triangle): its ten
// fixed-point sums to f32 (one rounding from the 64-bit integer, then an exact
// power-of-two scale), or NaN / an infinity where a flag bit is set; the sums
// and flags are cleared for the next launch.
__global__ void dr_det_finalize_kernel(long long* __restrict__ fx, int* __restrict__ nf,
                                       float* __restrict__ g, long long n_tris) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= n_tris) return;
  const int f = nf[t];
  nf[t] = 0;
#pragma unroll
  for (int p = 0; p < kParams; ++p) {
    const long long i = t * kParams + p;
    const int bits = (f >> (3 * p)) & 7;
    float v = __fmul_rn(__ll2float_rn(fx[i]), kDetInv);
    if ((bits & 1) || (bits & 6) == 6) v = __int_as_float(0x7fc00000);
    else if (bits & 2) v = __int_as_float(0x7f800000);
    else if (bits & 4) v = __int_as_float(0xff800000);
    g[i] = v;
    fx[i] = 0;
  }
}

cudaError_t launch_det_finalize(long long* fx, int* nf, float* grads, long long n, cudaStream_t s) {
  const long long n_tris = n / kParams;
  if (n_tris == 0) return cudaSuccess;
  const long long blocks = (n_tris + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  dr_det_finalize_kernel<<<(unsigned)blocks, 256, 0, s>>>(fx, nf, grads, n_tris);
  return cudaGetLastError();
}

// Per (scene, region) flags of the pixel tape for a launch over B scenes of
// tiles_x x tile_rows tiles: how many regions the region kernel uses.
long long tape_regions(int tiles_x, int tile_rows) {
  return (long long)((tiles_x + kRegionCols - 1) / kRegionCols) *
         ((tile_rows + kRegionRows - 1) / kRegionRows);
}

cudaError_t launch_raster(int mode, const RasterArgs& args, int n_tiles, cudaStream_t s) {
  if (args.B == 0 || n_tiles == 0) return cudaSuccess;
  if (args.tiles_x <= 0) return cudaErrorInvalidValue;
  RasterArgs a = args;
  a.tile_rows = n_tiles / a.tiles_x;
  switch (a.precision) {
    case kPrecRef: return launch_prec<kPrecRef>(mode, a, n_tiles, s);
    case kPrecStrict: return launch_prec<kPrecStrict>(mode, a, n_tiles, s);
    case kPrecFast: return launch_prec<kPrecFast>(mode, a, n_tiles, s);
  }
  return cudaErrorInvalidValue;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

size_t mse_partials_per_image(long long n) { return (size_t)((n + kMseChunk - 1) / kMseChunk); }

// partials: B * mse_partials_per_image(n) doubles; counters: B, zero between launches.
cudaError_t launch_mse(const float* img, const float* tgt, int B, long long n, float* losses,
                       double* partials, unsigned* counters, cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  if (n == 0) return cudaMemsetAsync(losses, 0xff, sizeof(float) * (size_t)B, s);  // 0/0: NaN
  const unsigned chunks = (unsigned)mse_partials_per_image(n);
  static_assert(kMseChunk % 4 == 0, "float4 chunks");
  const int vec = n % 4 == 0 && aligned16(img) && aligned16(tgt);
  for (int b0 = 0; b0 < B; b0 += 65535) {  // gridDim.y limit
    const int nb = min(B - b0, 65535);
    dim3 grid(chunks, nb);
    dr_mse_kernel<<<grid, 256, 0, s>>>(img + (size_t)b0 * n, tgt + (size_t)b0 * n, n, vec,
                                       partials, counters, losses + b0);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_adam(const AdamArgs& a, cudaStream_t s) {
  if (a.n == 0) return cudaSuccess;
  const int threads = 256;
  const bool vec = a.n % 4 == 0 && aligned16(a.params) && aligned16(a.m) && aligned16(a.v) &&
                   aligned16(a.grads) && (!a.copy_dst || aligned16(a.copy_dst));
  if (vec) {
    const long long blocks = (a.n / 4 + threads - 1) / threads;
    dr_adam4_kernel<<<(unsigned)blocks, threads, 0, s>>>(a);
  } else {
    const long long blocks = (a.n + threads - 1) / threads;
    dr_adam_kernel<<<(unsigned)blocks, threads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace dr

namespace dr {
size_t tri_rec_bytes() { return sizeof(TriRec); }
}  // namespace dr
