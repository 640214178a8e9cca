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

#include <cstdint>
#include <cstdio>

#include "dr_device.cuh"
#include "dr_internal.h"

namespace dr {

constexpr int kTile = 16;
constexpr int kThreads = 256;
constexpr int kChunk = 128;  // triangles binned per round (<= kThreads)
constexpr int kWarps = kThreads / 32;
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

__global__ void dr_setup_kernel(const float* __restrict__ params, int BT, int W, int H, float sigma,
                                int tape_semantics, TriRec* __restrict__ recs) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= BT) return;
  const float* p = params + (size_t)i * kParams;
  float v[6];
#pragma unroll
  for (int j = 0; j < 6; ++j) v[j] = p[j];
  float col[3] = {p[6], p[7], p[8]};
  float raw_alpha = p[9];

  TriRec r;
  for (int j = 0; j < 6; ++j) r.v[j] = v[j];
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

  // Edge vectors and squared lengths with the reference's rounding.
  for (int k = 0; k < 3; ++k) {
    int a = k, b = (k + 1) % 3;
    float ex = __fsub_rn(v[2 * b], v[2 * a]);
    float ey = __fsub_rn(v[2 * b + 1], v[2 * a + 1]);
    r.e[2 * k] = ex;
    r.e[2 * k + 1] = ey;
    r.len2[k] = __fadd_rn(__fmul_rn(ex, ex), __fmul_rn(ey, ey));
  }

  // Edge-line equations for the conservative fast paths, in double. Valid
  // only for a clearly non-degenerate triangle with a finite alpha.
  double ex0 = (double)v[2] - v[0], ey0 = (double)v[3] - v[1];
  double ex2 = (double)v[4] - v[0], ey2 = (double)v[5] - v[1];
  double area2 = ex0 * ey2 - ey0 * ex2;
  double maxl2 = 0.0, maxabs = 0.0;
  for (int k = 0; k < 3; ++k) {
    double l2 = (double)r.e[2 * k] * r.e[2 * k] + (double)r.e[2 * k + 1] * r.e[2 * k + 1];
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
    r.n[2 * k] = (float)nx;
    r.n[2 * k + 1] = (float)ny;
    r.c[k] = (float)(-(nx * v[2 * a] + ny * v[2 * a + 1]));
  }
  // Slack for evaluating n.p + c in f32 and for the reference's own f32
  // distance rounding: a few ulps of the largest magnitude involved.
  r.margin = (float)(4e-6 * (2.0 + maxabs));
  if (fast) flags |= kFastOk;
  r.flags = flags;
  r.pad[0] = r.pad[1] = r.pad[2] = 0;

  float4* dst = reinterpret_cast<float4*>(recs + i);
  const float4* src = reinterpret_cast<const float4*>(&r);
#pragma unroll
  for (int j = 0; j < kRecWords / 4; ++j) dst[j] = src[j];
}

// ---------------------------------------------------------------------------
// Raster kernel
// ---------------------------------------------------------------------------

struct Smem {
  TriRec rec[kChunk];
  int eflags[kChunk];
  int kidx[kChunk];
  float acc[kChunk][kParams];
  int warp_count[kWarps];
  double loss_part[kWarps];
  int is_last;
};

// Bin triangles [c0, c0 + kChunk) of scene b against tile [tx0,tx1)x[ty0,ty1)
// into shared memory, preserving triangle order. Returns the entry count.
__device__ int build_list(Smem& sm, const TriRec* __restrict__ recs, int T, int c0, int tx0,
                          int ty0, int tx1, int ty1, int W, int H, float rej, float acc) {
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int k = c0 + (int)threadIdx.x;
  bool keep = false;
  int ef = 0;
  const TriRec* r = recs + k;
  if ((int)threadIdx.x < kChunk && k < T) {
    int flags = r->flags;
    int bx0 = r->bbox[0], by0 = r->bbox[1], bx1 = r->bbox[2], by1 = r->bbox[3];
    keep = (flags & kLive) && bx0 < tx1 && bx1 > tx0 && by0 < ty1 && by1 > ty0;
    if (keep) {
      if (bx0 <= tx0 && bx1 >= tx1 && by0 <= ty0 && by1 >= ty1) ef |= kBoxCoversTile;
      if (flags & kFastOk) {
        float cx0 = pixel_center(tx0, W), cx1 = pixel_center(tx1 - 1, W);
        float cy0 = pixel_center(ty0, H), cy1 = pixel_center(ty1 - 1, H);
        float m = r->margin;
        float mn_all = __int_as_float(0x7f800000);
        bool far_out = false;
#pragma unroll
        for (int e = 0; e < 3; ++e) {
          float nx = r->n[2 * e], ny = r->n[2 * e + 1], c = r->c[e];
          float l00 = __fmaf_rn(nx, cx0, __fmaf_rn(ny, cy0, c));
          float l10 = __fmaf_rn(nx, cx1, __fmaf_rn(ny, cy0, c));
          float l01 = __fmaf_rn(nx, cx0, __fmaf_rn(ny, cy1, c));
          float l11 = __fmaf_rn(nx, cx1, __fmaf_rn(ny, cy1, c));
          float lmax = fmaxf(fmaxf(l00, l10), fmaxf(l01, l11));
          float lmin = fminf(fminf(l00, l10), fminf(l01, l11));
          if (lmax < -(rej + m)) far_out = true;
          mn_all = fminf(mn_all, lmin);
        }
        if (far_out) keep = false;
        if (mn_all > acc + m) ef |= kTileInside;
      }
    }
  }
  unsigned ballot = __ballot_sync(0xffffffffu, keep);
  if (lane == 0) sm.warp_count[warp] = __popc(ballot);
  __syncthreads();
  int base = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    int cnt = sm.warp_count[w];
    base += (w < warp) ? cnt : 0;
    total += cnt;
  }
  if (keep) {
    int slot = base + __popc(ballot & ((1u << lane) - 1u));
    sm.kidx[slot] = k;
    sm.eflags[slot] = ef;
    const float4* src = reinterpret_cast<const float4*>(r);
    float4* dst = reinterpret_cast<float4*>(&sm.rec[slot]);
#pragma unroll
    for (int j = 0; j < kRecWords / 4; ++j) dst[j] = src[j];
  }
  __syncthreads();
  return total;
}

// Per-pixel evaluation of one list entry: returns true when the pair
// contributes (w > MIN_WEIGHT) and fills w, cov and (if want_geo) the
// nearest-edge data. Mirrors raster.rs:53-59 with the box test of
// raster.rs:144-168 and the conservative fast paths described in
// dr_device.cuh.
struct PairEval {
  float w, cov;
  bool band;  // full geometry evaluated (else cov == 1 exactly)
  SdResult g;
};

__device__ __forceinline__ bool eval_pair(const TriRec& r, int ef, int px, int py, float ptx,
                                          float pty, float sigma_eff, float rej, float acc,
                                          PairEval& out) {
  if (!(ef & kBoxCoversTile)) {
    if (px < r.bbox[0] || px >= r.bbox[2] || py < r.bbox[1] || py >= r.bbox[3]) return false;
  }
  if (ef & kTileInside) {
    out.cov = 1.0f;
    out.w = r.alpha;
    out.band = false;
    return true;  // alpha > MIN_WEIGHT is guaranteed by the set-up cull
  }
  if (r.flags & kFastOk) {
    float l0 = __fmaf_rn(r.n[0], ptx, __fmaf_rn(r.n[1], pty, r.c[0]));
    float l1 = __fmaf_rn(r.n[2], ptx, __fmaf_rn(r.n[3], pty, r.c[1]));
    float l2 = __fmaf_rn(r.n[4], ptx, __fmaf_rn(r.n[5], pty, r.c[2]));
    float mn = fminf(fminf(l0, l1), l2);
    if (mn < -(rej + r.margin)) return false;
    if (mn > acc + r.margin) {
      out.cov = 1.0f;
      out.w = r.alpha;
      out.band = false;
      return true;
    }
  }
  out.g = signed_distance_ref(r.v, r.e, r.len2, ptx, pty);
  out.cov = sigmoid_ref(__fdiv_rn(out.g.sd, sigma_eff));
  out.w = __fmul_rn(r.alpha, out.cov);
  out.band = true;
  return !(out.w <= kMinWeight);
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
    if (f == 0.0f) {
      z0 = k;
      m = 1.0f;
      e = 0;
    } else if (f != f) {
      zn = k;
      m = 1.0f;
      e = 0;
    } else {
      m = __fmul_rn(m, f);
      if (m < kRenormInv) {
        m = __fmul_rn(m, kRenorm);
        e += 1;
      }
    }
  }
};

// A_k = prod over layers above k of (1 - w), given the full product P (after
// the last layer) and the running product Q (through layer k).
__device__ __forceinline__ float attenuation(const Prod& P, const Prod& Q, int k) {
  if (k < P.zn) return __int_as_float(0x7fc00000);
  if (k < P.z0) return 0.0f;
  float ratio = __fdiv_rn(P.m, Q.m);
  int de = P.e - Q.e;
  if (de == 0) return ratio;
  if (de == 1) return __fmul_rn(ratio, kRenormInv);
  if (de == 2) return __fmul_rn(__fmul_rn(ratio, kRenormInv), kRenormInv);
  return 0.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ size_t pix_index(int layout, int b, int ch, int px, int py, int W,
                                            int H) {
  if (layout == kLayoutBCHW) return (((size_t)b * 3 + ch) * H + py) * W + px;
  return (((size_t)b * H + py) * W + px) * 3 + ch;
}

template <int Mode>
__global__ void __launch_bounds__(kThreads) dr_raster_kernel(RasterArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  if (a.skip_flag && *a.skip_flag) return;

  const int b = blockIdx.y;
  const int local_tile = blockIdx.x;
  const int tile_col = local_tile % a.tiles_x;
  const int tile_row = a.tile_row0 + (local_tile / a.tiles_x) * a.tile_row_step;
  const int tx0 = tile_col * kTile, ty0 = tile_row * kTile;
  const int tx1 = min(tx0 + kTile, a.W), ty1 = min(ty0 + kTile, a.H);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Each warp covers an 8x4 block of the 16x16 tile.
  const int px = tx0 + (warp & 1) * 8 + (lane & 7);
  const int py = ty0 + (warp >> 1) * 4 + (lane >> 3);
  const bool active = px < a.W && py < a.H;
  const float ptx = pixel_center(px, a.W), pty = pixel_center(py, a.H);

  const TriRec* recs = a.recs + (size_t)b * a.T;
  float bg0 = a.bg3[0], bg1 = a.bg3[1], bg2 = a.bg3[2];
  if (a.bg_dev) {
    const float* q = a.bg_dev + (a.bg_per_scene ? 3 * b : 0);
    bg0 = q[0];
    bg1 = q[1];
    bg2 = q[2];
  }
  const float sig = a.sigma_eff;
  const float rej = a.rej, acc = a.acc;
  const int n_chunks = (a.T + kChunk - 1) / kChunk;

  // ---- pass 1: forward composite ------------------------------------------
  float c0 = bg0, c1 = bg1, c2 = bg2;
  Prod P;
  P.init();
  int count = 0;
  for (int ci = 0; ci < n_chunks; ++ci) {
    count = build_list(sm, recs, a.T, ci * kChunk, tx0, ty0, tx1, ty1, a.W, a.H, rej, acc);
    if (active) {
      for (int j = 0; j < count; ++j) {
        const TriRec& r = sm.rec[j];
        PairEval pe;
        if (!eval_pair(r, sm.eflags[j], px, py, ptx, pty, sig, rej, acc, pe)) continue;
        float w = pe.w, om = __fsub_rn(1.0f, w);
        c0 = __fadd_rn(__fmul_rn(r.color[0], w), __fmul_rn(c0, om));
        c1 = __fadd_rn(__fmul_rn(r.color[1], w), __fmul_rn(c1, om));
        c2 = __fadd_rn(__fmul_rn(r.color[2], w), __fmul_rn(c2, om));
        if (Mode != kModeRender) P.mul(om, sm.kidx[j]);
      }
    }
    if (ci + 1 < n_chunks) __syncthreads();
  }

  if (a.image && active) {
    a.image[pix_index(a.layout, b, 0, px, py, a.W, a.H)] = c0;
    a.image[pix_index(a.layout, b, 1, px, py, a.W, a.H)] = c1;
    a.image[pix_index(a.layout, b, 2, px, py, a.W, a.H)] = c2;
  }
  if (Mode == kModeRender) return;

  // ---- loss and the gradient reaching the top of the stack ----------------
  float G0 = 0.f, G1 = 0.f, G2 = 0.f;
  double sq = 0.0;
  if (active) {
    float o0 = a.other[pix_index(a.layout, b, 0, px, py, a.W, a.H)];
    float o1 = a.other[pix_index(a.layout, b, 1, px, py, a.W, a.H)];
    float o2 = a.other[pix_index(a.layout, b, 2, px, py, a.W, a.H)];
    if (Mode == kModeLoss) {
      float d0 = __fsub_rn(c0, o0), d1 = __fsub_rn(c1, o1), d2 = __fsub_rn(c2, o2);
      sq = (double)d0 * d0 + (double)d1 * d1 + (double)d2 * d2;
      G0 = __fmul_rn(a.grad_scale, d0);  // grad.rs:112-114
      G1 = __fmul_rn(a.grad_scale, d1);
      G2 = __fmul_rn(a.grad_scale, d2);
    } else {
      G0 = o0;
      G1 = o1;
      G2 = o2;
    }
  }
  if (Mode == kModeLoss) {
    double ws = warp_sum_d(sq);
    if (lane == 0) sm.loss_part[warp] = ws;
    // published after the next __syncthreads (inside build_list / below)
  }

  // ---- pass 2: recomposite in forward order and accumulate gradients ------
  float r0 = bg0, r1 = bg1, r2 = bg2;
  Prod Q;
  Q.init();
  for (int ci = 0; ci < n_chunks; ++ci) {
    if (n_chunks > 1) {
      __syncthreads();
      count = build_list(sm, recs, a.T, ci * kChunk, tx0, ty0, tx1, ty1, a.W, a.H, rej, acc);
    }
    for (int i = threadIdx.x; i < count * kParams; i += kThreads) (&sm.acc[0][0])[i] = 0.0f;
    __syncthreads();
    for (int j = 0; j < count; ++j) {
      const TriRec& r = sm.rec[j];
      const int ef = sm.eflags[j];
      const int k = sm.kidx[j];
      float gc0 = 0.f, gc1 = 0.f, gc2 = 0.f, ga = 0.f;
      float gv[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      bool contrib = false;
      if (active) {
        PairEval pe;
        if (eval_pair(r, ef, px, py, ptx, pty, sig, rej, acc, pe)) {
          contrib = true;
          float w = pe.w, om = __fsub_rn(1.0f, w);
          // A barrier layer resets Q to 1, so the same ratio yields the
          // product of the layers above it.
          Q.mul(om, k);
          const float A = attenuation(P, Q, k);
          float g0 = __fmul_rn(G0, A), g1 = __fmul_rn(G1, A), g2 = __fmul_rn(G2, A);
          // grad.rs:162-179
          gc0 = __fmul_rn(g0, w);
          gc1 = __fmul_rn(g1, w);
          gc2 = __fmul_rn(g2, w);
          float d_w = __fmul_rn(g0, __fsub_rn(r.color[0], r0));
          d_w = __fadd_rn(d_w, __fmul_rn(g1, __fsub_rn(r.color[1], r1)));
          d_w = __fadd_rn(d_w, __fmul_rn(g2, __fsub_rn(r.color[2], r2)));
          if (r.flags & kAlphaActive) ga = __fmul_rn(d_w, pe.cov);
          float d_cov = __fmul_rn(d_w, r.alpha);
          // coverage_with_grad (grad.rs:231-270): zero when cov == 1 exactly
          // (fast path) or dist < 1e-9; d_cov * 0 keeps NaN propagation.
          float coef[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (pe.band && !(pe.g.dist < 1e-9f)) {
            const float cov = pe.cov, t = pe.g.t, dist = pe.g.dist;
            const int ea = pe.g.edge, eb = (ea + 1) % 3;
            const float ax = r.v[2 * ea], ay = r.v[2 * ea + 1];
            const float cpx = __fadd_rn(ax, __fmul_rn(t, r.e[2 * ea]));
            const float cpy = __fadd_rn(ay, __fmul_rn(t, r.e[2 * ea + 1]));
            const float ux = __fdiv_rn(__fsub_rn(ptx, cpx), dist);
            const float uy = __fdiv_rn(__fsub_rn(pty, cpy), dist);
            const float sign = (pe.g.sd > 0.0f) ? 1.0f : -1.0f;
            const float chain =
                __fmul_rn(__fdiv_rn(__fmul_rn(cov, __fsub_rn(1.0f, cov)), sig), sign);
            const float ka = __fmul_rn(chain, -__fsub_rn(1.0f, t));
            const float kb = __fmul_rn(chain, -t);
            float cax = __fmul_rn(ka, ux), cay = __fmul_rn(ka, uy);
            float cbx = __fmul_rn(kb, ux), cby = __fmul_rn(kb, uy);
#pragma unroll
            for (int q = 0; q < 3; ++q) {
              coef[2 * q] = (q == ea) ? cax : ((q == eb) ? cbx : 0.0f);
              coef[2 * q + 1] = (q == ea) ? cay : ((q == eb) ? cby : 0.0f);
            }
          }
#pragma unroll
          for (int q = 0; q < 6; ++q) gv[q] = __fmul_rn(d_cov, coef[q]);
          // composite (raster.rs:63)
          r0 = __fadd_rn(__fmul_rn(r.color[0], w), __fmul_rn(r0, om));
          r1 = __fadd_rn(__fmul_rn(r.color[1], w), __fmul_rn(r1, om));
          r2 = __fadd_rn(__fmul_rn(r.color[2], w), __fmul_rn(r2, om));
        }
      }
      // Block reduction: warp shuffles, then one shared atomic per warp.
      if (__any_sync(0xffffffffu, contrib)) {
        float s6 = warp_sum(gc0), s7 = warp_sum(gc1), s8 = warp_sum(gc2), s9 = warp_sum(ga);
        if (lane == 0) {
          atomicAdd(&sm.acc[j][6], s6);
          atomicAdd(&sm.acc[j][7], s7);
          atomicAdd(&sm.acc[j][8], s8);
          atomicAdd(&sm.acc[j][9], s9);
        }
        if (!(ef & kTileInside)) {
#pragma unroll
          for (int q = 0; q < 6; ++q) {
            float s = warp_sum(gv[q]);
            if (lane == 0) atomicAdd(&sm.acc[j][q], s);
          }
        }
      }
    }
    __syncthreads();
    // One global atomic per (triangle, parameter) per block.
    float* g = a.grads + (size_t)b * a.T * kParams;
    for (int i = threadIdx.x; i < count * kParams; i += kThreads) {
      float v = (&sm.acc[0][0])[i];
      if (v != 0.0f) atomicAdd(&g[(size_t)sm.kidx[i / kParams] * kParams + (i % kParams)], v);
    }
  }

  // ---- per-scene loss: tile partials, summed by the last block ------------
  if (Mode == kModeLoss) {
    __syncthreads();
    const int n_tiles = gridDim.x;
    if (threadIdx.x == 0) {
      double s = 0.0;
      for (int w = 0; w < kWarps; ++w) s += sm.loss_part[w];
      a.loss_partials[(size_t)b * n_tiles + local_tile] = s;
      __threadfence();
      unsigned prev = atomicAdd(&a.loss_counters[b], 1u);
      sm.is_last = (prev == (unsigned)(n_tiles - 1));
    }
    __syncthreads();
    if (sm.is_last) {
      __threadfence();
      double s = 0.0;
      for (int t = threadIdx.x; t < n_tiles; t += kThreads)
        s += *((volatile double*)&a.loss_partials[(size_t)b * n_tiles + t]);
      s = warp_sum_d(s);
      if (lane == 0) sm.loss_part[warp] = s;
      __syncthreads();
      if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < kWarps; ++w) tot += sm.loss_part[w];
        if (a.loss_sums) a.loss_sums[b] = tot;
        if (a.losses) a.losses[b] = (float)(tot / a.n_values);  // canvas.rs:58
        a.loss_counters[b] = 0;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// MSE (canvas.rs:45-59) and Adam (optim.rs:40-60 + fit.rs:399-424)
// ---------------------------------------------------------------------------

__global__ void dr_mse_kernel(const float* __restrict__ img, const float* __restrict__ tgt,
                              long long n, float* __restrict__ losses) {
  __shared__ double part[kWarps];
  const float* x = img + (size_t)blockIdx.x * n;
  const float* y = tgt + (size_t)blockIdx.x * n;
  double s = 0.0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    double d = (double)__fsub_rn(x[i], y[i]);
    s += d * d;
  }
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    losses[blockIdx.x] = (float)(t / (double)n);
  }
}

__global__ void dr_adam_kernel(AdamArgs a) {
  if (a.skip_flag && *a.skip_flag) return;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  if (a.copy_flag && *a.copy_flag) a.copy_dst[i] = a.params[i];
  if (a.run_flag && !*a.run_flag) return;
  const int cls = (int)(i % kParams);
  const float lr = cls < 6 ? a.lr_pos : (cls < 9 ? a.lr_color : a.lr_alpha);
  float g = a.grads[i];
  float m = __fadd_rn(__fmul_rn(a.beta1, a.m[i]), __fmul_rn(a.one_minus_beta1, g));
  float v = __fadd_rn(__fmul_rn(a.beta2, a.v[i]), __fmul_rn(__fmul_rn(a.one_minus_beta2, g), g));
  a.m[i] = m;
  a.v[i] = v;
  float m_hat = __fdiv_rn(m, a.bc1);
  float v_hat = __fdiv_rn(v, a.bc2);
  float p = __fsub_rn(a.params[i],
                      __fdiv_rn(__fmul_rn(lr, m_hat), __fadd_rn(__fsqrt_rn(v_hat), a.eps)));
  if (a.project) {
    if (p != p) p = 0.5f;
    if (cls < 6) p = rclamp(p, -0.25f, 1.25f);
    else if (cls < 9) p = rclamp(p, 0.0f, 1.0f);
    else p = rclamp(p, 1e-3f, 0.999f);
  }
  a.params[i] = p;
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

__global__ void dr_fit_control_kernel(FitState* st, int iter, float min_delta, long long patience,
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

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

size_t raster_smem_bytes() { return sizeof(Smem); }

cudaError_t launch_fit_init(FitState* st, cudaStream_t s) {
  dr_fit_init_kernel<<<1, 1, 0, s>>>(st);
  return cudaGetLastError();
}

cudaError_t launch_fit_control(FitState* st, int iter, float min_delta, long long patience,
                               float* losses, cudaStream_t s) {
  dr_fit_control_kernel<<<1, 1, 0, s>>>(st, iter, min_delta, patience, losses);
  return cudaGetLastError();
}


cudaError_t launch_setup(const float* params, int BT, int W, int H, float sigma,
                         int tape_semantics, TriRec* recs, cudaStream_t s) {
  if (BT == 0) return cudaSuccess;
  int threads = 128;
  int blocks = (BT + threads - 1) / threads;
  dr_setup_kernel<<<blocks, threads, 0, s>>>(params, BT, W, H, sigma, tape_semantics, recs);
  return cudaGetLastError();
}

static_assert(sizeof(Smem) <= 48 * 1024, "raster smem must fit the default 48 KB limit");

template <int Mode> static cudaError_t launch_mode(const RasterArgs& a, int n_tiles, cudaStream_t s) {
  const size_t smem = sizeof(Smem);
  dim3 grid(n_tiles, a.B);
  dr_raster_kernel<Mode><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_raster(int mode, const RasterArgs& a, int n_tiles, cudaStream_t s) {
  if (a.B == 0 || n_tiles == 0) return cudaSuccess;
  switch (mode) {
    case kModeRender: return launch_mode<kModeRender>(a, n_tiles, s);
    case kModeLoss: return launch_mode<kModeLoss>(a, n_tiles, s);
    case kModeGrad: return launch_mode<kModeGrad>(a, n_tiles, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_mse(const float* img, const float* tgt, int B, long long n, float* losses,
                       cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  dr_mse_kernel<<<B, 512, 0, s>>>(img, tgt, n, losses);
  return cudaGetLastError();
}

cudaError_t launch_adam(const AdamArgs& a, cudaStream_t s) {
  if (a.n == 0) return cudaSuccess;
  int threads = 256;
  long long blocks = (a.n + threads - 1) / threads;
  dr_adam_kernel<<<(unsigned)blocks, threads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace dr

namespace dr {
size_t tri_rec_bytes() { return sizeof(TriRec); }
}  // namespace dr
