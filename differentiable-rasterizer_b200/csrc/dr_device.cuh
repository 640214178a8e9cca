// Device-side building blocks of the soft-triangle rasterizer (sm_100a).
//
// Semantics follow the reference CPU path (crates/diffrast/src/raster.rs,
// grad.rs). The arithmetic that decides a pixel's value is written with
// explicit round-to-nearest intrinsics (__fmul_rn, __fadd_rn, __fdiv_rn,
// __fsqrt_rn): nvcc may not contract them into FMAs, so every line computes
// exactly what the Rust expression computes, in the same order. Only expf
// differs (CUDA's expf vs libm's; both are within 2 ulp).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dr {

constexpr int kParams = 10;          // scene.rs:21 Triangle::N_PARAMS
constexpr float kMinWeight = 1e-6f;  // raster.rs:34 MIN_WEIGHT


// Triangle record written once per (scene, triangle) by the set-up kernel and
// staged into shared memory by the raster kernels. 40 words, 16-byte aligned.
// Each edge's data sits in one 32-byte run, so evaluating an edge whose index
// the code knows loads two 16-byte words instead of eight scattered ones.
struct __align__(16) EdgeRec {
  float ax, ay;  // the edge's first vertex (raw params)
  float ex, ey;  // edge vector b - a for edges (v0,v1), (v1,v2), (v2,v0)
  float nx, ny;  // unit inward normal (fast path only)
  float c;       // line offset: l(p) = n . p + c
  float il;      // 1 / len2 (0 when len2 <= 1e-20: t = 0, raster.rs:129-130)
};
struct __align__(16) TriRec {
  int bbox[4];      // x0 y0 x1 y1 of pixel_bounds (raster.rs:144-168); all 0 unless
                    // kLive. First, so that a tile's mask pass reads one 16-byte word.
  EdgeRec ed[3];
  float len2[3];    // |e|^2 as the reference computes it (raster.rs:127)
  float alpha;      // clamp(a, 0, 1) (raster.rs:48)
  float color[3];
  float margin;     // absolute slack on the edge-line tests, normalized units
  int flags;
  float rej;        // skip pixels with min edge-line distance below -rej
  float acc;        // w == alpha for pixels with min edge-line distance above acc
  float wind;       // sign of the signed area (+1 / -1): the sign of the reference's
                    // edge cross product on the inner side of every edge
};
static_assert(sizeof(TriRec) == 160, "TriRec layout");
constexpr int kRecWords = 40;

enum RecFlags : int {
  kLive = 1,         // has a non-empty box and a usable alpha
  kAlphaActive = 2,  // 0 < raw alpha < 1: alpha receives gradient (grad.rs:145)
  kFastOk = 4,       // non-degenerate, finite alpha: edge-line tests are valid
};

// f32::clamp (NaN passes through).
__device__ __forceinline__ float rclamp(float x, float lo, float hi) {
  x = (x < lo) ? lo : x;
  x = (x > hi) ? hi : x;
  return x;
}

// raster.rs:79-87
__device__ __forceinline__ float sigmoid_ref(float x) {
  if (x >= 0.0f) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  }
  float e = expf(x);
  return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

// raster.rs:124-134 / grad.rs:275-284 for edge (a, a + e), plus the winding
// cross product of raster.rs:119-122 (which reuses the same ab and ap).
__device__ __forceinline__ float segment_ref(float ax, float ay, float ex, float ey, float len2,
                                             float px, float py, float& t_out, float& cross_out) {
  float apx = __fsub_rn(px, ax);
  float apy = __fsub_rn(py, ay);
  float t;
  if (len2 <= 1e-20f) {
    t = 0.0f;
  } else {
    t = rclamp(__fdiv_rn(__fadd_rn(__fmul_rn(apx, ex), __fmul_rn(apy, ey)), len2), 0.0f, 1.0f);
  }
  float dx = __fsub_rn(apx, __fmul_rn(t, ex));
  float dy = __fsub_rn(apy, __fmul_rn(t, ey));
  t_out = t;
  cross_out = __fsub_rn(__fmul_rn(ex, apy), __fmul_rn(ey, apx));
  return __fsqrt_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)));
}

struct SdResult {
  float sd;    // signed distance (raster.rs:96-106)
  float dist;  // nearest-edge distance (strict < from +inf, grad.rs:236-242)
  float t;     // projection parameter on the nearest edge
  int edge;    // nearest edge index
};

// signed_distance + the nearest-edge bookkeeping of coverage_with_grad.
// fminf ignores NaN like f32::min, so `sd` folds exactly as the reference;
// the strict `<` walk picks the same edge value the fold lands on.
__device__ __forceinline__ SdResult signed_distance_ref(const EdgeRec* ed, const float* len2,
                                                        float px, float py) {
  float t0, t1, t2, c0, c1, c2;
  float d0 = segment_ref(ed[0].ax, ed[0].ay, ed[0].ex, ed[0].ey, len2[0], px, py, t0, c0);
  float d1 = segment_ref(ed[1].ax, ed[1].ay, ed[1].ex, ed[1].ey, len2[1], px, py, t1, c1);
  float d2 = segment_ref(ed[2].ax, ed[2].ay, ed[2].ex, ed[2].ey, len2[2], px, py, t2, c2);
  float d = fminf(fminf(fminf(__int_as_float(0x7f800000), d0), d1), d2);
  SdResult r;
  int edge = 0;
  float bt = 0.0f, bd = __int_as_float(0x7f800000);
  if (d0 < bd) { edge = 0; bt = t0; bd = d0; }
  if (d1 < bd) { edge = 1; bt = t1; bd = d1; }
  if (d2 < bd) { edge = 2; bt = t2; bd = d2; }
  bool inside = (c0 >= 0.0f && c1 >= 0.0f && c2 >= 0.0f) || (c0 <= 0.0f && c1 <= 0.0f && c2 <= 0.0f);
  r.sd = inside ? d : -d;
  r.dist = bd;
  r.t = bt;
  r.edge = edge;
  return r;
}

// Pixel centre (raster.rs:138-140), IEEE division like the reference.
__device__ __forceinline__ float pixel_center(int x, int n) {
  return __fdiv_rn(__fadd_rn((float)x, 0.5f), (float)n);
}

}  // namespace dr
