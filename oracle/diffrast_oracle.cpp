// CPU oracle for the soft-triangle rasterizer hot path.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity checker and the timed CPU
// baseline; nothing in the product path links, loads or calls it. Only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
// use it.
//
// It is an op-for-op restatement, in C++, of the reference's Rust CPU path
// (VivianSobers/Differentiable-Rasterizer, crates/diffrast/src):
//   raster.rs:26-168   cull radius, MIN_WEIGHT, render/composite, coverage,
//                      sigmoid, signed_distance, is_inside, cross,
//                      point_segment_distance, pixel_center, pixel_bounds
//   grad.rs:56-294     render_with_tape (per-triangle patches), backward,
//                      backward_one, backward_batch, coverage_with_grad,
//                      closest_point_on_segment, finite_difference
//   canvas.rs:45-59    mse with an f64 sum
//   optim.rs:40-60     Adam::step (f32, powi bias correction)
//   fit.rs:243-424     Fitter::step, sigma_at, mean_color, sample,
//                      learning_rates, project, validate
//   diffrast-py/src/lib.rs:301-318  grad-input backward by target inversion
//
// Floating point follows Rust's semantics: no FMA contraction (build with
// -ffp-contract=off, no fast-math), libm expf/powf, IEEE sqrt and division,
// left-to-right evaluation as written in the Rust source. f32::min/max ignore a
// NaN operand (fmin/fmax), f32::clamp propagates NaN, `as usize` saturates.
//
// Every kernel is a template on the arithmetic type F. F = float is the
// reference; F = double is a twin that keeps the reference's discrete decisions
// (the f32 bounding-box cull is always computed in f32) and measures the f32
// rounding noise floor the GPU results are judged against.
//
// Parity pinning: the reference ships no stored output vectors. The oracle is
// pinned by restating every known-answer test the reference holds for this
// path (raster.rs:170-241, grad.rs:325-495, optim.rs:63-98, fit.rs:426-636,
// tests/integration.rs) in tests/test_oracle.py.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#include <atomic>
#include <thread>

namespace {

constexpr int kParams = 10;           // scene.rs:21 Triangle::N_PARAMS
constexpr float kMinWeight = 1e-6f;   // raster.rs:34 MIN_WEIGHT

template <typename F> struct Tri {
  F v[3][2];
  F color[3];
  F alpha;
  float raw_v[3][2];  // the f32 vertices, for the f32 bbox cull
};

// P is the storage type of the parameters: f32 for every entry point, f64
// only for the f64 fit twin, whose box cull still takes the f32 vertices.
template <typename F, typename P = float> Tri<F> load_tri(const P* p) {
  Tri<F> t;
  for (int i = 0; i < 3; ++i) {
    t.v[i][0] = (F)p[2 * i];
    t.v[i][1] = (F)p[2 * i + 1];
    t.raw_v[i][0] = (float)p[2 * i];
    t.raw_v[i][1] = (float)p[2 * i + 1];
  }
  for (int c = 0; c < 3; ++c) t.color[c] = (F)p[6 + c];
  t.alpha = (F)p[9];
  return t;
}

// f32::clamp: NaN passes through (raster.rs:48 uses it on alpha).
template <typename F> inline F rclamp(F x, F lo, F hi) {
  if (x < lo) x = lo;
  if (x > hi) x = hi;
  return x;
}

// raster.rs:79-87 / grad.rs:287-294
template <typename F> inline F sigmoid(F x) {
  if (x >= (F)0) {
    return (F)1 / ((F)1 + std::exp(-x));
  }
  F e = std::exp(x);
  return e / ((F)1 + e);
}

// raster.rs:119-122
template <typename F> inline F cross(const F a[2], const F b[2], const F pt[2]) {
  return (b[0] - a[0]) * (pt[1] - a[1]) - (b[1] - a[1]) * (pt[0] - a[0]);
}

// raster.rs:111-116
template <typename F> inline bool is_inside(const F v[3][2], const F pt[2]) {
  F c0 = cross(v[0], v[1], pt);
  F c1 = cross(v[1], v[2], pt);
  F c2 = cross(v[2], v[0], pt);
  return (c0 >= (F)0 && c1 >= (F)0 && c2 >= (F)0) || (c0 <= (F)0 && c1 <= (F)0 && c2 <= (F)0);
}

// raster.rs:124-134 and grad.rs:275-284 (same arithmetic; returns t and d)
template <typename F> inline void segment(const F a[2], const F b[2], const F pt[2], F* t_out,
                                          F* d_out) {
  F ab0 = b[0] - a[0], ab1 = b[1] - a[1];
  F ap0 = pt[0] - a[0], ap1 = pt[1] - a[1];
  F len2 = ab0 * ab0 + ab1 * ab1;
  F t;
  if (len2 <= (F)1e-20f) {
    t = (F)0;
  } else {
    t = rclamp((ap0 * ab0 + ap1 * ab1) / len2, (F)0, (F)1);
  }
  F dx = ap0 - t * ab0;
  F dy = ap1 - t * ab1;
  *t_out = t;
  *d_out = std::sqrt(dx * dx + dy * dy);
}

// raster.rs:96-106 (fold from +inf with f32::min, which ignores NaN)
template <typename F> inline F signed_distance(const F v[3][2], const F pt[2]) {
  F d = std::numeric_limits<F>::infinity();
  for (int i = 0; i < 3; ++i) {
    F t, di;
    segment(v[i], v[(i + 1) % 3], pt, &t, &di);
    d = std::fmin(d, di);
  }
  return is_inside(v, pt) ? d : -d;
}

// raster.rs:74-76 (sigma.max(1e-8))
template <typename F> inline F coverage(const Tri<F>& t, const F pt[2], F sigma) {
  return sigmoid(signed_distance(t.v, pt) / std::fmax(sigma, (F)1e-8f));
}

// raster.rs:138-140
template <typename F> inline void pixel_center(size_t x, size_t y, size_t W, size_t H, F pt[2]) {
  pt[0] = ((F)x + (F)0.5f) / (F)W;
  pt[1] = ((F)y + (F)0.5f) / (F)H;
}

// Rust `f as usize` for a non-negative f32 (after .max(0.0)): saturating.
inline uint64_t sat_usize(float f) {
  if (!(f > 0.0f)) return 0;  // NaN and 0 -> 0
  if (f >= 18446744073709551616.0f) return UINT64_MAX;
  return (uint64_t)f;
}

struct Bounds {
  size_t x0, y0, x1, y1;
};

// raster.rs:144-168. Always evaluated in f32, as the reference does; `+ 1`
// wraps like a release-mode usize add.
inline bool pixel_bounds(const float v[3][2], size_t W, size_t H, float sigma, Bounds* b) {
  float pad = 6.0f * sigma;  // raster.rs:26-28 cull_radius
  float lo_x = INFINITY, lo_y = INFINITY, hi_x = -INFINITY, hi_y = -INFINITY;
  for (int i = 0; i < 3; ++i) {
    if (!std::isfinite(v[i][0]) || !std::isfinite(v[i][1])) return false;
    lo_x = std::fmin(lo_x, v[i][0]);
    hi_x = std::fmax(hi_x, v[i][0]);
    lo_y = std::fmin(lo_y, v[i][1]);
    hi_y = std::fmax(hi_y, v[i][1]);
  }
  float fw = (float)W, fh = (float)H;
  uint64_t x0 = sat_usize(std::fmax(std::floor((lo_x - pad) * fw), 0.0f));
  uint64_t y0 = sat_usize(std::fmax(std::floor((lo_y - pad) * fh), 0.0f));
  uint64_t x1 = std::min<uint64_t>(sat_usize(std::fmax(std::ceil((hi_x + pad) * fw), 0.0f)) + 1u, W);
  uint64_t y1 = std::min<uint64_t>(sat_usize(std::fmax(std::ceil((hi_y + pad) * fh), 0.0f)) + 1u, H);
  if (!(x0 < x1 && y0 < y1)) return false;
  b->x0 = x0;
  b->y0 = y0;
  b->x1 = x1;
  b->y1 = y1;
  return true;
}

template <typename F> struct Canvas {
  size_t W, H;
  std::vector<F> data;
  Canvas(size_t w, size_t h, const F bg[3]) : W(w), H(h), data(w * h * 3) {
    for (size_t i = 0; i < w * h; ++i) {
      data[3 * i] = bg[0];
      data[3 * i + 1] = bg[1];
      data[3 * i + 2] = bg[2];
    }
  }
  size_t idx(size_t x, size_t y) const { return (y * W + x) * 3; }
};

// raster.rs:46-68
template <typename F> void composite(Canvas<F>& c, const Tri<F>& t, F sigma) {
  Bounds bb;
  if (!pixel_bounds(t.raw_v, c.W, c.H, (float)sigma, &bb)) return;
  F alpha = rclamp(t.alpha, (F)0, (F)1);
  if (alpha <= (F)0) return;
  for (size_t y = bb.y0; y < bb.y1; ++y) {
    for (size_t x = bb.x0; x < bb.x1; ++x) {
      F pt[2];
      pixel_center(x, y, c.W, c.H, pt);
      F w = alpha * coverage(t, pt, sigma);
      if (w <= (F)kMinWeight) continue;
      size_t i = c.idx(x, y);
      for (int ch = 0; ch < 3; ++ch) {
        c.data[i + ch] = t.color[ch] * w + c.data[i + ch] * ((F)1 - w);
      }
    }
  }
}

// raster.rs:37-43
template <typename F>
void render(const float* params, int T, const float bg[3], size_t W, size_t H, F sigma, F* out) {
  F bgf[3] = {(F)bg[0], (F)bg[1], (F)bg[2]};
  Canvas<F> c(W, H, bgf);
  for (int k = 0; k < T; ++k) composite(c, load_tri<F>(params + (size_t)k * kParams), sigma);
  std::memcpy(out, c.data.data(), c.data.size() * sizeof(F));
}

// canvas.rs:45-59: sum of ((a - b) as f64)^2 in f64, / n, as f32 (kept in F's
// precision for the twin; the subtraction happens in F).
template <typename F> double mse_sum(const F* a, const F* b, size_t n) {
  double s = 0.0;
  for (size_t i = 0; i < n; ++i) {
    double d = (double)(a[i] - b[i]);
    s += d * d;
  }
  return s;
}

template <typename F> F mse(const F* a, const F* b, size_t n) {
  return (F)(mse_sum(a, b, n) / (double)n);
}

// grad.rs:28-35
template <typename F> struct Patch {
  bool present = false;
  Bounds bb{};
  std::vector<F> before;
};

// grad.rs:56-90
template <typename F>
void render_with_tape(const std::vector<Tri<F>>& tris, size_t W, size_t H, F sigma, Canvas<F>& c,
                      std::vector<Patch<F>>& tape) {
  tape.assign(tris.size(), Patch<F>());
  for (size_t k = 0; k < tris.size(); ++k) {
    const Tri<F>& t = tris[k];
    F alpha = rclamp(t.alpha, (F)0, (F)1);
    Bounds bb;
    if (!pixel_bounds(t.raw_v, W, H, (float)sigma, &bb) || !(alpha > (F)0)) continue;
    Patch<F>& p = tape[k];
    p.present = true;
    p.bb = bb;
    p.before.reserve((bb.x1 - bb.x0) * (bb.y1 - bb.y0) * 3);
    for (size_t y = bb.y0; y < bb.y1; ++y) {
      for (size_t x = bb.x0; x < bb.x1; ++x) {
        size_t i = c.idx(x, y);
        p.before.push_back(c.data[i]);
        p.before.push_back(c.data[i + 1]);
        p.before.push_back(c.data[i + 2]);
        F pt[2];
        pixel_center(x, y, W, H, pt);
        F w = alpha * coverage(t, pt, sigma);
        if (w <= (F)kMinWeight) continue;
        for (int ch = 0; ch < 3; ++ch) {
          c.data[i + ch] = t.color[ch] * w + c.data[i + ch] * ((F)1 - w);
        }
      }
    }
  }
}

// grad.rs:231-270
template <typename F>
F coverage_with_grad(const Tri<F>& tri, const F pt[2], F sigma_in, F d[3][2]) {
  const auto& v = tri.v;
  F sigma = std::fmax(sigma_in, (F)1e-8f);
  int edge = 0;
  F bt = (F)0, bd = std::numeric_limits<F>::infinity();
  for (int i = 0; i < 3; ++i) {
    F t, di;
    segment(v[i], v[(i + 1) % 3], pt, &t, &di);
    if (di < bd) {
      edge = i;
      bt = t;
      bd = di;
    }
  }
  F t = bt, dist = bd;
  bool inside = signed_distance(v, pt) > (F)0;
  F sign = inside ? (F)1 : (F)-1;
  F cov = sigmoid(sign * dist / sigma);
  for (int a = 0; a < 3; ++a) d[a][0] = d[a][1] = (F)0;
  if (dist < (F)1e-9f) return cov;
  const F* a = v[edge];
  const F* b = v[(edge + 1) % 3];
  F cp[2] = {a[0] + t * (b[0] - a[0]), a[1] + t * (b[1] - a[1])};
  F u[2] = {(pt[0] - cp[0]) / dist, (pt[1] - cp[1]) / dist};
  F chain = cov * ((F)1 - cov) / sigma * sign;
  for (int ax = 0; ax < 2; ++ax) {
    d[edge][ax] = chain * -((F)1 - t) * u[ax];
    d[(edge + 1) % 3][ax] += chain * -t * u[ax];
  }
  return cov;
}

// grad.rs:135-182
template <typename F>
void backward_one(const Tri<F>& tri, size_t W, size_t H, F sigma, const Patch<F>& patch,
                  std::vector<F>& d_canvas, F* g) {
  F alpha = rclamp(tri.alpha, (F)0, (F)1);
  bool alpha_active = tri.alpha > (F)0 && tri.alpha < (F)1;
  size_t row_len = (patch.bb.x1 - patch.bb.x0) * 3;
  for (size_t y = patch.bb.y0; y < patch.bb.y1; ++y) {
    for (size_t x = patch.bb.x0; x < patch.bb.x1; ++x) {
      F pt[2];
      pixel_center(x, y, W, H, pt);
      F dcv[3][2];
      F cov = coverage_with_grad(tri, pt, sigma, dcv);
      F w = alpha * cov;
      if (w <= (F)kMinWeight) continue;
      size_t off = (y - patch.bb.y0) * row_len + (x - patch.bb.x0) * 3;
      const F* dst = &patch.before[off];
      size_t di = (y * W + x) * 3;
      F d_out[3] = {d_canvas[di], d_canvas[di + 1], d_canvas[di + 2]};
      F d_w = (F)0;
      for (int ch = 0; ch < 3; ++ch) {
        g[6 + ch] += d_out[ch] * w;
        d_w += d_out[ch] * (tri.color[ch] - dst[ch]);
        d_canvas[di + ch] = d_out[ch] * ((F)1 - w);
      }
      if (alpha_active) g[9] += d_w * cov;
      F d_cov = d_w * alpha;
      for (int vv = 0; vv < 3; ++vv) {
        g[vv * 2] += d_cov * dcv[vv][0];
        g[vv * 2 + 1] += d_cov * dcv[vv][1];
      }
    }
  }
}

enum GradMode {
  kTarget = 0,        // d_canvas = 2/N (r - t), grad.rs:112-114
  kInvertGrad = 1,    // PyO3 CPU path: t = r - g*N/2, then kTarget
  kDirectGrad = 2,    // d_canvas = upstream gradient (GPU grad_input mode)
};

// One scene: render_with_tape + backward (grad.rs:98-131), with the d_canvas
// seeding chosen by `mode`. Writes T*10 grads, returns the loss as F.
template <typename F, typename P = float>
F scene_backward(const P* params, int T, const float bg[3], size_t W, size_t H, F sigma,
                 const float* other, int mode, F* grads, F* image_out) {
  std::vector<Tri<F>> tris;
  tris.reserve(T);
  for (int k = 0; k < T; ++k) tris.push_back(load_tri<F, P>(params + (size_t)k * kParams));
  F bgf[3] = {(F)bg[0], (F)bg[1], (F)bg[2]};
  Canvas<F> rendered(W, H, bgf);
  std::vector<Patch<F>> tape;
  render_with_tape(tris, W, H, sigma, rendered, tape);
  size_t n = W * H * 3;
  if (image_out) std::memcpy(image_out, rendered.data.data(), n * sizeof(F));

  std::vector<F> target(n);
  if (mode == kTarget) {
    for (size_t i = 0; i < n; ++i) target[i] = (F)other[i];
  } else if (mode == kInvertGrad) {
    // diffrast-py/src/lib.rs:281,311-313: rendered - g * n_pixels / 2.0
    F n_pixels = (F)(float)n;
    for (size_t i = 0; i < n; ++i) target[i] = rendered.data[i] - (F)other[i] * n_pixels / (F)2;
  }
  F loss = (F)0;
  std::vector<F> d_canvas(n);
  if (mode == kDirectGrad) {
    for (size_t i = 0; i < n; ++i) d_canvas[i] = (F)other[i];
  } else {
    loss = mse(rendered.data.data(), target.data(), n);
    F scale = (F)2 / (F)(float)n;
    for (size_t i = 0; i < n; ++i) d_canvas[i] = scale * (rendered.data[i] - target[i]);
  }
  std::fill(grads, grads + (size_t)T * kParams, (F)0);
  for (int k = T - 1; k >= 0; --k) {
    if (!tape[k].present) continue;
    backward_one(tris[k], W, H, sigma, tape[k], d_canvas, grads + (size_t)k * kParams);
  }
  return loss;
}

int clamp_threads(int threads) {
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  return threads;
}

// Scene-level parallelism, as rayon's par_iter over scenes (grad.rs:199-206):
// workers pull scene indices from a shared counter, results land by index so
// the output order is the input order.
template <typename Fn> void parallel_for(int n, int threads, Fn fn) {
  threads = std::min(clamp_threads(threads), std::max(n, 1));
  if (threads <= 1) {
    for (int i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int> next{0};
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int w = 0; w < threads; ++w) {
    pool.emplace_back([&]() {
      for (int i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    });
  }
  for (auto& th : pool) th.join();
}

// optim.rs:40-60 helper: f32 powi. Rust lowers `powi` with a runtime exponent
// to compiler-rt's square-and-multiply loop; restated here.
float powi_f32(float a, int b) {
  bool recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

}  // namespace

extern "C" {

// --- geometry probes (used by the known-answer tests) ----------------------

// raster.rs:144-168. Returns 1 and fills out[4] = {x0, y0, x1, y1} when the
// triangle has a non-empty box, else 0.
int oracle_pixel_bounds(const float* tri, int W, int H, float sigma, int64_t* out) {
  float v[3][2] = {{tri[0], tri[1]}, {tri[2], tri[3]}, {tri[4], tri[5]}};
  Bounds b;
  if (!pixel_bounds(v, (size_t)W, (size_t)H, sigma, &b)) return 0;
  out[0] = (int64_t)b.x0;
  out[1] = (int64_t)b.y0;
  out[2] = (int64_t)b.x1;
  out[3] = (int64_t)b.y1;
  return 1;
}

float oracle_signed_distance(const float* verts6, float px, float py) {
  float v[3][2] = {{verts6[0], verts6[1]}, {verts6[2], verts6[3]}, {verts6[4], verts6[5]}};
  float pt[2] = {px, py};
  return signed_distance<float>(v, pt);
}

float oracle_coverage(const float* tri, float px, float py, float sigma) {
  Tri<float> t = load_tri<float>(tri);
  float pt[2] = {px, py};
  return coverage<float>(t, pt, sigma);
}

// grad.rs:231-270; d6 receives d(cov)/d(x0,y0,x1,y1,x2,y2).
float oracle_coverage_with_grad(const float* tri, float px, float py, float sigma, float* d6) {
  Tri<float> t = load_tri<float>(tri);
  float pt[2] = {px, py};
  float d[3][2];
  float cov = coverage_with_grad<float>(t, pt, sigma, d);
  for (int i = 0; i < 3; ++i) {
    d6[2 * i] = d[i][0];
    d6[2 * i + 1] = d[i][1];
  }
  return cov;
}

// canvas.rs:45-59
float oracle_mse(const float* a, const float* b, int64_t n) { return mse<float>(a, b, (size_t)n); }

// --- batched render / backward (grad.rs:192-212, diffrast-py lib.rs) -------

// params (B,T,10); bg is 3 floats, or B*3 when bg_per_scene; out (B,H,W,3).
void oracle_render_batch(const float* params, const float* bg, int bg_per_scene, int B, int T,
                         int H, int W, float sigma, float* out, int threads) {
  size_t img = (size_t)H * W * 3;
  parallel_for(B, threads, [&](int b) {
    render<float>(params + (size_t)b * T * kParams, T, bg + (bg_per_scene ? 3 * b : 0), W, H,
                  sigma, out + (size_t)b * img);
  });
}

void oracle64_render_batch(const float* params, const float* bg, int bg_per_scene, int B, int T,
                           int H, int W, float sigma, double* out, int threads) {
  size_t img = (size_t)H * W * 3;
  parallel_for(B, threads, [&](int b) {
    render<double>(params + (size_t)b * T * kParams, T, bg + (bg_per_scene ? 3 * b : 0), W, H,
                   (double)sigma, out + (size_t)b * img);
  });
}

// mode: 0 = targets (fused_loss_backward / backward_batch), 1 = upstream
// gradient via target inversion (PyO3 CPU backward_batch), 2 = upstream
// gradient used directly. `other` is (B,H,W,3). losses (B) may be null;
// images_out (B,H,W,3) may be null.
void oracle_backward_batch(const float* params, const float* bg, int bg_per_scene, int B, int T,
                           int H, int W, float sigma, const float* other, int mode, float* losses,
                           float* grads, float* images_out, int threads) {
  size_t img = (size_t)H * W * 3;
  parallel_for(B, threads, [&](int b) {
    float l = scene_backward<float>(params + (size_t)b * T * kParams, T,
                                    bg + (bg_per_scene ? 3 * b : 0), W, H, sigma,
                                    other + (size_t)b * img, mode,
                                    grads + (size_t)b * T * kParams,
                                    images_out ? images_out + (size_t)b * img : nullptr);
    if (losses) losses[b] = l;
  });
}

void oracle64_backward_batch(const float* params, const float* bg, int bg_per_scene, int B, int T,
                             int H, int W, float sigma, const float* other, int mode,
                             double* losses, double* grads, double* images_out, int threads) {
  size_t img = (size_t)H * W * 3;
  parallel_for(B, threads, [&](int b) {
    double l = scene_backward<double>(params + (size_t)b * T * kParams, T,
                                      bg + (bg_per_scene ? 3 * b : 0), W, H, (double)sigma,
                                      other + (size_t)b * img, mode,
                                      grads + (size_t)b * T * kParams,
                                      images_out ? images_out + (size_t)b * img : nullptr);
    if (losses) losses[b] = l;
  });
}

// grad.rs:298-323 (single scene, central differences, f32).
float oracle_finite_difference(const float* params, const float* bg, int T, int H, int W,
                               float sigma, const float* target, float eps, float* grads) {
  size_t n = (size_t)H * W * 3;
  std::vector<float> img(n), probe(params, params + (size_t)T * kParams);
  render<float>(params, T, bg, W, H, sigma, img.data());
  float loss = mse<float>(img.data(), target, n);
  for (size_t i = 0; i < probe.size(); ++i) {
    float base = params[i];
    probe[i] = base + eps;
    render<float>(probe.data(), T, bg, W, H, sigma, img.data());
    float hi = mse<float>(img.data(), target, n);
    probe[i] = base - eps;
    render<float>(probe.data(), T, bg, W, H, sigma, img.data());
    float lo = mse<float>(img.data(), target, n);
    probe[i] = base;
    grads[i] = (hi - lo) / (2.0f * eps);
  }
  return loss;
}

// --- optimizer and fit driver ----------------------------------------------

float oracle_powi(float a, int b) { return powi_f32(a, b); }

// optim.rs:40-60. `t` is the step counter, incremented here.
void oracle_adam_step(float* params, float* m, float* v, const float* grads, const float* lr,
                      int64_t n, uint32_t* t, float beta1, float beta2, float eps) {
  *t += 1;
  float bc1 = 1.0f - powi_f32(beta1, (int)*t);
  float bc2 = 1.0f - powi_f32(beta2, (int)*t);
  for (int64_t i = 0; i < n; ++i) {
    float g = grads[i];
    m[i] = beta1 * m[i] + (1.0f - beta1) * g;
    v[i] = beta2 * v[i] + (1.0f - beta2) * g * g;
    float m_hat = m[i] / bc1;
    float v_hat = v[i] / bc2;
    params[i] -= lr[i] * m_hat / (std::sqrt(v_hat) + eps);
  }
}

// fit.rs:399-424
void oracle_project(float* params, int64_t n_tris) {
  for (int64_t k = 0; k < n_tris; ++k) {
    float* tri = params + k * kParams;
    for (int i = 0; i < kParams; ++i)
      if (std::isnan(tri[i])) tri[i] = 0.5f;
    for (int i = 0; i < 6; ++i) tri[i] = rclamp(tri[i], -0.25f, 1.25f);
    for (int i = 6; i < 9; ++i) tri[i] = rclamp(tri[i], 0.0f, 1.0f);
    tri[9] = rclamp(tri[9], 1e-3f, 0.999f);
  }
}

// fit.rs:343-349
float oracle_sigma_at(float sigma_start, float sigma_end, int64_t iters, int64_t i) {
  if (iters <= 1) return sigma_end;
  float t = (float)i / (float)(iters - 1);
  return sigma_start * std::pow(sigma_end / sigma_start, t);
}

// fit.rs:369-385 and 356-366: background = mean colour of the target; each
// triangle's colour = nearest-pixel sample of the target at its centroid.
// (The random vertices and alphas of seed_scene come from the caller.)
void oracle_seed_colors(const float* target, int H, int W, float* params, int T, float* bg_out) {
  double sum[3] = {0, 0, 0};
  size_t npx = (size_t)H * W;
  for (size_t i = 0; i < npx; ++i)
    for (int ch = 0; ch < 3; ++ch) sum[ch] += (double)target[3 * i + ch];
  float n = (float)npx;
  for (int ch = 0; ch < 3; ++ch) bg_out[ch] = (float)(sum[ch] / (double)n);
  for (int k = 0; k < T; ++k) {
    float* tri = params + (size_t)k * kParams;
    float cx = (tri[0] + tri[2] + tri[4]) / 3.0f;
    float cy = (tri[1] + tri[3] + tri[5]) / 3.0f;
    // fit.rs:381-385: `(x * w as f32) as isize` then clamp to the canvas.
    auto to_isize = [](float f) -> int64_t {
      if (std::isnan(f)) return 0;
      if (f >= 9.2233720368547758e18f) return INT64_MAX;
      if (f <= -9.2233720368547758e18f) return INT64_MIN;
      return (int64_t)f;
    };
    int64_t px = std::clamp<int64_t>(to_isize(cx * (float)W), 0, W - 1);
    int64_t py = std::clamp<int64_t>(to_isize(cy * (float)H), 0, H - 1);
    size_t i = ((size_t)py * W + (size_t)px) * 3;
    tri[6] = target[i];
    tri[7] = target[i + 1];
    tri[8] = target[i + 2];
  }
}

struct OracleFitConfig {
  int64_t iters;
  float sigma_start, sigma_end;
  float lr_pos, lr_color, lr_alpha;
  int64_t patience;  // < 0 means None
  float min_delta;
};

// fit.rs:98-117. 0 = ok, 1 NoTriangles, 2 NonPositiveSigma,
// 3 SigmaNotDecreasing, 4 NonPositiveLearningRate.
int oracle_fit_validate(const OracleFitConfig* c, int T) {
  if (T == 0) return 1;
  if (!(std::isfinite(c->sigma_start) && std::isfinite(c->sigma_end)) || c->sigma_start <= 0.0f ||
      c->sigma_end <= 0.0f)
    return 2;
  if (c->sigma_start < c->sigma_end) return 3;
  float lrs[3] = {c->lr_pos, c->lr_color, c->lr_alpha};
  for (float lr : lrs)
    if (!std::isfinite(lr) || lr <= 0.0f) return 4;
  return 0;
}

}  // extern "C"

namespace {

// powi in the arithmetic type F: the f32 square-and-multiply of powi_f32 for
// F = float, the same loop in f64 for the twin.
template <typename F> F powi_t(F a, int b) {
  bool recip = b < 0;
  F r = (F)1;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? (F)1 / r : r;
}

// fit.rs:166-181 + Fitter::new/step (fit.rs:214-288) in the arithmetic type F.
// F = float is the reference; F = double keeps the reference's discrete steps
// (the sigma schedule and box cull in f32) and carries parameters, moments and
// the loss in f64, which measures how far f32 rounding moves a fit.
template <typename F>
int fit_t(const float* target, int H, int W, const float* init_params, const float* bg, int T,
          const OracleFitConfig* cfg, F* losses, int64_t* n_losses, F* best_params,
          F* final_params, int64_t* best_iter, F* best_loss, int* stop_reason) {
  int err = oracle_fit_validate(cfg, T);
  if (err) return err;
  size_t np = (size_t)T * kParams;
  std::vector<F> params(np), m(np, (F)0), v(np, (F)0), lr(np), grads(np);
  for (size_t i = 0; i < np; ++i) params[i] = (F)init_params[i];
  std::vector<F> best(params);
  for (int k = 0; k < T; ++k) {  // fit.rs:388-396
    for (int i = 0; i < 6; ++i) lr[k * kParams + i] = (F)cfg->lr_pos;
    for (int i = 6; i < 9; ++i) lr[k * kParams + i] = (F)cfg->lr_color;
    lr[k * kParams + 9] = (F)cfg->lr_alpha;
  }
  const F beta1 = (F)0.9f, beta2 = (F)0.999f, eps = (F)1e-8f, min_delta = (F)cfg->min_delta;
  uint32_t t = 0;
  int64_t iter = 0, since = 0, bi = 0, count = 0;
  F bl = std::numeric_limits<F>::infinity();
  int stop = 0;
  for (;;) {
    if (iter >= cfg->iters) {
      stop = 0;
      break;
    }
    int64_t i = iter;
    F sigma = (F)oracle_sigma_at(cfg->sigma_start, cfg->sigma_end, cfg->iters, i);
    F loss = scene_backward<F, F>(params.data(), T, bg, W, H, sigma, target, kTarget,
                                  grads.data(), nullptr);
    if (!std::isfinite(loss)) {
      stop = 2;
      break;
    }
    losses[count++] = loss;
    if (loss + min_delta < bl) {  // fit.rs:268-275
      bl = loss;
      bi = i;
      best = params;
      since = 0;
    } else {
      since += 1;
    }
    iter += 1;
    if (cfg->patience >= 0 && since >= cfg->patience) {
      stop = 1;
      break;
    }
    // optim.rs:40-60
    t += 1;
    F bc1 = (F)1 - powi_t<F>(beta1, (int)t);
    F bc2 = (F)1 - powi_t<F>(beta2, (int)t);
    for (size_t j = 0; j < np; ++j) {
      F g = grads[j];
      m[j] = beta1 * m[j] + ((F)1 - beta1) * g;
      v[j] = beta2 * v[j] + ((F)1 - beta2) * g * g;
      F m_hat = m[j] / bc1;
      F v_hat = v[j] / bc2;
      params[j] -= lr[j] * m_hat / (std::sqrt(v_hat) + eps);
    }
    // fit.rs:399-424
    for (int k = 0; k < T; ++k) {
      F* tri = params.data() + (size_t)k * kParams;
      for (int q = 0; q < kParams; ++q)
        if (std::isnan(tri[q])) tri[q] = (F)0.5f;
      for (int q = 0; q < 6; ++q) tri[q] = rclamp(tri[q], (F)-0.25f, (F)1.25f);
      for (int q = 6; q < 9; ++q) tri[q] = rclamp(tri[q], (F)0, (F)1);
      tri[9] = rclamp(tri[9], (F)1e-3f, (F)0.999f);
    }
  }
  *n_losses = count;
  std::memcpy(best_params, best.data(), np * sizeof(F));
  std::memcpy(final_params, params.data(), np * sizeof(F));
  *best_iter = bi;
  *best_loss = bl;
  *stop_reason = stop;
  return 0;
}

}  // namespace

extern "C" {

// fit.rs:166-181 + Fitter::new/step (fit.rs:214-288), starting from the given
// seeded scene (params (T,10) + background). Returns the ConfigError code (or
// 0). Outputs: losses[iters] (n_losses filled), best_params (T,10),
// final_params (T,10), best_iter, best_loss, stop_reason (0 Completed,
// 1 Converged, 2 Diverged).
int oracle_fit(const float* target, int H, int W, const float* init_params, const float* bg,
               int T, const OracleFitConfig* cfg, float* losses, int64_t* n_losses,
               float* best_params, float* final_params, int64_t* best_iter, float* best_loss,
               int* stop_reason) {
  return fit_t<float>(target, H, W, init_params, bg, T, cfg, losses, n_losses, best_params,
                      final_params, best_iter, best_loss, stop_reason);
}

// The same fit with f64 parameters, moments and loss (the noise-floor twin).
int oracle64_fit(const float* target, int H, int W, const float* init_params, const float* bg,
                 int T, const OracleFitConfig* cfg, double* losses, int64_t* n_losses,
                 double* best_params, double* final_params, int64_t* best_iter,
                 double* best_loss, int* stop_reason) {
  return fit_t<double>(target, H, W, init_params, bg, T, cfg, losses, n_losses, best_params,
                       final_params, best_iter, best_loss, stop_reason);
}

int oracle_num_threads(void) { return clamp_threads(0); }

}  // extern "C"
