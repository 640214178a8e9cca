// Rounding helpers of the soft-edge arithmetic (sm_100a).
//
// Quotients, square roots and the sigmoid with the reference's rounding, built
// from the hardware approximations and one Newton-Raphson correction each, with
// no library slow path. Used by dr_kernels.cu; a test kernel
// (tests/cuda/rounding_check.cu) compares them with CUDA's IEEE operations.
#pragma once

#include <cuda_runtime.h>

namespace dr {

// Quotients and square roots rounded to nearest without the library's
// special-case branches: the hardware approximation (rcp.approx / rsqrt.approx,
// relative error below 2^-22) refined by one Newton-Raphson step with an FMA
// residual (Markstein's method). The refined value is within ~2^-44 of the
// exact result, so it rounds correctly except for inputs whose exact result
// lies that close to a rounding midpoint. Valid for normal, positive inputs.
__device__ __forceinline__ float rcp_approx(float y) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}
__device__ __forceinline__ float rsqrt_approx(float x) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// sqrt(x) for x >= 0; inputs below 1e-30 (distances far under the 1e-9 cut
// of grad.rs:252) return 0.
__device__ __forceinline__ float sqrt_nr(float x) {
  const float rs = rsqrt_approx(x);
  const float s = __fmul_rn(x, rs);
  const float res = __fmaf_rn(-s, s, x);
  const float out = __fmaf_rn(res, __fmul_rn(0.5f, rs), s);
  return x > 1e-30f ? out : 0.0f;
}

// a / b rounded to nearest, given inv_b within 2^-22 of 1 / b (rcp_approx, or
// a precomputed RN(1 / b)): one correction step on the product with an FMA
// residual. For a = 1 this is the Newton-refined reciprocal.
__device__ __forceinline__ float div_rn_inv(float a, float b, float inv_b) {
  const float q0 = __fmul_rn(a, inv_b);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, inv_b, q0);
}

// Sigmoid of raster.rs:79-87 with its rounding: RN(1 / RN(1 + e)) for x >= 0,
// RN(e / RN(1 + e)) below, e = exp(-|x|). The exponential may be approximate:
// its error moves 1 + e by far less than an ulp of 1 wherever e is small,
// while near cov == 1 the gradient uses 1 - cov, which depends on exactly how
// the reference rounded cov.
__device__ __forceinline__ float sigmoid_rounded(float x) {
  const float e = __expf(-fabsf(x));
  const float y = __fadd_rn(1.0f, e);
  return div_rn_inv(x >= 0.0f ? 1.0f : e, y, rcp_approx(y));
}

__device__ __forceinline__ float sigmoid_fast(float x) {
  const float e = __expf(-fabsf(x));
  return __fdividef(x >= 0.0f ? 1.0f : e, __fadd_rn(1.0f, e));
}

}  // namespace dr
