// Test kernel for the rounding helpers in dr_math.cuh (built by
// tests/test_gpu_rounding.py with nvcc; not part of the library).
//
// For n inputs it writes, per element, each helper's result next to CUDA's
// IEEE operation for the same input:
//   out[0] div_rn_inv(a, b, rcp.approx(b))   out[1] __fdiv_rn(a, b)
//   out[2] sqrt_nr(x)                         out[3] __fsqrt_rn(x)
//   out[4] sigmoid_rounded(s)                 out[5] sigmoid_ref(s) (expf, __fdiv_rn)
// with x = |a| and s = a (the sigmoid's argument).

#include <cuda_runtime.h>

#include "dr_device.cuh"
#include "dr_math.cuh"

__global__ void rounding_kernel(const float* __restrict__ a, const float* __restrict__ b, int n,
                                float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = a[i], y = b[i];
  out[0 * (size_t)n + i] = dr::div_rn_inv(x, y, dr::rcp_approx(y));
  out[1 * (size_t)n + i] = __fdiv_rn(x, y);
  out[2 * (size_t)n + i] = dr::sqrt_nr(fabsf(x));
  out[3 * (size_t)n + i] = __fsqrt_rn(fabsf(x));
  out[4 * (size_t)n + i] = dr::sigmoid_rounded(x);
  out[5 * (size_t)n + i] = dr::sigmoid_ref(x);
}

extern "C" int rounding_check(const float* a, const float* b, int n, float* out) {
  if (n <= 0) return 0;
  rounding_kernel<<<(n + 255) / 256, 256>>>(a, b, n, out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return (int)e;
}
