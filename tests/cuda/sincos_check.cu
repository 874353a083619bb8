// Test harness: evaluates sincos_big (the phase codes of the tensor-core kernels and of the
// short head) and CUDA's sincosf on the same inputs so the test can compare both against float64.
#include "../../sca2_b200/csrc/common.cuh"

__global__ void sincos_check_kernel(const float* x, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s, c, s2, c2;
  sca2::sincos_big(x[i], &s, &c);
  sincosf(x[i], &s2, &c2);
  out[4 * i + 0] = s;
  out[4 * i + 1] = c;
  out[4 * i + 2] = s2;
  out[4 * i + 3] = c2;
}

extern "C" int sincos_check(const float* x, float* out, int n) {
  sincos_check_kernel<<<(n + 255) / 256, 256>>>(x, out, n);
  return (int)cudaDeviceSynchronize();
}
