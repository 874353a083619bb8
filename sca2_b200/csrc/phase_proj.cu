// Backward of the projected-phase prologue (sm_100a).  With the phases formed inside the scan
// kernels as phi = K(h) theta + (pos + t) omega and psi = K(z) theta + (pos + t) omega, the
// scan's backward produces d(phi), d(psi) (fp32); this pass turns them into the gradients of
// the projections and of theta:
//
//   dK(h) = d(phi) theta,  dK(z) = d(psi) theta,  dtheta = sum_{b,t} d(phi) K(h) + d(psi) K(z)
//
// (the chain rule of the reference's K(x) theta + p omega; omega is a buffer, positions carry no
// gradient).  One thread per (token, head, 8 modes), 16-byte loads and stores; dtheta is summed
// per CTA in shared memory and across CTAs by a fixed-order pass (deterministic).
#include "common.cuh"

namespace sca2 {
namespace pproj {

constexpr int NT = 256;

__device__ __forceinline__ void ld8(const void* base, int64_t off, int dtype, float* x) {
  if (dtype == SCA2_BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) { x[2 * k] = __low2float(h2[k]); x[2 * k + 1] = __high2float(h2[k]); }
  } else {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
    const float4 a = q[0], c = q[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  }
}
__device__ __forceinline__ void st8(void* base, int64_t off, int dtype, const float* x) {
  if (dtype == SCA2_BF16) {
    uint4 u;
    __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) h2[k] = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + off) = u;
  } else {
    float4* q = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + off);
    q[0] = make_float4(x[0], x[1], x[2], x[3]);
    q[1] = make_float4(x[4], x[5], x[6], x[7]);
  }
}

// dphi, dpsi: (B,T,H,Mh) fp32 contiguous.  kh, kz: the projections (strided, dtype); dkh, dkz
// likewise.  part: gridDim.x x (H*Mh) partial sums of dtheta.
__global__ void __launch_bounds__(NT) proj_bwd_kernel(int B, int T, int H, int Mh, int dtype, const float* dphi,
                                                      const float* dpsi, sca2_tok kh, sca2_tok kz, const float* theta,
                                                      sca2_tok dkh, sca2_tok dkz, float* part) {
  extern __shared__ float red[];  // H * Mh
  const int HM = H * Mh, U = HM / 8;
  for (int u = threadIdx.x; u < HM; u += NT) red[u] = 0.f;
  __syncthreads();
  const int64_t units = (int64_t)B * T * U;
  for (int64_t u = (int64_t)blockIdx.x * NT + threadIdx.x; u < units; u += (int64_t)gridDim.x * NT) {
    const int64_t bt = u / U;
    const int r = (int)(u - bt * U), h = (r * 8) / Mh, m0 = r * 8 - h * Mh;
    const int b = (int)(bt / T), t = (int)(bt - (int64_t)b * T);
    const int64_t g = bt * HM + (int64_t)r * 8;
    float dp[8], dq[8], xh[8], xz[8], th[8], yh[8], yz[8];
    {
      const float4* a = reinterpret_cast<const float4*>(dphi + g);
      const float4* c = reinterpret_cast<const float4*>(dpsi + g);
      const float4 a0 = a[0], a1 = a[1], c0 = c[0], c1 = c[1];
      dp[0] = a0.x; dp[1] = a0.y; dp[2] = a0.z; dp[3] = a0.w; dp[4] = a1.x; dp[5] = a1.y; dp[6] = a1.z; dp[7] = a1.w;
      dq[0] = c0.x; dq[1] = c0.y; dq[2] = c0.z; dq[3] = c0.w; dq[4] = c1.x; dq[5] = c1.y; dq[6] = c1.z; dq[7] = c1.w;
    }
    ld8(kh.ptr, tok_off(kh, b, t, h) + m0, dtype, xh);
    ld8(kz.ptr, tok_off(kz, b, t, h) + m0, dtype, xz);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      th[k] = theta[h * Mh + m0 + k];
      yh[k] = dp[k] * th[k];
      yz[k] = dq[k] * th[k];
      atomicAdd(red + h * Mh + m0 + k, fmaf(dp[k], xh[k], dq[k] * xz[k]));
    }
    st8(const_cast<void*>(dkh.ptr), tok_off(dkh, b, t, h) + m0, dtype, yh);
    st8(const_cast<void*>(dkz.ptr), tok_off(dkz, b, t, h) + m0, dtype, yz);
  }
  __syncthreads();
  for (int u = threadIdx.x; u < HM; u += NT) part[(int64_t)blockIdx.x * HM + u] = red[u];
}

__global__ void proj_reduce_kernel(const float* part, int nparts, int HM, float* dtheta) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= HM) return;
  float acc = 0.f;
  for (int k = 0; k < nparts; ++k) acc += part[(int64_t)k * HM + u];
  dtheta[u] = acc;
}

constexpr int kGrid = 296;  // 2 CTAs per SM

}  // namespace pproj

size_t proj_work_floats(int B, int T, int H, int Mh) {
  return 2 * (size_t)B * T * H * Mh + (size_t)pproj::kGrid * H * Mh;
}

// dphi / dpsi scratch at the start of `work`, then the partials
cudaError_t proj_bwd(int B, int T, int H, int Mh, int dtype, const float* work, const sca2_tok& kh,
                     const sca2_tok& kz, const float* theta, const sca2_tok& dkh, const sca2_tok& dkz, float* dtheta,
                     cudaStream_t st) {
  const size_t n = (size_t)B * T * H * Mh;
  const float* dphi = work;
  const float* dpsi = work + n;
  float* part = const_cast<float*>(work) + 2 * n;
  const int HM = H * Mh;
  pproj::proj_bwd_kernel<<<pproj::kGrid, pproj::NT, HM * sizeof(float), st>>>(B, T, H, Mh, dtype, dphi, dpsi, kh,
                                                                              kz, theta, dkh, dkz, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  pproj::proj_reduce_kernel<<<(HM + 127) / 128, 128, 0, st>>>(part, pproj::kGrid, HM, dtheta);
  return cudaGetLastError();
}

}  // namespace sca2
