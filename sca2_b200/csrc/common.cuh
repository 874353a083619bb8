// Shared device helpers for the sca2b200 scan kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sca2b200.h"

namespace sca2 {

// ---- element access -------------------------------------------------------------
__device__ __forceinline__ float ld_io(const void* p, int64_t i, int dt) {
  return dt == SCA2_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                         : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_io(void* p, int64_t i, float x, int dt) {
  if (dt == SCA2_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else
    reinterpret_cast<float*>(p)[i] = x;
}
__device__ __forceinline__ int64_t tok_off(const sca2_tok& t, int b, int tt, int h) {
  return (int64_t)b * t.sb + (int64_t)tt * t.st + (int64_t)h * t.sh;
}
__device__ __forceinline__ int64_t out_off(const sca2_out& t, int b, int tt, int h, int r) {
  return (int64_t)b * t.sb + (int64_t)tt * t.st + (int64_t)h * t.sh + (int64_t)r * t.sr;
}

// ---- division by a runtime divisor ------------------------------------------------------
// floor(u / d) by a multiply-high with m = magic(d) = ceil(2^32 / d): u m / 2^32 = u / d +
// u e / (d 2^32) with e = m d - 2^32 < d, so the floor is exact while u e < 2^32 (u < 2^32 / d
// suffices).  d = 1 would need m = 2^32: it is encoded as m = 0 and returns u.
__host__ __device__ constexpr uint32_t magic(uint32_t d) { return d > 1 ? 0xFFFFFFFFu / d + 1u : 0u; }
__device__ __forceinline__ int qdiv(int u, uint32_t m) { return m ? (int)__umulhi((uint32_t)u, m) : u; }

// ---- sine and cosine of large phases -----------------------------------------------------
// Cody and Waite's additive reduction (W. J. Cody, W. Waite, "Software Manual for the Elementary
// Functions", 1980): r = x - k 2pi with k = rint(x / 2pi) and 2pi split into three parts, the
// first with only 9 significant bits so k * part1 is exact for |k| < 2^15 (|x| < 2e5), then the
// SFU sine / cosine on r in [-pi, pi] (absolute error about 1e-6 for the phases of this scan).
__device__ __forceinline__ void sincos_big(float x, float* s, float* c) {
  constexpr float kInv2Pi = 0.15915494309189535f;
  constexpr float kP1 = 6.28125f;                   // 2pi rounded to 9 bits
  constexpr float kP2 = 1.9353071795864769e-3f;     // 2pi - kP1, rounded to fp32
  constexpr float kP3 = 1.0253131677018246e-11f;    // 2pi - kP1 - kP2, rounded to fp32
  const float k = rintf(x * kInv2Pi);
  float r = fmaf(-k, kP1, x);
  r = fmaf(-k, kP2, r);
  r = fmaf(-k, kP3, r);
  __sincosf(r, s, c);
}

// Slots of the saved-state buffer (B,H,slots,K,V) for T tokens: four per 64-token chunk.  The
// fp32 path keeps the state entering its 32-token chunk c in slot c; the tensor-core path keeps
// the state entering its 64-token chunk c in slot 2c, its saved T and E in slot 2c+1 and its
// masked, decayed read kernel P (bf16, operand layout) in slot 2 NC + c; the chunk-parallel
// explicit-key path (K = V = 128) uses slots 4c .. 4c+3 (gdn_cp.cu).
__host__ __device__ inline int state_slots(int T) { return 4 * ((T + 63) / 64); }

// Phases formed inside the kernels from the head's projections (phase flavour): when `on`,
// phw / phq hold K(h) / K(z) in `dtype` and phi = K(h) theta + (pos + t) omega, psi likewise,
// each product rounded to fp32 and then summed (the reference's fp32 expression).
struct PhaseProj {
  int on;
  int dtype;             // SCA2_F32 or SCA2_BF16
  const float* theta;    // (H, Mh)
  const float* omega;    // (H, Mh)
  const float* pos;      // device scalar, or nullptr = 0
};

// exp of a difference of cumulative log-decays, clamped at 0 before exp so masked
// (anti-causal) entries never overflow (sca2/versions/README.md:69-75).
__device__ __forceinline__ float exp_le0(float x) { return expf(fminf(x, 0.f)); }

// ---- small shared-memory GEMM -------------------------------------------------------
// acc(i, j) = sum_{k < KD} A(i, k) * B(k, j) for i < M, j < N, handed to epi(i, j, acc).
// Each thread owns a TM x TN micro tile with STRIDED rows / columns (row i = tm + ii*M/TM,
// column j = tn + jj*N/TN) so that a warp reads consecutive columns of B (no bank
// conflicts) and broadcasts rows of A.  M % TM == 0 and N % TN == 0 are required; all
// operands live in shared memory and are accessed through the load functors.
template <int TM, int TN, class LA, class LB, class EPI>
__device__ __forceinline__ void smem_gemm(int M, int N, int KD, LA la, LB lb, EPI epi) {
  const int tiles_m = M / TM, tiles_n = N / TN;
  const int ntiles = tiles_m * tiles_n;
  for (int t = threadIdx.x; t < ntiles; t += blockDim.x) {
    const int tm = t / tiles_n, tn = t - (t / tiles_n) * tiles_n;
    float acc[TM][TN];
#pragma unroll
    for (int ii = 0; ii < TM; ++ii)
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) acc[ii][jj] = 0.f;
    for (int k = 0; k < KD; ++k) {
      float av[TM], bv[TN];
#pragma unroll
      for (int ii = 0; ii < TM; ++ii) av[ii] = la(tm + ii * tiles_m, k);
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) bv[jj] = lb(k, tn + jj * tiles_n);
#pragma unroll
      for (int ii = 0; ii < TM; ++ii)
#pragma unroll
        for (int jj = 0; jj < TN; ++jj) acc[ii][jj] = fmaf(av[ii], bv[jj], acc[ii][jj]);
    }
#pragma unroll
    for (int ii = 0; ii < TM; ++ii)
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) epi(tm + ii * tiles_m, tn + jj * tiles_n, acc[ii][jj]);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// inclusive prefix sum over the 32 lanes of a warp
__device__ __forceinline__ float warp_incl_scan(float x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

}  // namespace sca2
