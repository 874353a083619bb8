// Single-token decode step: one CTA per (batch, head); the fp32 state is read once and
// written once (the kernel is HBM-bound: 2 * K * V * 4 bytes per (b, h)).
//
//   S~ = gamma .* S                        gamma[m] = exp(g) exp(-lam[m])
//   e  = v - beta (k^T S~) / kappa         (GDN form: v pre-scaled by beta)
//   o_r = (Q_r^T S~ + (Q_r . k) e) / kappa  == Q_r^T S_new / kappa
//   S_new = S~ + k e^T
// Follows lapa/layer.py:387-412 (LongHead.step), sca2/arch_gatedc.py:171-193
// (CHeadGated.step) and fla's recurrent GDN step.
#include "common.cuh"

namespace sca2 {
namespace step {

constexpr int NT = 256;
constexpr int MAXR = 32;  // largest number of state rows held in registers per thread

template <int FL, int VEC, int MAXR>
__global__ void __launch_bounds__(NT) step_kernel(sca2_scan_args p, const float* S_in,
                                                  float* S_out, sca2_out o) {
  extern __shared__ float sm[];
  constexpr int R = FL == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int K = p.K, V = p.V;
  const int slots = V / VEC;
  const int rg = max(1, min(NT / slots, K));
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)(K / 2) : 1.f;
  const float ik = 1.f / kappa;
  float* kk = sm;                 // K
  float* Q = kk + K;              // R*K
  float* gam = Q + R * K;         // K
  float* vv = gam + K;            // V
  float* red = vv + V;            // (1+R) * rg * V
  float* ee = red + (1 + R) * rg * V;  // V
  float* scal = ee + V;           // 4

  // ---- prologue
  const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
  const float* gp = reinterpret_cast<const float*>(p.g.ptr);
  const float bt = bp ? bp[tok_off(p.beta, b, 0, h)] : 0.f;
  const float gdec = gp ? expf(gp[tok_off(p.g, b, 0, h)]) : 1.f;
  if (FL == SCA2_FLAVOR_PHASE) {
    const int Mh = K / 2;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
    for (int m = threadIdx.x; m < Mh; m += blockDim.x) {
      float s, c, sq, cq;
      sincosf(phw[tok_off(p.phw, b, 0, h) + m], &s, &c);
      sincosf(phq[tok_off(p.phq, b, 0, h) + m], &sq, &cq);
      const float wr = p.wr[h * Mh + m], wi = p.wi[h * Mh + m];
      const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
      kk[m] = c;
      kk[m + Mh] = s;
      Q[m] = c1;
      Q[m + Mh] = c2;
      Q[K + m] = -c2;
      Q[K + m + Mh] = c1;
      const float l = p.lam ? p.lam[h * Mh + m] : 0.f;
      gam[m] = gam[m + Mh] = gdec * expf(-l);
    }
  } else {
    for (int m = threadIdx.x; m < K; m += blockDim.x) {
      kk[m] = ld_io(p.phw.ptr, tok_off(p.phw, b, 0, h) + m, p.io_dtype);
      Q[m] = p.q_scale * ld_io(p.phq.ptr, tok_off(p.phq, b, 0, h) + m, p.io_dtype);
      const float l = p.lam ? p.lam[h * K + m] : 0.f;
      gam[m] = gdec * expf(-l);
    }
  }
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float x = ld_io(p.v.ptr, tok_off(p.v, b, 0, h) + j, p.io_dtype);
    if (p.v_times_beta) x *= bt;
    vv[j] = x;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // Q_r . k
    for (int r = 0; r < R; ++r) {
      float s = 0.f;
      for (int m = threadIdx.x; m < K; m += 32) s += Q[r * K + m] * kk[m];
      s = warp_sum(s);
      if (threadIdx.x == 0) scal[r] = s;
    }
  }

  // ---- pass over the state: decay, partial reductions over rows
  const int tx = threadIdx.x % slots, ty = threadIdx.x / slots;
  const bool active = threadIdx.x < slots * rg;
  const int64_t base = (int64_t)bh * K * V;
  float s_reg[MAXR][VEC];
  float pk[VEC], pq[R][VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
    pk[c] = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) pq[r][c] = 0.f;
  }
  if (active) {
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      const int m = ty + q * rg;
      if (m < K) {
        float x[VEC];
        if (VEC == 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(S_in + base + (int64_t)m * V + tx * 4);
          x[0] = t4.x; x[1] = t4.y; x[2] = t4.z; x[3] = t4.w;
        } else {
          x[0] = S_in[base + (int64_t)m * V + tx];
        }
        const float gm = gam[m], km = kk[m];
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
          const float s = gm * x[c];
          s_reg[q][c] = s;
          pk[c] = fmaf(km, s, pk[c]);
#pragma unroll
          for (int r = 0; r < R; ++r) pq[r][c] = fmaf(Q[r * K + m], s, pq[r][c]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const int j = tx * VEC + c;
      red[ty * V + j] = pk[c];
#pragma unroll
      for (int r = 0; r < R; ++r) red[((1 + r) * rg + ty) * V + j] = pq[r][c];
    }
  }
  __syncthreads();
  // ---- column reductions: e, o
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float sk = 0.f;
    for (int y = 0; y < rg; ++y) sk += red[y * V + j];
    const float e = vv[j] - bt * sk * ik;
    ee[j] = e;
    for (int r = 0; r < R; ++r) {
      float sq = 0.f;
      for (int y = 0; y < rg; ++y) sq += red[((1 + r) * rg + y) * V + j];
      st_io(o.ptr, out_off(o, b, 0, h, r) + j, (sq + scal[r] * e) * ik, p.io_dtype);
    }
  }
  __syncthreads();
  // ---- write the new state
  if (active) {
    float ev[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) ev[c] = ee[tx * VEC + c];
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      const int m = ty + q * rg;
      if (m < K) {
        const float km = kk[m];
        if (VEC == 4) {
          float4 t4;
          t4.x = fmaf(km, ev[0], s_reg[q][0]);
          t4.y = fmaf(km, ev[1], s_reg[q][1]);
          t4.z = fmaf(km, ev[2], s_reg[q][2]);
          t4.w = fmaf(km, ev[3], s_reg[q][3]);
          *reinterpret_cast<float4*>(S_out + base + (int64_t)m * V + tx * 4) = t4;
        } else {
          S_out[base + (int64_t)m * V + tx] = fmaf(km, ev[0], s_reg[q][0]);
        }
      }
    }
  }
}

}  // namespace step

// Rows of state each thread must hold; the launcher rejects shapes needing more than MAXR.
int step_rows_per_thread(int K, int V, int vec) {
  const int slots = V / vec;
  if (slots > step::NT) return 1 << 30;
  const int rg = slots > 0 ? (step::NT / slots < K ? step::NT / slots : K) : 1;
  return (K + rg - 1) / (rg > 0 ? rg : 1);
}
int step_max_rows() { return step::MAXR; }  // rows per thread of the widest variant

size_t step_smem_bytes(int K, int V, int R, int vec) {
  const int slots = V / vec;
  int rg = step::NT / slots;
  if (rg > K) rg = K;
  if (rg < 1) rg = 1;
  return (size_t)(K + R * K + K + V + (1 + R) * rg * V + V + 4) * 4;
}

template <int FL, int VEC, int MR>
static void launch_step_t(const sca2_scan_args& p, const float* S_in, float* S_out,
                          const sca2_out& o, size_t smem, cudaStream_t st) {
  auto k = step::step_kernel<FL, VEC, MR>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k<<<dim3(p.B * p.H), step::NT, smem, st>>>(p, S_in, S_out, o);
}

template <int FL, int VEC>
static void launch_step_v(const sca2_scan_args& p, const float* S_in, float* S_out,
                          const sca2_out& o, size_t smem, int rows, cudaStream_t st) {
  if (rows <= 4)
    launch_step_t<FL, VEC, 4>(p, S_in, S_out, o, smem, st);
  else if (rows <= 16)
    launch_step_t<FL, VEC, 16>(p, S_in, S_out, o, smem, st);
  else
    launch_step_t<FL, VEC, 32>(p, S_in, S_out, o, smem, st);
}

cudaError_t launch_step(const sca2_scan_args& p, const float* S_in, float* S_out,
                        const sca2_out& o, int vec, cudaStream_t st) {
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  const size_t smem = step_smem_bytes(p.K, p.V, R, vec);
  const int rows = step_rows_per_thread(p.K, p.V, vec);
  if (p.flavor == SCA2_FLAVOR_PHASE) {
    if (vec == 4) launch_step_v<SCA2_FLAVOR_PHASE, 4>(p, S_in, S_out, o, smem, rows, st);
    else launch_step_v<SCA2_FLAVOR_PHASE, 1>(p, S_in, S_out, o, smem, rows, st);
  } else {
    if (vec == 4) launch_step_v<SCA2_FLAVOR_KEY, 4>(p, S_in, S_out, o, smem, rows, st);
    else launch_step_v<SCA2_FLAVOR_KEY, 1>(p, S_in, S_out, o, smem, rows, st);
  }
  return cudaGetLastError();
}

// ---- RMS read-out ---------------------------------------------------------------------
namespace rms {
constexpr int NT = 256;
// one warp per row
__global__ void __launch_bounds__(NT) rms_fwd_kernel(const void* x, void* u, int64_t N, int D,
                                                     float eps, int dt) {
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const int64_t off = row * D;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    ss = fmaf(a, a, ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  for (int j = lane; j < D; j += 32) st_io(u, off + j, ld_io(x, off + j, dt) * r, dt);
}

__global__ void __launch_bounds__(NT) rms_bwd_kernel(const void* x, const void* du, void* dx,
                                                     int64_t N, int D, float eps, int dt) {
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const int64_t off = row * D;
  float ss = 0.f, sd = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    ss = fmaf(a, a, ss);
    sd = fmaf(a, ld_io(du, off + j, dt), sd);
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  const float r = rsqrtf(ss / (float)D + eps);
  const float c = r * r * sd / (float)D;  // mean(du * u) / r
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    const float g = ld_io(du, off + j, dt);
    st_io(dx, off + j, r * (g - a * c), dt);
  }
}
}  // namespace rms

cudaError_t launch_rms_fwd(const void* x, void* u, int64_t N, int D, float eps, int dt,
                           cudaStream_t st) {
  const int64_t blocks = (N + rms::NT / 32 - 1) / (rms::NT / 32);
  rms::rms_fwd_kernel<<<(unsigned)blocks, rms::NT, 0, st>>>(x, u, N, D, eps, dt);
  return cudaGetLastError();
}
cudaError_t launch_rms_bwd(const void* x, const void* du, void* dx, int64_t N, int D, float eps,
                           int dt, cudaStream_t st) {
  const int64_t blocks = (N + rms::NT / 32 - 1) / (rms::NT / 32);
  rms::rms_bwd_kernel<<<(unsigned)blocks, rms::NT, 0, st>>>(x, du, dx, N, D, eps, dt);
  return cudaGetLastError();
}

}  // namespace sca2
