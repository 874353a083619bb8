// Short head (sm_100a): the exact L-tap window read of the LapA / SCA2 short head, forward
// (prefill and decode), backward, and the ring-buffer update.
//
//   phi_t = K(h_t) theta + ((pos + t) mod L) omega,   psi_t = K(z_t) theta + ((pos + t) mod L) omega
//   kappa(t, s) = (1/L) sum_m (wr + i wi)_m e^{i (phi_s - psi_t)}
//   o_t = [ sum_{s=t-L+1..t} Re kappa(t,s) e_s  |  sum Im kappa(t,s) e_s ]
//
// (lapa/layer.py:418-545 ShortHead._read/_banded/step; sca2/arch_short.py:45-158).  The
// L-1 previous writes come from the state (c = cos phi, s = sin phi, e = value, oldest
// first) and are prepended to the call's own writes ("extended" index x = s + L - 1).
//
// Everything is fp32 on the CUDA cores: the DFT grid's comb (sum over m of e^{i m 2pi k / L})
// cancels to zero at every lag k != 0 only to fp32 rounding, and bf16 tensor-core operands
// would turn that exact zero into a visible leak between lags.  The work is small (L (2L + 2dv)
// multiply-adds per token) and independent across tokens, so each CTA takes TT consecutive
// queries of one sequence and the L-1 keys before them; the codes (sin / cos of the phases,
// computed here from K(h), K(z), theta, omega and the position), kappa and the values sit in
// shared memory with odd row strides so that lanes walking different keys hit different banks.
// Values and output gradients are processed in slices of DS columns, so dv is unbounded.
#include "common.cuh"

namespace sca2 {
namespace shortk {

constexpr int NT = 256;
constexpr int DS = 64;  // value columns per slice
constexpr int DSP = DS + 1;

__device__ __forceinline__ int pmod(long long p, int L) {
  long long r = p % L;
  return (int)(r < 0 ? r + L : r);
}

struct Geo {
  int L, n, LP, dv, T, TT, t0, tq;
};
__device__ __forceinline__ Geo geo(const sca2_short_args& p, int TT) {
  Geo g;
  g.L = p.L;
  g.n = p.L - 1;
  g.LP = p.L + 1;
  g.dv = p.dv;
  g.T = p.T;
  g.TT = TT;
  g.t0 = blockIdx.x * TT;
  g.tq = min(TT, p.T - g.t0);
  return g;
}

// cos / sin of the write phase of extended key x of this CTA (token s = t0 - n + x), from
// the state for s < 0
__device__ __forceinline__ void key_code(const sca2_short_args& p, const Geo& g, int b, long long p0, int s, int l,
                                         float* c, float* sn) {
  if (s < 0) {
    const int64_t k = ((int64_t)b * g.n + g.n + s) * g.L + l;
    *c = p.c0 ? p.c0[k] : 1.f;
    *sn = p.s0 ? p.s0[k] : 0.f;
  } else {
    const float ph = p.kh[((int64_t)b * g.T + s) * g.L + l] * p.theta[l] + (float)pmod(p0 + s, g.L) * p.omega[l];
    sincosf(ph, sn, c);
  }
}
__device__ __forceinline__ float key_value(const sca2_short_args& p, const Geo& g, int b, int s, int j) {
  if (s < 0) return p.e0 ? p.e0[((int64_t)b * g.n + g.n + s) * g.dv + j] : 0.f;
  return p.v[((int64_t)b * g.T + s) * g.dv + j];
}

size_t fwd_smem_floats(int L, int TT) {
  const int n = L - 1, LP = L + 1;
  return (size_t)(TT + n) * (2 * LP + DSP) + (size_t)TT * (2 * LP + 2 * L);
}
size_t bwd_smem_floats(int L, int TT) {
  const int n = L - 1, LP = L + 1, NX = TT + n;
  return (size_t)NX * (2 * LP + DSP) + (size_t)NX * (4 * LP + 4 * L + 2 * DSP) + 3 * L;
}

__global__ void __launch_bounds__(NT) short_fwd_kernel(sca2_short_args p, float* o, int TT) {
  extern __shared__ float sm[];
  const Geo g = geo(p, TT);
  const int tid = threadIdx.x, b = blockIdx.y, L = g.L, n = g.n, LP = g.LP, dv = g.dv;
  const int NX = g.tq + n;
  float* KC = sm;                    // keys: cos, sin  [x][l]  (stride LP)
  float* KS = KC + (TT + n) * LP;
  float* E = KS + (TT + n) * LP;     // values slice [x][j]  (stride DSP)
  float* Q1 = E + (TT + n) * DSP;    // read codes c1, c2  [i][l]
  float* Q2 = Q1 + TT * LP;
  float* KR = Q2 + TT * LP;          // kappa [i][lag]
  float* KI = KR + TT * L;
  const long long p0 = p.pos ? *p.pos : 0;
  for (int u = tid; u < NX * L; u += NT) {
    const int x = u / L, l = u - (u / L) * L;
    float c, s;
    key_code(p, g, b, p0, g.t0 - n + x, l, &c, &s);
    KC[x * LP + l] = c;
    KS[x * LP + l] = s;
  }
  for (int u = tid; u < g.tq * L; u += NT) {
    const int i = u / L, l = u - (u / L) * L, t = g.t0 + i;
    const float ph = p.kz[((int64_t)b * g.T + t) * L + l] * p.theta[l] + (float)pmod(p0 + t, L) * p.omega[l];
    float s, c;
    sincosf(ph, &s, &c);
    const float wr = p.wr[l], wi = p.wi[l];
    Q1[i * LP + l] = wr * c + wi * s;
    Q2[i * LP + l] = wr * s - wi * c;
  }
  __syncthreads();
  const float iL = 1.f / (float)L;
  for (int u = tid; u < g.tq * L; u += NT) {
    const int i = u / L, lag = u - (u / L) * L, x = i + n - lag;
    float kr = 0.f, ki = 0.f;
    for (int l = 0; l < L; ++l) {
      const float kc = KC[x * LP + l], ks = KS[x * LP + l], q1 = Q1[i * LP + l], q2 = Q2[i * LP + l];
      kr = fmaf(kc, q1, fmaf(ks, q2, kr));
      ki = fmaf(ks, q1, fmaf(-kc, q2, ki));
    }
    KR[i * L + lag] = kr * iL;
    KI[i * L + lag] = ki * iL;
  }
  for (int j0 = 0; j0 < dv; j0 += DS) {
    const int w = min(DS, dv - j0);
    __syncthreads();  // kappa written / previous slice consumed
    for (int u = tid; u < NX * w; u += NT) {
      const int x = u / w, j = u - (u / w) * w;
      E[x * DSP + j] = key_value(p, g, b, g.t0 - n + x, j0 + j);
    }
    __syncthreads();
    for (int u = tid; u < g.tq * w; u += NT) {
      const int i = u / w, j = u - (u / w) * w;
      float ar = 0.f, ai = 0.f;
      for (int lag = 0; lag < L; ++lag) {
        const float ev = E[(i + n - lag) * DSP + j];
        ar = fmaf(KR[i * L + lag], ev, ar);
        ai = fmaf(KI[i * L + lag], ev, ai);
      }
      float* orow = o + ((int64_t)b * g.T + g.t0 + i) * 2 * dv;
      orow[j0 + j] = ar;
      orow[dv + j0 + j] = ai;
    }
  }
}

// new ring buffer: entry k (0 <= k < n) is extended index T + k, i.e. token T - n + k
__global__ void __launch_bounds__(NT) short_state_kernel(sca2_short_args p, float* c1, float* s1, float* e1) {
  const int b = blockIdx.x, L = p.L, n = L - 1, dv = p.dv, T = p.T;
  Geo g;
  g.L = L; g.n = n; g.LP = L + 1; g.dv = dv; g.T = T; g.TT = 0; g.t0 = 0; g.tq = 0;
  const long long p0 = p.pos ? *p.pos : 0;
  for (int u = threadIdx.x; u < n * L; u += NT) {
    const int k = u / L, l = u - (u / L) * L;
    float c, s;
    key_code(p, g, b, p0, T - n + k, l, &c, &s);
    c1[((int64_t)b * n + k) * L + l] = c;
    s1[((int64_t)b * n + k) * L + l] = s;
  }
  for (int u = threadIdx.x; u < n * dv; u += NT) {
    const int k = u / dv, j = u - (u / dv) * dv;
    e1[((int64_t)b * n + k) * dv + j] = key_value(p, g, b, T - n + k, j);
  }
}

// Backward of one CTA: queries [t0, t0 + tq) and the keys it owns, [t0, t0 + tq) plus the
// buffered keys [-n, 0) for the first CTA.  Key s is read by queries s .. s + n, so the CTA
// also loads the n queries after its own (up to T) and recomputes their kappa for the pairs
// that reach its keys.  Pairs are indexed (y, lag): query t = t0 + y, key s = t - lag,
// extended key x = y + n - lag (< NX = tq + n for the pairs this CTA needs).
__global__ void __launch_bounds__(NT) short_bwd_kernel(sca2_short_args p, const float* dO, const float* dc1,
                                                       const float* ds1, const float* de1, sca2_short_grads gr,
                                                       float* part, int TT) {
  extern __shared__ float sm[];
  const Geo g = geo(p, TT);
  const int tid = threadIdx.x, b = blockIdx.y, L = g.L, n = g.n, LP = g.LP, dv = g.dv, T = g.T;
  const int NX = g.tq + n;                // keys  s = t0 - n + x
  const int NY = min(g.tq + n, T - g.t0);  // queries t = t0 + y
  float* KC = sm;
  float* KS = KC + (TT + n) * LP;
  float* E = KS + (TT + n) * LP;          // values slice [x][j]
  float* Q1 = E + (TT + n) * DSP;         // [y][l]
  float* Q2 = Q1 + (TT + n) * LP;
  float* CQ = Q2 + (TT + n) * LP;
  float* SQ = CQ + (TT + n) * LP;
  float* KR = SQ + (TT + n) * LP;         // kappa and its gradient [y][lag]
  float* KI = KR + (TT + n) * L;
  float* DKR = KI + (TT + n) * L;
  float* DKI = DKR + (TT + n) * L;
  float* GR = DKI + (TT + n) * L;         // dO slice [y][j], re then im
  float* GI = GR + (TT + n) * DSP;
  float* RED = GI + (TT + n) * DSP;       // dtheta, dwr, dwi partials of this CTA
  const long long p0 = p.pos ? *p.pos : 0;
  const float iL = 1.f / (float)L;
  for (int u = tid; u < 3 * L; u += NT) RED[u] = 0.f;
  for (int u = tid; u < NX * L; u += NT) {
    const int x = u / L, l = u - (u / L) * L;
    float c, s;
    key_code(p, g, b, p0, g.t0 - n + x, l, &c, &s);
    KC[x * LP + l] = c;
    KS[x * LP + l] = s;
  }
  for (int u = tid; u < NY * L; u += NT) {
    const int y = u / L, l = u - (u / L) * L, t = g.t0 + y;
    const float ph = p.kz[((int64_t)b * T + t) * L + l] * p.theta[l] + (float)pmod(p0 + t, L) * p.omega[l];
    float s, c;
    sincosf(ph, &s, &c);
    const float wr = p.wr[l], wi = p.wi[l];
    CQ[y * LP + l] = c;
    SQ[y * LP + l] = s;
    Q1[y * LP + l] = wr * c + wi * s;
    Q2[y * LP + l] = wr * s - wi * c;
  }
  __syncthreads();
  // kappa of every needed pair (zero for the pairs outside this CTA's keys)
  for (int u = tid; u < NY * L; u += NT) {
    const int y = u / L, lag = u - (u / L) * L, x = y + n - lag;
    float kr = 0.f, ki = 0.f;
    if (x < NX) {
      for (int l = 0; l < L; ++l) {
        const float kc = KC[x * LP + l], ks = KS[x * LP + l], q1 = Q1[y * LP + l], q2 = Q2[y * LP + l];
        kr = fmaf(kc, q1, fmaf(ks, q2, kr));
        ki = fmaf(ks, q1, fmaf(-kc, q2, ki));
      }
    }
    KR[y * L + lag] = kr * iL;
    KI[y * L + lag] = ki * iL;
    DKR[y * L + lag] = 0.f;
    DKI[y * L + lag] = 0.f;
  }
  // d kappa(t, s) = dO_t . e_s, accumulated over value slices (each thread keeps its pairs)
  for (int j0 = 0; j0 < dv; j0 += DS) {
    const int w = min(DS, dv - j0);
    __syncthreads();
    for (int u = tid; u < NX * w; u += NT) {
      const int x = u / w, j = u - (u / w) * w;
      E[x * DSP + j] = key_value(p, g, b, g.t0 - n + x, j0 + j);
    }
    for (int u = tid; u < NY * w; u += NT) {
      const int y = u / w, j = u - (u / w) * w;
      const float* row = dO + ((int64_t)b * T + g.t0 + y) * 2 * dv;
      GR[y * DSP + j] = row[j0 + j];
      GI[y * DSP + j] = row[dv + j0 + j];
    }
    __syncthreads();
    for (int u = tid; u < NY * L; u += NT) {
      const int y = u / L, lag = u - (u / L) * L, x = y + n - lag;
      if (x >= NX) continue;
      float ar = 0.f, ai = 0.f;
      for (int j = 0; j < w; ++j) {
        const float ev = E[x * DSP + j];
        ar = fmaf(GR[y * DSP + j], ev, ar);
        ai = fmaf(GI[y * DSP + j], ev, ai);
      }
      DKR[y * L + lag] += ar;
      DKI[y * L + lag] += ai;
    }
  }
  __syncthreads();
  // queries: d c1, d c2 -> d psi -> d K(z), and the theta / wr / wi partials
  for (int u = tid; u < g.tq * L; u += NT) {
    const int y = u / L, l = u - (u / L) * L, t = g.t0 + y;
    float a1 = 0.f, a2 = 0.f;
    for (int lag = 0; lag < L; ++lag) {
      const int x = y + n - lag;
      const float dr = DKR[y * L + lag], di = DKI[y * L + lag], kc = KC[x * LP + l], ks = KS[x * LP + l];
      a1 = fmaf(dr, kc, fmaf(di, ks, a1));
      a2 = fmaf(dr, ks, fmaf(-di, kc, a2));
    }
    a1 *= iL;
    a2 *= iL;
    const float cq = CQ[y * LP + l], sq = SQ[y * LP + l], wr = p.wr[l], wi = p.wi[l];
    const float dcq = a1 * wr - a2 * wi, dsq = a1 * wi + a2 * wr;
    const float dpsi = -sq * dcq + cq * dsq;
    const int64_t ti = ((int64_t)b * T + t) * L + l;
    gr.dkz[ti] = dpsi * p.theta[l];
    atomicAdd(RED + l, dpsi * p.kz[ti]);
    atomicAdd(RED + L + l, a1 * cq + a2 * sq);
    atomicAdd(RED + 2 * L + l, a1 * sq - a2 * cq);
  }
  // owned keys: x in [n, NX) (s = t0 .. t0 + tq - 1) and, for the first CTA, [0, n) (the buffer)
  const int x0 = g.t0 == 0 ? 0 : n;
  for (int u = tid; u < (NX - x0) * L; u += NT) {
    const int x = x0 + u / L, l = u - (u / L) * L, s = g.t0 - n + x;
    float dcw = 0.f, dsw = 0.f;
    for (int lag = 0; lag < L; ++lag) {
      const int y = x - n + lag;
      if (y < 0 || y >= NY) continue;
      const float dr = DKR[y * L + lag], di = DKI[y * L + lag], q1 = Q1[y * LP + l], q2 = Q2[y * LP + l];
      dcw = fmaf(dr, q1, fmaf(-di, q2, dcw));
      dsw = fmaf(dr, q2, fmaf(di, q1, dsw));
    }
    dcw *= iL;
    dsw *= iL;
    if (s >= T - n) {  // the key is also in the new ring buffer
      const int64_t k = ((int64_t)b * n + (s - (T - n))) * L + l;
      if (dc1) dcw += dc1[k];
      if (ds1) dsw += ds1[k];
    }
    if (s >= 0) {
      const float dphi = -KS[x * LP + l] * dcw + KC[x * LP + l] * dsw;
      const int64_t si = ((int64_t)b * T + s) * L + l;
      gr.dkh[si] = dphi * p.theta[l];
      atomicAdd(RED + l, dphi * p.kh[si]);
    } else {
      const int64_t k = ((int64_t)b * n + n + s) * L + l;
      if (gr.dc0) gr.dc0[k] = dcw;
      if (gr.ds0) gr.ds0[k] = dsw;
    }
  }
  // owned keys' values: d e_s = sum over the queries reading s of kappa . dO
  for (int j0 = 0; j0 < dv; j0 += DS) {
    const int w = min(DS, dv - j0);
    __syncthreads();
    for (int u = tid; u < NY * w; u += NT) {
      const int y = u / w, j = u - (u / w) * w;
      const float* row = dO + ((int64_t)b * T + g.t0 + y) * 2 * dv;
      GR[y * DSP + j] = row[j0 + j];
      GI[y * DSP + j] = row[dv + j0 + j];
    }
    __syncthreads();
    for (int u = tid; u < (NX - x0) * w; u += NT) {
      const int x = x0 + u / w, j = u - (u / w) * w, s = g.t0 - n + x;
      float acc = 0.f;
      for (int lag = 0; lag < L; ++lag) {
        const int y = x - n + lag;
        if (y < 0 || y >= NY) continue;
        acc = fmaf(KR[y * L + lag], GR[y * DSP + j], fmaf(KI[y * L + lag], GI[y * DSP + j], acc));
      }
      if (s >= T - n && de1) acc += de1[((int64_t)b * n + (s - (T - n))) * dv + j0 + j];
      if (s >= 0)
        gr.dv[((int64_t)b * T + s) * dv + j0 + j] = acc;
      else if (gr.de0)
        gr.de0[((int64_t)b * n + n + s) * dv + j0 + j] = acc;
    }
  }
  __syncthreads();
  float* dst = part + ((int64_t)b * gridDim.x + blockIdx.x) * 3 * L;
  for (int u = tid; u < 3 * L; u += NT) dst[u] = RED[u];
}

// dtheta, dwr, dwi = sums of the per-CTA partials (fixed order: deterministic)
__global__ void short_reduce_kernel(const float* part, int nparts, int L, sca2_short_grads gr) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= 3 * L) return;
  float acc = 0.f;
  for (int k = 0; k < nparts; ++k) acc += part[(int64_t)k * 3 * L + u];
  float* out = u < L ? gr.dtheta : u < 2 * L ? gr.dwr : gr.dwi;
  out[u % L] = acc;
}

}  // namespace shortk

int short_tokens_per_cta(int L, bool bwd, int max_smem) {
  const int cand[3] = {64, 32, 16};
  for (int i = 0; i < 3; ++i) {
    const size_t f = bwd ? shortk::bwd_smem_floats(L, cand[i]) : shortk::fwd_smem_floats(L, cand[i]);
    if (f * sizeof(float) <= 112u * 1024u || (i == 2 && f * sizeof(float) <= (size_t)max_smem)) return cand[i];
  }
  return 0;
}

size_t short_work_floats(int B, int T, int L, int max_smem) {
  const int TT = short_tokens_per_cta(L, true, max_smem);
  if (TT == 0 || T < 1) return 0;
  return (size_t)B * ((T + TT - 1) / TT) * 3 * L;
}

cudaError_t short_fwd(const sca2_short_args& p, float* o, float* c1, float* s1, float* e1, int max_smem,
                      cudaStream_t st) {
  if (p.T > 0) {
    const int TT = short_tokens_per_cta(p.L, false, max_smem);
    const int smem = (int)(shortk::fwd_smem_floats(p.L, TT) * sizeof(float));
    cudaError_t e = cudaFuncSetAttribute(shortk::short_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.T + TT - 1) / TT, p.B);
    shortk::short_fwd_kernel<<<grid, shortk::NT, smem, st>>>(p, o, TT);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (p.L > 1 && (c1 || s1 || e1)) {
    shortk::short_state_kernel<<<p.B, shortk::NT, 0, st>>>(p, c1, s1, e1);
    return cudaGetLastError();
  }
  return cudaSuccess;
}

cudaError_t short_bwd(const sca2_short_args& p, const float* dO, const float* dc1, const float* ds1,
                      const float* de1, const sca2_short_grads& g, float* work, int max_smem, cudaStream_t st) {
  const int TT = short_tokens_per_cta(p.L, true, max_smem);
  const int smem = (int)(shortk::bwd_smem_floats(p.L, TT) * sizeof(float));
  cudaError_t e = cudaFuncSetAttribute(shortk::short_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int nch = (p.T + TT - 1) / TT;
  dim3 grid(nch, p.B);
  shortk::short_bwd_kernel<<<grid, shortk::NT, smem, st>>>(p, dO, dc1, ds1, de1, g, work, TT);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  shortk::short_reduce_kernel<<<(3 * p.L + 127) / 128, 128, 0, st>>>(work, p.B * nch, p.L, g);
  return cudaGetLastError();
}

}  // namespace sca2
