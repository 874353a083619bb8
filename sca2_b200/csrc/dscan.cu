// D-head diagonal scan (sm_100a): the complex diagonal recurrence of the SCA2 D head and its
// read-out contracted over the M memory rows, forward (prefill and decode) and backward.
//
//   s_t[m, j] = a_t[m, g(j)] s_{t-1}[m, j] + v_t[j]          (complex s, real v; g(j) = j / gs)
//   A_t[j]  = mean_m Re(s_t[m, j] conj(c_t[m, j]))  = mean_m (sr cr + si ci)
//   Bv_t[j] = mean_m Im(s_t[m, j] conj(c_t[m, j]))  = mean_m (si cr - sr ci)
//
// with c = the normalised query (DHeadRef, sca2/ref.py:239-275: c per (t, m, j)) or its
// separable factor over m (DHeadSepQ, sca2/arch_sepq.py:100-104: c per (t, m), the factor
// over j applied afterwards).  The gate a is the cartesian complex gate of the head
// (tanh / sqrt(2) of two projections, or exp(-softplus) e^{i phase} for the polar gate).
//
// One thread per (b, m, j); a warp holds all M rows of 32/M consecutive channels, so the
// contraction over m is a butterfly of shuffles.  The recurrence runs sequentially over t
// per thread (the work per token is tiny; parallelism comes from B * M * V threads).  The
// forward keeps the state entering every 16-token block for the backward, which recomputes
// each block's states in registers and walks it in reverse with the adjoint of s.
#include "common.cuh"

namespace sca2 {
namespace dscan {

constexpr int NT = 256;
constexpr int CK = 16;  // tokens per checkpoint block

struct Map {
  int b, m, j, g, jj;
  bool live;
};
template <int M>
__device__ __forceinline__ Map thread_map(const sca2_dscan_args& p) {
  constexpr int JW = 32 / M;  // channels per warp
  Map r;
  const int idx = blockIdx.y * NT + threadIdx.x;
  const int lane = idx & 31, wid = idx >> 5;
  r.b = blockIdx.x;
  r.m = lane % M;
  r.jj = lane / M;
  r.j = wid * JW + r.jj;
  r.live = r.j < p.V;
  r.g = r.live ? r.j / (p.V / p.G) : 0;
  return r;
}

// sum over the M rows of a warp (lanes with the same channel)
template <int M>
__device__ __forceinline__ float sum_m(float x) {
#pragma unroll
  for (int o = 1; o < M; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
// sum over the channels of a warp with the same row (all in one gate group)
template <int M>
__device__ __forceinline__ float sum_j(float x) {
#pragma unroll
  for (int o = M; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int M, bool SEP>
__global__ void __launch_bounds__(NT) dscan_fwd_kernel(sca2_dscan_args p, float* ab, float* S_re, float* S_im,
                                                       float* ckpt) {
  const Map q = thread_map<M>(p);
  const int T = p.T, V = p.V, G = p.G;
  const int64_t bT = (int64_t)q.b * T;
  const int jc = q.live ? q.j : 0;
  float sr = 0.f, si = 0.f;
  const int64_t sidx = ((int64_t)q.b * M + q.m) * V + jc;
  if (p.S0_re && q.live) {
    sr = p.S0_re[sidx];
    si = p.S0_im[sidx];
  }
  const int NK = (T + CK - 1) / CK;
  for (int t = 0; t < T; ++t) {
    if (ckpt && (t % CK) == 0 && q.live) {
      const int64_t c0 = (((int64_t)q.b * NK + t / CK) * 2) * M * V + (int64_t)q.m * V + q.j;
      ckpt[c0] = sr;
      ckpt[c0 + (int64_t)M * V] = si;
    }
    const int64_t tm = (bT + t) * M + q.m;
    const float ar = p.a_re[tm * G + q.g], ai = p.a_im[tm * G + q.g];
    const float vt = p.v[(bT + t) * V + jc];
    const float cr = SEP ? p.c_re[tm] : p.c_re[tm * V + jc];
    const float ci = SEP ? p.c_im[tm] : p.c_im[tm * V + jc];
    const float nr = fmaf(ar, sr, fmaf(-ai, si, vt));
    const float ni = fmaf(ar, si, ai * sr);
    sr = nr;
    si = ni;
    const float pa = sum_m<M>(q.live ? sr * cr + si * ci : 0.f);
    const float pb = sum_m<M>(q.live ? si * cr - sr * ci : 0.f);
    if (q.m == 0 && q.live) {
      ab[((bT + t) * 2) * V + q.j] = pa * (1.f / M);
      ab[((bT + t) * 2 + 1) * V + q.j] = pb * (1.f / M);
    }
  }
  if (q.live) {
    S_re[sidx] = sr;
    S_im[sidx] = si;
  }
}

template <int M, bool SEP>
__global__ void __launch_bounds__(NT) dscan_bwd_kernel(sca2_dscan_args p, const float* dab, const float* dS_re,
                                                       const float* dS_im, const float* ckpt, sca2_dscan_grads gr) {
  const Map q = thread_map<M>(p);
  const int T = p.T, V = p.V, G = p.G;
  const int64_t bT = (int64_t)q.b * T;
  const int jc = q.live ? q.j : 0;
  const int64_t sidx = ((int64_t)q.b * M + q.m) * V + jc;
  float dsr = (dS_re && q.live) ? dS_re[sidx] : 0.f;
  float dsi = (dS_im && q.live) ? dS_im[sidx] : 0.f;
  const int NK = (T + CK - 1) / CK;
  constexpr float iM = 1.f / M;
  for (int k = NK - 1; k >= 0; --k) {
    const int t0 = k * CK, n = min(CK, T - t0);
    float pr[CK], pi[CK];  // state entering each token of the block
    {
      const int64_t c0 = (((int64_t)q.b * NK + k) * 2) * M * V + (int64_t)q.m * V + jc;
      float sr = ckpt[c0], si = ckpt[c0 + (int64_t)M * V];
#pragma unroll
      for (int u = 0; u < CK; ++u) {
        pr[u] = sr;
        pi[u] = si;
        if (u < n) {
          const int64_t tm = (bT + t0 + u) * M + q.m;
          const float ar = p.a_re[tm * G + q.g], ai = p.a_im[tm * G + q.g];
          const float vt = p.v[(bT + t0 + u) * V + jc];
          const float nr = fmaf(ar, sr, fmaf(-ai, si, vt));
          si = fmaf(ar, si, ai * sr);
          sr = nr;
        }
      }
    }
#pragma unroll
    for (int u = CK - 1; u >= 0; --u) {
      if (u >= n) continue;
      const int t = t0 + u;
      const int64_t tm = (bT + t) * M + q.m;
      const float ar = p.a_re[tm * G + q.g], ai = p.a_im[tm * G + q.g];
      const float vt = p.v[(bT + t) * V + jc];
      const float sr = fmaf(ar, pr[u], fmaf(-ai, pi[u], vt)), si = fmaf(ar, pi[u], ai * pr[u]);
      const float gA = dab[((bT + t) * 2) * V + jc] * iM, gB = dab[((bT + t) * 2 + 1) * V + jc] * iM;
      const float cr = SEP ? p.c_re[tm] : p.c_re[tm * V + jc];
      const float ci = SEP ? p.c_im[tm] : p.c_im[tm * V + jc];
      // read at t
      dsr = q.live ? dsr + gA * cr - gB * ci : 0.f;
      dsi = q.live ? dsi + gA * ci + gB * cr : 0.f;
      const float dcr = q.live ? gA * sr + gB * si : 0.f, dci = q.live ? gA * si - gB * sr : 0.f;
      if (SEP) {
        const float xr = sum_j<M>(dcr), xi = sum_j<M>(dci);
        if (q.jj == 0) {
          atomicAdd(gr.dc_re + tm, xr);
          atomicAdd(gr.dc_im + tm, xi);
        }
      } else if (q.live) {
        gr.dc_re[tm * V + q.j] = dcr;
        gr.dc_im[tm * V + q.j] = dci;
      }
      // v_t and the gate a_t
      const float dvt = sum_m<M>(dsr);
      if (q.m == 0 && q.live) gr.dv[(bT + t) * V + q.j] = dvt;
      const float dar = sum_j<M>(dsr * pr[u] + dsi * pi[u]);
      const float dai = sum_j<M>(-dsr * pi[u] + dsi * pr[u]);
      if (q.jj == 0) {
        atomicAdd(gr.da_re + tm * G + q.g, dar);
        atomicAdd(gr.da_im + tm * G + q.g, dai);
      }
      // adjoint to the state entering token t
      const float ndr = ar * dsr + ai * dsi;
      dsi = -ai * dsr + ar * dsi;
      dsr = ndr;
    }
  }
  if (q.live) {
    if (gr.dS0_re) gr.dS0_re[sidx] = dsr;
    if (gr.dS0_im) gr.dS0_im[sidx] = dsi;
  }
}

template <int M>
cudaError_t launch_fwd_m(const sca2_dscan_args& p, float* ab, float* S_re, float* S_im, float* ckpt,
                         cudaStream_t st) {
  const int per_b = M * p.V;
  dim3 grid(p.B, (per_b + NT - 1) / NT);
  if (p.sep)
    dscan_fwd_kernel<M, true><<<grid, NT, 0, st>>>(p, ab, S_re, S_im, ckpt);
  else
    dscan_fwd_kernel<M, false><<<grid, NT, 0, st>>>(p, ab, S_re, S_im, ckpt);
  return cudaGetLastError();
}
template <int M>
cudaError_t launch_bwd_m(const sca2_dscan_args& p, const float* dab, const float* dS_re, const float* dS_im,
                         const float* ckpt, const sca2_dscan_grads& g, cudaStream_t st) {
  const int per_b = M * p.V;
  dim3 grid(p.B, (per_b + NT - 1) / NT);
  if (p.sep)
    dscan_bwd_kernel<M, true><<<grid, NT, 0, st>>>(p, dab, dS_re, dS_im, ckpt, g);
  else
    dscan_bwd_kernel<M, false><<<grid, NT, 0, st>>>(p, dab, dS_re, dS_im, ckpt, g);
  return cudaGetLastError();
}

}  // namespace dscan

cudaError_t dscan_fwd(const sca2_dscan_args& p, float* ab, float* S_re, float* S_im, float* ckpt, cudaStream_t st) {
  switch (p.M) {
    case 1: return dscan::launch_fwd_m<1>(p, ab, S_re, S_im, ckpt, st);
    case 2: return dscan::launch_fwd_m<2>(p, ab, S_re, S_im, ckpt, st);
    case 4: return dscan::launch_fwd_m<4>(p, ab, S_re, S_im, ckpt, st);
    case 8: return dscan::launch_fwd_m<8>(p, ab, S_re, S_im, ckpt, st);
    case 16: return dscan::launch_fwd_m<16>(p, ab, S_re, S_im, ckpt, st);
    case 32: return dscan::launch_fwd_m<32>(p, ab, S_re, S_im, ckpt, st);
  }
  return cudaErrorInvalidValue;
}
cudaError_t dscan_bwd(const sca2_dscan_args& p, const float* dab, const float* dS_re, const float* dS_im,
                      const float* ckpt, const sca2_dscan_grads& g, cudaStream_t st) {
  switch (p.M) {
    case 1: return dscan::launch_bwd_m<1>(p, dab, dS_re, dS_im, ckpt, g, st);
    case 2: return dscan::launch_bwd_m<2>(p, dab, dS_re, dS_im, ckpt, g, st);
    case 4: return dscan::launch_bwd_m<4>(p, dab, dS_re, dS_im, ckpt, g, st);
    case 8: return dscan::launch_bwd_m<8>(p, dab, dS_re, dS_im, ckpt, g, st);
    case 16: return dscan::launch_bwd_m<16>(p, dab, dS_re, dS_im, ckpt, g, st);
    case 32: return dscan::launch_bwd_m<32>(p, dab, dS_re, dS_im, ckpt, g, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sca2
