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
// One thread per (b, m, j) (and, for long sequences, per 16-token block); a warp holds all M
// rows of 32/M consecutive channels, so the contraction over m is a butterfly of shuffles.
// Short sequences and decode run the recurrence sequentially over t per thread.  Long ones
// split T into 16-token blocks that run in parallel, joined by a short pass over the blocks
// (the recurrence is linear, so a block is the affine map s -> P s + e).  The forward keeps
// the state entering every block for the backward, which recomputes each block's states in
// registers and walks it in reverse with the adjoint of s.
#include "common.cuh"

namespace sca2 {
namespace dscan {

constexpr int NT = 256;
constexpr int CK = 16;  // tokens per checkpoint block
constexpr int OUT_TOK = 8;  // tokens per round of the output pass's row sums (16 to 17 KB of shared memory)
__host__ __device__ constexpr int out_stride(int M) { return M >= 16 ? M + 1 : M; }

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

// ---- chunk-parallel forms (long sequences) --------------------------------------------------
// Blocks of CK tokens run in parallel.  Forward: (1) every block scans from a zero state,
// giving its end state e and the product P of its gates; (2) one pass over the blocks folds
// S_in(k+1) = P_k S_in(k) + e_k, which are the checkpoints; (3) every block rescans from
// S_in(k) and writes the read.  Backward: (1) every block runs its adjoint from a zero
// adjoint at its end, giving the adjoint q it sends to the left and the product Q of its
// conjugate gates; (2) one reverse pass folds R(k-1) = Q_k R(k) + q_k (R = adjoint entering a
// block from the right; R(last) = dS, R(-1) = dS0); (3) every block runs the gradient pass of
// dscan_bwd_kernel from R(k).  Workspace (floats): fwd e, P; bwd q, Q, R.

template <int M>
__device__ __forceinline__ Map thread_map_c(const sca2_dscan_args& p) {
  constexpr int JW = 32 / M;
  Map r;
  const int idx = blockIdx.z * NT + threadIdx.x;
  const int lane = idx & 31, wid = idx >> 5;
  r.b = blockIdx.x;
  r.m = lane % M;
  r.jj = lane / M;
  r.j = wid * JW + r.jj;
  r.live = r.j < p.V;
  r.g = r.live ? r.j / (p.V / p.G) : 0;
  return r;
}

// Gate groups a CTA's channels can touch: its 256 / M channels in groups of gs = V / G
__host__ __device__ inline int ngl_max(int M, int gs) { return (NT / M) / gs + 2; }

// Inputs of one 16-token block for a CTA's channels [j0, j0 + 256 / M), staged in shared memory
// with coalesced loads before the dependent passes: v and dab [CK][JC] per token row, the gates
// of the groups those channels touch [CK][M][NGL][re, im] and the separable read factor
// [CK][M][re, im] (each part on request); zeros past the sequence, the value width or the gate
// groups.
template <int M>
struct Stage {
  static constexpr int JC = NT / M;
  float *v, *d, *a, *c;
  int g0, ngl;
  __host__ __device__ static constexpr int floats(int ngl) { return CK * JC * 3 + CK * M * ngl * 2 + CK * M * 2; }
  __device__ void load(const sca2_dscan_args& p, const float* dab, int b, int t0, int n, int j0, float* base,
                       int ngl_max, bool with_v = true, bool with_c = true) {
    const int V = p.V, G = p.G, gs = V / G;
    ngl = ngl_max;
    g0 = j0 / gs;
    v = base;
    d = v + CK * JC;
    a = d + 2 * CK * JC;
    c = a + CK * M * ngl * 2;
    const int64_t bT = (int64_t)b * p.T;
    for (int u = threadIdx.x; u < CK * JC; u += NT) {
      const int t = u / JC, jl = u % JC, j = j0 + jl;
      const bool live = t < n && j < V;
      const int64_t row = bT + t0 + t;
      if (with_v) v[u] = live ? p.v[row * V + j] : 0.f;
      if (dab) {
        d[t * 2 * JC + jl] = live ? dab[(row * 2) * V + j] : 0.f;
        d[t * 2 * JC + JC + jl] = live ? dab[(row * 2 + 1) * V + j] : 0.f;
      }
    }
    for (int u = threadIdx.x; u < CK * M * ngl; u += NT) {
      const int gl = u % ngl, tm = u / ngl, t = tm / M, m = tm % M, g = g0 + gl;
      const bool live = t < n && g < G;
      const int64_t idx = ((bT + t0 + t) * M + m) * G + g;
      a[2 * u] = live ? p.a_re[idx] : 0.f;
      a[2 * u + 1] = live ? p.a_im[idx] : 0.f;
    }
    for (int u = threadIdx.x; with_c && u < CK * M; u += NT) {
      const int t = u / M;
      const int64_t idx = (bT + t0 + t) * M + (u % M);
      c[2 * u] = t < n ? p.c_re[idx] : 0.f;
      c[2 * u + 1] = t < n ? p.c_im[idx] : 0.f;
    }
  }
  __device__ float2 gate(int t, int m, int g) const {
    const float* q = a + ((t * M + m) * ngl + (g - g0)) * 2;
    return make_float2(q[0], q[1]);
  }
};

// The folds reduce nothing over rows and read no per-token input, so their threads take channels
// fastest: their loads and stores of the [M][V] planes coalesce.  `blk` is the grid index that
// enumerates (m, j) tiles of NT threads.
template <int M>
__device__ __forceinline__ Map chan_map(const sca2_dscan_args& p, int blk) {
  Map r;
  const int idx = blk * NT + threadIdx.x;
  r.b = blockIdx.x;
  r.m = idx / p.V;
  r.j = idx - r.m * p.V;
  r.jj = 0;
  r.live = r.m < M;
  if (!r.live) r.m = M - 1, r.j = 0;  // idle threads of the last tile read row M - 1, channel 0
  r.g = r.j / (p.V / p.G);
  return r;
}

// complex product of a block's gates, kept per (b, k, m, g) by the group's first channel
template <int M>
__global__ void __launch_bounds__(NT) dscan_fwd_local(sca2_dscan_args p, float* e, float* P) {
  extern __shared__ float sst[];
  const Map q = thread_map_c<M>(p);
  const int k = blockIdx.y, NK = gridDim.y, T = p.T, V = p.V, G = p.G;
  const int t0 = k * CK, n = min(CK, T - t0);
  Stage<M> sg;
  sg.load(p, nullptr, q.b, t0, n, blockIdx.z * (NT / M), sst, ngl_max(M, V / G), true, false);
  __syncthreads();
  const int jl = q.j - blockIdx.z * (NT / M), gq = q.live ? q.g : sg.g0;
  float sr = 0.f, si = 0.f, pr = 1.f, pi = 0.f;
#pragma unroll 4
  for (int u = 0; u < n; ++u) {
    const float2 a = sg.gate(u, q.m, gq);
    const float ar = a.x, ai = a.y;
    const float vt = sg.v[u * Stage<M>::JC + jl];
    const float nr = fmaf(ar, sr, fmaf(-ai, si, vt));
    si = fmaf(ar, si, ai * sr);
    sr = nr;
    const float qr = ar * pr - ai * pi;
    pi = ar * pi + ai * pr;
    pr = qr;
  }
  if (!q.live) return;
  const int64_t base = ((int64_t)q.b * NK + k) * 2;
  e[base * M * V + (int64_t)q.m * V + q.j] = sr;
  e[(base + 1) * M * V + (int64_t)q.m * V + q.j] = si;
  if (q.j % (V / G) == 0) {
    P[base * M * G + (int64_t)q.m * G + q.g] = pr;
    P[(base + 1) * M * G + (int64_t)q.m * G + q.g] = pi;
  }
}

// fold over the blocks (sequential per (b, m, j)): checkpoints and the final state.  The fold's
// inputs are loaded CU blocks at a time into registers before the dependent updates, so a
// thread waits for one round of loads per CU blocks instead of one per block.
constexpr int CU = 16;
template <int M>
__global__ void __launch_bounds__(NT) dscan_fwd_carry(sca2_dscan_args p, const float* __restrict__ e,
                                                     const float* __restrict__ P, float* __restrict__ ckpt,
                                                     float* S_re, float* S_im) {
  const Map q = chan_map<M>(p, blockIdx.y);
  if (!q.live) return;
  const int V = p.V, G = p.G, NK = (p.T + CK - 1) / CK;
  const int64_t sidx = ((int64_t)q.b * M + q.m) * V + q.j;
  float sr = p.S0_re ? p.S0_re[sidx] : 0.f, si = p.S0_im ? p.S0_im[sidx] : 0.f;
  for (int k0 = 0; k0 < NK; k0 += CU) {
    float pr[CU], pi[CU], er[CU], ei[CU];
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      const int64_t base = ((int64_t)q.b * NK + min(k0 + u, NK - 1)) * 2;
      pr[u] = P[base * M * G + (int64_t)q.m * G + q.g];
      pi[u] = P[(base + 1) * M * G + (int64_t)q.m * G + q.g];
      er[u] = e[base * M * V + (int64_t)q.m * V + q.j];
      ei[u] = e[(base + 1) * M * V + (int64_t)q.m * V + q.j];
    }
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      if (k0 + u >= NK) break;
      const int64_t base = ((int64_t)q.b * NK + k0 + u) * 2;
      ckpt[base * M * V + (int64_t)q.m * V + q.j] = sr;
      ckpt[(base + 1) * M * V + (int64_t)q.m * V + q.j] = si;
      const float nr = pr[u] * sr - pi[u] * si + er[u];
      si = pr[u] * si + pi[u] * sr + ei[u];
      sr = nr;
    }
  }
  S_re[sidx] = sr;
  S_im[sidx] = si;
}

// every block from its incoming state: the read
template <int M, bool SEP>
__global__ void __launch_bounds__(NT) dscan_fwd_out(sca2_dscan_args p, const float* ckpt, float* ab) {
  extern __shared__ float sst[];
  const Map q = thread_map_c<M>(p);
  const int k = blockIdx.y, NK = gridDim.y, T = p.T, V = p.V, G = p.G;
  const int t0 = k * CK, n = min(CK, T - t0);
  const int jc = q.live ? q.j : 0;
  const int64_t bT = (int64_t)q.b * T;
  const int64_t base = ((int64_t)q.b * NK + k) * 2;
  // rows of M >= 16 padded to an odd stride (the sums' loads conflict-free); narrower rows stay
  // 16-byte aligned for vector loads
  constexpr int JC = NT / M, HT = OUT_TOK, MP = out_stride(M);
  Stage<M> sg;
  float* pout = sst;  // [HT][re, im][JC][MP]: the rows' terms of the read, summed over m after each round
  if (SEP) {  // separable read: the block's inputs staged once, coalesced
    sg.load(p, nullptr, q.b, t0, n, blockIdx.z * JC, sst, ngl_max(M, V / G));
    pout = sst + Stage<M>::floats(sg.ngl);
    __syncthreads();
  }
  const int cj0 = blockIdx.z * JC, jl = q.j - cj0;
  float sr = ckpt[base * M * V + (int64_t)q.m * V + jc], si = ckpt[(base + 1) * M * V + (int64_t)q.m * V + jc];
  for (int h0 = 0; h0 < n; h0 += HT) {
#pragma unroll
    for (int uu = 0; uu < HT; ++uu) {
      const int u = h0 + uu;
      if (u >= n) break;
      const int t = t0 + u;
      const int64_t tm = (bT + t) * M + q.m;
      float ar, ai, vt, cr, ci;
      if (SEP) {
        const float2 a = sg.gate(u, q.m, q.live ? q.g : sg.g0);
        ar = a.x, ai = a.y;
        vt = sg.v[u * JC + jl];
        cr = sg.c[(u * M + q.m) * 2];
        ci = sg.c[(u * M + q.m) * 2 + 1];
      } else {
        ar = p.a_re[tm * G + q.g], ai = p.a_im[tm * G + q.g];
        vt = p.v[(bT + t) * V + jc];
        cr = p.c_re[tm * V + jc];
        ci = p.c_im[tm * V + jc];
      }
      const float nr = fmaf(ar, sr, fmaf(-ai, si, vt));
      si = fmaf(ar, si, ai * sr);
      sr = nr;
      // lane order (jl, m) is consecutive within a warp: stores nearly conflict-free
      pout[((uu * 2) * JC + jl) * MP + q.m] = q.live ? sr * cr + si * ci : 0.f;
      pout[((uu * 2 + 1) * JC + jl) * MP + q.m] = q.live ? si * cr - sr * ci : 0.f;
    }
    __syncthreads();
    const int nu = min(HT, n - h0);
    for (int o = threadIdx.x; o < nu * 2 * JC; o += NT) {  // (token, re / im, channel): coalesced writes
      const int c = o % JC, rr = (o / JC) & 1, uu = o / (2 * JC), j = cj0 + c;
      const float* src = pout + ((uu * 2 + rr) * JC + c) * MP;
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < M; ++m) acc += src[m];
      if (j < V) ab[((bT + t0 + h0 + uu) * 2 + rr) * V + j] = acc * (1.f / M);
    }
    __syncthreads();  // the buffer is rewritten by the next round
  }
}

// adjoint of a block from zero at its end: q (to the left) and Q = prod conj(a)
template <int M, bool SEP>
__global__ void __launch_bounds__(NT) dscan_bwd_local(sca2_dscan_args p, const float* dab, float* qv, float* Qg) {
  extern __shared__ float sst[];
  const Map q = thread_map_c<M>(p);
  const int k = blockIdx.y, NK = gridDim.y, T = p.T, V = p.V, G = p.G;
  const int t0 = k * CK, n = min(CK, T - t0);
  const int jc = q.live ? q.j : 0;
  const int64_t bT = (int64_t)q.b * T;
  constexpr float iM = 1.f / M;
  constexpr int JC = Stage<M>::JC;
  Stage<M> sg;
  sg.load(p, dab, q.b, t0, n, blockIdx.z * JC, sst, ngl_max(M, V / G), false, SEP);
  __syncthreads();
  const int jl = q.j - blockIdx.z * JC, gq = q.live ? q.g : sg.g0;
  float dr = 0.f, di = 0.f, Pr = 1.f, Pi = 0.f;
#pragma unroll 4
  for (int u = n - 1; u >= 0; --u) {
    const int t = t0 + u;
    const int64_t tm = (bT + t) * M + q.m;
    const float2 a = sg.gate(u, q.m, gq);
    const float ar = a.x, ai = a.y;
    const float gA = sg.d[u * 2 * JC + jl] * iM, gB = sg.d[u * 2 * JC + JC + jl] * iM;
    const float cr = SEP ? sg.c[(u * M + q.m) * 2] : p.c_re[tm * V + jc];
    const float ci = SEP ? sg.c[(u * M + q.m) * 2 + 1] : p.c_im[tm * V + jc];
    dr += gA * cr - gB * ci;
    di += gA * ci + gB * cr;
    const float nr = ar * dr + ai * di;
    di = -ai * dr + ar * di;
    dr = nr;
    const float qr = ar * Pr + ai * Pi;  // conj(a) * P
    Pi = ar * Pi - ai * Pr;
    Pr = qr;
  }
  if (!q.live) return;
  const int64_t base = ((int64_t)q.b * NK + k) * 2;
  qv[base * M * V + (int64_t)q.m * V + q.j] = dr;
  qv[(base + 1) * M * V + (int64_t)q.m * V + q.j] = di;
  if (q.j % (V / G) == 0) {
    Qg[base * M * G + (int64_t)q.m * G + q.g] = Pr;
    Qg[(base + 1) * M * G + (int64_t)q.m * G + q.g] = Pi;
  }
}

// reverse fold: R(k) = adjoint entering block k from the right; R(-1) = dS0 (inputs loaded CU
// blocks at a time, as in the forward fold)
template <int M>
__global__ void __launch_bounds__(NT) dscan_bwd_carry(sca2_dscan_args p, const float* dS_re, const float* dS_im,
                                                     const float* __restrict__ qv, const float* __restrict__ Qg,
                                                     float* __restrict__ R, sca2_dscan_grads gr) {
  const Map q = chan_map<M>(p, blockIdx.y);
  if (!q.live) return;
  const int V = p.V, G = p.G, NK = (p.T + CK - 1) / CK;
  const int64_t sidx = ((int64_t)q.b * M + q.m) * V + q.j;
  float rr = dS_re ? dS_re[sidx] : 0.f, ri = dS_im ? dS_im[sidx] : 0.f;
  for (int k1 = NK - 1; k1 >= 0; k1 -= CU) {
    float Pr[CU], Pi[CU], xr[CU], xi[CU];
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      const int64_t base = ((int64_t)q.b * NK + max(k1 - u, 0)) * 2;
      Pr[u] = Qg[base * M * G + (int64_t)q.m * G + q.g];
      Pi[u] = Qg[(base + 1) * M * G + (int64_t)q.m * G + q.g];
      xr[u] = qv[base * M * V + (int64_t)q.m * V + q.j];
      xi[u] = qv[(base + 1) * M * V + (int64_t)q.m * V + q.j];
    }
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      if (k1 - u < 0) break;
      const int64_t base = ((int64_t)q.b * NK + k1 - u) * 2;
      R[base * M * V + (int64_t)q.m * V + q.j] = rr;
      R[(base + 1) * M * V + (int64_t)q.m * V + q.j] = ri;
      const float nr = Pr[u] * rr - Pi[u] * ri + xr[u];
      ri = Pr[u] * ri + Pi[u] * rr + xi[u];
      rr = nr;
    }
  }
  if (gr.dS0_re) gr.dS0_re[sidx] = rr;
  if (gr.dS0_im) gr.dS0_im[sidx] = ri;
}

// gradient pass of one block from its incoming adjoint R(k).  The gradients summed over
// channels (da per (t, m, g), and dc per (t, m) with the separable read) are reduced per warp by
// shuffles and stored per warp (plain stores: a warp's channels lie in one gate group); after
// the block, one pass adds the warps' partials (those of each gate group for da) and the CTA
// issues one global atomic per (t, m[, g]).
template <int M, bool SEP>
__global__ void __launch_bounds__(NT) dscan_bwd_block(sca2_dscan_args p, const float* dab, const float* ckpt,
                                                     const float* R, sca2_dscan_grads gr) {
  extern __shared__ float sred[];
  const Map q = thread_map_c<M>(p);
  const int k = blockIdx.y, NK = gridDim.y, T = p.T, V = p.V, G = p.G;
  const int t0 = k * CK, n = min(CK, T - t0);
  const int jc = q.live ? q.j : 0;
  const int64_t bT = (int64_t)q.b * T;
  const int64_t base = ((int64_t)q.b * NK + k) * 2;
  constexpr float iM = 1.f / M;
  const int gs = V / G, NGL = ngl_max(M, gs);
  constexpr int NW = NT / 32;
  const int warp = threadIdx.x >> 5;
  float* pdc = sred;                                  // [NW][CK][M][2] per-warp partials (separable read)
  float* pda = sred + (SEP ? NW * CK * M * 2 : 0);    // [NW][CK][M][2]
  const int nred = (SEP ? 2 : 1) * NW * CK * M * 2;  // every entry read is written (rows t < n)
  Stage<M> sg;
  if (SEP) sg.load(p, dab, q.b, t0, n, blockIdx.z * (NT / M), sred + nred, NGL);
  __syncthreads();
  const int jl = q.j - blockIdx.z * (NT / M);  // channel within the CTA
  auto gate = [&](int u, int64_t tm) -> float2 {
    return SEP ? sg.gate(u, q.m, q.live ? q.g : sg.g0) : make_float2(p.a_re[tm * G + q.g], p.a_im[tm * G + q.g]);
  };
  auto val = [&](int u, int t) -> float { return SEP ? sg.v[u * Stage<M>::JC + jl] : p.v[(bT + t) * V + jc]; };
  float dsr = q.live ? R[base * M * V + (int64_t)q.m * V + jc] : 0.f;
  float dsi = q.live ? R[(base + 1) * M * V + (int64_t)q.m * V + jc] : 0.f;
  float pr[CK], pi[CK];
  {
    float sr = ckpt[base * M * V + (int64_t)q.m * V + jc], si = ckpt[(base + 1) * M * V + (int64_t)q.m * V + jc];
#pragma unroll
    for (int u = 0; u < CK; ++u) {
      pr[u] = sr;
      pi[u] = si;
      if (u < n) {
        const int64_t tm = (bT + t0 + u) * M + q.m;
        const float2 a = gate(u, tm);
        const float vt = val(u, t0 + u);
        const float nr = fmaf(a.x, sr, fmaf(-a.y, si, vt));
        si = fmaf(a.x, si, a.y * sr);
        sr = nr;
      }
    }
  }
#pragma unroll
  for (int u = CK - 1; u >= 0; --u) {
    if (u >= n) continue;
    const int t = t0 + u;
    const int64_t tm = (bT + t) * M + q.m;
    const float2 a = gate(u, tm);
    const float ar = a.x, ai = a.y;
    const float vt = val(u, t);
    const float sr = fmaf(ar, pr[u], fmaf(-ai, pi[u], vt)), si = fmaf(ar, pi[u], ai * pr[u]);
    const float gA = (SEP ? sg.d[u * 2 * Stage<M>::JC + jl] : dab[((bT + t) * 2) * V + jc]) * iM;
    const float gB = (SEP ? sg.d[u * 2 * Stage<M>::JC + Stage<M>::JC + jl] : dab[((bT + t) * 2 + 1) * V + jc]) * iM;
    const float cr = SEP ? sg.c[(u * M + q.m) * 2] : p.c_re[tm * V + jc];
    const float ci = SEP ? sg.c[(u * M + q.m) * 2 + 1] : p.c_im[tm * V + jc];
    dsr = q.live ? dsr + gA * cr - gB * ci : 0.f;
    dsi = q.live ? dsi + gA * ci + gB * cr : 0.f;
    const float dcr = q.live ? gA * sr + gB * si : 0.f, dci = q.live ? gA * si - gB * sr : 0.f;
    if (SEP) {
      const float xr = sum_j<M>(dcr), xi = sum_j<M>(dci);
      if (q.jj == 0) {  // lane jj = 0 holds the warp's sum (zeros past the value width)
        float* d = pdc + ((warp * CK + u) * M + q.m) * 2;
        d[0] = xr;
        d[1] = xi;
      }
    } else if (q.live) {
      gr.dc_re[tm * V + q.j] = dcr;
      gr.dc_im[tm * V + q.j] = dci;
    }
    const float dvt = sum_m<M>(dsr);
    if (q.m == 0 && q.live) gr.dv[(bT + t) * V + q.j] = dvt;
    const float dar = sum_j<M>(dsr * pr[u] + dsi * pi[u]);
    const float dai = sum_j<M>(-dsr * pi[u] + dsi * pr[u]);
    if (q.jj == 0) {
      float* d = pda + ((warp * CK + u) * M + q.m) * 2;
      d[0] = dar;
      d[1] = dai;
    }
    const float ndr = ar * dsr + ai * dsi;
    dsi = -ai * dsr + ar * dsi;
    dsr = ndr;
  }
  __syncthreads();
  const int cj0 = blockIdx.z * (NT / M);  // the CTA's first channel; warp w's is cj0 + w (32 / M)
  for (int u = threadIdx.x; u < n * M; u += NT) {  // u = t M + m
    const int64_t tm = (bT + t0 + u / M) * M + (u % M);
    if (SEP) {
      float xr = 0.f, xi = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) xr += pdc[(w * CK * M + u) * 2], xi += pdc[(w * CK * M + u) * 2 + 1];
      atomicAdd(gr.dc_re + tm, xr);
      atomicAdd(gr.dc_im + tm, xi);
    }
    // da: the warps in channel order, one atomic per gate group they cover
    int gc = -1;
    float xr = 0.f, xi = 0.f;
    for (int w = 0; w < NW; ++w) {
      const int jw = cj0 + w * (32 / M);
      if (jw >= V) break;
      const int gw = jw / gs;
      if (gw != gc) {
        if (gc >= 0) {
          atomicAdd(gr.da_re + tm * G + gc, xr);
          atomicAdd(gr.da_im + tm * G + gc, xi);
        }
        gc = gw, xr = 0.f, xi = 0.f;
      }
      xr += pda[(w * CK * M + u) * 2];
      xi += pda[(w * CK * M + u) * 2 + 1];
    }
    if (gc >= 0) {
      atomicAdd(gr.da_re + tm * G + gc, xr);
      atomicAdd(gr.da_im + tm * G + gc, xi);
    }
  }
}

// the chunk-parallel form pays off once there are several blocks per sequence
inline bool use_blocks(const sca2_dscan_args& p, const float* work) {
  return work != nullptr && p.T > 4 * CK && (p.T + CK - 1) / CK <= 65535;
}

// ---- the folds over the blocks in three passes (long sequences) -------------------------
// out[k] = s; s = A_k s + c_k over the blocks k in fold order (ascending: the forward's
// checkpoints, A = P, c = e; descending: the adjoint entering each block from the right,
// A = Q, c = q).  With NK blocks one thread per (b, m, j) would take NK dependent steps, so
// the blocks are taken in groups of FG: (1) every group's composed map (A_g, c_g) in
// parallel, (2) one fold over the groups giving the state entering each group and the final
// state, (3) every group's blocks from its entering state in parallel.  Each pass loads its
// group's inputs into registers before the dependent updates.
constexpr int FG = 16;
// floats of e + P + checkpoints (forward) or q + R + Q (backward)
inline size_t dscan_base_floats(int B, int NK, int M, int G, int V) {
  return (size_t)B * NK * 2 * (2 * (size_t)M * V + (size_t)M * G);
}
struct FoldIO {
  const float* A;  // [(b NK + k) 2 + r][M][G]
  const float* c;  // [(b NK + k) 2 + r][M][V]
  float* Ag;       // [(b NG + g) 2 + r][M][G]  group maps (pass 1 -> 2)
  float* cg;       // [(b NG + g) 2 + r][M][V]
  float* Sg;       // [(b NG + g) 2 + r][M][V]  state entering each group (pass 2 -> 3)
  int NK, NG;
  bool rev;
};
// block of the i-th step of group gi in fold order, or -1 past the sequence
__device__ __forceinline__ int fold_block(const FoldIO& f, int gi, int i) {
  const int k0 = gi * FG + i;
  if (k0 >= f.NK) return -1;
  return f.rev ? f.NK - 1 - k0 : k0;
}

template <int M>
__device__ __forceinline__ void fold_load(const sca2_dscan_args& p, const FoldIO& f, const Map& q, int gi, float* ar,
                                          float* ai, float* cr, float* ci) {
  const int V = p.V, G = p.G;
#pragma unroll
  for (int u = 0; u < FG; ++u) {
    const int k = fold_block(f, gi, u);
    const int64_t base = ((int64_t)q.b * f.NK + (k < 0 ? 0 : k)) * 2;
    ar[u] = k < 0 ? 1.f : f.A[base * M * G + (int64_t)q.m * G + q.g];
    ai[u] = k < 0 ? 0.f : f.A[(base + 1) * M * G + (int64_t)q.m * G + q.g];
    cr[u] = k < 0 ? 0.f : f.c[base * M * V + (int64_t)q.m * V + q.j];
    ci[u] = k < 0 ? 0.f : f.c[(base + 1) * M * V + (int64_t)q.m * V + q.j];
  }
}

template <int M>
__global__ void __launch_bounds__(NT) dscan_fold_groups(sca2_dscan_args p, FoldIO f) {
  const Map q = chan_map<M>(p, blockIdx.z);
  if (!q.live) return;
  const int gi = blockIdx.y, V = p.V, G = p.G;
  float ar[FG], ai[FG], cr[FG], ci[FG];
  fold_load<M>(p, f, q, gi, ar, ai, cr, ci);
  float Pr = 1.f, Pi = 0.f, xr = 0.f, xi = 0.f;  // the composed map s -> (Pr + i Pi) s + (xr + i xi)
#pragma unroll
  for (int u = 0; u < FG; ++u) {
    const float nPr = ar[u] * Pr - ai[u] * Pi, nPi = ar[u] * Pi + ai[u] * Pr;
    const float nxr = ar[u] * xr - ai[u] * xi + cr[u], nxi = ar[u] * xi + ai[u] * xr + ci[u];
    Pr = nPr, Pi = nPi, xr = nxr, xi = nxi;
  }
  const int64_t gb = ((int64_t)q.b * f.NG + gi) * 2;
  f.cg[gb * M * V + (int64_t)q.m * V + q.j] = xr;
  f.cg[(gb + 1) * M * V + (int64_t)q.m * V + q.j] = xi;
  if (q.j % (V / G) == 0) {
    f.Ag[gb * M * G + (int64_t)q.m * G + q.g] = Pr;
    f.Ag[(gb + 1) * M * G + (int64_t)q.m * G + q.g] = Pi;
  }
}

template <int M>
__global__ void __launch_bounds__(NT) dscan_fold_top(sca2_dscan_args p, FoldIO f, const float* s_re, const float* s_im,
                                                     float* fin_re, float* fin_im) {
  const Map q = chan_map<M>(p, blockIdx.y);
  if (!q.live) return;
  const int V = p.V, G = p.G;
  const int64_t sidx = ((int64_t)q.b * M + q.m) * V + q.j;
  float sr = s_re ? s_re[sidx] : 0.f, si = s_im ? s_im[sidx] : 0.f;
  for (int g0 = 0; g0 < f.NG; g0 += FG) {
    float ar[FG], ai[FG], cr[FG], ci[FG];
#pragma unroll
    for (int u = 0; u < FG; ++u) {
      const int64_t gb = ((int64_t)q.b * f.NG + min(g0 + u, f.NG - 1)) * 2;
      ar[u] = f.Ag[gb * M * G + (int64_t)q.m * G + q.g];
      ai[u] = f.Ag[(gb + 1) * M * G + (int64_t)q.m * G + q.g];
      cr[u] = f.cg[gb * M * V + (int64_t)q.m * V + q.j];
      ci[u] = f.cg[(gb + 1) * M * V + (int64_t)q.m * V + q.j];
    }
#pragma unroll
    for (int u = 0; u < FG; ++u) {
      if (g0 + u >= f.NG) break;
      const int64_t gb = ((int64_t)q.b * f.NG + g0 + u) * 2;
      f.Sg[gb * M * V + (int64_t)q.m * V + q.j] = sr;
      f.Sg[(gb + 1) * M * V + (int64_t)q.m * V + q.j] = si;
      const float nr = ar[u] * sr - ai[u] * si + cr[u];
      si = ar[u] * si + ai[u] * sr + ci[u];
      sr = nr;
    }
  }
  if (fin_re) fin_re[sidx] = sr;
  if (fin_im) fin_im[sidx] = si;
}

template <int M>
__global__ void __launch_bounds__(NT) dscan_fold_blocks(sca2_dscan_args p, FoldIO f, float* out) {
  const Map q = chan_map<M>(p, blockIdx.z);
  if (!q.live) return;
  const int gi = blockIdx.y, V = p.V;
  float ar[FG], ai[FG], cr[FG], ci[FG];
  fold_load<M>(p, f, q, gi, ar, ai, cr, ci);
  const int64_t gb = ((int64_t)q.b * f.NG + gi) * 2;
  float sr = f.Sg[gb * M * V + (int64_t)q.m * V + q.j], si = f.Sg[(gb + 1) * M * V + (int64_t)q.m * V + q.j];
#pragma unroll
  for (int u = 0; u < FG; ++u) {
    const int k = fold_block(f, gi, u);
    if (k < 0) break;
    const int64_t base = ((int64_t)q.b * f.NK + k) * 2;
    out[base * M * V + (int64_t)q.m * V + q.j] = sr;
    out[(base + 1) * M * V + (int64_t)q.m * V + q.j] = si;
    const float nr = ar[u] * sr - ai[u] * si + cr[u];
    si = ar[u] * si + ai[u] * sr + ci[u];
    sr = nr;
  }
}

// the three passes; `gw` holds Ag, cg, Sg (dscan_fold_floats)
inline size_t fold_floats(int B, int NK, int M, int G, int V) {
  const size_t NG = (size_t)((NK + FG - 1) / FG);
  return (size_t)B * NG * 2 * (2 * (size_t)M * V + (size_t)M * G);
}
template <int M>
cudaError_t launch_fold(const sca2_dscan_args& p, const float* A, const float* c, float* out, const float* s_re,
                        const float* s_im, float* fin_re, float* fin_im, bool rev, float* gw, cudaStream_t st) {
  const int NK = (p.T + CK - 1) / CK, NG = (NK + FG - 1) / FG, tiles = (M * p.V + NT - 1) / NT;
  FoldIO f;
  f.A = A, f.c = c, f.NK = NK, f.NG = NG, f.rev = rev;
  f.cg = gw;
  f.Sg = gw + (size_t)p.B * NG * 2 * M * p.V;
  f.Ag = f.Sg + (size_t)p.B * NG * 2 * M * p.V;
  dscan_fold_groups<M><<<dim3(p.B, NG, tiles), NT, 0, st>>>(p, f);
  dscan_fold_top<M><<<dim3(p.B, tiles), NT, 0, st>>>(p, f, s_re, s_im, fin_re, fin_im);
  dscan_fold_blocks<M><<<dim3(p.B, NG, tiles), NT, 0, st>>>(p, f, out);
  return cudaGetLastError();
}

// dynamic shared memory of a staged block pass, and the opt-in for more than 48 KB
template <int M>
inline int stage_bytes(const sca2_dscan_args& p) {
  return Stage<M>::floats(ngl_max(M, p.V / p.G)) * (int)sizeof(float);
}
template <typename Kernel>
inline cudaError_t allow_smem(Kernel k, int bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int M>
cudaError_t launch_fwd_m(const sca2_dscan_args& p, float* ab, float* S_re, float* S_im, float* ckpt, float* work,
                         cudaStream_t st) {
  const int per_b = M * p.V, NK = (p.T + CK - 1) / CK;
  if (!use_blocks(p, work)) {  // short sequences (and decode): one sequential pass
    dim3 grid(p.B, (per_b + NT - 1) / NT);
    if (p.sep)
      dscan_fwd_kernel<M, true><<<grid, NT, 0, st>>>(p, ab, S_re, S_im, ckpt);
    else
      dscan_fwd_kernel<M, false><<<grid, NT, 0, st>>>(p, ab, S_re, S_im, ckpt);
    return cudaGetLastError();
  }
  float* e = work;
  float* P = e + (size_t)p.B * NK * 2 * M * p.V;
  float* ck = ckpt ? ckpt : P + (size_t)p.B * NK * 2 * M * p.G;  // inference: checkpoints in the workspace
  dim3 gl(p.B, NK, (per_b + NT - 1) / NT), gc(p.B, (per_b + NT - 1) / NT);
  const int sm = stage_bytes<M>(p);
  cudaError_t err = allow_smem(dscan_fwd_local<M>, sm);
  if (err != cudaSuccess) return err;
  dscan_fwd_local<M><<<gl, NT, sm, st>>>(p, e, P);
  if (NK > 2 * FG) {  // long sequences: the fold in three passes
    float* gw = e + dscan_base_floats(p.B, NK, M, p.G, p.V);
    if ((err = launch_fold<M>(p, P, e, ck, p.S0_re, p.S0_im, S_re, S_im, false, gw, st)) != cudaSuccess) return err;
  } else {
    dscan_fwd_carry<M><<<gc, NT, 0, st>>>(p, e, P, ck, S_re, S_im);
  }
  const int ob = OUT_TOK * 2 * (NT / M) * out_stride(M) * (int)sizeof(float);  // the output pass's row sums
  if (p.sep) {
    if ((err = allow_smem(dscan_fwd_out<M, true>, sm + ob)) != cudaSuccess) return err;
    dscan_fwd_out<M, true><<<gl, NT, sm + ob, st>>>(p, ck, ab);
  } else {
    if ((err = allow_smem(dscan_fwd_out<M, false>, ob)) != cudaSuccess) return err;
    dscan_fwd_out<M, false><<<gl, NT, ob, st>>>(p, ck, ab);
  }
  return cudaGetLastError();
}
template <int M>
cudaError_t launch_bwd_m(const sca2_dscan_args& p, const float* dab, const float* dS_re, const float* dS_im,
                         const float* ckpt, float* work, const sca2_dscan_grads& g, cudaStream_t st) {
  const int per_b = M * p.V, NK = (p.T + CK - 1) / CK;
  if (!use_blocks(p, work)) {
    dim3 grid(p.B, (per_b + NT - 1) / NT);
    if (p.sep)
      dscan_bwd_kernel<M, true><<<grid, NT, 0, st>>>(p, dab, dS_re, dS_im, ckpt, g);
    else
      dscan_bwd_kernel<M, false><<<grid, NT, 0, st>>>(p, dab, dS_re, dS_im, ckpt, g);
    return cudaGetLastError();
  }
  float* qv = work;
  float* R = qv + (size_t)p.B * NK * 2 * M * p.V;
  float* Qg = R + (size_t)p.B * NK * 2 * M * p.V;
  dim3 gl(p.B, NK, (per_b + NT - 1) / NT), gc(p.B, (per_b + NT - 1) / NT);
  const int sm = stage_bytes<M>(p);
  auto kl = p.sep ? dscan_bwd_local<M, true> : dscan_bwd_local<M, false>;
  cudaError_t err = allow_smem(kl, sm);
  if (err != cudaSuccess) return err;
  kl<<<gl, NT, sm, st>>>(p, dab, qv, Qg);
  if (NK > 2 * FG) {  // long sequences: the reverse fold in three passes
    float* gw = qv + dscan_base_floats(p.B, NK, M, p.G, p.V);
    if ((err = launch_fold<M>(p, Qg, qv, R, dS_re, dS_im, g.dS0_re, g.dS0_im, true, gw, st)) != cudaSuccess) return err;
  } else {
    dscan_bwd_carry<M><<<gc, NT, 0, st>>>(p, dS_re, dS_im, qv, Qg, R, g);
  }
  const int red = (p.sep ? 2 : 1) * (NT / 32) * CK * M * 2 * (int)sizeof(float) + (p.sep ? sm : 0);
  auto kb = p.sep ? dscan_bwd_block<M, true> : dscan_bwd_block<M, false>;
  if ((err = allow_smem(kb, red)) != cudaSuccess) return err;
  kb<<<gl, NT, red, st>>>(p, dab, ckpt, R, g);
  return cudaGetLastError();
}

}  // namespace dscan

// workspace of the chunk-parallel forms (floats): fwd e + P (+ checkpoints when the caller
// keeps none), bwd q + R + Q; then the three-pass fold's group maps and entering states
size_t dscan_work_floats(int B, int T, int M, int G, int V) {
  const int NK = (T + dscan::CK - 1) / dscan::CK;
  return dscan::dscan_base_floats(B, NK, M, G, V) + dscan::fold_floats(B, NK, M, G, V);
}

cudaError_t dscan_fwd(const sca2_dscan_args& p, float* ab, float* S_re, float* S_im, float* ckpt, float* work,
                      cudaStream_t st) {
  switch (p.M) {
    case 1: return dscan::launch_fwd_m<1>(p, ab, S_re, S_im, ckpt, work, st);
    case 2: return dscan::launch_fwd_m<2>(p, ab, S_re, S_im, ckpt, work, st);
    case 4: return dscan::launch_fwd_m<4>(p, ab, S_re, S_im, ckpt, work, st);
    case 8: return dscan::launch_fwd_m<8>(p, ab, S_re, S_im, ckpt, work, st);
    case 16: return dscan::launch_fwd_m<16>(p, ab, S_re, S_im, ckpt, work, st);
    case 32: return dscan::launch_fwd_m<32>(p, ab, S_re, S_im, ckpt, work, st);
  }
  return cudaErrorInvalidValue;
}
cudaError_t dscan_bwd(const sca2_dscan_args& p, const float* dab, const float* dS_re, const float* dS_im,
                      const float* ckpt, float* work, const sca2_dscan_grads& g, cudaStream_t st) {
  switch (p.M) {
    case 1: return dscan::launch_bwd_m<1>(p, dab, dS_re, dS_im, ckpt, work, g, st);
    case 2: return dscan::launch_bwd_m<2>(p, dab, dS_re, dS_im, ckpt, work, g, st);
    case 4: return dscan::launch_bwd_m<4>(p, dab, dS_re, dS_im, ckpt, work, g, st);
    case 8: return dscan::launch_bwd_m<8>(p, dab, dS_re, dS_im, ckpt, work, g, st);
    case 16: return dscan::launch_bwd_m<16>(p, dab, dS_re, dS_im, ckpt, work, g, st);
    case 32: return dscan::launch_bwd_m<32>(p, dab, dS_re, dS_im, ckpt, work, g, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sca2
