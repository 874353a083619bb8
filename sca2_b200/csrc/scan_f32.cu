// fp32 chunked scan (forward + backward) on CUDA cores: the exact-precision path.
//
// One CTA per (batch*head, block of VB value columns); it walks the chunks of its
// sequence in order (forward) or in reverse (backward).  Every value column of the
// recurrence is independent given the codes (S, e, o are column-separable), so the
// value axis is split across CTAs; per-token key-side gradients are summed over the
// value blocks with fp32 atomics.
//
// Chunk algebra (chunk of Cl tokens, i = 0..Cl-1, incoming state S; same as the
// numpy oracle's forward_chunked / backward_chunked):
//   kr = k * exp(-lam i), kw = k * exp(+lam i), qr = Q * exp(-lam i)   (scaled codes,
//        lapa/layer.py:319-326)
//   Gc = cumsum(g), a_i = exp(Gc_i), w_j = exp(Gc_{Cl-1} - Gc_j), Dg = exp(Gc_i - Gc_j)
//        (scalar decay as a C x C mask, sca2/arch_gatedc.py:136-139)
//   Sp = exp(-lam) S                                                  (lapa/layer.py:354)
//   Gr = (kr kw^T / kappa) .* Dg, strictly lower;  L = diag(beta) Gr   (Gram, :327)
//   E  = (I + L)^{-1} (v - beta .* a .* (kr Sp) / kappa)              (delta solve, :329-356)
//   P_r = (qr_r kw^T / kappa) .* Dg, lower incl.                      (K2, :345-348)
//   O_r = a .* (qr_r Sp) / kappa + P_r E                              (:357-362)
//   S'  = exp(-lam (Cl-1)) .* (a_{Cl-1} Sp + kw^T (w .* E))           (:363-364)
#include <cstdio>

#include "common.cuh"

namespace sca2 {
namespace f32 {

constexpr int CK = 32;    // internal chunk (the math is chunk-size invariant)
constexpr int VB = 32;    // value columns per CTA
constexpr int VBP = VB + 1;
constexpr int CKP = CK + 1;
constexpr int NT = 256;

struct Layout {
  int KP, R;
  // float offsets
  int kr, kw, qr, S, dS, dS0p, Gr, P, dL, dQK, E, R0, dY, dO, dK, dQ;
  int lam, d1, dCm1, dlam, dwr, dwi;
  int beta, Gc, a, w, da, dw, rows, cols, dbeta, misc;
  int total;
};

__host__ __device__ inline Layout make_layout(int K, int R, bool bwd) {
  Layout L{};
  L.KP = (K + 3) & ~3;
  L.R = R;
  int o = 0;
  auto take = [&](int n) { int r = o; o += (n + 3) & ~3; return r; };
  L.kr = take(CK * L.KP);
  L.kw = take(CK * L.KP);
  L.qr = take(R * CK * L.KP);
  L.S = take(L.KP * VBP);
  L.Gr = take(CK * CKP);
  L.P = take(R * CK * CKP);
  L.E = take(CK * VBP);
  L.lam = take(L.KP);
  L.d1 = take(L.KP);
  L.dCm1 = take(L.KP);
  L.beta = take(CK);
  L.Gc = take(CK);
  L.a = take(CK);
  L.w = take(CK);
  if (bwd) {
    L.dS = take(L.KP * VBP);
    L.dS0p = take(L.KP * VBP);
    L.dL = take(CK * CKP);
    L.dQK = take(R * CK * CKP);
    L.R0 = take(CK * VBP);
    L.dY = take(CK * VBP);
    L.dO = take(R * CK * VBP);
    L.dK = take(CK * L.KP);
    L.dQ = take(R * CK * L.KP);
    L.dlam = take(L.KP);
    L.dwr = take(L.KP);
    L.dwi = take(L.KP);
    L.da = take(CK);
    L.dw = take(CK);
    L.rows = take(CK);
    L.cols = take(CK);
    L.dbeta = take(CK);
    L.misc = take(8);
  }
  L.total = o;
  return L;
}

// ---- chunk prologue: codes, scaled codes, gates, values --------------------------------
// Rows i >= Cl are zero (codes, values, beta, g) so a ragged last chunk needs no special
// case in the contractions.
template <int FL>
__device__ void load_chunk(const sca2_scan_args& p, const Layout& Lo, float* sm, int b, int h,
                           int t0, int Cl, int vb0) {
  const int K = p.K, KP = Lo.KP;
  float* kr = sm + Lo.kr;
  float* kw = sm + Lo.kw;
  float* qr = sm + Lo.qr;
  float* Y = sm + Lo.E;
  const float* lam = sm + Lo.lam;
  if (FL == SCA2_FLAVOR_PHASE) {
    const int Mh = K / 2;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
    for (int idx = threadIdx.x; idx < CK * Mh; idx += blockDim.x) {
      const int i = idx / Mh, m = idx - (idx / Mh) * Mh;
      float c = 0.f, s = 0.f, c1 = 0.f, c2 = 0.f, ell = 1.f, elli = 1.f;
      if (i < Cl) {
        const float phi = phw[tok_off(p.phw, b, t0 + i, h) + m];
        const float psi = phq[tok_off(p.phq, b, t0 + i, h) + m];
        float cq, sq;
        sincosf(phi, &s, &c);
        sincosf(psi, &sq, &cq);
        const float wr = p.wr[h * Mh + m], wi = p.wi[h * Mh + m];
        c1 = wr * cq + wi * sq;
        c2 = wr * sq - wi * cq;
        const float l = lam[m];
        ell = expf(-l * (float)i);
        elli = expf(l * (float)i);
      }
      kr[i * KP + m] = c * ell;
      kr[i * KP + m + Mh] = s * ell;
      kw[i * KP + m] = c * elli;
      kw[i * KP + m + Mh] = s * elli;
      qr[(0 * CK + i) * KP + m] = c1 * ell;
      qr[(0 * CK + i) * KP + m + Mh] = c2 * ell;
      qr[(1 * CK + i) * KP + m] = -c2 * ell;
      qr[(1 * CK + i) * KP + m + Mh] = c1 * ell;
    }
  } else {
    for (int idx = threadIdx.x; idx < CK * K; idx += blockDim.x) {
      const int i = idx / K, m = idx - (idx / K) * K;
      float kk = 0.f, qq = 0.f, ell = 1.f, elli = 1.f;
      if (i < Cl) {
        kk = ld_io(p.phw.ptr, tok_off(p.phw, b, t0 + i, h) + m, p.io_dtype);
        qq = p.q_scale * ld_io(p.phq.ptr, tok_off(p.phq, b, t0 + i, h) + m, p.io_dtype);
        const float l = lam[m];
        ell = expf(-l * (float)i);
        elli = expf(l * (float)i);
      }
      kr[i * KP + m] = kk * ell;
      kw[i * KP + m] = kk * elli;
      qr[i * KP + m] = qq * ell;
    }
  }
  // gates (CK == 32: one warp)
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
    const float* gp = reinterpret_cast<const float*>(p.g.ptr);
    const float bt = (bp && i < Cl) ? bp[tok_off(p.beta, b, t0 + i, h)] : 0.f;
    const float gi = (gp && i < Cl) ? gp[tok_off(p.g, b, t0 + i, h)] : 0.f;
    const float Gc = warp_incl_scan(gi);
    const float Glast = __shfl_sync(0xffffffffu, Gc, Cl - 1);
    sm[Lo.beta + i] = bt;
    sm[Lo.Gc + i] = Gc;
    sm[Lo.a + i] = expf(Gc);
    sm[Lo.w + i] = i < Cl ? exp_le0(Glast - Gc) : 0.f;
  }
  for (int m = threadIdx.x; m < KP; m += blockDim.x)
    sm[Lo.dCm1 + m] = expf(-lam[m] * (float)(Cl - 1));
  // values (GDN form: pre-scaled by beta)
  const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
  for (int idx = threadIdx.x; idx < CK * VB; idx += blockDim.x) {
    const int i = idx / VB, j = idx - (idx / VB) * VB;
    float x = 0.f;
    if (i < Cl && vb0 + j < p.V) {
      x = ld_io(p.v.ptr, tok_off(p.v, b, t0 + i, h) + vb0 + j, p.io_dtype);
      if (p.v_times_beta) x *= bp[tok_off(p.beta, b, t0 + i, h)];
    }
    Y[i * VBP + j] = x;
  }
}

// per-channel constants of head h: lam (0 if none), d1 = exp(-lam); zero padding columns
template <int FL>
__device__ void init_head(const sca2_scan_args& p, const Layout& Lo, float* sm, int h) {
  const int K = p.K, KP = Lo.KP;
  const int KH = FL == SCA2_FLAVOR_PHASE ? K / 2 : K;
  for (int m = threadIdx.x; m < KP; m += blockDim.x) {
    float l = 0.f;
    if (m < K && p.lam) l = p.lam[h * KH + (m % KH)];
    sm[Lo.lam + m] = l;
    sm[Lo.d1 + m] = expf(-l);
  }
  if (KP != K) {
    const int R = Lo.R;
    for (int idx = threadIdx.x; idx < CK * KP; idx += blockDim.x) {
      if (idx % KP >= K) {
        sm[Lo.kr + idx] = 0.f;
        sm[Lo.kw + idx] = 0.f;
        for (int r = 0; r < R; ++r) sm[Lo.qr + r * CK * KP + idx] = 0.f;
      }
    }
  }
}

// E = (I + diag(beta) Gr)^{-1} Y in place (forward substitution; one warp per 4 columns,
// lane = row).  Gr is strictly lower with zeros elsewhere.
__device__ __forceinline__ void solve_lower(const float* Gr, const float* beta, float* Y) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const float bl = beta[lane];
  float y[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) y[q] = Y[lane * VBP + wid + 8 * q];
  for (int jj = 0; jj < CK - 1; ++jj) {
    const float l = bl * Gr[lane * CKP + jj];
#pragma unroll
    for (int q = 0; q < 4; ++q) y[q] -= l * __shfl_sync(0xffffffffu, y[q], jj);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) Y[lane * VBP + wid + 8 * q] = y[q];
}

// dY = (I + diag(beta) Gr)^{-T} dE in place (backward substitution).
__device__ __forceinline__ void solve_upper_T(const float* Gr, const float* beta, float* Y) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float y[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) y[q] = Y[lane * VBP + wid + 8 * q];
  for (int jj = CK - 1; jj > 0; --jj) {
    const float l = beta[jj] * Gr[jj * CKP + lane];  // zero for lane >= jj
#pragma unroll
    for (int q = 0; q < 4; ++q) y[q] -= l * __shfl_sync(0xffffffffu, y[q], jj);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) Y[lane * VBP + wid + 8 * q] = y[q];
}

// ======================================================================================
//  forward
// ======================================================================================
template <int FL>
__global__ void __launch_bounds__(NT) scan_fwd_kernel(sca2_scan_args p, sca2_out o,
                                                      float* S_final, float* cstates, int NC, int NCS,
                                                      Layout Lo) {
  extern __shared__ float sm[];
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int vb0 = blockIdx.y * VB;
  const int K = p.K, V = p.V, KP = Lo.KP;
  constexpr int R = FL == SCA2_FLAVOR_PHASE ? 2 : 1;
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)(K / 2) : 1.f;
  const float ik = 1.f / kappa;
  float* kr = sm + Lo.kr;
  float* kw = sm + Lo.kw;
  float* qr = sm + Lo.qr;
  float* S = sm + Lo.S;
  float* Gr = sm + Lo.Gr;
  float* P = sm + Lo.P;
  float* Y = sm + Lo.E;
  const float* d1 = sm + Lo.d1;
  const float* dCm1 = sm + Lo.dCm1;
  const float* beta = sm + Lo.beta;
  const float* Gc = sm + Lo.Gc;
  const float* av = sm + Lo.a;
  const float* wv = sm + Lo.w;

  init_head<FL>(p, Lo, sm, h);
  const int64_t sbase = ((int64_t)b * p.H + h) * K * (int64_t)V;
  for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
    const int m = idx / VB, j = idx - (idx / VB) * VB;
    float x = 0.f;
    if (p.S0 && m < K && vb0 + j < V) x = p.S0[sbase + (int64_t)m * V + vb0 + j];
    S[m * VBP + j] = x;
  }
  __syncthreads();

  for (int c = 0; c < NC; ++c) {
    const int t0 = c * CK, Cl = min(CK, p.T - t0);
    if (cstates) {
      const int64_t cb = (((int64_t)b * p.H + h) * NCS + c) * K * (int64_t)V;
      for (int idx = threadIdx.x; idx < K * VB; idx += blockDim.x) {
        const int m = idx / VB, j = idx - (idx / VB) * VB;
        if (vb0 + j < V) cstates[cb + (int64_t)m * V + vb0 + j] = S[m * VBP + j];
      }
    }
    load_chunk<FL>(p, Lo, sm, b, h, t0, Cl, vb0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
      const int m = idx / VB, j = idx - (idx / VB) * VB;
      S[m * VBP + j] *= d1[m];
    }
    __syncthreads();
    // ---- Gram, intra-chunk read kernel, state read-back
    smem_gemm<2, 2>(CK, CK, KP, [&](int i, int k) { return kr[i * KP + k]; },
                    [&](int k, int j) { return kw[j * KP + k]; },
                    [&](int i, int j, float acc) {
                      Gr[i * CKP + j] = j < i ? acc * ik * exp_le0(Gc[i] - Gc[j]) : 0.f;
                    });
    for (int r = 0; r < R; ++r) {
      const float* q = qr + r * CK * KP;
      float* Pr = P + r * CK * CKP;
      smem_gemm<2, 2>(CK, CK, KP, [&](int i, int k) { return q[i * KP + k]; },
                      [&](int k, int j) { return kw[j * KP + k]; },
                      [&](int i, int j, float acc) {
                        Pr[i * CKP + j] = j <= i ? acc * ik * exp_le0(Gc[i] - Gc[j]) : 0.f;
                      });
    }
    smem_gemm<2, 2>(CK, VB, KP, [&](int i, int k) { return kr[i * KP + k]; },
                    [&](int k, int j) { return S[k * VBP + j]; },
                    [&](int i, int j, float acc) { Y[i * VBP + j] -= beta[i] * av[i] * acc * ik; });
    __syncthreads();
    solve_lower(Gr, beta, Y);
    __syncthreads();
    // ---- outputs: O_r = a qr_r Sp / kappa + P_r E
    for (int r = 0; r < R; ++r) {
      const float* q = qr + r * CK * KP;
      const float* Pr = P + r * CK * CKP;
      smem_gemm<2, 2>(
          CK, VB, KP + CK,
          [&](int i, int k) { return k < KP ? av[i] * ik * q[i * KP + k] : Pr[i * CKP + (k - KP)]; },
          [&](int k, int j) { return k < KP ? S[k * VBP + j] : Y[(k - KP) * VBP + j]; },
          [&](int i, int j, float acc) {
            if (i < Cl && vb0 + j < V) st_io(o.ptr, out_off(o, b, t0 + i, h, r) + vb0 + j, acc, p.io_dtype);
          });
    }
    __syncthreads();
    // ---- state update
    const float aC = av[Cl - 1];
    smem_gemm<2, 2>(KP, VB, CK, [&](int m, int i) { return kw[i * KP + m]; },
                    [&](int i, int j) { return wv[i] * Y[i * VBP + j]; },
                    [&](int m, int j, float acc) {
                      S[m * VBP + j] = dCm1[m] * (aC * S[m * VBP + j] + acc);
                    });
    __syncthreads();
  }
  if (S_final) {
    for (int idx = threadIdx.x; idx < K * VB; idx += blockDim.x) {
      const int m = idx / VB, j = idx - (idx / VB) * VB;
      if (vb0 + j < V) S_final[sbase + (int64_t)m * V + vb0 + j] = S[m * VBP + j];
    }
  }
}

// ======================================================================================
//  backward
// ======================================================================================
template <int FL>
__global__ void __launch_bounds__(NT) scan_bwd_kernel(sca2_scan_args p, sca2_out dO,
                                                      const float* dS_final, const float* cstates,
                                                      sca2_scan_grads gr, int NC, int NCS, Layout Lo) {
  extern __shared__ float sm[];
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int vb0 = blockIdx.y * VB;
  const int K = p.K, V = p.V, KP = Lo.KP;
  constexpr int R = FL == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int Mh = K / 2;
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)Mh : 1.f;
  const float ik = 1.f / kappa;
  float* kr = sm + Lo.kr;
  float* kw = sm + Lo.kw;
  float* qr = sm + Lo.qr;
  float* Sp = sm + Lo.S;
  float* dS = sm + Lo.dS;
  float* dS0p = sm + Lo.dS0p;
  float* Gr = sm + Lo.Gr;
  float* P = sm + Lo.P;
  float* dL = sm + Lo.dL;
  float* dQK = sm + Lo.dQK;
  float* E = sm + Lo.E;
  float* R0 = sm + Lo.R0;
  float* dY = sm + Lo.dY;
  float* dOs = sm + Lo.dO;
  float* dK = sm + Lo.dK;
  float* dQ = sm + Lo.dQ;
  const float* lam = sm + Lo.lam;
  const float* d1 = sm + Lo.d1;
  const float* dCm1 = sm + Lo.dCm1;
  float* dlam = sm + Lo.dlam;
  float* dwr = sm + Lo.dwr;
  float* dwi = sm + Lo.dwi;
  const float* beta = sm + Lo.beta;
  const float* Gc = sm + Lo.Gc;
  const float* av = sm + Lo.a;
  const float* wv = sm + Lo.w;
  float* da = sm + Lo.da;
  float* dw = sm + Lo.dw;
  float* rows = sm + Lo.rows;
  float* cols = sm + Lo.cols;
  float* dbeta = sm + Lo.dbeta;
  float* misc = sm + Lo.misc;

  init_head<FL>(p, Lo, sm, h);
  for (int m = threadIdx.x; m < KP; m += blockDim.x) {
    dlam[m] = 0.f;
    dwr[m] = 0.f;
    dwi[m] = 0.f;
  }
  const int64_t sbase = ((int64_t)b * p.H + h) * K * (int64_t)V;
  for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
    const int m = idx / VB, j = idx - (idx / VB) * VB;
    float x = 0.f;
    if (dS_final && m < K && vb0 + j < V) x = dS_final[sbase + (int64_t)m * V + vb0 + j];
    dS[m * VBP + j] = x;
  }
  __syncthreads();

  for (int c = NC - 1; c >= 0; --c) {
    const int t0 = c * CK, Cl = min(CK, p.T - t0);
    load_chunk<FL>(p, Lo, sm, b, h, t0, Cl, vb0);  // values land in E (as Y)
    {
      const int64_t cb = (((int64_t)b * p.H + h) * NCS + c) * K * (int64_t)V;
      for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
        const int m = idx / VB, j = idx - (idx / VB) * VB;
        float x = 0.f;
        if (m < K && vb0 + j < V) x = cstates[cb + (int64_t)m * V + vb0 + j];
        Sp[m * VBP + j] = x;  // scaled by d1 below
      }
      for (int idx = threadIdx.x; idx < R * CK * VB; idx += blockDim.x) {
        const int r = idx / (CK * VB), rem = idx - r * (CK * VB);
        const int i = rem / VB, j = rem - (rem / VB) * VB;
        float x = 0.f;
        if (i < Cl && vb0 + j < V) x = ld_io(dO.ptr, out_off(dO, b, t0 + i, h, r) + vb0 + j, p.io_dtype);
        dOs[(r * CK + i) * VBP + j] = x;
      }
      if (threadIdx.x < CK) {
        da[threadIdx.x] = 0.f;
        dw[threadIdx.x] = 0.f;
        rows[threadIdx.x] = 0.f;
        cols[threadIdx.x] = 0.f;
        dbeta[threadIdx.x] = 0.f;
      }
      if (threadIdx.x == 0) misc[0] = 0.f;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
      const int m = idx / VB, j = idx - (idx / VB) * VB;
      Sp[m * VBP + j] *= d1[m];
    }
    __syncthreads();
    // ---- A: Gram (no beta), P, R0 = a kr Sp / kappa, da += a sum_r dO_r . (qr_r Sp)/kappa
    smem_gemm<2, 2>(CK, CK, KP, [&](int i, int k) { return kr[i * KP + k]; },
                    [&](int k, int j) { return kw[j * KP + k]; },
                    [&](int i, int j, float acc) {
                      Gr[i * CKP + j] = j < i ? acc * ik * exp_le0(Gc[i] - Gc[j]) : 0.f;
                    });
    for (int r = 0; r < R; ++r) {
      const float* q = qr + r * CK * KP;
      float* Pr = P + r * CK * CKP;
      const float* dOr = dOs + r * CK * VBP;
      smem_gemm<2, 2>(CK, CK, KP, [&](int i, int k) { return q[i * KP + k]; },
                      [&](int k, int j) { return kw[j * KP + k]; },
                      [&](int i, int j, float acc) {
                        Pr[i * CKP + j] = j <= i ? acc * ik * exp_le0(Gc[i] - Gc[j]) : 0.f;
                      });
      if (p.g.ptr) {
        smem_gemm<2, 2>(CK, VB, KP, [&](int i, int k) { return q[i * KP + k]; },
                        [&](int k, int j) { return Sp[k * VBP + j]; },
                        [&](int i, int j, float acc) {
                          atomicAdd(&da[i], av[i] * ik * acc * dOr[i * VBP + j]);
                        });
      }
    }
    smem_gemm<2, 2>(CK, VB, KP, [&](int i, int k) { return kr[i * KP + k]; },
                    [&](int k, int j) { return Sp[k * VBP + j]; },
                    [&](int i, int j, float acc) {
                      const float r0 = av[i] * acc * ik;
                      R0[i * VBP + j] = r0;
                      E[i * VBP + j] -= beta[i] * r0;
                    });
    __syncthreads();
    // ---- B: recompute E
    solve_lower(Gr, beta, E);
    __syncthreads();
    // ---- C: dE = w .* (kw dSc) + sum_r P_r^T dO_r, with dSc = exp(-lam (Cl-1)) dS
    smem_gemm<2, 2>(CK, VB, KP, [&](int jr, int m) { return kw[jr * KP + m] * dCm1[m]; },
                    [&](int m, int j) { return dS[m * VBP + j]; },
                    [&](int jr, int j, float acc) {
                      const float x = wv[jr] * acc;
                      dY[jr * VBP + j] = x;
                      if (p.g.ptr) atomicAdd(&dw[jr], x * E[jr * VBP + j]);
                    });
    __syncthreads();
    smem_gemm<2, 2>(CK, VB, R * CK,
                    [&](int jr, int k) {
                      const int r = k / CK, i = k - (k / CK) * CK;
                      return P[(r * CK + i) * CKP + jr];
                    },
                    [&](int k, int j) {
                      const int r = k / CK, i = k - (k / CK) * CK;
                      return dOs[(r * CK + i) * VBP + j];
                    },
                    [&](int jr, int j, float acc) { dY[jr * VBP + j] += acc; });
    __syncthreads();
    // ---- D: dY = (I + L)^{-T} dE
    solve_upper_T(Gr, beta, dY);
    __syncthreads();
    // ---- E: dL (strict) and dP (lower incl.) plus the row-wise beta / decay terms
    smem_gemm<2, 2>(CK, CK, VB, [&](int i, int v) { return dY[i * VBP + v]; },
                    [&](int v, int j) { return E[j * VBP + v]; },
                    [&](int i, int j, float acc) {
                      float out = 0.f;
                      if (j < i) {
                        const float dl = -acc;                       // dL = -dY E^T
                        const float g = Gr[i * CKP + j];
                        atomicAdd(&dbeta[i], dl * g);
                        if (p.g.ptr) {
                          const float gc = beta[i] * dl * g;
                          atomicAdd(&rows[i], gc);
                          atomicAdd(&cols[j], gc);
                        }
                        out = beta[i] * dl * exp_le0(Gc[i] - Gc[j]);  // d(kr kw^T / kappa)
                      }
                      dL[i * CKP + j] = out;
                    });
    for (int r = 0; r < R; ++r) {
      const float* dOr = dOs + r * CK * VBP;
      const float* Pr = P + r * CK * CKP;
      float* dQr = dQK + r * CK * CKP;
      smem_gemm<2, 2>(CK, CK, VB, [&](int i, int v) { return dOr[i * VBP + v]; },
                      [&](int v, int j) { return E[j * VBP + v]; },
                      [&](int i, int j, float acc) {
                        float out = 0.f;
                        if (j <= i) {
                          if (p.g.ptr) {
                            const float gc = acc * Pr[i * CKP + j];
                            atomicAdd(&rows[i], gc);
                            atomicAdd(&cols[j], gc);
                          }
                          out = acc * exp_le0(Gc[i] - Gc[j]);
                        }
                        dQr[i * CKP + j] = out;
                      });
    }
    // row terms: s_i = sum_v dY R0; dbeta -= s_i; da -= beta s_i (dR0 = -beta dY); dv
    {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
      for (int i = wid; i < CK; i += NT / 32) {
        float s = dY[i * VBP + lane] * R0[i * VBP + lane];
        float sv = 0.f;
        const bool ok = i < Cl && vb0 + lane < V;
        float dvv = dY[i * VBP + lane];
        if (p.v_times_beta && ok) {
          const float vr = ld_io(p.v.ptr, tok_off(p.v, b, t0 + i, h) + vb0 + lane, p.io_dtype);
          sv = dvv * vr;
          dvv *= bp[tok_off(p.beta, b, t0 + i, h)];
        }
        if (ok) st_io(const_cast<void*>(gr.dv.ptr), tok_off(gr.dv, b, t0 + i, h) + vb0 + lane, dvv, p.io_dtype);
        s = warp_sum(s);
        sv = warp_sum(sv);
        if (lane == 0) {  // other threads add into the same rows in this phase
          atomicAdd(&dbeta[i], sv - s);
          atomicAdd(&da[i], -beta[i] * s);
        }
      }
    }
    __syncthreads();
    // ---- F: key-side gradients per (token i, channel m), and dS0p per (m, v)
    for (int idx = threadIdx.x; idx < CK * KP; idx += blockDim.x) {
      const int i = idx / KP, m = idx - (idx / KP) * KP;
      float dkr = 0.f, dkw = 0.f, dq0 = 0.f, dq1 = 0.f, tS = 0.f, sR = 0.f, sO0 = 0.f, sO1 = 0.f;
      for (int j = 0; j < CK; ++j) {
        dkr = fmaf(dL[i * CKP + j], kw[j * KP + m], dkr);
        dkw = fmaf(dL[j * CKP + i], kr[j * KP + m], dkw);
        dq0 = fmaf(dQK[i * CKP + j], kw[j * KP + m], dq0);
        dkw = fmaf(dQK[j * CKP + i], qr[j * KP + m], dkw);
        if (R == 2) {
          dq1 = fmaf(dQK[(CK + i) * CKP + j], kw[j * KP + m], dq1);
          dkw = fmaf(dQK[(CK + j) * CKP + i], qr[(CK + j) * KP + m], dkw);
        }
      }
      for (int v = 0; v < VB; ++v) {
        const float sp = Sp[m * VBP + v];
        tS = fmaf(E[i * VBP + v], dS[m * VBP + v], tS);
        sR = fmaf(dY[i * VBP + v], sp, sR);
        sO0 = fmaf(dOs[i * VBP + v], sp, sO0);
        if (R == 2) sO1 = fmaf(dOs[(CK + i) * VBP + v], sp, sO1);
      }
      const float ai = av[i];
      tS *= wv[i] * dCm1[m];
      dkr = dkr * ik - ai * beta[i] * sR * ik;
      dkw = dkw * ik + tS;
      dq0 = (dq0 + ai * sO0) * ik;
      dq1 = (dq1 + ai * sO1) * ik;
      const float l = lam[m], fi = (float)i;
      const float ell = expf(-l * fi), elli = expf(l * fi);
      dK[i * KP + m] = dkr * ell + dkw * elli;
      dQ[i * KP + m] = dq0 * ell;
      if (R == 2) dQ[(CK + i) * KP + m] = dq1 * ell;
      if (p.lam && m < K) {
        float dl = fi * (dkw * kw[i * KP + m] - dkr * kr[i * KP + m] - dq0 * qr[i * KP + m]);
        if (R == 2) dl -= fi * dq1 * qr[(CK + i) * KP + m];
        dl -= (float)(Cl - 1) * kw[i * KP + m] * tS;
        atomicAdd(&dlam[m], dl);
      }
    }
    smem_gemm<2, 2>(KP, VB, (R + 1) * CK,
                    [&](int m, int k) {
                      const int r = k / CK, i = k - (k / CK) * CK;
                      return r < R ? qr[(r * CK + i) * KP + m] * av[i]
                                   : -kr[i * KP + m] * av[i] * beta[i];
                    },
                    [&](int k, int j) {
                      const int r = k / CK, i = k - (k / CK) * CK;
                      return r < R ? dOs[(r * CK + i) * VBP + j] : dY[i * VBP + j];
                    },
                    [&](int m, int j, float acc) { dS0p[m * VBP + j] = acc * ik; });
    __syncthreads();
    // ---- G: adjoint state to the previous chunk, state-side decay gradients
    {
      const float aC = av[Cl - 1];
      float daC = 0.f;
      for (int idx = threadIdx.x; idx < KP * VB; idx += blockDim.x) {
        const int m = idx / VB, j = idx - (idx / VB) * VB;
        const float sp = Sp[m * VBP + j], ds = dS[m * VBP + j], d0 = dS0p[m * VBP + j];
        const float t = aC * dCm1[m] * sp * ds;  // aC exp(-lam Cl) S0 dS
        daC += t;
        if (p.lam && m < K) atomicAdd(&dlam[m], -d0 * sp - (float)Cl * t);
        dS[m * VBP + j] = aC * dCm1[m] * d1[m] * ds + d1[m] * d0;
      }
      if (p.g.ptr) {
        daC = warp_sum(daC);
        if ((threadIdx.x & 31) == 0) atomicAdd(&misc[0], daC);
      }
    }
    __syncthreads();
    // ---- H: per-token outputs
    if (p.g.ptr && threadIdx.x < 32) {
      const int i = threadIdx.x;
      const float dwi_ = dw[i];
      const float dwsum = warp_sum(dwi_);
      float dG = rows[i] - cols[i] + da[i] - dwi_;
      if (i == Cl - 1) dG += dwsum + misc[0];
      if (i >= Cl) dG = 0.f;
      // reverse inclusive cumsum: dg_i = sum_{u >= i} dG_u
      float tot = warp_sum(dG);
      float incl = warp_incl_scan(dG);
      const float dg = tot - incl + dG;
      if (i < Cl) {
        float* gp = reinterpret_cast<float*>(const_cast<void*>(gr.dg.ptr));
        atomicAdd(&gp[tok_off(gr.dg, b, t0 + i, h)], dg);
      }
    }
    if (p.beta.ptr && gr.dbeta.ptr && threadIdx.x >= 32 && threadIdx.x < 64) {
      const int i = threadIdx.x - 32;
      if (i < Cl) {
        float* bp = reinterpret_cast<float*>(const_cast<void*>(gr.dbeta.ptr));
        atomicAdd(&bp[tok_off(gr.dbeta, b, t0 + i, h)], dbeta[i]);
      }
    }
    if (FL == SCA2_FLAVOR_PHASE) {
      const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
      const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
      float* dphw = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
      float* dphq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
      for (int idx = threadIdx.x; idx < CK * Mh; idx += blockDim.x) {
        const int i = idx / Mh, m = idx - (idx / Mh) * Mh;
        if (i >= Cl) continue;
        float s, c, sq, cq;
        sincosf(phw[tok_off(p.phw, b, t0 + i, h) + m], &s, &c);
        sincosf(phq[tok_off(p.phq, b, t0 + i, h) + m], &sq, &cq);
        const float dphi = -s * dK[i * KP + m] + c * dK[i * KP + m + Mh];
        const float dc1 = dQ[i * KP + m] + dQ[(CK + i) * KP + m + Mh];
        const float dc2 = dQ[i * KP + m + Mh] - dQ[(CK + i) * KP + m];
        const float wr = p.wr[h * Mh + m], wi = p.wi[h * Mh + m];
        atomicAdd(&dwr[m], dc1 * cq + dc2 * sq);
        atomicAdd(&dwi[m], dc1 * sq - dc2 * cq);
        const float dcq = dc1 * wr - dc2 * wi, dsq = dc1 * wi + dc2 * wr;
        atomicAdd(&dphw[tok_off(gr.dphw, b, t0 + i, h) + m], dphi);
        atomicAdd(&dphq[tok_off(gr.dphq, b, t0 + i, h) + m], -sq * dcq + cq * dsq);
      }
    } else {
      float* dk = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
      float* dq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
      for (int idx = threadIdx.x; idx < CK * K; idx += blockDim.x) {
        const int i = idx / K, m = idx - (idx / K) * K;
        if (i >= Cl) continue;
        atomicAdd(&dk[tok_off(gr.dphw, b, t0 + i, h) + m], dK[i * KP + m]);
        atomicAdd(&dq[tok_off(gr.dphq, b, t0 + i, h) + m], p.q_scale * dQ[i * KP + m]);
      }
    }
    __syncthreads();
  }
  // incoming-state gradient and per-head gradients
  if (gr.dS0) {
    for (int idx = threadIdx.x; idx < K * VB; idx += blockDim.x) {
      const int m = idx / VB, j = idx - (idx / VB) * VB;
      if (vb0 + j < V) gr.dS0[sbase + (int64_t)m * V + vb0 + j] = dS[m * VBP + j];
    }
  }
  const int KH = FL == SCA2_FLAVOR_PHASE ? Mh : K;
  for (int m = threadIdx.x; m < K; m += blockDim.x) {
    if (gr.dlam && p.lam) atomicAdd(&gr.dlam[h * KH + (m % KH)], dlam[m]);
    if (FL == SCA2_FLAVOR_PHASE && m < Mh) {
      if (gr.dwr) atomicAdd(&gr.dwr[h * Mh + m], dwr[m]);
      if (gr.dwi) atomicAdd(&gr.dwi[h * Mh + m], dwi[m]);
    }
  }
}

}  // namespace f32

// ---- host launchers ------------------------------------------------------------------
int f32_smem_bytes(int K, int R, bool bwd) { return f32::make_layout(K, R, bwd).total * 4; }
int f32_num_chunks(int T) { return (T + f32::CK - 1) / f32::CK; }

cudaError_t f32_scan_fwd(const sca2_scan_args& p, const sca2_out& o, float* S_final,
                         float* cstates, cudaStream_t st) {
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  f32::Layout Lo = f32::make_layout(p.K, R, false);
  const int NC = f32_num_chunks(p.T);
  dim3 grid(p.B * p.H, (p.V + f32::VB - 1) / f32::VB);
  const size_t smem = (size_t)Lo.total * 4;
  if (p.flavor == SCA2_FLAVOR_PHASE) {
    auto k = f32::scan_fwd_kernel<SCA2_FLAVOR_PHASE>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, f32::NT, smem, st>>>(p, o, S_final, cstates, NC, state_slots(p.T), Lo);
  } else {
    auto k = f32::scan_fwd_kernel<SCA2_FLAVOR_KEY>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, f32::NT, smem, st>>>(p, o, S_final, cstates, NC, state_slots(p.T), Lo);
  }
  return cudaGetLastError();
}

cudaError_t f32_scan_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final,
                         const float* cstates, const sca2_scan_grads& gr, cudaStream_t st) {
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  f32::Layout Lo = f32::make_layout(p.K, R, true);
  const int NC = f32_num_chunks(p.T);
  dim3 grid(p.B * p.H, (p.V + f32::VB - 1) / f32::VB);
  const size_t smem = (size_t)Lo.total * 4;
  if (p.flavor == SCA2_FLAVOR_PHASE) {
    auto k = f32::scan_bwd_kernel<SCA2_FLAVOR_PHASE>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, f32::NT, smem, st>>>(p, dO, dS_final, cstates, gr, NC, state_slots(p.T), Lo);
  } else {
    auto k = f32::scan_bwd_kernel<SCA2_FLAVOR_KEY>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, f32::NT, smem, st>>>(p, dO, dS_final, cstates, gr, NC, state_slots(p.T), Lo);
  }
  return cudaGetLastError();
}

}  // namespace sca2
