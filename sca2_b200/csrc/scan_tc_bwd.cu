// Tensor-core (tcgen05 / TMEM) backward scan for bf16 inputs on sm_100a.
//
// One CTA per (batch*head, block of VB value columns); chunks of 64 tokens are walked in
// reverse.  Per chunk, with S the state entering the chunk (saved by the forward at slot 2c)
// and dS the adjoint of the state leaving it (carried in fp32 registers):
//
//   forward recompute   G = KR KW^T, T = (I + beta Gr)^{-1}, U^T = V'^T T^T, Wk = T Z^T,
//                       X^T = Sp^T Wk^T, E = U - X, R0^T = Sp^T KR^T (a/kappa),
//                       Os = QR Sp                                  (Sp = d1 .* S)
//   adjoint chain       dE^T = dSc^T (KW diag w)^T + dO^T P          (dSc = dCm1 .* dS)
//                       dY^T = dE^T T
//                       dS0p^T = dO^T (QR a/kappa) - dY^T Z^T
//                       dS <- a_last dCm1 d1 .* dS + d1 .* dS0p
//   gradients           dL = -dY E^T, dP = dO E^T, dKK = beta dL .* Dg, dQK = dP .* Dg
//                       dkr = dKK KW / kappa - (beta a / kappa) dY Sp^T
//                       dqr = dQK KW / kappa + (a / kappa) dO Sp^T
//                       dkw = (dKK^T KR + dQK^T QR) / kappa + w E dSc^T
//                       Lw = (((j - i) dKK)^T KR + ((j - i) dQK)^T QR) / kappa: the
//                       intra-chunk part of d(lam) is sum_j kw_j .* Lw_j, taken in this
//                       relative-position form because i (kr, qr) and j (kw) weighted
//                       sums cancel to a few percent of their size
//                       then d(phi, psi | k, q), d(beta), d(g), d(lam), d(wr, wi), dv = dY
//
// Same algebra as the oracle's backward_chunked.  All products are bf16 MMAs with fp32
// accumulation in TMEM; the inversion, masks, decays and reductions run on CUDA cores in
// fp32.  Shared memory is carved into a persistent area and two pools that alias each other
// (pool A lives until the third MMA batch completes, pool B is written after it).  Every
// mbarrier wait is bounded: on a timeout the CTA records a fault bit, frees its TMEM and
// returns.  Key-side gradients are accumulated into zero-filled fp32 buffers with atomics.
#include "tc_common.cuh"

namespace sca2 {
namespace tc {

extern __device__ unsigned int g_fault;

template <int KD, int VB, int R>
struct BwdLayout {
  static constexpr int al(int x) { return (x + 1023) & ~1023; }
  static constexpr int mx(int a, int b) { return a > b ? a : b; }
  static constexpr int RC = R * C;
  // persistent
  static constexpr int PT = 0;                                  // C x RC   [j][(r,i)]  P^T
  static constexpr int TBT = PT + al(C * RC * 2);               // C x C    [i][j] = T[j][i]
  static constexpr int DOA = TBT + al(C * C * 2);               // RC x VB  [(r,i)][v]  dO
  static constexpr int Z = DOA + al(RC * VB * 2);               // KD x C   [m][i]
  static constexpr int POOL = Z + al(KD * C * 2);
  // pool A: prologue .. third MMA batch
  static constexpr int KR = POOL;                               // C x KD
  static constexpr int KW = KR + al(C * KD * 2);                // C x KD
  static constexpr int QR = KW + al(C * KD * 2);                // RC x KD
  static constexpr int VT = QR + al(RC * KD * 2);               // VB x C
  static constexpr int SB = VT + al(VB * C * 2);                // VB x KD  Sp^T
  static constexpr int DSB = SB + al(VB * KD * 2);              // VB x KD  dSc^T
  static constexpr int DOT = DSB + al(VB * KD * 2);             // VB x RC  dO^T
  static constexpr int KWW = DOT + al(VB * RC * 2);             // C x KD   kw w
  static constexpr int QRAT = KWW + al(C * KD * 2);             // KD x RC  qr a / kappa
  static constexpr int TB = QRAT + al(KD * RC * 2);             // C x C
  static constexpr int WK = TB + al(C * C * 2);                 // C x KD
  static constexpr int LS = WK + al(C * KD * 2);                // fp32 C x LDF
  static constexpr int TS = LS + al(C * LDF * 4);
  static constexpr int WS = TS + al(C * LDF * 4);
  static constexpr int A_END = WS + al(3 * 256 * 4);
  // pool B: after the third batch
  static constexpr int EA = POOL;                               // C x VB   [i][v]  E
  static constexpr int DEB = EA + al(C * VB * 2);               // VB x C   dE^T
  static constexpr int DYA = DEB + al(VB * C * 2);              // C x VB   dY
  static constexpr int DYB = DYA + al(C * VB * 2);              // VB x C   -dY^T
  static constexpr int KWT = DYB + al(VB * C * 2);              // KD x C   kw^T
  static constexpr int KRT = KWT + al(KD * C * 2);              // KD x C   kr^T
  static constexpr int QRT = KRT + al(KD * C * 2);              // KD x RC  qr^T
  static constexpr int SBT = QRT + al(KD * RC * 2);             // KD x VB  Sp
  static constexpr int DSBT = SBT + al(KD * VB * 2);            // KD x VB  dSc
  static constexpr int DKKA = DSBT + al(KD * VB * 2);           // C x C    dKK
  static constexpr int DKKT = DKKA + al(C * C * 2);             // C x C    dKK^T
  static constexpr int DQKA = DKKT + al(C * C * 2);             // RC x C   dQK
  static constexpr int DQKT = DQKA + al(RC * C * 2);            // C x RC   dQK^T
  static constexpr int DKKWT = DQKT + al(C * RC * 2);           // C x C    ((j - i) dKK)^T
  static constexpr int DQKWT = DKKWT + al(C * C * 2);           // C x RC   ((j - i) dQK)^T
  static constexpr int B_END = DQKWT + al(C * RC * 2);
  // fp32 staging of the key-side gradients (after the sixth batch, aliases pool B)
  static constexpr int GKR = POOL;                              // C x KD
  static constexpr int GKW = GKR + C * KD * 4;                  // C x KD
  static constexpr int GKW3 = GKW + C * KD * 4;                 // C x KD  (w E dSc^T part)
  static constexpr int GQR = GKW3 + C * KD * 4;                 // RC x KD
  static constexpr int GKRS = GQR + RC * KD * 4;                // C x KD  (state part of dkr)
  static constexpr int GQRS = GKRS + C * KD * 4;                // RC x KD (state part of dqr)
  static constexpr int GLW = GQRS + RC * KD * 4;                // C x KD  (position-weighted dkw)
  static constexpr int G_END = GLW + C * KD * 4;
  static constexpr int SC = al(mx(mx(A_END, B_END), G_END));
  // scalars (floats): beta, Gc, a, w, dbeta, da, dw, rows, cols [C each]; d1, dCm1, lam, wr,
  // wi, dlam, dwr, dwi [KD each]; misc[8]
  static constexpr int SC_FLOATS = 9 * C + 8 * KD + 8;
  static constexpr int MBAR = SC + al(SC_FLOATS * 4);
  static constexpr int TOTAL = MBAR + 64;
};

// TMEM columns (see the lifetime plan in the kernel body)
struct BCols {
  static constexpr int G = 0, PT = 64, UT = 192, WK = 256;                       // batches 1-2
  static constexpr int XT = 64, R0T = 128, DE1 = 192, DE2 = 256, DS0 = 320, OS = 384;  // batch 3
  static constexpr int DYT = 64;                                                  // batch 4
  static constexpr int DL = 128, DP = 192;                                        // batch 5
  static constexpr int DKR1 = 0, DKR2 = 64, DQR1 = 128, DQR2 = 192, DKW12 = 256, DKW3 = 384,
                       DLW = 448;                                                 // batch 6
  static constexpr int ALLOC = 512;
};


// ---- code operands of the backward ---------------------------------------------------------
//   KR[i][m] = kr, KW[i][m] = kw, QR[(r,i)][m] = qr, KWW[i][m] = w kw   (16-byte stores)
//   Z[m][i] = beta a kr / kappa, QRAT[m][(r,i)] = a qr / kappa           (element stores)
template <int FL, int KD, int R>
__device__ void build_codes_bwd(const sca2_scan_args& p, bf16* KR, bf16* KW, bf16* QR, bf16* Z, bf16* KWW,
                                bf16* QRAT, const Gates& g, const float* s_lam, const float* s_wr,
                                const float* s_wi, int flags, int b, int h, int t0, int Cl, float ik) {
  constexpr int RC = R * C;
  const int tid = threadIdx.x;
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2, MB = Mh / 8, NU = C * MB / NT;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int unit = tid + u * NT, i = unit / MB, m0 = (unit % MB) * 8;
      const bool live = i < Cl;
      float rw[8], rq[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        rw[k] = live ? phw[tok_off(p.phw, b, t0 + i, h) + m0 + k] : 0.f;
        rq[k] = live ? phq[tok_off(p.phq, b, t0 + i, h) + m0 + k] : 0.f;
      }
      const float fi = (float)i, zb = g.beta[i] * g.a[i] * ik, fa = g.a[i] * ik, wv = g.w[i];
      float kc[8], ks[8], wc[8], ws[8], q0a[8], q0b[8], q1a[8], q1b[8], wwc[8], wws[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int m = m0 + k;
        float c = 0.f, s = 0.f, cq = 0.f, sq = 0.f;
        if (live) {
          sincosf(rw[k], &s, &c);
          sincosf(rq[k], &sq, &cq);
        }
        const float l = s_lam[m];
        const float ell = __expf(-l * fi), elli = __expf(l * fi);
        const float c1 = s_wr[m] * cq + s_wi[m] * sq, c2 = s_wr[m] * sq - s_wi[m] * cq;
        kc[k] = c * ell; ks[k] = s * ell; wc[k] = c * elli; ws[k] = s * elli;
        wwc[k] = wc[k] * wv; wws[k] = ws[k] * wv;
        q0a[k] = c1 * ell; q0b[k] = c2 * ell; q1a[k] = -c2 * ell; q1b[k] = c1 * ell;
      }
      st8(KR, umma::kmaj(i, m0, KD), kc);
      st8(KR, umma::kmaj(i, Mh + m0, KD), ks);
      st8(KW, umma::kmaj(i, m0, KD), wc);
      st8(KW, umma::kmaj(i, Mh + m0, KD), ws);
      st8(KWW, umma::kmaj(i, m0, KD), wwc);
      st8(KWW, umma::kmaj(i, Mh + m0, KD), wws);
      st8(QR, umma::kmaj(i, m0, KD), q0a);
      st8(QR, umma::kmaj(i, Mh + m0, KD), q0b);
      st8(QR, umma::kmaj(C + i, m0, KD), q1a);
      st8(QR, umma::kmaj(C + i, Mh + m0, KD), q1b);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        st1(Z, umma::kmaj(m0 + k, i, C), kc[k] * zb);
        st1(Z, umma::kmaj(Mh + m0 + k, i, C), ks[k] * zb);
        st1(QRAT, umma::kmaj(m0 + k, i, RC), q0a[k] * fa);
        st1(QRAT, umma::kmaj(Mh + m0 + k, i, RC), q0b[k] * fa);
        st1(QRAT, umma::kmaj(m0 + k, C + i, RC), q1a[k] * fa);
        st1(QRAT, umma::kmaj(Mh + m0 + k, C + i, RC), q1b[k] * fa);
      }
    }
  } else {
    constexpr int MB = KD / 8, NU = C * MB / NT;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int unit = tid + u * NT, i = unit / MB, m0 = (unit % MB) * 8;
      const bool live = i < Cl;
      const int64_t ok_ = tok_off(p.phw, b, t0 + i, h) + m0, oq = tok_off(p.phq, b, t0 + i, h) + m0;
      const float fi = (float)i, zb = g.beta[i] * g.a[i] * ik, fa = g.a[i] * ik, wv = g.w[i];
      float kc[8], wc[8], qc[8], ww[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float kk = live ? ld_io(p.phw.ptr, ok_ + k, p.io_dtype) : 0.f;
        const float qq = live ? p.q_scale * ld_io(p.phq.ptr, oq + k, p.io_dtype) : 0.f;
        const float l = s_lam[m0 + k];
        const float ell = __expf(-l * fi), elli = __expf(l * fi);
        kc[k] = kk * ell; wc[k] = kk * elli; qc[k] = qq * ell; ww[k] = wc[k] * wv;
      }
      st8(KR, umma::kmaj(i, m0, KD), kc);
      st8(KW, umma::kmaj(i, m0, KD), wc);
      st8(KWW, umma::kmaj(i, m0, KD), ww);
      st8(QR, umma::kmaj(i, m0, KD), qc);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        st1(Z, umma::kmaj(m0 + k, i, C), kc[k] * zb);
        st1(QRAT, umma::kmaj(m0 + k, i, RC), qc[k] * fa);
      }
    }
  }
}

// ---- transposed code operands: KWT[m][i] = kw, KRT[m][i] = kr, QRT[m][(r,i)] = qr ----------
// Units of (one mode, 8 consecutive tokens) so every row is written with 16-byte stores.
template <int FL, int KD, int R>
__device__ void build_codes_T(const sca2_scan_args& p, bf16* KWT, bf16* KRT, bf16* QRT, const float* s_lam,
                              const float* s_wr, const float* s_wi, int flags, int b, int h, int t0, int Cl) {
  constexpr int RC = R * C;
  const int tid = threadIdx.x;
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2, NU = Mh * (C / 8) / NT;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
#pragma unroll
    for (int u = 0; u < (NU > 0 ? NU : 1); ++u) {
      const int unit = tid + u * NT;
      if (unit >= Mh * (C / 8)) break;
      const int m = unit % Mh, i0 = (unit / Mh) * 8;
      const float l = s_lam[m], wr = s_wr[m], wi = s_wi[m];
      float kc[8], ks[8], wc[8], ws[8], q0a[8], q0b[8], q1a[8], q1b[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k;
        float c = 0.f, s = 0.f, cq = 0.f, sq = 0.f;
        if (i < Cl) {
          sincosf(phw[tok_off(p.phw, b, t0 + i, h) + m], &s, &c);
          sincosf(phq[tok_off(p.phq, b, t0 + i, h) + m], &sq, &cq);
        }
        const float ell = __expf(-l * (float)i), elli = __expf(l * (float)i);
        const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
        kc[k] = c * ell; ks[k] = s * ell; wc[k] = c * elli; ws[k] = s * elli;
        q0a[k] = c1 * ell; q0b[k] = c2 * ell; q1a[k] = -c2 * ell; q1b[k] = c1 * ell;
      }
      st8(KRT, umma::kmaj(m, i0, C), kc);
      st8(KRT, umma::kmaj(Mh + m, i0, C), ks);
      st8(KWT, umma::kmaj(m, i0, C), wc);
      st8(KWT, umma::kmaj(Mh + m, i0, C), ws);
      st8(QRT, umma::kmaj(m, i0, RC), q0a);
      st8(QRT, umma::kmaj(Mh + m, i0, RC), q0b);
      st8(QRT, umma::kmaj(m, C + i0, RC), q1a);
      st8(QRT, umma::kmaj(Mh + m, C + i0, RC), q1b);
    }
  } else {
    constexpr int NU = KD * (C / 8) / NT;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int unit = tid + u * NT, m = unit % KD, i0 = (unit / KD) * 8;
      const float l = s_lam[m];
      float kc[8], wc[8], qc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k;
        const float kk = i < Cl ? ld_io(p.phw.ptr, tok_off(p.phw, b, t0 + i, h) + m, p.io_dtype) : 0.f;
        const float qq = i < Cl ? p.q_scale * ld_io(p.phq.ptr, tok_off(p.phq, b, t0 + i, h) + m, p.io_dtype) : 0.f;
        const float ell = __expf(-l * (float)i), elli = __expf(l * (float)i);
        kc[k] = kk * ell; wc[k] = kk * elli; qc[k] = qq * ell;
      }
      st8(KRT, umma::kmaj(m, i0, C), kc);
      st8(KWT, umma::kmaj(m, i0, C), wc);
      st8(QRT, umma::kmaj(m, i0, RC), qc);
    }
  }
}

// ---- chain rule from the code-space gradients to the inputs, per (token, mode) --------------
template <int FL, int KD, int R>
__device__ void finish_key_grads(const sca2_scan_args& p, const sca2_scan_grads& gr, const float* GKR,
                                 const float* GKW, const float* GKW3, const float* GQR, const float* GKRS,
                                 const float* GQRS, const float* GLW, const Gates& g,
                                 const float* s_lam, const float* s_wr, const float* s_wi, float* s_dlam,
                                 float* s_dwr, float* s_dwi, int b, int h, int t0, int Cl) {
  const int tid = threadIdx.x;
  const float fCl1 = (float)(Cl - 1);
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
    float* dphw = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
    float* dphq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
    for (int idx = tid; idx < C * Mh; idx += NT) {
      const int i = idx / Mh, m = idx % Mh;
      if (i >= Cl) continue;
      float s, c, sq, cq;
      sincosf(phw[tok_off(p.phw, b, t0 + i, h) + m], &s, &c);
      sincosf(phq[tok_off(p.phq, b, t0 + i, h) + m], &sq, &cq);
      const float l = s_lam[m], fi = (float)i;
      const float ell = __expf(-l * fi), elli = __expf(l * fi);
      const float wr = s_wr[m], wi = s_wi[m];
      const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
      const float krc = c * ell, krs = s * ell, kwc = c * elli, kws = s * elli;
      const float q00 = c1 * ell, q01 = c2 * ell, q10 = -c2 * ell, q11 = c1 * ell;
      const float dkrc = GKR[i * KD + m], dkrs = GKR[i * KD + m + Mh];
      const float dkwc = GKW[i * KD + m], dkws = GKW[i * KD + m + Mh];
      const float d3c = GKW3[i * KD + m], d3s = GKW3[i * KD + m + Mh];
      const float dq00 = GQR[i * KD + m], dq01 = GQR[i * KD + m + Mh];
      const float dq10 = GQR[(C + i) * KD + m], dq11 = GQR[(C + i) * KD + m + Mh];
      const float dkc = dkrc * ell + dkwc * elli, dks = dkrs * ell + dkws * elli;
      const float dc1 = (dq00 + dq11) * ell, dc2 = (dq01 - dq10) * ell;
      atomicAdd(&dphw[tok_off(gr.dphw, b, t0 + i, h) + m], -s * dkc + c * dks);
      atomicAdd(&dphq[tok_off(gr.dphq, b, t0 + i, h) + m],
                -sq * (dc1 * wr - dc2 * wi) + cq * (dc1 * wi + dc2 * wr));
      atomicAdd(&s_dwr[m], dc1 * cq + dc2 * sq);
      atomicAdd(&s_dwi[m], dc1 * sq - dc2 * cq);
      if (p.lam) {
        // intra-chunk pairs enter through the position-weighted product GLW (no cancellation
        // between the i-weighted read side and the j-weighted write side); the state-side
        // parts keep their own position weights
        const float sr0 = GKRS[i * KD + m], sr1 = GKRS[i * KD + m + Mh];
        const float sq00 = GQRS[i * KD + m], sq01 = GQRS[i * KD + m + Mh];
        const float sq10 = GQRS[(C + i) * KD + m], sq11 = GQRS[(C + i) * KD + m + Mh];
        const float dl = kwc * GLW[i * KD + m] + kws * GLW[i * KD + m + Mh] -
                         fi * (sr0 * krc + sr1 * krs + sq00 * q00 + sq01 * q01 + sq10 * q10 + sq11 * q11) +
                         (fi - fCl1) * (kwc * d3c + kws * d3s);
        atomicAdd(&s_dlam[m], dl);
      }
    }
  } else {
    float* dk = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
    float* dq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
    for (int idx = tid; idx < C * KD; idx += NT) {
      const int i = idx / KD, m = idx % KD;
      if (i >= Cl) continue;
      const float kk = ld_io(p.phw.ptr, tok_off(p.phw, b, t0 + i, h) + m, p.io_dtype);
      const float qq = p.q_scale * ld_io(p.phq.ptr, tok_off(p.phq, b, t0 + i, h) + m, p.io_dtype);
      const float l = s_lam[m], fi = (float)i;
      const float ell = __expf(-l * fi), elli = __expf(l * fi);
      const float dkr = GKR[i * KD + m], dkw = GKW[i * KD + m], dqr = GQR[i * KD + m];
      atomicAdd(&dk[tok_off(gr.dphw, b, t0 + i, h) + m], dkr * ell + dkw * elli);
      atomicAdd(&dq[tok_off(gr.dphq, b, t0 + i, h) + m], p.q_scale * dqr * ell);
      if (p.lam) {
        const float dl = kk * elli * GLW[i * KD + m] -
                         fi * ell * (GKRS[i * KD + m] * kk + GQRS[i * KD + m] * qq) +
                         (fi - fCl1) * kk * elli * GKW3[i * KD + m];
        atomicAdd(&s_dlam[m], dl);
      }
    }
  }
}

// sum over the 16 row-owning lanes of an M = 64 fragment (lanes 0..15); result in lane 0
__device__ __forceinline__ float sum16(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int FL, int KD, int VB, int R>
__global__ void __launch_bounds__(NT, 1) scan_bwd_tc(sca2_scan_args p, sca2_out dO, const float* dS_final,
                                                    const float* cstates, sca2_scan_grads gr, int NCS,
                                                    int flags) {
  using L = BwdLayout<KD, VB, R>;
  using CO = BCols;
  constexpr int RC = R * C;
  constexpr int Mh = KD / 2;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, sub = warp & 3;
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int vb0 = blockIdx.y * VB;
  const int V = p.V;
  const bool has_g = p.g.ptr != nullptr;
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)Mh : 1.f;
  const float ik = 1.f / kappa;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  Gates gates{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* s_dbeta = sc + 4 * C;
  float* s_da = sc + 5 * C;
  float* s_dw = sc + 6 * C;
  float* s_rows = sc + 7 * C;
  float* s_cols = sc + 8 * C;
  float* s_d1 = sc + 9 * C;
  float* s_dCm1 = s_d1 + KD;
  float* s_lam = s_dCm1 + KD;
  float* s_wr = s_lam + KD;
  float* s_wi = s_wr + KD;
  float* s_dlam = s_wi + KD;
  float* s_dwr = s_dlam + KD;
  float* s_dwi = s_dwr + KD;
  float* s_misc = s_dwi + KD;
  auto BF = [&](int off) { return reinterpret_cast<bf16*>(sm + off); };
  float* LS = reinterpret_cast<float*>(sm + L::LS);
  float* TS = reinterpret_cast<float*>(sm + L::TS);
  float* WS = reinterpret_cast<float*>(sm + L::WS);
  float* GKR = reinterpret_cast<float*>(sm + L::GKR);
  float* GKW = reinterpret_cast<float*>(sm + L::GKW);
  float* GKW3 = reinterpret_cast<float*>(sm + L::GKW3);
  float* GQR = reinterpret_cast<float*>(sm + L::GQR);
  float* GKRS = reinterpret_cast<float*>(sm + L::GKRS);
  float* GQRS = reinterpret_cast<float*>(sm + L::GQRS);
  float* GLW = reinterpret_cast<float*>(sm + L::GLW);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  volatile int* s_err = reinterpret_cast<volatile int*>(sm + L::MBAR + 12);

  // ---- set-up
  constexpr int KH = FL == SCA2_FLAVOR_PHASE ? Mh : KD;
  for (int m = tid; m < KD; m += NT) {
    const float l = p.lam ? p.lam[h * KH + (m % KH)] : 0.f;
    s_lam[m] = l;
    s_d1[m] = expf(-l);
    s_wr[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wr[h * KH + m] : 0.f;
    s_wi[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wi[h * KH + m] : 0.f;
    s_dlam[m] = 0.f;
    s_dwr[m] = 0.f;
    s_dwi[m] = 0.f;
  }
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
    *s_err = 0;
  }
  if (tid < 32) umma::tmem_alloc(s_tmem, CO::ALLOC);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  uint32_t phase = 0;

  // state-layout registers (rows v of an M = VB fragment, columns m): adjoint dS and Sp
  constexpr int NS = KD / 2;
  float dSreg[NS], Spreg[NS];
  const int srow = frag_row<VB>();
  const bool sown = owns_rows<VB>();
  const int64_t bhKV = ((int64_t)b * p.H + h) * KD * (int64_t)V;
#pragma unroll
  for (int q = 0; q < KD / 32; ++q)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int m = frag_col0<VB, KD>(q) + j;
      dSreg[16 * q + j] = (sown && dS_final) ? dS_final[bhKV + (int64_t)m * V + vb0 + srow] : 0.f;
    }
  float Ureg[C / 2], R0reg[C / 2];

  auto wait_mma = [&]() -> bool {
    if (!umma::mbar_wait(mbar, phase)) *s_err = 1;
    phase ^= 1u;
    __syncthreads();
    umma::fence_after_sync();
    return *s_err == 0;
  };
  auto Dg = [&](int i, int j) -> float { return has_g ? __expf(fminf(gates.Gc[i] - gates.Gc[j], 0.f)) : 1.f; };

  const int NC = (p.T + C - 1) / C;
  bool ok = true;
  for (int c = NC - 1; c >= 0 && ok; --c) {
    const int t0 = c * C, Cl = min(C, p.T - t0);
    const int64_t cb = (((int64_t)b * p.H + h) * NCS + 2 * c) * KD * (int64_t)V;
    // ================= prologue =================
    ValueLoad<VB> vl;
    load_values<VB>(p, vl, b, h, t0, Cl, vb0);
    load_gates(p, gates, b, h, t0, Cl);
    for (int m = tid; m < KD; m += NT) s_dCm1[m] = expf(-s_lam[m] * (float)(Cl - 1));
    if (tid < C) {
      s_dbeta[tid] = 0.f;
      s_da[tid] = 0.f;
      s_dw[tid] = 0.f;
      s_rows[tid] = 0.f;
      s_cols[tid] = 0.f;
    }
    if (tid == 0) s_misc[0] = 0.f;
    // Sp = d1 .* S (state entering the chunk) in the state layout
#pragma unroll
    for (int q = 0; q < KD / 32; ++q)
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = frag_col0<VB, KD>(q) + j;
        Spreg[16 * q + j] = sown ? cstates[cb + (int64_t)m * V + vb0 + srow] * s_d1[m] : 0.f;
      }
    // dO: [(r,i)][v] (16-byte loads from global when aligned) and dO^T [v][(r,i)]
    for (int u = tid; u < RC * (VB / 8); u += NT) {
      const int row = u / (VB / 8), v0 = (u % (VB / 8)) * 8, r = row / C, i = row % C;
      float x[8];
      if (i < Cl) {
        const int64_t off = out_off(dO, b, t0 + i, h, r) + vb0 + v0;
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = ld_io(dO.ptr, off + k, p.io_dtype);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = 0.f;
      }
      st8(BF(L::DOA), umma::kmaj(row, v0, VB), x);
#pragma unroll
      for (int k = 0; k < 8; ++k) st1(BF(L::DOT), umma::kmaj(v0 + k, row, RC), x[k]);
    }
    __syncthreads();  // gates, dCm1 ready
    build_codes_bwd<FL, KD, R>(p, BF(L::KR), BF(L::KW), BF(L::QR), BF(L::Z), BF(L::KWW), BF(L::QRAT), gates,
                               s_lam, s_wr, s_wi, flags, b, h, t0, Cl, ik);
    store_values<VB>(p, vl, gates.beta, BF(L::VT));
    // Sp^T and dSc^T (bf16, rows v)
    if (sown) {
#pragma unroll
      for (int q = 0; q < KD / 32; ++q) {
        float xs[16], xd[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = frag_col0<VB, KD>(q) + j;
          xs[j] = Spreg[16 * q + j];
          xd[j] = s_dCm1[m] * dSreg[16 * q + j];
        }
        const int m0 = frag_col0<VB, KD>(q);
        st8(BF(L::SB), umma::kmaj(srow, m0, KD), xs);
        st8(BF(L::SB), umma::kmaj(srow, m0 + 8, KD), xs + 8);
        st8(BF(L::DSB), umma::kmaj(srow, m0, KD), xd);
        st8(BF(L::DSB), umma::kmaj(srow, m0 + 8, KD), xd + 8);
      }
    }
    publish_smem();
    // ================= batch 1: G, P^T =================
    if (tid == 0) {
      umma::gemm(tb + CO::G, sm + L::KR, sm + L::KW, 64, 64, KD, false);
      umma::gemm(tb + CO::PT, sm + L::KW, sm + L::QR, 64, RC, KD, false);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    for_frag<64, 64>(tb + CO::G, [&](int i, int j0, int, const float* x) {
      const float bi = gates.beta[i] * ik;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * Dg(i, jj) : 0.f;
      }
    });
    for_frag<64, RC>(tb + CO::PT, [&](int jr, int c0, int, const float* x) {
      float y[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int i = (c0 + k) % C;
        y[k] = jr <= i ? x[k] * ik * Dg(i, jr) : 0.f;
      }
      st8(BF(L::PT), umma::kmaj(jr, c0, RC), y);
      st8(BF(L::PT), umma::kmaj(jr, c0 + 8, RC), y + 8);
    });
    __syncthreads();
    invert_unit_lower(LS, TS, WS);
    store_T<false>(TS, BF(L::TB));
    store_T<true>(TS, BF(L::TBT));
    publish_smem();
    // ================= batch 2: U^T, Wk =================
    if (tid == 0) {
      umma::gemm(tb + CO::UT, sm + L::VT, sm + L::TB, VB, C, C, false);
      umma::gemm(tb + CO::WK, sm + L::TB, sm + L::Z, 64, KD, C, false);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    for_frag<VB, C>(tb + CO::UT, [&](int, int, int q, const float* x) {
#pragma unroll
      for (int j = 0; j < 16; ++j) Ureg[16 * q + j] = x[j];
    });
    for_frag<64, KD>(tb + CO::WK, [&](int i, int m0, int, const float* x) {
      st8(BF(L::WK), umma::kmaj(i, m0, KD), x);
      st8(BF(L::WK), umma::kmaj(i, m0 + 8, KD), x + 8);
    });
    publish_smem();
    // ================= batch 3: X^T, R0^T, dE^T (two parts), dS0p^T (part 1), Os =================
    if (tid == 0) {
      umma::gemm(tb + CO::XT, sm + L::SB, sm + L::WK, VB, C, KD, false);
      umma::gemm(tb + CO::R0T, sm + L::SB, sm + L::KR, VB, C, KD, false);
      umma::gemm(tb + CO::DE1, sm + L::DSB, sm + L::KWW, VB, C, KD, false);
      umma::gemm(tb + CO::DE2, sm + L::DOT, sm + L::PT, VB, C, RC, false);
      umma::gemm(tb + CO::DS0, sm + L::DOT, sm + L::QRAT, VB, KD, RC, false);
      umma::gemm(tb + CO::OS, sm + L::QR, sm + L::SB, RC, VB, KD, false);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    // ---- pool A is free from here on
    // E = U - X (rows v) -> EA [i][v]; R0 -> regs; dE^T -> DEB; dw_j = sum_v E dE1
    {
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int i0 = frag_col0<VB, C>(q);
        float xx[16], r0[16], d1v[16], d2v[16];
        umma::ld16(umma::taddr(tb + CO::XT, 32 * sub, i0), xx);
        umma::ld16(umma::taddr(tb + CO::R0T, 32 * sub, i0), r0);
        umma::ld16(umma::taddr(tb + CO::DE1, 32 * sub, i0), d1v);
        umma::ld16(umma::taddr(tb + CO::DE2, 32 * sub, i0), d2v);
        float e[16], de[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int i = i0 + j;
          e[j] = Ureg[16 * q + j] - xx[j];
          R0reg[16 * q + j] = r0[j] * gates.a[i] * ik;
          de[j] = d1v[j] + d2v[j];
        }
        if (sown) {
#pragma unroll
          for (int j = 0; j < 16; ++j) st1(BF(L::EA), umma::kmaj(i0 + j, srow, VB), e[j]);
          st8(BF(L::DEB), umma::kmaj(srow, i0, C), de);
          st8(BF(L::DEB), umma::kmaj(srow, i0 + 8, C), de + 8);
        }
        if (has_g) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float t = sum16(sown ? e[j] * d1v[j] : 0.f);
            if (lane == 0) atomicAdd(&s_dw[i0 + j], t);
          }
        }
      }
      // da (first term): sum_r sum_v dO * Os * a / kappa over rows (r, i)
      if (has_g) {
        const int row = frag_row<RC>(), i = row % C;
#pragma unroll
        for (int q = 0; q < VB / 32; ++q) {
          const int v0 = frag_col0<RC, VB>(q);
          float os[16];
          umma::ld16(umma::taddr(tb + CO::OS, 32 * sub, v0), os);
          if (owns_rows<RC>()) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              s += os[j] * __bfloat162float(BF(L::DOA)[umma::kmaj(row, v0 + j, VB)]);
            atomicAdd(&s_da[i], s * gates.a[i] * ik);
          }
        }
      }
    }
    // late operands for batch 6 (pool B): kw^T, kr^T, qr^T, Sp, dSc
    build_codes_T<FL, KD, R>(p, BF(L::KWT), BF(L::KRT), BF(L::QRT), s_lam, s_wr, s_wi, flags, b, h, t0, Cl);
    if (sown) {
#pragma unroll
      for (int q = 0; q < KD / 32; ++q)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = frag_col0<VB, KD>(q) + j;
          st1(BF(L::SBT), umma::kmaj(m, srow, VB), Spreg[16 * q + j]);
          st1(BF(L::DSBT), umma::kmaj(m, srow, VB), s_dCm1[m] * dSreg[16 * q + j]);
        }
    }
    publish_smem();
    // ================= batch 4: dY^T = dE^T T =================
    if (tid == 0) {
      umma::gemm(tb + CO::DYT, sm + L::DEB, sm + L::TBT, VB, C, C, false);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    {
      const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int i0 = frag_col0<VB, C>(q);
        float dy[16];
        umma::ld16(umma::taddr(tb + CO::DYT, 32 * sub, i0), dy);
        float ndy[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int i = i0 + j;
          ndy[j] = -dy[j];
          float s = sown ? dy[j] * R0reg[16 * q + j] : 0.f;
          float sv = 0.f;
          if (sown && i < Cl && vb0 + srow < V) {
            const int64_t off = tok_off(p.v, b, t0 + i, h) + vb0 + srow;
            float dv = dy[j];
            if (p.v_times_beta) {
              sv = dy[j] * ld_io(p.v.ptr, off, p.io_dtype);
              dv *= bp[tok_off(p.beta, b, t0 + i, h)];
            }
            st_io(const_cast<void*>(gr.dv.ptr), tok_off(gr.dv, b, t0 + i, h) + vb0 + srow, dv, p.io_dtype);
          }
          s = sum16(s);
          if (p.v_times_beta) sv = sum16(sv);
          if (lane == 0) {
            atomicAdd(&s_dbeta[i], sv - s);
            atomicAdd(&s_da[i], -gates.beta[i] * s);
          }
          if (sown) st1(BF(L::DYA), umma::kmaj(i, srow, VB), dy[j]);
        }
        if (sown) {
          st8(BF(L::DYB), umma::kmaj(srow, i0, C), ndy);
          st8(BF(L::DYB), umma::kmaj(srow, i0 + 8, C), ndy + 8);
        }
      }
    }
    publish_smem();
    // ================= batch 5: dL, dP, dS0p^T (part 2) =================
    if (tid == 0) {
      umma::gemm(tb + CO::DL, sm + L::DYA, sm + L::EA, 64, C, VB, false);
      umma::gemm(tb + CO::DP, sm + L::DOA, sm + L::EA, RC, C, VB, false);
      umma::gemm(tb + CO::DS0, sm + L::DYB, sm + L::Z, VB, KD, C, true);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    // dL with Gr -> dKK, dbeta, decay sums
    {
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int j0 = frag_col0<64, C>(q);
        float dl[16], gg[16];
        umma::ld16(umma::taddr(tb + CO::DL, 32 * sub, j0), dl);
        umma::ld16(umma::taddr(tb + CO::G, 32 * sub, j0), gg);
        const int i = frag_row<64>();
        const bool own = owns_rows<64>();
        float dkk[16];
        float sb = 0.f, srow_ = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          float val = 0.f, gcol = 0.f;
          if (own && jj < i) {
            const float d = Dg(i, jj);
            const float l = -dl[j];
            const float grv = gg[j] * ik * d;
            sb += l * grv;
            gcol = gates.beta[i] * l * grv;
            srow_ += gcol;
            val = gates.beta[i] * l * d;
          }
          dkk[j] = val;
          if (has_g) {
            const float t = sum16(gcol);
            if (lane == 0) atomicAdd(&s_cols[jj], t);
          }
        }
        if (own) {
          atomicAdd(&s_dbeta[i], sb);
          if (has_g) atomicAdd(&s_rows[i], srow_);
          st8(BF(L::DKKA), umma::kmaj(i, j0, C), dkk);
          st8(BF(L::DKKA), umma::kmaj(i, j0 + 8, C), dkk + 8);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            st1(BF(L::DKKT), umma::kmaj(j0 + j, i, C), dkk[j]);
            st1(BF(L::DKKWT), umma::kmaj(j0 + j, i, C), dkk[j] * (float)(j0 + j - i));
          }
        }
      }
      // dP -> dQK and decay sums
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int j0 = frag_col0<RC, C>(q);
        float dp[16];
        umma::ld16(umma::taddr(tb + CO::DP, 32 * sub, j0), dp);
        const int row = frag_row<RC>(), i = row % C;
        const bool own = owns_rows<RC>();
        float dqk[16];
        float srow_ = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          float val = 0.f, gcol = 0.f;
          if (own && jj <= i) {
            val = dp[j] * Dg(i, jj);
            if (has_g) {
              gcol = dp[j] * __bfloat162float(BF(L::PT)[umma::kmaj(jj, row, RC)]);
              srow_ += gcol;
            }
          }
          dqk[j] = val;
          if (has_g) {
            float t = gcol;
            if (RC == 128) {
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            } else {
              t = sum16(t);
            }
            if (lane == 0) atomicAdd(&s_cols[jj], t);
          }
        }
        if (own) {
          if (has_g) atomicAdd(&s_rows[i], srow_);
          st8(BF(L::DQKA), umma::kmaj(row, j0, C), dqk);
          st8(BF(L::DQKA), umma::kmaj(row, j0 + 8, C), dqk + 8);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            st1(BF(L::DQKT), umma::kmaj(j0 + j, row, RC), dqk[j]);
            st1(BF(L::DQKWT), umma::kmaj(j0 + j, row, RC), dqk[j] * (float)(j0 + j - i));
          }
        }
      }
      // dS0p^T -> adjoint update, state-side decay gradients
      const float aC = gates.a[Cl - 1];
      float daC = 0.f;
#pragma unroll
      for (int q = 0; q < KD / 32; ++q) {
        const int m0 = frag_col0<VB, KD>(q);
        float d0[16];
        umma::ld16(umma::taddr(tb + CO::DS0, 32 * sub, m0), d0);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + j;
          float dl = 0.f;
          if (sown) {
            const float sp = Spreg[16 * q + j], ds = dSreg[16 * q + j];
            const float t = aC * s_dCm1[m] * sp * ds;
            daC += t;
            dl = -d0[j] * sp - (float)Cl * t;
            dSreg[16 * q + j] = aC * s_dCm1[m] * s_d1[m] * ds + s_d1[m] * d0[j];
          }
          if (p.lam) {
            const float t = sum16(dl);
            if (lane == 0) atomicAdd(&s_dlam[m], t);
          }
        }
      }
      if (has_g) {
        daC = warp_sum(sown ? daC : 0.f);
        if (lane == 0) atomicAdd(&s_misc[0], daC);
      }
    }
    publish_smem();
    // ================= batch 6: dkr, dqr, dkw =================
    if (tid == 0) {
      umma::gemm(tb + CO::DKR1, sm + L::DKKA, sm + L::KWT, 64, KD, C, false);
      umma::gemm(tb + CO::DKR2, sm + L::DYA, sm + L::SBT, 64, KD, VB, false);
      umma::gemm(tb + CO::DQR1, sm + L::DQKA, sm + L::KWT, RC, KD, C, false);
      umma::gemm(tb + CO::DQR2, sm + L::DOA, sm + L::SBT, RC, KD, VB, false);
      umma::gemm(tb + CO::DKW12, sm + L::DKKT, sm + L::KRT, 64, KD, C, false);
      umma::gemm(tb + CO::DKW12, sm + L::DQKT, sm + L::QRT, 64, KD, RC, true);
      umma::gemm(tb + CO::DKW3, sm + L::EA, sm + L::DSBT, 64, KD, VB, false);
      if (p.lam) {
        umma::gemm(tb + CO::DLW, sm + L::DKKWT, sm + L::KRT, 64, KD, C, false);
        umma::gemm(tb + CO::DLW, sm + L::DQKWT, sm + L::QRT, 64, KD, RC, true);
      }
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    // ---- stage fp32 key-side gradients (pool B is free); tcgen05.ld is warp-collective, so
    // every lane loads and only row owners store
    {
      const int i = frag_row<64>();
      const bool own = owns_rows<64>();
#pragma unroll
      for (int q = 0; q < KD / 32; ++q) {
        const int m0 = frag_col0<64, KD>(q);
        float x[16], y[16];
        umma::ld16(umma::taddr(tb + CO::DKR1, 32 * sub, m0), x);
        umma::ld16(umma::taddr(tb + CO::DKR2, 32 * sub, m0), y);
        if (own) {
          const float f = gates.beta[i] * gates.a[i] * ik;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            GKR[i * KD + m0 + j] = x[j] * ik - f * y[j];
            GKRS[i * KD + m0 + j] = -f * y[j];
          }
        }
        umma::ld16(umma::taddr(tb + CO::DKW12, 32 * sub, m0), x);
        umma::ld16(umma::taddr(tb + CO::DKW3, 32 * sub, m0), y);
        if (own) {
          const float wv = gates.w[i];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            GKW3[i * KD + m0 + j] = wv * y[j];
            GKW[i * KD + m0 + j] = x[j] * ik + wv * y[j];
          }
        }
        if (p.lam) {
          umma::ld16(umma::taddr(tb + CO::DLW, 32 * sub, m0), x);
          if (own) {
#pragma unroll
            for (int j = 0; j < 16; ++j) GLW[i * KD + m0 + j] = x[j] * ik;
          }
        }
      }
      const int row = frag_row<RC>();
      const bool ownq = owns_rows<RC>();
#pragma unroll
      for (int q = 0; q < KD / 32; ++q) {
        const int m0 = frag_col0<RC, KD>(q);
        float x[16], y[16];
        umma::ld16(umma::taddr(tb + CO::DQR1, 32 * sub, m0), x);
        umma::ld16(umma::taddr(tb + CO::DQR2, 32 * sub, m0), y);
        if (ownq) {
          const float f = gates.a[row % C] * ik;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            GQR[row * KD + m0 + j] = x[j] * ik + f * y[j];
            GQRS[row * KD + m0 + j] = f * y[j];
          }
        }
      }
    }
    __syncthreads();
    // ---- per (token, mode): chain rule to the inputs, lambda / w gradients
    finish_key_grads<FL, KD, R>(p, gr, GKR, GKW, GKW3, GQR, GKRS, GQRS, GLW, gates, s_lam, s_wr, s_wi, s_dlam,
                                s_dwr, s_dwi, b, h, t0, Cl);
    // ---- per-token beta and decay gradients
    if (tid < 32) {
      float dGv[2], dwv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = tid + 32 * u;
        dwv[u] = i < Cl ? s_dw[i] : 0.f;
        dGv[u] = i < Cl ? s_rows[i] - s_cols[i] + s_da[i] - s_dw[i] : 0.f;
      }
      const float dwsum = warp_sum(dwv[0] + dwv[1]);
      if (has_g) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (tid + 32 * u == Cl - 1) dGv[u] += dwsum + s_misc[0];
        // reverse inclusive cumsum over the 64 tokens: dg_i = sum_{u >= i} dG_u
        const float tot1 = warp_sum(dGv[1]);
        const float inc1 = warp_incl_scan(dGv[1]);
        const float tot0 = warp_sum(dGv[0]);
        const float inc0 = warp_incl_scan(dGv[0]);
        const float g1 = tot1 - inc1 + dGv[1];
        const float g0 = tot0 - inc0 + dGv[0] + tot1;
        float* gp = reinterpret_cast<float*>(const_cast<void*>(gr.dg.ptr));
        if (tid < Cl) atomicAdd(&gp[tok_off(gr.dg, b, t0 + tid, h)], g0);
        if (tid + 32 < Cl) atomicAdd(&gp[tok_off(gr.dg, b, t0 + tid + 32, h)], g1);
      }
      if (p.beta.ptr && gr.dbeta.ptr) {
        float* bpp = reinterpret_cast<float*>(const_cast<void*>(gr.dbeta.ptr));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = tid + 32 * u;
          if (i < Cl) atomicAdd(&bpp[tok_off(gr.dbeta, b, t0 + i, h)], s_dbeta[i]);
        }
      }
    }
    publish_smem();
  }
  // ---- incoming-state gradient and per-head gradients
  if (ok) {
    if (gr.dS0 && sown) {
#pragma unroll
      for (int q = 0; q < KD / 32; ++q)
#pragma unroll
        for (int j = 0; j < 16; ++j)
          gr.dS0[bhKV + (int64_t)(frag_col0<VB, KD>(q) + j) * V + vb0 + srow] = dSreg[16 * q + j];
    }
    for (int m = tid; m < KD; m += NT) {
      if (gr.dlam && p.lam) atomicAdd(&gr.dlam[h * KH + (m % KH)], s_dlam[m]);
      if (FL == SCA2_FLAVOR_PHASE && m < Mh) {
        if (gr.dwr) atomicAdd(&gr.dwr[h * Mh + m], s_dwr[m]);
        if (gr.dwi) atomicAdd(&gr.dwi[h * Mh + m], s_dwi[m]);
      }
    }
  } else {
    if (tid == 0) atomicOr(&g_fault, 1u);
    umma::mbar_wait(mbar, phase ^ 1u);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tb, CO::ALLOC);
}

template <int FL, int KD, int VB, int R>
cudaError_t launch_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final, const float* cstates,
                       const sca2_scan_grads& gr, int NCS, int flags, cudaStream_t st) {
  auto k = scan_bwd_tc<FL, KD, VB, R>;
  const int smem = BwdLayout<KD, VB, R>::TOTAL;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, p.V / VB);
  k<<<grid, NT, smem, st>>>(p, dO, dS_final, cstates, gr, NCS, flags);
  return cudaGetLastError();
}

}  // namespace tc

int tc_bwd_smem(int K, int VB, int R) {
  if (K == 64 && VB == 64 && R == 2) return tc::BwdLayout<64, 64, 2>::TOTAL;
  if (K == 64 && VB == 64 && R == 1) return tc::BwdLayout<64, 64, 1>::TOTAL;
  return 1 << 30;
}

// Whether a bf16 training pass (forward with saved chunk states + backward) runs on the tensor
// cores: K = 64, V a multiple of 64, both kernels within the shared-memory limit.
bool tc_train_ok(const sca2_scan_args& p, int max_smem) {
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  return p.io_dtype == SCA2_BF16 && p.K == 64 && p.V % 64 == 0 && tc_bwd_smem(64, 64, R) <= max_smem;
}

cudaError_t tc_scan_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final, const float* cstates,
                        const sca2_scan_grads& gr, int NCS, cudaStream_t st) {
  if (p.flavor == SCA2_FLAVOR_PHASE)
    return tc::launch_bwd<SCA2_FLAVOR_PHASE, 64, 64, 2>(p, dO, dS_final, cstates, gr, NCS, 0, st);
  return tc::launch_bwd<SCA2_FLAVOR_KEY, 64, 64, 1>(p, dO, dS_final, cstates, gr, NCS, 0, st);
}

}  // namespace sca2
