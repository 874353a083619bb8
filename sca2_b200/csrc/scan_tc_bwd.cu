// Tensor-core (tcgen05 / TMEM) backward scan for bf16 inputs on sm_100a.
//
// One CTA per (batch*head, block of 64 value columns); chunks of 64 tokens are walked in
// reverse.  The forward saved, per chunk c: the state entering the chunk (slot 2c of the
// chunk-state buffer, fp32) and, in slot 2c+1, the inverse T = (I + beta Gr)^{-1} and the
// corrected values E = T (V' - beta a kr Sp / kappa) in bf16, already in the operand layout,
// and in slot 2 NC + c the masked, decayed read kernel P = (QR KW^T / kappa) .* Dg (bf16).
// With Sp = d1 .* S (state entering the chunk, decayed once) and dS the adjoint of the state
// leaving the chunk (fp32 registers), one chunk is:
//
//   batch 1   G = KR KW^T, DS0 = dO^T QRA, DQR2 = dO Sp^T, DKW3 = E dSc^T,
//             dE = KWW dSc + P^T dO                              (dSc = dCm1 .* dS)
//   batch 3   dY = T^T dE           (dv = dY, beta dY for the GDN write)
//   batch 4   DL = dY E^T, DP = dO E^T, DS0 += dY^T ZN, DKR2 = dY Sp^T
//             -> dKK = beta (-DL) .* Dg (strict), dQK = DP .* Dg (incl),
//                dS <- a_last dCm1 d1 .* dS + d1 .* DS0
//   batch 5   DKR1 = dKK KW, DQR1 = dQK KW, DKW12 = dKK^T KR + dQK^T QR,
//             DLW = ((j - i) dKK)^T KR + ((j - i) dQK)^T QR
//   finish    dkr = DKR1 / kappa - beta a / kappa DKR2,  dqr = DQR1 / kappa + a / kappa DQR2,
//             dkw = DKW12 / kappa + w DKW3, then the chain rule to (phi, psi | k, q), and the
//             row reductions that give d(beta), d(a), d(w) from the same products
//             (sum_v dY R0 = a / kappa sum_m kr DKR2, sum_v E (kw dSc) = sum_m kw DKW3, ...)
//
// where ZN = -beta a kr / kappa, QRA = a qr / kappa, KWW = w kw.  The intra-chunk part of
// d(lam) is sum_j kw_j .* DLW_j / kappa: the relative-position form, because the separately
// i-weighted (kr, qr) and j-weighted (kw) sums cancel to a few percent of their size.
//
// Every product is a bf16 MMA with fp32 accumulation in TMEM.  Operands used both ways are
// stored once, K-major, and read through MN-major descriptors for the transposed use.  The
// next chunk's state, T, E, P and dO are copied in while the current chunk runs: dO of a full
// chunk by TMA (phase flavour, one 5-D tensor copy per read column into operand layout, completion
// on an mbarrier whose wait is bounded) where the tensor map can address dO, the rest by cp.async;
// its phases (keys) and gates are loaded into registers.  Every mbarrier wait is bounded: on a
// timeout the CTA records a fault bit, frees its TMEM and returns.
#include <cstring>

#include "tc_common.cuh"

namespace sca2 {
namespace tc {

// bit 0: a bounded mbarrier wait of the backward timed out (one fault word per translation
// unit: the library is built without relocatable device code)
__device__ unsigned int g_fault_bwd;

constexpr int BVB = 64;  // value columns per CTA

// byte offsets of the shared-memory carve-up; regions R1..R5 are reused by operands with
// disjoint lifetimes (noted per region)
template <int FL, int R>
struct BwdLayout {
  static constexpr int KD = 64, VB = BVB, RC = R * C, Mh = KD / 2;
  static constexpr int KR = 0;                     // C x KD   kr             [i][m]
  static constexpr int KW = KR + C * KD * 2;       // C x KD   kw             [i][m]
  static constexpr int QR = KW + C * KD * 2;       // RC x KD  qr             [(r,i)][m]
  static constexpr int TB = QR + RC * KD * 2;      // C x C    T (saved)      [i][j]
  static constexpr int EB = TB + C * C * 2;        // VB x C   E^T (saved)    [v][j]
  static constexpr int DOA = EB + VB * C * 2;      // RC x VB  dO             [(r,i)][v]
  static constexpr int CST = DOA + RC * VB * 2;    // fp32 KD x VB staged state [m][v]
  static constexpr int PP = CST + KD * VB * 4;     // RC x C   P (saved)      [(r,i)][j]
  static constexpr int CACHE = PP + RC * C * 2;    // fp32 phase: cos/sin phi, cos/sin psi [4][C][CS]
                                                   //      key:   k, q * scale [2][C][CS]
  // cache row stride: 4 floats of padding put the rows of 8 consecutive tokens in distinct
  // 16-byte bank groups, so the finish's 16-byte loads (one token row per lane) do not conflict
  static constexpr int CS = (FL == SCA2_FLAVOR_PHASE ? Mh : KD) + 4;
  static constexpr int CACHE_BYTES = FL == SCA2_FLAVOR_PHASE ? 4 * C * CS * 4 : 2 * C * CS * 4;
  static constexpr int R1 = CACHE + CACHE_BYTES;   // QRA (b1) | dQK (epi4-b5)
  static constexpr int R2 = R1 + RC * 64 * 2;      // KWW (b1) | dE (epi2-b3) | dKK (epi4-b5) | PQ (finish)
  static constexpr int R3 = R2 + C * 64 * 2;       // ZN (codes-b4) | (j-i) dKK (epi4-b5)
  static constexpr int R4 = R3 + C * 64 * 2;       // Sp^T, dSc^T [v][m] (prologue-b4) | (j-i) dQK (epi4-b5)
  static constexpr int R5 = R4 + 2 * VB * KD * 2;  // dY [i][v] (epi3-b4)
  static constexpr int KH = FL == SCA2_FLAVOR_PHASE ? Mh : KD;
  static constexpr int GRW = R5 + C * VB * 2;      // fp32 C x KH  staged dphw / dk rows of the chunk
  static constexpr int GRQ = GRW + C * KH * 4;     // fp32 C x KH  staged dphq / dq rows
  static constexpr int ELL = GRQ + C * KH * 4;     // fp32 C x CS  exp(-lam_m i), chunk-independent
  static constexpr int SC = ELL + C * CS * 4;
  // scalars (floats): beta, Gc, a, w, dbeta, da, dw, rows, cols [C]; d1, dCm1, lam, wr, wi,
  // dlam, dwr, dwi [KD]; misc[8]; a second set of beta, Gc, a, w [C] (the next chunk's); the
  // column factors of the decay mask [C]; the head's theta and omega [Mh] (phases from projections)
  static constexpr int SC_FLOATS = 14 * C + 8 * KD + 8 + 2 * Mh;
  static constexpr int MBAR = SC + ((SC_FLOATS * 4 + 1023) & ~1023);
  static constexpr int TOTAL = MBAR + 64;  // MMA mbarrier, TMEM base, error flag, dO-tile mbarrier
  static_assert(TOTAL <= 227 * 1024, "shared memory");
  static_assert(RC * 64 * 2 >= RC * KD * 2, "R1 holds QRA");
  static_assert(2 * VB * KD * 2 >= RC * C * 2, "R4 holds the weighted dQK");
  static_assert(C * 64 * 2 >= C * Mh * 4, "R2, R3 and R5 each hold a C x Mh fp32 staging array (phase)");
  static_assert(2 * C * 64 * 2 >= C * KD * 4 && 2 * VB * KD * 2 >= C * KD * 4,
                "R2..R3 and R4 hold a C x K fp32 staging array (key)");
};

// TMEM columns (fp32).  Lifetimes: batch 1 writes G, P, DS0, DQR2, DKW3, DE; DY reuses P's
// columns after the first epilogue; DL and DP follow DE; the batch-5 results reuse G, DY, DL, DP.
struct BCols {
  static constexpr int G = 0, P = 64, DS0 = 128, DQR2 = 192, DKW3 = 256, DE = 320;
  static constexpr int DY = 64, DL = 320, DP = 384, DKR2 = 448;
  static constexpr int DKR1 = 0, DQR1 = 64, DKW12 = 320, DLW = 384;
  static constexpr int ALLOC = 512;
};

// launch flags of the backward (host-computed)
// B_OVERWRITE: write the key-side gradient rows instead of accumulating (this CTA owns them)
enum : int { B_PH_VEC = 1, B_DO_VEC = 2, B_DV_VEC = 4, B_G_VEC = 8, B_K_VEC = 16, B_OVERWRITE = 32 };

// ---- asynchronous copies of the next chunk's saved data ------------------------------------
// element (m, v) of the staged state: rows m of BVB floats, v XOR-swizzled in 8-float groups by
// (m / 2) % 4, so the state-layout reads (8 rows v by 4 column pairs m per instruction) hit 32
// distinct banks; 16-byte runs stay contiguous
__device__ __forceinline__ int cst_idx(int m, int v) { return m * BVB + (v ^ (((m >> 1) & 3) << 3)); }
template <int KD>
__device__ __forceinline__ void pf_state(uint8_t* dst, const float* cstates, int64_t slot_base, int V, int vb0) {
  // 64 rows m of 64 fp32 columns -> [m][v] (16 copies per row)
  for (int u = threadIdx.x; u < KD * 16; u += NT) {
    const int m = u >> 4, v4 = (u & 15) * 4;
    cp16(dst + cst_idx(m, v4) * 4, cstates + slot_base + (int64_t)m * V + vb0 + v4, true);
  }
}
__device__ __forceinline__ void pf_bytes(uint8_t* dst, const uint8_t* src, int nbytes) {
  for (int u = threadIdx.x * 16; u < nbytes; u += NT * 16) cp16(dst + u, src + u, true);
}
template <int R>
__device__ __forceinline__ void pf_dO(const sca2_scan_args& p, const sca2_out& dO, bf16* DOA, int flags, int b,
                                      int h, int t0, int Cl, int vb0) {
  constexpr int RC = R * C;
  for (int u = threadIdx.x; u < RC * (BVB / 8); u += NT) {
    const int row = u >> 3, v0 = (u & 7) * 8, r = row >> 6, i = row & 63;
    const bool live = i < Cl;
    const int64_t off = live ? out_off(dO, b, t0 + i, h, r) + vb0 + v0 : 0;
    bf16* dst = DOA + umma::kmaj(row, v0, BVB);
    if (flags & B_DO_VEC) {
      cp16(dst, reinterpret_cast<const bf16*>(dO.ptr) + off, live);
    } else {
      float x[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = (live && vb0 + v0 + k < p.V) ? ld_io(dO.ptr, off + k, p.io_dtype) : 0.f;
      st8(dst, 0, x);
    }
  }
}

// the chunk's rows of an fp32 key-side gradient (accumulated into) -> G[i][m], zero rows i >= Cl
template <int KH>
__device__ __forceinline__ void pf_grad_rows(float* G, const sca2_tok& t, int b, int h, int t0, int Cl) {
  const float* base = reinterpret_cast<const float*>(t.ptr);
  for (int u = threadIdx.x; u < C * (KH / 4); u += NT) {
    const int i = u / (KH / 4), m4 = (u % (KH / 4)) * 4;
    const bool live = i < Cl;
    cp16(G + i * KH + m4, base + (live ? tok_off(t, b, t0 + i, h) + m4 : 0), live);
  }
}

// ---- code operands and the per-chunk cache --------------------------------------------------
//   KR[i][m] = kr, KW[i][m] = kw, QR[(r,i)][m] = qr, ZN[i][m] = -beta a kr / kappa,
//   KWW[i][m] = w kw, QRA[(r,i)][m] = a qr / kappa; cache: cos / sin of phi and psi (phase)
//   or k and q * scale (key), fp32 [.][i][m]
template <int FL, int KD, int R>
__device__ __forceinline__ void build_codes2(const CodeRegs<FL, KD>& cr, uint8_t* sm, const Gates& g, const float* s_lam,
                                             const float* s_wr, const float* s_wi, float q_scale, int Cl, float ik) {
  const float* ELL = reinterpret_cast<const float*>(sm + BwdLayout<FL, R>::ELL);
  using L = BwdLayout<FL, R>;
  bf16* KR = reinterpret_cast<bf16*>(sm + L::KR);
  bf16* KW = reinterpret_cast<bf16*>(sm + L::KW);
  bf16* QR = reinterpret_cast<bf16*>(sm + L::QR);
  bf16* QRA = reinterpret_cast<bf16*>(sm + L::R1);
  bf16* KWW = reinterpret_cast<bf16*>(sm + L::R2);
  bf16* ZN = reinterpret_cast<bf16*>(sm + L::R3);
  float* cache = reinterpret_cast<float*>(sm + L::CACHE);
  const int tid = threadIdx.x;
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2;
    int i, m0;
    code_unit<Mh / 8>(tid, i, m0);
    const bool live = i < Cl;
    const float fi = (float)i, zb = -g.beta[i] * g.a[i] * ik, fa = g.a[i] * ik, wv = g.w[i];
    float c[8], s[8], cq[8], sq[8];
    float kc[8], ks[8], wc[8], ws[8], q0a[8], q0b[8], q1a[8], q1b[8];
    float el[8];
    {
      const float4 e0 = *reinterpret_cast<const float4*>(ELL + i * L::CS + m0);
      const float4 e1 = *reinterpret_cast<const float4*>(ELL + i * L::CS + m0 + 4);
      el[0] = e0.x; el[1] = e0.y; el[2] = e0.z; el[3] = e0.w; el[4] = e1.x; el[5] = e1.y; el[6] = e1.z; el[7] = e1.w;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int m = m0 + k;
      c[k] = s[k] = cq[k] = sq[k] = 0.f;
      if (live) {
        sincos_big(cr.w[0][k], &s[k], &c[k]);
        sincos_big(cr.q[0][k], &sq[k], &cq[k]);
      }
      const float l = s_lam[m];
      const float ell = el[k], elli = __expf(l * fi);
      const float c1 = s_wr[m] * cq[k] + s_wi[m] * sq[k], c2 = s_wr[m] * sq[k] - s_wi[m] * cq[k];
      kc[k] = c[k] * ell; ks[k] = s[k] * ell; wc[k] = c[k] * elli; ws[k] = s[k] * elli;
      q0a[k] = c1 * ell; q0b[k] = c2 * ell; q1a[k] = -c2 * ell; q1b[k] = c1 * ell;
    }
    constexpr int CS = L::CS;
    float4* cw = reinterpret_cast<float4*>(cache + (0 * C + i) * CS + m0);
    float4* sw = reinterpret_cast<float4*>(cache + (1 * C + i) * CS + m0);
    float4* cqp = reinterpret_cast<float4*>(cache + (2 * C + i) * CS + m0);
    float4* sqp = reinterpret_cast<float4*>(cache + (3 * C + i) * CS + m0);
    cw[0] = make_float4(c[0], c[1], c[2], c[3]); cw[1] = make_float4(c[4], c[5], c[6], c[7]);
    sw[0] = make_float4(s[0], s[1], s[2], s[3]); sw[1] = make_float4(s[4], s[5], s[6], s[7]);
    cqp[0] = make_float4(cq[0], cq[1], cq[2], cq[3]); cqp[1] = make_float4(cq[4], cq[5], cq[6], cq[7]);
    sqp[0] = make_float4(sq[0], sq[1], sq[2], sq[3]); sqp[1] = make_float4(sq[4], sq[5], sq[6], sq[7]);
    st8(KR, umma::kmaj(i, m0, KD), kc);
    st8(KR, umma::kmaj(i, Mh + m0, KD), ks);
    st8(KW, umma::kmaj(i, m0, KD), wc);
    st8(KW, umma::kmaj(i, Mh + m0, KD), ws);
    st8(QR, umma::kmaj(i, m0, KD), q0a);
    st8(QR, umma::kmaj(i, Mh + m0, KD), q0b);
    st8(QR, umma::kmaj(C + i, m0, KD), q1a);
    st8(QR, umma::kmaj(C + i, Mh + m0, KD), q1b);
    float t[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = zb * kc[k];
    st8(ZN, umma::kmaj(i, m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = zb * ks[k];
    st8(ZN, umma::kmaj(i, Mh + m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = wv * wc[k];
    st8(KWW, umma::kmaj(i, m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = wv * ws[k];
    st8(KWW, umma::kmaj(i, Mh + m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = fa * q0a[k];
    st8(QRA, umma::kmaj(i, m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = fa * q0b[k];
    st8(QRA, umma::kmaj(i, Mh + m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = fa * q1a[k];
    st8(QRA, umma::kmaj(C + i, m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = fa * q1b[k];
    st8(QRA, umma::kmaj(C + i, Mh + m0, KD), t);
  } else {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      int i, m0;
      code_unit<KD / 8>(tid + u * NT, i, m0);
      const float fi = (float)i, zb = -g.beta[i] * g.a[i] * ik, fa = g.a[i] * ik, wv = g.w[i];
      float kk[8], qq[8], kc[8], wc[8], qc[8], t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float l = s_lam[m0 + k];
        const float ell = ELL[i * L::CS + m0 + k], elli = __expf(l * fi);
        kk[k] = cr.w[u][k];
        qq[k] = q_scale * cr.q[u][k];
        kc[k] = kk[k] * ell; wc[k] = kk[k] * elli; qc[k] = qq[k] * ell;
      }
      float4* kp = reinterpret_cast<float4*>(cache + (0 * C + i) * L::CS + m0);
      float4* qp = reinterpret_cast<float4*>(cache + (1 * C + i) * L::CS + m0);
      kp[0] = make_float4(kk[0], kk[1], kk[2], kk[3]); kp[1] = make_float4(kk[4], kk[5], kk[6], kk[7]);
      qp[0] = make_float4(qq[0], qq[1], qq[2], qq[3]); qp[1] = make_float4(qq[4], qq[5], qq[6], qq[7]);
      st8(KR, umma::kmaj(i, m0, KD), kc);
      st8(KW, umma::kmaj(i, m0, KD), wc);
      st8(QR, umma::kmaj(i, m0, KD), qc);
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = zb * kc[k];
      st8(ZN, umma::kmaj(i, m0, KD), t);
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = wv * wc[k];
      st8(KWW, umma::kmaj(i, m0, KD), t);
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = fa * qc[k];
      st8(QRA, umma::kmaj(i, m0, KD), t);
    }
  }
}

// Position of element m of token row i in the finish's fp32 staging arrays (rows of KH >= 32
// floats): the 16-byte chunk index is XORed with i mod 8, so the rows of 8 consecutive tokens
// put a given chunk in 8 distinct bank groups (the staging stores have one token row per lane).
__device__ __forceinline__ int swz(int i, int m) { return ((((m >> 2) ^ (i & 7))) << 2) | (m & 3); }

// sum over the 16 row-owning lanes of an M = 64 fragment (lanes 0..15); result in lane 0
__device__ __forceinline__ float sum16(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// fp32 gradient rows: += 8 consecutive values.  staged: the row's previous values were copied
// into shared memory at the start of the chunk (only CTA writing them, 16-byte aligned); else
// plain read-add-write when this CTA is the only writer, atomics otherwise.
__device__ __forceinline__ void acc_row8(float* dst, const float* x, bool vec, bool exclusive,
                                         const float* staged) {
  if (staged) {
    const float4 a = reinterpret_cast<const float4*>(staged)[0], b = reinterpret_cast<const float4*>(staged)[1];
    float4* d = reinterpret_cast<float4*>(dst);
    d[0] = make_float4(a.x + x[0], a.y + x[1], a.z + x[2], a.w + x[3]);
    d[1] = make_float4(b.x + x[4], b.y + x[5], b.z + x[6], b.w + x[7]);
  } else if (exclusive && vec) {
    float4* d = reinterpret_cast<float4*>(dst);
    float4 a = d[0], b = d[1];
    a.x += x[0]; a.y += x[1]; a.z += x[2]; a.w += x[3];
    b.x += x[4]; b.y += x[5]; b.z += x[6]; b.w += x[7];
    d[0] = a;
    d[1] = b;
  } else if (exclusive) {
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] += x[k];
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) atomicAdd(dst + k, x[k]);
  }
}

// HG: a per-token scalar decay (p.g) is present; PJ: phases formed from projections (PhaseProj::on,
// phase flavour).  Both are compile-time variants, so a kernel carries only the code its inputs use.
template <int FL, int R, bool HG, bool PJ>
__global__ void __launch_bounds__(NT, 1) scan_bwd_tc(sca2_scan_args p, sca2_out dO, const float* dS_final,
                                                    const float* cstates, sca2_scan_grads gr, int NCS,
                                                    int flags, PhaseProj pp_in,
                                                    const __grid_constant__ CUtensorMap omap, int use_tma) {
  PhaseProj pp = pp_in;
  pp.on = PJ;
  using L = BwdLayout<FL, R>;
  using CO = BCols;
  constexpr int KD = 64, VB = BVB, RC = R * C, Mh = KD / 2;
  constexpr int KH = FL == SCA2_FLAVOR_PHASE ? Mh : KD;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, sub = warp & 3, half = tid >> 7;
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int vb0 = blockIdx.y * VB;
  // MMA issue: lane 0 of warps 0..NISS-1 each issue the products of their own accumulators and
  // commit (or arrive, when they have none in a batch) on the batch's mbarrier
  constexpr int NISS = 4;
  const bool issuer = lane == 0 && warp < NISS;
  // the next chunk's gates: loaded and formed by the last warp, which issues no products
  constexpr int GW = NT / 32 - 1;
  const int V = p.V;
  constexpr bool has_g = HG;  // a per-token scalar decay (p.g) is present: its gradient terms
  const bool excl = gridDim.y == 1;  // the only CTA writing this (b, h)'s key-side gradients
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)Mh : 1.f;
  const float ik = 1.f / kappa;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  // gates of chunk c in set c & 1: the next chunk's are formed while this one runs
  auto gset = [&](int k) -> Gates {
    float* g0 = (k & 1) ? sc + 9 * C + 8 * KD + 8 : sc;
    return Gates{g0, g0 + C, g0 + 2 * C, g0 + 3 * C};
  };
  Gates gates = gset(0);
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
  float* s_fdec = s_misc + 8 + 4 * C;  // column factors of the decay mask (decay_block)
  float* s_th = s_fdec + C;            // theta, omega of the head (phases from projections)
  float* s_om = s_th + Mh;
  auto BF = [&](int off) { return reinterpret_cast<bf16*>(sm + off); };
  float* CST = reinterpret_cast<float*>(sm + L::CST);
  float* cache = reinterpret_cast<float*>(sm + L::CACHE);
  float* ELL = reinterpret_cast<float*>(sm + L::ELL);
  bf16* PA = BF(L::PP);
  bf16* DQKA = BF(L::R1);
  bf16* DEA = BF(L::R2);
  bf16* DKKA = BF(L::R2);
  float* PQ = reinterpret_cast<float*>(sm + L::R2);
  bf16* DKKW = BF(L::R3);
  bf16* SB = BF(L::R4);
  bf16* DSB = BF(L::R4 + VB * KD * 2);
  bf16* DQKW = BF(L::R4);
  bf16* DYA = BF(L::R5);
  float* GRW = reinterpret_cast<float*>(sm + L::GRW);
  float* GRQ = reinterpret_cast<float*>(sm + L::GRQ);
  const bool gwrite = excl && (flags & B_OVERWRITE) && (flags & B_G_VEC);  // rows written, not accumulated
  const bool gstage = excl && (flags & B_G_VEC) && !gwrite;  // gradient rows staged in shared memory
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  volatile int* s_err = reinterpret_cast<volatile int*>(sm + L::MBAR + 12);
  // dO tiles of full chunks by TMA (phase flavour: one copy per read column r into its 64-row half
  // of DOA), issued by thread 0, completion on obar, waited by every thread at the top of the
  // chunk; the ragged chunk takes 16-byte cp.async copies
  uint64_t* obar = reinterpret_cast<uint64_t*>(sm + L::MBAR + 16);
  const CUtensorMap* omp = &omap;
  uint32_t oph = 0;
  bool opend = false;  // a dO tile is in flight (uniform over the CTA)
  const bool otma = FL == SCA2_FLAVOR_PHASE && use_tma;  // compiled out of the key flavour
  auto tma_dO = [&](int t0c) {
    if (tid == 0) {
      tma_expect(obar, (uint32_t)(RC * VB * 2));
#pragma unroll
      for (int r = 0; r < R; ++r)
        tma_load5(sm + L::DOA + r * (C * VB * 2), omp, vb0 / 8, (b * p.T + t0c) / 8, R * h + r, obar);
    }
    opend = true;
  };

  // ---- set-up
  for (int m = tid; m < KD; m += NT) {
    const float l = p.lam ? p.lam[h * KH + (m % KH)] : 0.f;
    s_lam[m] = l;
    s_d1[m] = expf(-l);
    s_wr[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wr[h * KH + m] : 0.f;
    s_wi[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wi[h * KH + m] : 0.f;
    if (FL == SCA2_FLAVOR_PHASE && pp.on && m < Mh) {
      s_th[m] = pp.theta[h * Mh + m];
      s_om[m] = pp.omega[h * Mh + m];
    }
    s_dlam[m] = 0.f;
    s_dwr[m] = 0.f;
    s_dwi[m] = 0.f;
  }
  if (tid == 0) {
    umma::mbar_init(mbar, NISS);
    umma::mbar_init(obar, 1);
    umma::fence_mbar_init();
    *s_err = 0;
  }
  if (tid < 32) umma::tmem_alloc(s_tmem, CO::ALLOC);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  uint32_t phase = 0;
  // exp(-lam_m i) for the 64 positions of a chunk (read from here by the code build and the
  // finish; visible after the first chunk's barriers)
  for (int u = tid; u < C * KH; u += NT) {
    const int i = u / KH, m = u - (u / KH) * KH;
    ELL[i * L::CS + m] = __expf(-s_lam[m] * (float)i);
  }

  // state-layout registers: the M = VB (rows v) x N = KD (columns m) accumulator layout over all
  // 32 lanes (for_frag16): element k at row s_v(k), column s_m(k); adjoint dS and Sp
  constexpr int NS = KD / 4;
  float dSreg[NS], Spreg[NS], Lreg[NS];  // Lreg: state-side d(lam) terms summed over the chunks
  const int sv0 = 16 * sub + (lane >> 2), sm0 = half * (KD / 2) + 2 * (lane & 3);
  auto s_v = [&](int k) { return sv0 + 8 * ((k >> 1) & 1); };
  auto s_m = [&](int k) { return sm0 + 8 * (k >> 2) + (k & 1); };
  const int64_t bhKV = ((int64_t)b * p.H + h) * KD * (int64_t)V;
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    dSreg[k] = dS_final ? dS_final[bhKV + (int64_t)s_m(k) * V + vb0 + s_v(k)] : 0.f;
    Lreg[k] = 0.f;
  }

  auto wait_mma = [&]() -> bool {
    if (!umma::mbar_wait(mbar, phase)) *s_err = 1;
    phase ^= 1u;
    __syncthreads();
    umma::fence_after_sync();
    return *s_err == 0;
  };
  // Dg of row i over the 16 columns j0.. (zeros right of the row; 1 without a decay)
  auto dg_block = [&](int i, int j0, float* d) {
    if (!has_g) {
#pragma unroll
      for (int j = 0; j < 16; ++j) d[j] = 1.f;
    } else {
      decay_block(gates.Gc, s_fdec, i, j0, d);
    }
  };
  const int64_t bhs = ((int64_t)b * p.H + h) * NCS;
  auto slot = [&](int s) -> int64_t { return (bhs + s) * KD * (int64_t)V; };
  auto saved = [&](int c) -> const uint8_t* { return reinterpret_cast<const uint8_t*>(cstates + slot(2 * c + 1)); };
  const int NC = (p.T + C - 1) / C;
  // the chunk's masked, decayed read kernel P as the forward formed it (slot 2 NC + c)
  auto saved_P = [&](int c) -> const uint8_t* {
    return reinterpret_cast<const uint8_t*>(cstates + slot(2 * NC + c));
  };

  // prefetch of the last chunk
  CodeRegs<FL, KD> creg;
  GateRegs greg;
  {
    const int c = NC - 1, t0 = c * C, Cl = min(C, p.T - t0);
    pf_state<KD>(sm + L::CST, cstates, slot(2 * c), V, vb0);
    pf_bytes(sm + L::TB, saved(c), C * C * 2);
    pf_bytes(sm + L::EB, saved(c) + C * C * 2 + blockIdx.y * (VB * C * 2), VB * C * 2);
    pf_bytes(sm + L::PP, saved_P(c), RC * C * 2);
    if (otma && Cl == C)
      tma_dO(t0);
    else
      pf_dO<R>(p, dO, BF(L::DOA), flags, b, h, t0, Cl, vb0);
    cp_commit();
    load_code_regs<FL, KD>(p, creg, flags & (FL == SCA2_FLAVOR_PHASE ? B_PH_VEC : B_K_VEC), b, h, t0, Cl, pp);
    if (warp == 0) {
      load_gate_regs(p, greg, b, h, t0, Cl);
      gates_from_regs(greg, gset(c), Cl);
    }
  }

  bool ok = true;
  for (int c = NC - 1; c >= 0 && ok; --c) {
    const int t0 = c * C, Cl = min(C, p.T - t0);
    const float fi_last = (float)(Cl - 1);
    // ================= prologue =================
    cp_wait_all();
    if (opend) {  // this chunk's dO tile (TMA)
      if (!umma::mbar_wait(obar, oph)) *s_err = 1;
      oph ^= 1u;
      opend = false;
    }
    gates = gset(c);
    for (int m = tid; m < KD; m += NT) s_dCm1[m] = expf(-s_lam[m] * fi_last);
    if (tid < C) {
      s_dbeta[tid] = 0.f;
      s_da[tid] = 0.f;
      s_dw[tid] = 0.f;
      s_rows[tid] = 0.f;
      s_cols[tid] = 0.f;
    }
    if (tid == 0) s_misc[0] = 0.f;
    if (has_g) decay_factors(gates.Gc, s_fdec);
    __syncthreads();  // staged copies, gates, dCm1 and the decay factors visible
    if (gstage) {  // this chunk's gradient rows, needed by the finish (first group of the chunk)
      pf_grad_rows<KH>(GRW, gr.dphw, b, h, t0, Cl);
      pf_grad_rows<KH>(GRQ, gr.dphq, b, h, t0, Cl);
    }
    cp_commit();
    // Sp = d1 .* S (state layout registers) and the bf16 operands Sp^T, dSc^T [v][m]
#pragma unroll
    for (int g = 0; g < NS / 4; ++g) {
      float xs[4], xd[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = 4 * g + e, m = s_m(k);
        Spreg[k] = CST[cst_idx(m, s_v(k))] * s_d1[m];
        xs[e] = Spreg[k];
        xd[e] = s_dCm1[m] * dSreg[k];
      }
      const int m = sm0 + 8 * g;
      st2(SB, umma::kmaj(sv0, m, KD), xs[0], xs[1]);
      st2(SB, umma::kmaj(sv0 + 8, m, KD), xs[2], xs[3]);
      st2(DSB, umma::kmaj(sv0, m, KD), xd[0], xd[1]);
      st2(DSB, umma::kmaj(sv0 + 8, m, KD), xd[2], xd[3]);
    }
    finish_code_regs<FL, KD>(creg, pp, h, t0, Cl, s_th, s_om);
    build_codes2<FL, KD, R>(creg, sm, gates, s_lam, s_wr, s_wi, p.q_scale, Cl, ik);
    publish_smem();
    // ================= batch 1 =================
    if (issuer) {  // independent accumulators issued from NISS threads in parallel
      if (warp == 0) {
        umma::gemm_t(tb + CO::G, sm + L::KR, false, sm + L::KW, false, C, C, KD, false);
      } else if (warp == 1) {
        umma::gemm_t(tb + CO::DS0, sm + L::DOA, true, sm + L::R1, true, VB, KD, RC, false);
      } else if (warp == 2) {
        umma::gemm_t(tb + CO::DQR2, sm + L::DOA, false, SB, true, RC, KD, VB, false);
        umma::gemm_t(tb + CO::DKW3, sm + L::EB, true, DSB, true, C, KD, VB, false);
      } else {
        umma::gemm_t(tb + CO::DE, sm + L::R2, false, DSB, false, C, VB, KD, false);
        umma::gemm_t(tb + CO::DE, PA, true, sm + L::DOA, true, C, VB, RC, true);  // += P^T dO
      }
      umma::commit(mbar);
    }
    // next chunk: staged state (CST is free once the prologue has read it), codes and gates
    if (c > 0) {
      const int t1 = t0 - C;
      pf_state<KD>(sm + L::CST, cstates, slot(2 * (c - 1)), V, vb0);
      cp_commit();
      load_code_regs<FL, KD>(p, creg, flags & (FL == SCA2_FLAVOR_PHASE ? B_PH_VEC : B_K_VEC), b, h, t1, C, pp);
      if (warp == GW) load_gate_regs(p, greg, b, h, t1, C);
    }
    if (!(ok = wait_mma())) break;
    for_frag16<VB>(tb + CO::DE, [&](int, int j0, int v, const float* x) {
      st2(DEA, umma::kmaj(j0, v, VB), x[0], x[1]);
      st2(DEA, umma::kmaj(j0 + 8, v, VB), x[2], x[3]);
    });
    publish_smem();
    // ================= batch 3: dY = T^T dE =================
    if (issuer) {
      if (warp == 0) {
        umma::gemm_t(tb + CO::DY, sm + L::TB, true, DEA, true, C, VB, C, false);
        umma::commit(mbar);
      } else {
        umma::mbar_arrive(mbar);
      }
    }
    if (warp == GW && c > 0) gates_from_regs(greg, gset(c - 1), C);  // the next chunk's gates
    if (!(ok = wait_mma())) break;
    if (c > 0) {  // TB is free: the next chunk's T
      pf_bytes(sm + L::TB, saved(c - 1), C * C * 2);
      cp_commit();
    }
    {
      const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
      for_frag<C, VB>(tb + CO::DY, [&](int i, int v0, int, const float* x) {
        st8(DYA, umma::kmaj(i, v0, VB), x);
        st8(DYA, umma::kmaj(i, v0 + 8, VB), x + 8);
        if (i < Cl) {
          float y[16];
          float sv = 0.f;
          const float bi = p.v_times_beta ? bp[tok_off(p.beta, b, t0 + i, h)] : 1.f;
          const int64_t off = tok_off(gr.dv, b, t0 + i, h) + vb0 + v0;
          if (p.v_times_beta) {
            const int64_t ov = tok_off(p.v, b, t0 + i, h) + vb0 + v0;
#pragma unroll
            for (int j = 0; j < 16; ++j) sv += x[j] * ld_io(p.v.ptr, ov + j, p.io_dtype);
            atomicAdd(&s_dbeta[i], sv);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) y[j] = bi * x[j];
          if (flags & B_DV_VEC) {
            bf16* dst = reinterpret_cast<bf16*>(const_cast<void*>(gr.dv.ptr)) + off;
            st8(dst, 0, y);
            st8(dst, 8, y + 8);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (vb0 + v0 + j < V) st_io(const_cast<void*>(gr.dv.ptr), off + j, y[j], p.io_dtype);
          }
        }
      });
    }
    publish_smem();
    // ================= batch 4: DL, DP, DS0 += dY^T ZN, DKR2 =================
    if (issuer) {
      if (warp == 0)
        umma::gemm_t(tb + CO::DL, DYA, false, sm + L::EB, true, C, C, VB, false);
      else if (warp == 1)
        umma::gemm_t(tb + CO::DP, sm + L::DOA, false, sm + L::EB, true, RC, C, VB, false);
      else if (warp == 2)
        umma::gemm_t(tb + CO::DS0, DYA, true, sm + L::R3, true, VB, KD, C, true);
      else
        umma::gemm_t(tb + CO::DKR2, DYA, false, SB, true, C, KD, VB, false);
      umma::commit(mbar);
    }
    if (!(ok = wait_mma())) break;
    if (c > 0) {  // EB and DOA are free: the next chunk's E and dO
      pf_bytes(sm + L::EB, saved(c - 1) + C * C * 2 + blockIdx.y * (VB * C * 2), VB * C * 2);
      if (otma)
        tma_dO(t0 - C);
      else
        pf_dO<R>(p, dO, BF(L::DOA), flags, b, h, t0 - C, C, vb0);
      cp_commit();
    }
    // ---- dL with G -> dKK (+ position-weighted), d(beta) row term, decay sums
    if constexpr (!HG) {
      // the 16 rows of each sub-partition over all 32 lanes (16x256b loads): lane t holds rows
      // r0 = t/4 and r0 + 8, columns 2(t%4) and 2(t%4) + 1 of every 8-column group
      const int i0 = 16 * sub + (lane >> 2), i1 = i0 + 8, cw = (warp >> 2) * 32, c2 = 2 * (lane & 3);
      const float b0 = gates.beta[i0], b1 = gates.beta[i1];
      uint32_t ud[4][4], ug[4][4];
#pragma unroll
      for (int gi = 0; gi < 4; ++gi) {
        umma::ld4_rows16_issue(umma::taddr(tb + CO::DL, 32 * sub, cw + 8 * gi), ud[gi]);
        umma::ld4_rows16_issue(umma::taddr(tb + CO::G, 32 * sub, cw + 8 * gi), ug[gi]);
      }
      umma::ld_wait();
      float sb0 = 0.f, sb1 = 0.f;
#pragma unroll
      for (int gi = 0; gi < 4; ++gi) {
        const int j = cw + 8 * gi + c2;  // columns j, j + 1
        float dl[4], gg[4], kk[4], kw[4];
        umma::take<4>(ud[gi], dl);
        umma::take<4>(ug[gi], gg);
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // (i0, j), (i0, j + 1), (i1, j), (i1, j + 1)
          const int i = e < 2 ? i0 : i1, jj = j + (e & 1);
          float val = 0.f;
          if (jj < i) {
            const float l = -dl[e];
            if (e < 2)
              sb0 = fmaf(l, gg[e] * ik, sb0);
            else
              sb1 = fmaf(l, gg[e] * ik, sb1);
            val = (e < 2 ? b0 : b1) * l;
          }
          kk[e] = val;
          kw[e] = val * (float)(jj - i);
        }
        *reinterpret_cast<__nv_bfloat162*>(DKKA + umma::kmaj(i0, j, C)) = __floats2bfloat162_rn(kk[0], kk[1]);
        *reinterpret_cast<__nv_bfloat162*>(DKKA + umma::kmaj(i1, j, C)) = __floats2bfloat162_rn(kk[2], kk[3]);
        *reinterpret_cast<__nv_bfloat162*>(DKKW + umma::kmaj(i0, j, C)) = __floats2bfloat162_rn(kw[0], kw[1]);
        *reinterpret_cast<__nv_bfloat162*>(DKKW + umma::kmaj(i1, j, C)) = __floats2bfloat162_rn(kw[2], kw[3]);
      }
      // the row terms of d(beta): the four lanes of a row, then one atomic per row and warp
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        sb0 += __shfl_xor_sync(0xffffffffu, sb0, o);
        sb1 += __shfl_xor_sync(0xffffffffu, sb1, o);
      }
      if ((lane & 3) == 0) {
        atomicAdd(&s_dbeta[i0], sb0);
        atomicAdd(&s_dbeta[i1], sb1);
      }
    } else {
      const int i = frag_row<C>();
      const bool own = owns_rows<C>();
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int j0 = frag_col0<C, C>(q);
        float dl[16], gg[16];
        {
          uint32_t u[2][16];
          umma::ld16_issue(umma::taddr(tb + CO::DL, 32 * sub, j0), u[0]);
          umma::ld16_issue(umma::taddr(tb + CO::G, 32 * sub, j0), u[1]);
          umma::ld_wait();
          umma::take<16>(u[0], dl);
          umma::take<16>(u[1], gg);
        }
        float dkk[16], dkw[16], gcol[16], dgv[16];
        float sb = 0.f, srow_ = 0.f;
        dg_block(i, j0, dgv);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          float val = 0.f;
          gcol[j] = 0.f;
          if (own && jj < i) {
            const float d = dgv[j];
            const float l = -dl[j];
            const float grv = gg[j] * ik * d;
            sb += l * grv;
            gcol[j] = gates.beta[i] * l * grv;
            srow_ += gcol[j];
            val = gates.beta[i] * l * d;
          }
          dkk[j] = val;
          dkw[j] = val * (float)(jj - i);
        }
        if (has_g) {  // column sums of the 16 columns over the warp's rows: one transpose-reduce
          const float t = warp_transpose_sum<16>(gcol);
          if ((lane & 1) == 0) atomicAdd(&s_cols[j0 + red_index<16>(lane)], t);
        }
        if (own) {
          atomicAdd(&s_dbeta[i], sb);
          if (has_g) atomicAdd(&s_rows[i], srow_);
          st8(DKKA, umma::kmaj(i, j0, C), dkk);
          st8(DKKA, umma::kmaj(i, j0 + 8, C), dkk + 8);
          st8(DKKW, umma::kmaj(i, j0, C), dkw);
          st8(DKKW, umma::kmaj(i, j0 + 8, C), dkw + 8);
        }
      }
    }
    // ---- dP -> dQK (+ weighted) and decay sums
    {
      const int row = frag_row<RC>(), i = row & 63;
      const bool own = owns_rows<RC>();
#pragma unroll
      for (int q = 0; q < C / 32; ++q) {
        const int j0 = frag_col0<RC, C>(q);
        float dp[16];
        {
          uint32_t udp[16];
          umma::ld16_issue(umma::taddr(tb + CO::DP, 32 * sub, j0), udp);
          umma::ld_wait();
          umma::take<16>(udp, dp);
        }
        float dqk[16], dqw[16], gcol[16], dgv[16];
        float srow_ = 0.f;
        dg_block(i, j0, dgv);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float pa[8];  // P of the row's 8 columns (one 16-byte load)
          if (has_g && own) ld8_bf16(PA, umma::kmaj(row, j0 + 8 * hh, C), pa);
#pragma unroll
          for (int j8 = 0; j8 < 8; ++j8) {
            const int j = 8 * hh + j8, jj = j0 + j;
            float val = 0.f;
            gcol[j] = 0.f;
            if (own && jj <= i) {
              val = dp[j] * dgv[j];
              if (has_g) {
                gcol[j] = dp[j] * pa[j8];
                srow_ += gcol[j];
              }
            }
            dqk[j] = val;
            dqw[j] = val * (float)(jj - i);
          }
        }
        if (has_g) {  // column sums over the warp's rows (lanes without rows add zeros)
          const float t = warp_transpose_sum<16>(gcol);
          if ((lane & 1) == 0) atomicAdd(&s_cols[j0 + red_index<16>(lane)], t);
        }
        if (own) {
          if (has_g) atomicAdd(&s_rows[i], srow_);
          st8(DQKA, umma::kmaj(row, j0, C), dqk);
          st8(DQKA, umma::kmaj(row, j0 + 8, C), dqk + 8);
          st8(DQKW, umma::kmaj(row, j0, C), dqw);
          st8(DQKW, umma::kmaj(row, j0 + 8, C), dqw + 8);
        }
      }
    }
    // ---- DS0 -> adjoint update and state-side lambda / decay terms
    {
      const float aC = gates.a[Cl - 1];
      const float fCl = (float)Cl;
      float daC = 0.f;
      for_frag16<KD>(tb + CO::DS0, [&](int g, int, int, const float* d0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * g + e, m = s_m(k);
          const float sp = Spreg[k], ds = dSreg[k];
          const float t = aC * s_dCm1[m] * sp * ds;
          daC += t;
          Lreg[k] += -d0[e] * sp - fCl * t;
          dSreg[k] = aC * s_dCm1[m] * s_d1[m] * ds + s_d1[m] * d0[e];
        }
      });
      if (has_g) {
        daC = warp_sum(daC);
        if (lane == 0) atomicAdd(&s_misc[0], daC);
      }
    }
    publish_smem();
    if (c > 0) {  // every thread is past the dP epilogue, PA's last reader: the next chunk's P
      pf_bytes(sm + L::PP, saved_P(c - 1), RC * C * 2);
      cp_commit();
    }
    // ================= batch 5: DKR1, DQR1, DKW12, DLW =================
    if (issuer) {
      if (warp == 0) {
        umma::gemm_t(tb + CO::DKR1, DKKA, false, sm + L::KW, true, C, KD, C, false);
      } else if (warp == 1) {
        umma::gemm_t(tb + CO::DQR1, DQKA, false, sm + L::KW, true, RC, KD, C, false);
      } else if (warp == 2) {
        umma::gemm_t(tb + CO::DKW12, DKKA, true, sm + L::KR, true, C, KD, C, false);
        umma::gemm_t(tb + CO::DKW12, DQKA, true, sm + L::QR, true, C, KD, RC, true);
      } else if (p.lam) {
        umma::gemm_t(tb + CO::DLW, DKKW, true, sm + L::KR, true, C, KD, C, false);
        umma::gemm_t(tb + CO::DLW, DQKW, true, sm + L::QR, true, C, KD, RC, true);
      }
      if (warp < 3 || p.lam)
        umma::commit(mbar);
      else
        umma::mbar_arrive(mbar);
    }
    // the gradient rows (oldest group of this chunk); later groups hold the next chunk's data
    if (c > 0)
      cp_wait_group<4>();
    else
      cp_wait_group<0>();
    if (!(ok = wait_mma())) break;
    // ================= finish =================
    // (the loops over mode groups below are deliberately not unrolled: the unrolled bodies
    //  overflow the instruction cache and cost more than the loop overhead)
    // Per-element key / query gradients go to shared memory first (PK, PQ0 | PQ1) and are
    // written out once, coalesced, after one barrier.
    float* PK = FL == SCA2_FLAVOR_PHASE ? reinterpret_cast<float*>(sm + L::R5) : reinterpret_cast<float*>(sm + L::R4);
    float* PQ0 = reinterpret_cast<float*>(sm + L::R2);
    float* PQ1 = reinterpret_cast<float*>(sm + L::R3);  // phase: second read column's part
    // ---- key side: the 16 rows of each sub-partition over all 32 lanes (2 rows x 2 modes of an
    // 8-column group per thread)
    {
      const int r0 = lane >> 2, qq = lane & 3;
      const int rows[2] = {16 * sub + r0, 16 * sub + r0 + 8};
      float bsum[2] = {0.f, 0.f}, wsum[2] = {0.f, 0.f};
      constexpr int NG = FL == SCA2_FLAVOR_PHASE ? 2 : 4;  // groups of 8 modes (dims) per warp
#pragma unroll 1
      for (int g8 = 0; g8 < NG; ++g8) {
        const int mg = FL == SCA2_FLAVOR_PHASE ? 16 * half + 8 * g8 : 32 * half + 8 * g8;
        const int m0 = mg + 2 * qq;
        constexpr int NP = FL == SCA2_FLAVOR_PHASE ? 2 : 1;  // code columns per mode (cos, sin)
        float a1[NP][4], a2[NP][4], w12[NP][4], w3[NP][4], lw[NP][4];
        {
          uint32_t u[5 * NP][4];
          const uint32_t ta = umma::taddr(tb, 32 * sub, 0);
#pragma unroll
          for (int pp = 0; pp < NP; ++pp) {
            const int col = mg + pp * Mh;
            umma::ld4_rows16_issue(ta + CO::DKR1 + col, u[5 * pp + 0]);
            umma::ld4_rows16_issue(ta + CO::DKR2 + col, u[5 * pp + 1]);
            umma::ld4_rows16_issue(ta + CO::DKW12 + col, u[5 * pp + 2]);
            umma::ld4_rows16_issue(ta + CO::DKW3 + col, u[5 * pp + 3]);
            umma::ld4_rows16_issue(ta + CO::DLW + col, u[5 * pp + 4]);
          }
          umma::ld_wait();
#pragma unroll
          for (int pp = 0; pp < NP; ++pp) {
            umma::take<4>(u[5 * pp + 0], a1[pp]);
            umma::take<4>(u[5 * pp + 1], a2[pp]);
            umma::take<4>(u[5 * pp + 2], w12[pp]);
            umma::take<4>(u[5 * pp + 3], w3[pp]);
            umma::take<4>(u[5 * pp + 4], lw[pp]);
          }
        }
        float dl[2] = {0.f, 0.f};
#pragma unroll
        for (int ri = 0; ri < 2; ++ri) {
          const int i = rows[ri];
          const bool own = i < Cl;
          const float fi = (float)i, bi = gates.beta[i], aik = gates.a[i] * ik, wi_ = gates.w[i];
          // the two modes' cached codes as one 8-byte load (rows padded: conflict-free)
          const float2 c2 = *reinterpret_cast<const float2*>(cache + (0 * C + i) * L::CS + m0);
          const float2 s2 = FL == SCA2_FLAVOR_PHASE
                                ? *reinterpret_cast<const float2*>(cache + (1 * C + i) * L::CS + m0)
                                : c2;
          float dv2[2];
#pragma unroll
          for (int mi = 0; mi < 2; ++mi) {
            const int e = 2 * ri + mi, m = m0 + mi;
            const float l = s_lam[m];
            const float ell = ELL[i * L::CS + m], elli = __expf(l * fi);
            float dvv = 0.f;
            if constexpr (FL == SCA2_FLAVOR_PHASE) {
              const float c = mi ? c2.y : c2.x, s = mi ? s2.y : s2.x;
              const float krc = c * ell, krs = s * ell, kwc = c * elli, kws = s * elli;
              const float rc = aik * a2[0][e], rs = aik * a2[1][e];
              const float dkrc = a1[0][e] * ik - bi * rc, dkrs = a1[1][e] * ik - bi * rs;
              const float dkwc = w12[0][e] * ik + wi_ * w3[0][e], dkws = w12[1][e] * ik + wi_ * w3[1][e];
              const float dkc = dkrc * ell + dkwc * elli, dks = dkrs * ell + dkws * elli;
              dvv = -s * dkc + c * dks;
              const float kr_r = krc * rc + krs * rs, kw_w3 = kwc * w3[0][e] + kws * w3[1][e];
              if (own) {
                bsum[ri] += kr_r;
                wsum[ri] += kw_w3;
                if (p.lam) dl[mi] += ik * (kwc * lw[0][e] + kws * lw[1][e]) + fi * bi * kr_r + (fi - fi_last) * wi_ * kw_w3;
              }
            } else {
              const float kk = mi ? c2.y : c2.x;
              const float kr = kk * ell, kw = kk * elli;
              const float rr = aik * a2[0][e];
              const float dkr = a1[0][e] * ik - bi * rr, dkw = w12[0][e] * ik + wi_ * w3[0][e];
              dvv = dkr * ell + dkw * elli;
              if (own) {
                bsum[ri] += kr * rr;
                wsum[ri] += kw * w3[0][e];
                if (p.lam) dl[mi] += ik * kw * lw[0][e] + fi * bi * kr * rr + (fi - fi_last) * wi_ * kw * w3[0][e];
              }
            }
            dv2[mi] = own ? dvv : 0.f;
          }
          *reinterpret_cast<float2*>(PK + i * KH + swz(i, m0)) = make_float2(dv2[0], dv2[1]);
        }
        if (p.lam) {  // sum over the 16 rows: lanes with the same column pair
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            dl[0] += __shfl_xor_sync(0xffffffffu, dl[0], o);
            dl[1] += __shfl_xor_sync(0xffffffffu, dl[1], o);
          }
          if (r0 == 0) {
            atomicAdd(&s_dlam[m0], dl[0]);
            atomicAdd(&s_dlam[m0 + 1], dl[1]);
          }
        }
      }
      // row sums over this warp's modes: the four lanes of a row group
#pragma unroll
      for (int ri = 0; ri < 2; ++ri) {
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
          bsum[ri] += __shfl_xor_sync(0xffffffffu, bsum[ri], o);
          if (has_g) wsum[ri] += __shfl_xor_sync(0xffffffffu, wsum[ri], o);
        }
        const int i = rows[ri];
        if (qq == 0 && i < Cl) {
          atomicAdd(&s_dbeta[i], -bsum[ri]);
          if (has_g) {
            atomicAdd(&s_da[i], -gates.beta[i] * bsum[ri]);
            atomicAdd(&s_dw[i], gates.w[i] * wsum[ri]);
          }
        }
      }
    }
    // ---- query side (rows (r, i) of the M = R*64 accumulators)
    {
      const int row = frag_row<RC>(), r = row >> 6, i = row & 63;
      const bool own = owns_rows<RC>() && i < Cl;
      const float fi = (float)i, aik = gates.a[i] * ik;
      float asum = 0.f;
      if constexpr (FL == SCA2_FLAVOR_PHASE) {
#pragma unroll 1
        for (int g8 = 0; g8 < 2; ++g8) {
          const int mg = 16 * half + 8 * g8;
          float q1c[8], q1s[8], q2c[8], q2s[8];
          {
            uint32_t u[4][8];
            const uint32_t ta = umma::taddr(tb, 32 * sub, 0);
            umma::ld8_issue(ta + CO::DQR1 + mg, u[0]);
            umma::ld8_issue(ta + CO::DQR1 + Mh + mg, u[1]);
            umma::ld8_issue(ta + CO::DQR2 + mg, u[2]);
            umma::ld8_issue(ta + CO::DQR2 + Mh + mg, u[3]);
            umma::ld_wait();
            umma::take<8>(u[0], q1c); umma::take<8>(u[1], q1s);
            umma::take<8>(u[2], q2c); umma::take<8>(u[3], q2s);
          }
          float pq[8], dwr[8], dwi[8], dl[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            pq[k] = dwr[k] = dwi[k] = dl[k] = 0.f;
          }
          if (own) {
            float cqp[8], sqp[8];
            {
              const float4* c4 = reinterpret_cast<const float4*>(cache + (2 * C + i) * L::CS + mg);
              const float4* s4 = reinterpret_cast<const float4*>(cache + (3 * C + i) * L::CS + mg);
              const float4 a = c4[0], b = c4[1], cc = s4[0], d = s4[1];
              cqp[0] = a.x; cqp[1] = a.y; cqp[2] = a.z; cqp[3] = a.w; cqp[4] = b.x; cqp[5] = b.y; cqp[6] = b.z; cqp[7] = b.w;
              sqp[0] = cc.x; sqp[1] = cc.y; sqp[2] = cc.z; sqp[3] = cc.w; sqp[4] = d.x; sqp[5] = d.y; sqp[6] = d.z; sqp[7] = d.w;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int m = mg + k;
              const float cq = cqp[k], sq = sqp[k];
              const float wr = s_wr[m], wi = s_wi[m];
              const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
              const float ell = ELL[i * L::CS + m];
              const float gc = aik * q2c[k], gs = aik * q2s[k];
              const float dqc = (q1c[k] * ik + gc) * ell, dqs = (q1s[k] * ik + gs) * ell;
              const float dc1 = r ? dqs : dqc, dc2 = r ? -dqc : dqs;
              const float qrc = (r ? -c2 : c1) * ell, qrs = (r ? c1 : c2) * ell;
              pq[k] = -sq * (dc1 * wr - dc2 * wi) + cq * (dc1 * wi + dc2 * wr);
              dwr[k] = dc1 * cq + dc2 * sq;
              dwi[k] = dc1 * sq - dc2 * cq;
              const float gq = gc * qrc + gs * qrs;
              dl[k] = -fi * gq;
              asum += gq;
            }
          }
          // each read column's part of d(psi) -> PQ0 / PQ1 (zero rows beyond the chunk)
          {
            float* d = (r ? PQ1 : PQ0) + i * Mh;
            *reinterpret_cast<float4*>(d + swz(i, mg)) = make_float4(pq[0], pq[1], pq[2], pq[3]);
            *reinterpret_cast<float4*>(d + swz(i, mg + 4)) = make_float4(pq[4], pq[5], pq[6], pq[7]);
          }
          float x = warp_transpose_sum<8>(dwr);
          if ((lane & 3) == 0) atomicAdd(&s_dwr[mg + red_index<8>(lane)], x);
          x = warp_transpose_sum<8>(dwi);
          if ((lane & 3) == 0) atomicAdd(&s_dwi[mg + red_index<8>(lane)], x);
          if (p.lam) {
            x = warp_transpose_sum<8>(dl);
            if ((lane & 3) == 0) atomicAdd(&s_dlam[mg + red_index<8>(lane)], x);
          }
        }
      } else {
#pragma unroll 1
        for (int g8 = 0; g8 < 4; ++g8) {
          const int m0 = 32 * half + 8 * g8;
          float q1[8], q2[8];
          {
            uint32_t u[2][8];
            const uint32_t ta = umma::taddr(tb, 32 * sub, 0);
            umma::ld8_issue(ta + CO::DQR1 + m0, u[0]);
            umma::ld8_issue(ta + CO::DQR2 + m0, u[1]);
            umma::ld_wait();
            umma::take<8>(u[0], q1); umma::take<8>(u[1], q2);
          }
          float dl[8], dqv[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            dl[k] = 0.f;
            dqv[k] = 0.f;
          }
          if (own) {
            float qp[8];
            {
              const float4* q4 = reinterpret_cast<const float4*>(cache + (1 * C + i) * L::CS + m0);
              const float4 a = q4[0], b = q4[1];
              qp[0] = a.x; qp[1] = a.y; qp[2] = a.z; qp[3] = a.w; qp[4] = b.x; qp[5] = b.y; qp[6] = b.z; qp[7] = b.w;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int m = m0 + k;
              const float ell = ELL[i * L::CS + m];
              const float gqs = aik * q2[k];
              dqv[k] = p.q_scale * (q1[k] * ik + gqs) * ell;
              const float gq = gqs * qp[k] * ell;
              dl[k] = -fi * gq;
              asum += gq;
            }
          }
          if (owns_rows<RC>()) {
            float* d = PQ0 + i * KD;
            *reinterpret_cast<float4*>(d + swz(i, m0)) = make_float4(dqv[0], dqv[1], dqv[2], dqv[3]);
            *reinterpret_cast<float4*>(d + swz(i, m0 + 4)) = make_float4(dqv[4], dqv[5], dqv[6], dqv[7]);
          }
          if (p.lam) {
            const float x = warp_transpose_sum<8>(dl);
            if ((lane & 3) == 0) atomicAdd(&s_dlam[m0 + red_index<8>(lane)], x);
          }
        }
      }
      if (own && has_g) atomicAdd(&s_da[i], asum);
    }
    __syncthreads();
    // ---- key-side gradients out: 8 consecutive modes (dims) of one token per unit, coalesced;
    // warps 1..7 (warp 0 forms the per-token gradients below at the same time)
    if (warp > 0) {
      const bool gvec = flags & B_G_VEC;
      float* dk = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
      float* dq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
      for (int u = tid - 32; u < C * (KH / 8); u += NT - 32) {
        const int i = u / (KH / 8), m0 = (u % (KH / 8)) * 8;
        if (i >= Cl) continue;
        float y[8], z[8];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int o = i * KH + swz(i, m0 + 4 * hh);
          const float4 a = *reinterpret_cast<const float4*>(PK + o);
          float4 q = *reinterpret_cast<const float4*>(PQ0 + o);
          if (FL == SCA2_FLAVOR_PHASE) {
            const float4 q1 = *reinterpret_cast<const float4*>(PQ1 + o);
            q.x += q1.x; q.y += q1.y; q.z += q1.z; q.w += q1.w;
          }
          y[4 * hh] = a.x; y[4 * hh + 1] = a.y; y[4 * hh + 2] = a.z; y[4 * hh + 3] = a.w;
          z[4 * hh] = q.x; z[4 * hh + 1] = q.y; z[4 * hh + 2] = q.z; z[4 * hh + 3] = q.w;
        }
        if (gwrite) {
          float4* dk4 = reinterpret_cast<float4*>(dk + tok_off(gr.dphw, b, t0 + i, h) + m0);
          float4* dq4 = reinterpret_cast<float4*>(dq + tok_off(gr.dphq, b, t0 + i, h) + m0);
          dk4[0] = make_float4(y[0], y[1], y[2], y[3]);
          dk4[1] = make_float4(y[4], y[5], y[6], y[7]);
          dq4[0] = make_float4(z[0], z[1], z[2], z[3]);
          dq4[1] = make_float4(z[4], z[5], z[6], z[7]);
        } else {
          acc_row8(dk + tok_off(gr.dphw, b, t0 + i, h) + m0, y, gvec, excl, gstage ? GRW + i * KH + m0 : nullptr);
          acc_row8(dq + tok_off(gr.dphq, b, t0 + i, h) + m0, z, gvec, excl, gstage ? GRQ + i * KH + m0 : nullptr);
        }
      }
    }
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
  cp_wait_all();
  __syncthreads();
  // ---- incoming-state gradient and per-head gradients
  if (ok) {
    if (gr.dS0) {
#pragma unroll
      for (int k = 0; k < NS; ++k) gr.dS0[bhKV + (int64_t)s_m(k) * V + vb0 + s_v(k)] = dSreg[k];
    }
    if (p.lam) {  // state-side lambda terms: sum over the value rows (a lane's two rows, then the
                  // eight lanes sharing its column pairs)
#pragma unroll
      for (int g = 0; g < NS / 4; ++g) {
        float l0 = Lreg[4 * g] + Lreg[4 * g + 2], l1 = Lreg[4 * g + 1] + Lreg[4 * g + 3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          l0 += __shfl_xor_sync(0xffffffffu, l0, o);
          l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        if (lane < 4) {
          atomicAdd(&s_dlam[sm0 + 8 * g], l0);
          atomicAdd(&s_dlam[sm0 + 8 * g + 1], l1);
        }
      }
      __syncthreads();
    }
    for (int m = tid; m < KD; m += NT) {
      if (gr.dlam && p.lam) atomicAdd(&gr.dlam[h * KH + (m % KH)], s_dlam[m]);
      if (FL == SCA2_FLAVOR_PHASE && m < Mh) {
        if (gr.dwr) atomicAdd(&gr.dwr[h * Mh + m], s_dwr[m]);
        if (gr.dwi) atomicAdd(&gr.dwi[h * Mh + m], s_dwi[m]);
      }
    }
  } else {
    if (tid == 0) atomicOr(&g_fault_bwd, 1u);
    umma::mbar_wait(mbar, phase ^ 1u);
  }
  if (opend) umma::mbar_wait(obar, oph);  // bounded: a dO tile still in flight lands first
  umma::fence_before_sync();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tb, CO::ALLOC);
}

template <int FL, int R, bool HG>
auto bwd_kernel(bool pj) {
  if constexpr (FL == SCA2_FLAVOR_PHASE)
    return pj ? scan_bwd_tc<FL, R, HG, true> : scan_bwd_tc<FL, R, HG, false>;
  else
    return scan_bwd_tc<FL, R, HG, false>;
}

template <int FL, int R>
cudaError_t launch_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final, const float* cstates,
                       const sca2_scan_grads& gr, int NCS, int flags, const PhaseProj& pp, const CUtensorMap& omap,
                       int use_tma, cudaStream_t st) {
  const bool pj = pp.on != 0;
  auto k = p.g.ptr ? bwd_kernel<FL, R, true>(pj) : bwd_kernel<FL, R, false>(pj);
  const int smem = BwdLayout<FL, R>::TOTAL;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, p.V / BVB);
  k<<<grid, NT, smem, st>>>(p, dO, dS_final, cstates, gr, NCS, flags, pp, omap, use_tma);
  return cudaGetLastError();
}

}  // namespace tc

int tc_bwd_smem(int K, int R) {
  if (K != 64) return 1 << 30;
  return R == 2 ? tc::BwdLayout<SCA2_FLAVOR_PHASE, 2>::TOTAL : tc::BwdLayout<SCA2_FLAVOR_KEY, 1>::TOTAL;
}

// read and clear the backward's device fault word (synchronous)
cudaError_t tc_read_faults_bwd(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, tc::g_fault_bwd, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(tc::g_fault_bwd, &zero, sizeof(unsigned int));
}

// Whether a bf16 training pass (forward with saved chunk data + backward) runs on the tensor
// cores: K = 64, V a multiple of 64, both kernels within the shared-memory limit.  The decision
// depends on the arguments shared by the forward and the backward only, so the pair agrees.
bool tc_train_ok(const sca2_scan_args& p, int max_smem) {
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  return p.io_dtype == SCA2_BF16 && p.K == 64 && p.V % 64 == 0 && tc_bwd_smem(64, R) <= max_smem;
}

// phase_cp.cu: the tensor map of the dO tiles (phase flavour)
bool dO_tile_map(const sca2_scan_args& p, const sca2_out& dO, CUtensorMap* map);

cudaError_t tc_scan_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final, const float* cstates,
                        const sca2_scan_grads& gr, int NCS, cudaStream_t st, const PhaseProj& pp) {
  auto a16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
  int f = 0;
  if (p.flavor == SCA2_FLAVOR_PHASE && a16(p.phw.ptr) && a16(p.phq.ptr) && p.phw.sb % 4 == 0 &&
      p.phw.st % 4 == 0 && p.phw.sh % 4 == 0 && p.phq.sb % 4 == 0 && p.phq.st % 4 == 0 && p.phq.sh % 4 == 0)
    f |= tc::B_PH_VEC;
  if (p.flavor == SCA2_FLAVOR_KEY && a16(p.phw.ptr) && a16(p.phq.ptr) && p.phw.sb % 8 == 0 &&
      p.phw.st % 8 == 0 && p.phw.sh % 8 == 0 && p.phq.sb % 8 == 0 && p.phq.st % 8 == 0 && p.phq.sh % 8 == 0)
    f |= tc::B_K_VEC;
  if (a16(dO.ptr) && dO.sb % 8 == 0 && dO.st % 8 == 0 && dO.sh % 8 == 0 && dO.sr % 8 == 0) f |= tc::B_DO_VEC;
  if (a16(gr.dv.ptr) && gr.dv.sb % 8 == 0 && gr.dv.st % 8 == 0 && gr.dv.sh % 8 == 0) f |= tc::B_DV_VEC;
  if (a16(gr.dphw.ptr) && a16(gr.dphq.ptr) && gr.dphw.sb % 4 == 0 && gr.dphw.st % 4 == 0 && gr.dphw.sh % 4 == 0 &&
      gr.dphq.sb % 4 == 0 && gr.dphq.st % 4 == 0 && gr.dphq.sh % 4 == 0)
    f |= tc::B_G_VEC;
  if (gr.overwrite && p.V == tc::BVB && (f & tc::B_G_VEC)) f |= tc::B_OVERWRITE;
  // phase flavour: the dO tile of every full chunk by TMA where the map can address dO
  alignas(64) CUtensorMap omap;
  memset(&omap, 0, sizeof(omap));
  const int use_tma = (p.flavor == SCA2_FLAVOR_PHASE && dO_tile_map(p, dO, &omap)) ? 1 : 0;
  if (p.flavor == SCA2_FLAVOR_PHASE)
    return tc::launch_bwd<SCA2_FLAVOR_PHASE, 2>(p, dO, dS_final, cstates, gr, NCS, f, pp, omap, use_tma, st);
  return tc::launch_bwd<SCA2_FLAVOR_KEY, 1>(p, dO, dS_final, cstates, gr, NCS, f, pp, omap, 0, st);
}

}  // namespace sca2
