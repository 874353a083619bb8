// Chunk-parallel training forward of the phase-coded scan at K = 2 Mh = 64, V = 64, bf16 values,
// fp32 state (sm_100a): the LapA long head / CHeadDeltaDamp / CHeadGated form (per-mode decay
// lam, erase gate beta, scalar log-decay g, R = 2 read rows).
//
// The one-CTA-per-sequence walk leaves each 64-token chunk's work (codes, Gram, inversion,
// a dozen dependent products) exposed as latency on one SM.  Here the chunk algebra is
// regrouped so that only one small product per chunk stays sequential:
//
//   chunk c, tokens i, j < 64, modes m (k = [cos phi ; sin phi], kappa = Mh), S = state entering:
//     G   = (kr kw^T / kappa) .* Dg,  kr = k e^{-lam i},  kw = k e^{+lam i}
//     T   = (I + diag(beta) G_strict)^{-1}
//     W'  = T Z,   Z = diag(beta a / kappa) k e^{-lam (i+1)}        (so E = U - W' S)
//     U   = T v
//     Kc  = diag(w) k e^{-lam (Cl-1-i)},   d = a_last e^{-lam Cl}
//     S'  = d .* S - M S + B,   M = Kc^T W',   B = Kc^T U          (the only sequential step)
//     O_r = Qa_r S + P_r E,    E = T (v - Z S),   P_r = (qr_r kw^T / kappa) .* Dg (incl.),
//           qr = Q e^{-lam i},  Qa = diag(a / kappa) Q e^{-lam (i+1)}
//
// which is the reference's chunk closed form (lapa/layer.py:298-366 with the scalar-decay mask
// of sca2/arch_gatedc.py:136-139), with its state loop rewritten as S' = A S + B.  Three kernels:
//
//   pcp_prep   one CTA per (b, h, chunk), three per SM: codes, G (tcgen05), the fp32 inversion,
//              W' and U (tcgen05), M and B (tcgen05).  Writes T to slot 2c+1, B to slot 2c and
//              M (bf16, operand layout) with d to slot 3 NC + c.
//   pcp_state  one CTA of 4 warps per (b, h, 32 value columns), sequential over chunks: the
//              state in fp32 registers, M S as one tcgen05 product per chunk with the state
//              split hi + lo (stacked along N), the M, B, d of the chunk two ahead copied in
//              meanwhile.  Writes the state
//              entering chunk c over B_c in slot 2c, and the final state.
//   pcp_out    one CTA per (b, h, chunk), two per SM: E = T (v - Z S) and O = Qa S + P E
//              (tcgen05), the outputs, and E^T and P (hi parts) for the backward (slot 2c+1
//              after T, slot 2 NC + c) in the layout the tensor-core backward reads.
//
// Precision: every MMA accumulates in fp32; the state is carried in fp32 and enters its
// products as a hi + lo bf16 pair; so do, for the reads, the codes of P, P and E in P E, Qa, and
// v - Z S, and, for the state's inputs, U and Kc (the pair's three products hi*hi + hi*lo +
// lo*hi keep about 16 mantissa bits); T, Z, W' and M are single bf16.  A float64 emulation of
// exactly these roundings at the benchmark shape (B = 8, T = 4096, H = 16, Mh = 32, V = 64) gives
// a max-abs error of 0.9e-2 on the unit-RMS outputs of the checked sequences, against 1.8e-2
// with every chunk operand single bf16 (the bar is 2e-2).
// Every mbarrier wait is bounded; on a timeout the CTA sets a fault bit, drains its products
// and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "tc_common.cuh"

namespace sca2 {
namespace pcp {

using tc::C;
using tc::LDF;
using tc::NT;
using tc::Gates;
using tc::bf16;

constexpr int KD = 64, VD = 64, MH = 32, KV = KD * VD;
constexpr int VBS = 32;   // value columns per CTA of the state recurrence
constexpr int NTS = 128;  // threads per CTA of the state recurrence

// bit 0: a bounded mbarrier wait of a chunk-parallel phase kernel timed out
__device__ unsigned int g_fault_pcp;

__device__ __forceinline__ float* slot(float* cs, int bh, int NS, int s) { return cs + ((int64_t)bh * NS + s) * KV; }

// bounded wait on a batch; false (in every thread) after a timeout, with the fault bit set
__device__ __forceinline__ bool batch_wait(uint64_t* mbar, uint32_t parity) {
  const bool ok = umma::mbar_wait(mbar, parity);
  const bool bad = __syncthreads_or(!ok) != 0;
  umma::fence_after_sync();
  if (bad && threadIdx.x == 0) atomicOr(&g_fault_pcp, 1u);
  return !bad;
}

__device__ __forceinline__ void copy16(uint8_t* dst, const uint8_t* src, int nbytes, int nthr) {
  for (int u = threadIdx.x * 16; u < nbytes; u += nthr * 16)
    *reinterpret_cast<uint4*>(dst + u) = *reinterpret_cast<const uint4*>(src + u);
}

// per-head constants: lam per key row (cos and sin halves share a mode's lam), wr, wi per mode
__device__ __forceinline__ void load_head(const sca2_scan_args& p, int h, float* s_lam, float* s_wr, float* s_wi) {
  for (int m = threadIdx.x; m < KD; m += blockDim.x) {
    s_lam[m] = p.lam ? p.lam[h * MH + (m % MH)] : 0.f;
    if (s_wr && m < MH) {
      s_wr[m] = p.wr[h * MH + m];
      s_wi[m] = p.wi[h * MH + m];
    }
  }
}

// ======================================================================================
//  pcp_prep: T, M, B, d of every chunk
// ======================================================================================
// Region A holds the codes of the Gram product, then the inversion's input L, then W' and U
// (bf16); the lo parts of U and Kc go over Z and the values once W' and U are formed; about
// 71 KB in all, three CTAs per SM; 128 TMEM columns.
struct PrepL {
  static constexpr int A = 0;                      // KR | KW (bf16 C x KD each) -> LS -> WP | UB
  static constexpr int A_BYTES = C * LDF * 4;      // 17408 >= 2 * 8192
  static constexpr int KR = A, KW = A + C * KD * 2, LS = A, WP = A, UB = A + C * KD * 2;
  static constexpr int ZA = A + A_BYTES;           // C x KD  Z = beta a k e^{-lam (i+1)} / kappa [i][m]
  static constexpr int KC = ZA + C * KD * 2;       // C x KD  Kc [j][m]
  static constexpr int VA = KC + C * KD * 2;       // C x VD  values [j][v]
  static constexpr int TB = VA + C * VD * 2;       // C x C   T (bf16) [i][j]
  static constexpr int UBL = ZA, KCL = VA;         // after W', U: U lo over Z, Kc lo over the values
  static constexpr int TS = TB + C * C * 2;        // fp32 C x LDF
  static constexpr int WS = TS + C * LDF * 4;      // fp32 1024
  static constexpr int SC = WS + 1024 * 4;         // beta, Gc, a, w [C], lam [KD], decay factors [C]
  static constexpr int MBAR = SC + (5 * C + KD) * 4;  // batch mbarrier, TMEM base, value-tile mbarrier
  static constexpr int TOTAL = MBAR + 32;
  static_assert(2 * C * KD * 2 <= A_BYTES, "KR and KW fit region A");
  static_assert(TOTAL <= 74 * 1024, "three CTAs per SM");
};

__global__ void __launch_bounds__(NT, 3) pcp_prep(sca2_scan_args p, float* cs, int NS, int flags, PhaseProj pp,
                                                  const __grid_constant__ CUtensorMap vmap, int use_tma) {
  using L = PrepL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  const bool has_g = p.g.ptr != nullptr;
  constexpr float ik = 1.f / (float)MH;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* s_lam = sc + 4 * C;
  float* s_fdec = s_lam + KD;  // column factors of the decay mask (tc::decay_block)
  bf16* KR = reinterpret_cast<bf16*>(sm + L::KR);
  bf16* KW = reinterpret_cast<bf16*>(sm + L::KW);
  bf16* ZA = reinterpret_cast<bf16*>(sm + L::ZA);
  bf16* KC = reinterpret_cast<bf16*>(sm + L::KC);
  bf16* VA = reinterpret_cast<bf16*>(sm + L::VA);
  bf16* TB = reinterpret_cast<bf16*>(sm + L::TB);
  bf16* WP = reinterpret_cast<bf16*>(sm + L::WP);
  bf16* UB = reinterpret_cast<bf16*>(sm + L::UB);
  bf16* UBL = reinterpret_cast<bf16*>(sm + L::UBL);
  bf16* KCL = reinterpret_cast<bf16*>(sm + L::KCL);
  float* LS = reinterpret_cast<float*>(sm + L::LS);
  float* TS = reinterpret_cast<float*>(sm + L::TS);
  float* WS = reinterpret_cast<float*>(sm + L::WS);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  uint64_t* vbar = reinterpret_cast<uint64_t*>(sm + L::MBAR + 16);
  const bool tma = use_tma && Cl == C;  // full chunks take the value tile by TMA

  load_head(p, h, s_lam, nullptr, nullptr);
  if (warp == 0) {
    tc::GateRegs gr;
    tc::load_gate_regs(p, gr, b, h, t0, Cl);
    tc::gates_from_regs(gr, gt, Cl);
    if (has_g) tc::decay_factors_warp(gt.Gc, s_fdec);
  }
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::mbar_init(vbar, 1);
    umma::fence_mbar_init();
    if (tma) tc::tma_value_tile<VD>(VA, &vmap, b * p.T + t0, h, vbar);
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 128);
  if (!tma) tc::pf_values<VD>(p, VA, flags & tc::F_V_VEC, b, h, t0, Cl, 0);
  tc::cp_commit();
  tc::CodeRegs<SCA2_FLAVOR_PHASE, KD> cr;
  tc::load_code_regs<SCA2_FLAVOR_PHASE, KD>(p, cr, flags & tc::F_PH_VEC, b, h, t0, Cl, pp);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  int ui, um0;  // this thread's code unit: token ui, modes um0 .. um0 + 7
  tc::code_unit<KD / 16>(tid, ui, um0);
  float cc[8], cs8[8];  // its Kc values (cos, sin halves), kept for the lo part
  tc::finish_code_regs<SCA2_FLAVOR_PHASE, KD>(cr, pp, h, t0, Cl);
  {  // codes
    const int i = ui, m0 = um0;
    const float fi = (float)i;
    const float zb = gt.beta[i] * gt.a[i] * ik, wv = gt.w[i];
    float kc[8], ks[8], wc[8], ws[8], zc[8], zs[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float s = 0.f, co = 0.f;
      if (i < Cl) sincos_big(cr.w[0][k], &s, &co);
      const float l = s_lam[m0 + k];
      const float ell = __expf(-l * fi), elli = __expf(l * fi);
      const float el1 = __expf(-l * (fi + 1.f)), ec = wv * __expf(-l * (float)(Cl - 1 - i));
      kc[k] = co * ell; ks[k] = s * ell; wc[k] = co * elli; ws[k] = s * elli;
      zc[k] = zb * co * el1; zs[k] = zb * s * el1;
      cc[k] = ec * co; cs8[k] = ec * s;
    }
    tc::st8(KR, umma::kmaj(i, m0, KD), kc);
    tc::st8(KR, umma::kmaj(i, MH + m0, KD), ks);
    tc::st8(KW, umma::kmaj(i, m0, KD), wc);
    tc::st8(KW, umma::kmaj(i, MH + m0, KD), ws);
    tc::st8(ZA, umma::kmaj(i, m0, KD), zc);
    tc::st8(ZA, umma::kmaj(i, MH + m0, KD), zs);
    tc::st8(KC, umma::kmaj(i, m0, KD), cc);
    tc::st8(KC, umma::kmaj(i, MH + m0, KD), cs8);
  }
  tc::cp_wait_all();
  bool ok = !tma || batch_wait(vbar, 0);
  const bool tma_pending = tma && !ok;  // the tile copy must land before the CTA leaves
  int inflight = -1;                    // parity of a batch issued and not yet waited for
  tc::publish_smem();
  if (ok && tid == 0) {
    umma::gemm(tb, KR, KW, 64, 64, KD, false);  // G = KR KW^T
    umma::commit(mbar);
  }
  if (ok) {
    inflight = 0;
    if ((ok = batch_wait(mbar, 0))) inflight = -1;
  }
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int i, int j0, int, const float* x) {  // L = beta G .* Dg, strict
      const float bi = gt.beta[i] * ik;
      float dg[16];
      if (has_g) tc::decay_block(gt.Gc, s_fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
    });
    __syncthreads();
    tc::invert_unit_lower(LS, TS, WS);
    tc::store_T<false>(TS, TB);
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, TB, false, ZA, true, 64, KD, C, false);       // W' = T Z      [i][m]
      umma::gemm_t(tb + 64, TB, false, VA, true, 64, VD, C, false);  // U  = T v      [i][v]
      umma::commit(mbar);
    }
    copy16(reinterpret_cast<uint8_t*>(slot(cs, bh, NS, 2 * c + 1)), reinterpret_cast<const uint8_t*>(TB),
           C * C * 2, NT);
    inflight = 1;
    if ((ok = batch_wait(mbar, 1))) inflight = -1;
  }
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int i, int m0, int, const float* x) {
      tc::st8(WP, umma::kmaj(i, m0, KD), x);
      tc::st8(WP, umma::kmaj(i, m0 + 8, KD), x + 8);
    });
    tc::for_frag<64, 64>(tb + 64, [&](int i, int v0, int, const float* x) {  // U as hi + lo
      tc::st8_split(UB, UBL, umma::kmaj(i, v0, VD), x);
      tc::st8_split(UB, UBL, umma::kmaj(i, v0 + 8, VD), x + 8);
    });
    {  // Kc's lo part (the values' region is free)
      float l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) l[k] = cc[k] - __bfloat162float(__float2bfloat16_rn(cc[k]));
      tc::st8(KCL, umma::kmaj(ui, um0, KD), l);
#pragma unroll
      for (int k = 0; k < 8; ++k) l[k] = cs8[k] - __bfloat162float(__float2bfloat16_rn(cs8[k]));
      tc::st8(KCL, umma::kmaj(ui, MH + um0, KD), l);
    }
    tc::publish_smem();
    if (tid == 0) {  // M = Kc^T W' [m][m'],  B = Kc^T U [m][v]  (Kc and U split hi + lo)
      umma::gemm_t(tb, KC, true, WP, true, KD, KD, C, false);
      umma::gemm_t(tb, KCL, true, WP, true, KD, KD, C, true);
      umma::gemm_t(tb + 64, KC, true, UB, true, KD, VD, C, false);
      umma::gemm_t(tb + 64, KC, true, UBL, true, KD, VD, C, true);
      umma::gemm_t(tb + 64, KCL, true, UB, true, KD, VD, C, true);
      umma::commit(mbar);
    }
    inflight = 0;
    if ((ok = batch_wait(mbar, 0))) inflight = -1;
  }
  if (ok) {
    bf16* Mg = reinterpret_cast<bf16*>(slot(cs, bh, NS, 3 * NC + c));
    float* Bg = slot(cs, bh, NS, 2 * c);
    tc::for_frag<64, 64>(tb, [&](int m, int j0, int, const float* x) {
      tc::st8(Mg, umma::kmaj(m, j0, KD), x);
      tc::st8(Mg, umma::kmaj(m, j0 + 8, KD), x + 8);
    });
    tc::for_frag<64, 64>(tb + 64, [&](int m, int v0, int, const float* x) {
      float4* dst = reinterpret_cast<float4*>(Bg + m * VD + v0);
#pragma unroll
      for (int k = 0; k < 4; ++k) dst[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
    });
    if (tid < KD) {  // d = a_last e^{-lam Cl}, after M in the same slot
      float* dg = slot(cs, bh, NS, 3 * NC + c) + KD * KD / 2;
      dg[tid] = gt.a[Cl - 1] * expf(-s_lam[tid] * (float)Cl);
    }
  }
  // after a timeout: bounded waits for what is still in flight before TMEM and shared memory go
  if (inflight >= 0) umma::mbar_wait(mbar, (uint32_t)inflight);
  if (tma_pending) umma::mbar_wait(vbar, 0);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 128);
}

// ======================================================================================
//  pcp_state: S' = d .* S - M S + B over the chunks of one (b, h, 32 value columns)
// ======================================================================================
// NSTG stages of (M, B, d): chunk c + 2 is copied in while chunk c runs, so a copy has two
// chunk steps to arrive.  The state enters its product as [S hi | S lo] stacked along N (one
// 64 x 64 x 64 product, the two halves summed after), the B rows are padded by 4 floats (rows
// of 8 consecutive key rows fall in distinct bank groups), and the issuing thread does not
// take part in the copies (it is on the chain's critical path).
constexpr int NSTG = 3;
constexpr int BSR = VBS + 4;  // padded fp32 row of a stage's B
struct StateL {
  static constexpr int MA = 0;                          // NSTG x M (bf16 KD x KD, operand layout)
  static constexpr int BS = MA + NSTG * KD * KD * 2;    // NSTG x B (fp32 KD x BSR)
  static constexpr int SB = BS + NSTG * KD * BSR * 4;   // [S hi | S lo] (bf16 [m][2 VBS], read MN-major)
  static constexpr int DS = SB + KD * 2 * VBS * 2;      // NSTG x d [KD]
  static constexpr int MBAR = DS + NSTG * KD * 4;
  static constexpr int TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NTS) pcp_state(sca2_scan_args p, float* cs, int NS, float* S_final) {
  using L = StateL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, vb0 = blockIdx.y * VBS;
  const int NC = (p.T + C - 1) / C;
  bf16* SB = reinterpret_cast<bf16*>(sm + L::SB);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  // rows of the M = 64 accumulator: warp w's sub-partition, lanes < 16 hold rows 16 w + lane
  const bool own = lane < 16;
  const int m = 16 * warp + (lane & 15);

  // copy chunk cc's M, B (this CTA's columns) and d into stage cc % NSTG, spread over threads
  // 1..NTS-1; every thread commits one group per call (empty past the last chunk or for the
  // issuing thread) so that the wait_group counts stay uniform
  auto prefetch = [&](int cc) {
    if (cc < NC && tid > 0) {
      const int st = cc % NSTG, w = tid - 1;
      constexpr int NW = NTS - 1;
      const uint8_t* mg = reinterpret_cast<const uint8_t*>(slot(cs, bh, NS, 3 * NC + cc));
      uint8_t* ma = sm + L::MA + st * KD * KD * 2;
      for (int u = w; u < KD * KD * 2 / 16; u += NW) tc::cp16(ma + 16 * u, mg + 16 * u, true);
      const float* bg = slot(cs, bh, NS, 2 * cc) + vb0;
      float* bs = reinterpret_cast<float*>(sm + L::BS) + st * KD * BSR;
      for (int u = w; u < KD * VBS / 4; u += NW) {
        const int r = u / (VBS / 4), c4 = (u % (VBS / 4)) * 4;
        tc::cp16(bs + r * BSR + c4, bg + r * VD + c4, true);
      }
      if (w < KD / 4) tc::cp16(sm + L::DS + st * KD * 4 + 16 * w, mg + KD * KD * 2 + 16 * w, true);
    }
    tc::cp_commit();
  };

  float S[VBS];
  const int64_t srow = ((int64_t)bh * KD + m) * VD + vb0;
#pragma unroll
  for (int j = 0; j < VBS; ++j) S[j] = (own && p.S0) ? p.S0[srow + j] : 0.f;
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 2 * VBS);
  for (int k = 0; k < NSTG - 1; ++k) prefetch(k);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  uint32_t phase = 0;
  bool ok = true;
  for (int c = 0; c < NC; ++c) {
    const int st = c % NSTG;
    tc::cp_wait_group<NSTG - 2>();  // this thread's copies of chunk c have landed
    if (own)
#pragma unroll
      for (int v0 = 0; v0 < VBS; v0 += 8) {
        float h[8], l[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          h[k] = __bfloat162float(__float2bfloat16_rn(S[v0 + k]));
          l[k] = S[v0 + k] - h[k];
        }
        tc::st8(SB, umma::kmaj(m, v0, 2 * VBS), h);
        tc::st8(SB, umma::kmaj(m, VBS + v0, 2 * VBS), l);
      }
    tc::publish_smem();  // every thread's copies of chunk c and its S operand are visible
    if (tid == 0) {
      const bf16* ma = reinterpret_cast<const bf16*>(sm + L::MA + st * KD * KD * 2);
      umma::gemm_t(tb, ma, false, SB, true, KD, 2 * VBS, KD, false);  // M [S hi | S lo]
      umma::commit(mbar);
    }
    if (own) {
      // the state entering chunk c replaces B_c in slot 2c: every copy of B_c has landed (above)
      float4* dst = reinterpret_cast<float4*>(slot(cs, bh, NS, 2 * c) + m * VD + vb0);
#pragma unroll
      for (int k = 0; k < VBS / 4; ++k) dst[k] = make_float4(S[4 * k], S[4 * k + 1], S[4 * k + 2], S[4 * k + 3]);
    }
    prefetch(c + NSTG - 1);  // into the stage of chunk c - 1, whose reads ended before the barrier
    if (!(ok = batch_wait(mbar, phase))) break;
    phase ^= 1u;
    uint32_t r[4][16];
#pragma unroll
    for (int q = 0; q < 4; ++q) umma::ld16_issue(umma::taddr(tb, 32 * warp, 16 * q), r[q]);
    umma::ld_wait();
    float x[2 * VBS];
#pragma unroll
    for (int q = 0; q < 4; ++q) umma::take<16>(r[q], x + 16 * q);
    if (own) {
      const float d = reinterpret_cast<const float*>(sm + L::DS)[st * KD + m];
      const float4* bs = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sm + L::BS) +
                                                         st * KD * BSR + m * BSR);
#pragma unroll
      for (int k = 0; k < VBS / 4; ++k) {
        const float4 b4 = bs[k];
        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 4 * k + e;
          S[j] = fmaf(d, S[j], bb[e] - (x[j] + x[VBS + j]));
        }
      }
    }
    umma::fence_before_sync();
  }
  tc::cp_wait_all();
  if (!ok) umma::mbar_wait(mbar, phase);  // bounded drain of the product in flight
  if (ok && own && S_final) {
    float4* dst = reinterpret_cast<float4*>(S_final + srow);
#pragma unroll
    for (int k = 0; k < VBS / 4; ++k) dst[k] = make_float4(S[4 * k], S[4 * k + 1], S[4 * k + 2], S[4 * k + 3]);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 2 * VBS);
}

// ======================================================================================
//  pcp_out: outputs of every chunk from the state entering it
// ======================================================================================
struct OutL {
  // regions (bytes); later tenants follow the arrow once the earlier one is dead
  static constexpr int SH = 0;                     // S hi, lo (bf16 [m][v], read MN-major)
  static constexpr int SL = SH + KD * VD * 2;
  static constexpr int ZA = SL + KD * VD * 2;      // Z [i][m]                    -> E^T hi [v][j]
  static constexpr int QR = ZA + C * KD * 2;       // qr hi, lo [(r,i)][m]        -> P hi, lo [(r,i)][j]
  static constexpr int QRL = QR + 2 * C * KD * 2;
  static constexpr int KW = QRL + 2 * C * KD * 2;  // kw hi, lo [j][m]            -> Y hi, lo [j][v] -> Qa hi
  static constexpr int KWL = KW + C * KD * 2;
  static constexpr int VA = KWL + C * KD * 2;      // values [j][v]               -> E^T lo
  static constexpr int TB = VA + C * VD * 2;       // T [i][j]                    -> Qa lo (with the next 8 KB)
  static constexpr int XR = TB + C * C * 2;        // (8 KB, second half of Qa lo)
  static constexpr int EB = ZA, EL = VA, PB = QR, PL = QRL, YB = KW, YL = KWL, QA = KW, QAL = TB;
  static constexpr int SC = XR + C * KD * 2;       // beta, Gc, a, w [C], lam [KD], wr, wi [MH], decay factors [C]
  static constexpr int MBAR = SC + (5 * C + KD + 2 * MH) * 4;  // batch mbarrier, TMEM base, value-tile mbarrier
  static constexpr int TOTAL = MBAR + 32;
  static_assert(2 * C * KD * 2 == 2 * C * C * 2, "P hi / lo take the places of qr hi / lo");
  static_assert(TOTAL <= 113 * 1024, "two CTAs per SM");
};

__global__ void __launch_bounds__(NT, 2) pcp_out(sca2_scan_args p, sca2_out o, float* cs, int NS, int flags,
                                                 PhaseProj pp, const __grid_constant__ CUtensorMap vmap, int use_tma) {
  using L = OutL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  const bool has_g = p.g.ptr != nullptr;
  constexpr float ik = 1.f / (float)MH;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* s_lam = sc + 4 * C;
  float* s_wr = s_lam + KD;
  float* s_wi = s_wr + MH;
  float* s_fdec = s_wi + MH;  // column factors of the decay mask (tc::decay_block)
  bf16* SH = reinterpret_cast<bf16*>(sm + L::SH);
  bf16* SL = reinterpret_cast<bf16*>(sm + L::SL);
  bf16* ZA = reinterpret_cast<bf16*>(sm + L::ZA);
  bf16* KW = reinterpret_cast<bf16*>(sm + L::KW);
  bf16* KWL = reinterpret_cast<bf16*>(sm + L::KWL);
  bf16* QR = reinterpret_cast<bf16*>(sm + L::QR);
  bf16* QRL = reinterpret_cast<bf16*>(sm + L::QRL);
  bf16* YB = reinterpret_cast<bf16*>(sm + L::YB);
  bf16* YL = reinterpret_cast<bf16*>(sm + L::YL);
  bf16* PB = reinterpret_cast<bf16*>(sm + L::PB);
  bf16* PL = reinterpret_cast<bf16*>(sm + L::PL);
  bf16* VA = reinterpret_cast<bf16*>(sm + L::VA);
  bf16* EB = reinterpret_cast<bf16*>(sm + L::EB);
  bf16* EL = reinterpret_cast<bf16*>(sm + L::EL);
  bf16* TB = reinterpret_cast<bf16*>(sm + L::TB);
  bf16* QA = reinterpret_cast<bf16*>(sm + L::QA);
  bf16* QAL = reinterpret_cast<bf16*>(sm + L::QAL);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  uint64_t* vbar = reinterpret_cast<uint64_t*>(sm + L::MBAR + 16);
  const bool tma = use_tma && Cl == C;  // full chunks take the value tile by TMA

  load_head(p, h, s_lam, s_wr, s_wi);
  if (warp == 0) {
    tc::GateRegs gr;
    tc::load_gate_regs(p, gr, b, h, t0, Cl);
    tc::gates_from_regs(gr, gt, Cl);
    if (has_g) tc::decay_factors_warp(gt.Gc, s_fdec);
  }
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::mbar_init(vbar, 1);
    umma::fence_mbar_init();
    if (tma) tc::tma_value_tile<VD>(VA, &vmap, b * p.T + t0, h, vbar);
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 128);
  if (!tma) tc::pf_values<VD>(p, VA, flags & tc::F_V_VEC, b, h, t0, Cl, 0);
  {
    const uint8_t* tg = reinterpret_cast<const uint8_t*>(slot(cs, bh, NS, 2 * c + 1));
    for (int u = tid; u < C * C * 2 / 16; u += NT) tc::cp16(reinterpret_cast<uint8_t*>(TB) + 16 * u, tg + 16 * u, true);
  }
  tc::cp_commit();
  {  // the state entering the chunk (fp32, slot 2c) -> hi + lo bf16; 8 lanes take 8 rows
    const float* sg = slot(cs, bh, NS, 2 * c);
#pragma unroll
    for (int k = 0; k < KD * VD / 8 / NT; ++k) {
      const int u = tid + k * NT;
      const int mm = (u & 7) + 8 * (u / 64), v0 = ((u >> 3) & 7) * 8;
      const float4 a0 = reinterpret_cast<const float4*>(sg + mm * VD + v0)[0];
      const float4 a1 = reinterpret_cast<const float4*>(sg + mm * VD + v0)[1];
      const float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      tc::st8_split(SH, SL, umma::kmaj(mm, v0, VD), x);
    }
  }
  tc::CodeRegs<SCA2_FLAVOR_PHASE, KD> cr;
  tc::load_code_regs<SCA2_FLAVOR_PHASE, KD>(p, cr, flags & tc::F_PH_VEC, b, h, t0, Cl, pp);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  int ci, cm0;
  tc::code_unit<KD / 16>(tid, ci, cm0);
  float q1[8], q2[8];  // read columns c1, c2 of this thread's (token, 8 modes), kept for Qa
  tc::finish_code_regs<SCA2_FLAVOR_PHASE, KD>(cr, pp, h, t0, Cl);
  {
    const float fi = (float)ci;
    const float zb = gt.beta[ci] * gt.a[ci] * ik;
    float wc[8], ws[8], zc[8], zs[8], r0a[8], r0b[8], r1a[8], r1b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float s = 0.f, co = 0.f, sq = 0.f, cq = 0.f;
      if (ci < Cl) {
        sincos_big(cr.w[0][k], &s, &co);
        sincos_big(cr.q[0][k], &sq, &cq);
      }
      const float l = s_lam[cm0 + k];
      const float ell = __expf(-l * fi), elli = __expf(l * fi), el1 = __expf(-l * (fi + 1.f));
      const float wr = s_wr[cm0 + k], wi = s_wi[cm0 + k];
      q1[k] = wr * cq + wi * sq;
      q2[k] = wr * sq - wi * cq;
      wc[k] = co * elli; ws[k] = s * elli;
      zc[k] = zb * co * el1; zs[k] = zb * s * el1;
      r0a[k] = q1[k] * ell; r0b[k] = q2[k] * ell; r1a[k] = -q2[k] * ell; r1b[k] = q1[k] * ell;
    }
    tc::st8_split(KW, KWL, umma::kmaj(ci, cm0, KD), wc);
    tc::st8_split(KW, KWL, umma::kmaj(ci, MH + cm0, KD), ws);
    tc::st8(ZA, umma::kmaj(ci, cm0, KD), zc);
    tc::st8(ZA, umma::kmaj(ci, MH + cm0, KD), zs);
    tc::st8_split(QR, QRL, umma::kmaj(ci, cm0, KD), r0a);
    tc::st8_split(QR, QRL, umma::kmaj(ci, MH + cm0, KD), r0b);
    tc::st8_split(QR, QRL, umma::kmaj(C + ci, cm0, KD), r1a);
    tc::st8_split(QR, QRL, umma::kmaj(C + ci, MH + cm0, KD), r1b);
  }
  tc::cp_wait_all();
  bool ok = !tma || batch_wait(vbar, 0);
  const bool tma_pending = tma && !ok;  // the tile copy must land before the CTA leaves
  int inflight = -1;                    // parity of a batch issued and not yet waited for
  tc::publish_smem();
  if (ok && tid == 0) {
    umma::gemm_t(tb, ZA, false, SH, true, 64, VD, KD, false);  // X0 = Z S  [i][v]
    umma::gemm_t(tb, ZA, false, SL, true, 64, VD, KD, true);
    umma::gemm(tb + 64, QR, KW, 2 * 64, C, KD, false);        // P = qr kw^T [(r,i)][j] (codes hi + lo)
    umma::gemm(tb + 64, QR, KWL, 2 * 64, C, KD, true);
    umma::gemm(tb + 64, QRL, KW, 2 * 64, C, KD, true);
    umma::commit(mbar);
  }
  if (ok) {
    inflight = 0;
    if ((ok = batch_wait(mbar, 0))) inflight = -1;
  }
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int i, int v0, int, const float* x) {  // Y = v - X0
      float vv[16];
      tc::ld8_bf16(VA, umma::kmaj(i, v0, VD), vv);
      tc::ld8_bf16(VA, umma::kmaj(i, v0 + 8, VD), vv + 8);
#pragma unroll
      for (int j = 0; j < 16; ++j) vv[j] -= x[j];
      tc::st8_split(YB, YL, umma::kmaj(i, v0, VD), vv);
      tc::st8_split(YB, YL, umma::kmaj(i, v0 + 8, VD), vv + 8);
    });
    tc::for_frag<2 * 64, 64>(tb + 64, [&](int row, int j0, int, const float* x) {  // P masked, decayed
      const int i = row & 63;
      float y[16], dg[16];
      if (has_g) tc::decay_block(gt.Gc, s_fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        y[j] = jj <= i ? x[j] * ik * (has_g ? dg[j] : 1.f) : 0.f;
      }
      tc::st8_split(PB, PL, umma::kmaj(row, j0, C), y);
      tc::st8_split(PB, PL, umma::kmaj(row, j0 + 8, C), y + 8);
    });
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, YB, true, TB, false, VD, C, C, false);  // E^T = Y^T T^T  [v][i]  (Y hi + lo)
      umma::gemm_t(tb, YL, true, TB, false, VD, C, C, true);
      umma::commit(mbar);
    }
    // P for the backward (slot 2 NC + c), while E^T is computed
    copy16(reinterpret_cast<uint8_t*>(slot(cs, bh, NS, 2 * NC + c)), reinterpret_cast<const uint8_t*>(PB),
           2 * C * C * 2, NT);
    inflight = 1;
    if ((ok = batch_wait(mbar, 1))) inflight = -1;
  }
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int v, int i0, int, const float* x) {
      tc::st8_split(EB, EL, umma::kmaj(v, i0, C), x);
      tc::st8_split(EB, EL, umma::kmaj(v, i0 + 8, C), x + 8);
    });
    {  // Qa = (a / kappa) Q e^{-lam (i+1)} (hi + lo) over Y and T (both dead)
      const float fa = gt.a[ci] * ik, fi = (float)ci;
      float r0a[8], r0b[8], r1a[8], r1b[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float e = fa * __expf(-s_lam[cm0 + k] * (fi + 1.f));
        r0a[k] = q1[k] * e; r0b[k] = q2[k] * e; r1a[k] = -q2[k] * e; r1b[k] = q1[k] * e;
      }
      tc::st8_split(QA, QAL, umma::kmaj(ci, cm0, KD), r0a);
      tc::st8_split(QA, QAL, umma::kmaj(ci, MH + cm0, KD), r0b);
      tc::st8_split(QA, QAL, umma::kmaj(C + ci, cm0, KD), r1a);
      tc::st8_split(QA, QAL, umma::kmaj(C + ci, MH + cm0, KD), r1b);
    }
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb + 64, QA, false, SH, true, 2 * 64, VD, KD, false);  // O = Qa S + P E
      umma::gemm_t(tb + 64, QA, false, SL, true, 2 * 64, VD, KD, true);
      umma::gemm_t(tb + 64, QAL, false, SH, true, 2 * 64, VD, KD, true);
      umma::gemm(tb + 64, PB, EB, 2 * 64, VD, C, true);  // P E with both split hi + lo
      umma::gemm(tb + 64, PB, EL, 2 * 64, VD, C, true);
      umma::gemm(tb + 64, PL, EB, 2 * 64, VD, C, true);
      umma::commit(mbar);
    }
    // E^T for the backward, after T in slot 2c+1
    copy16(reinterpret_cast<uint8_t*>(slot(cs, bh, NS, 2 * c + 1)) + C * C * 2, reinterpret_cast<const uint8_t*>(EB),
           VD * C * 2, NT);
    inflight = 0;
    if ((ok = batch_wait(mbar, 0))) inflight = -1;
  }
  if (ok) {
    tc::for_frag<2 * 64, 64>(tb + 64, [&](int row, int v0, int, const float* x) {
      const int r = row >> 6, i = row & 63;
      if (i < Cl) {
        const int64_t off = out_off(o, b, t0 + i, h, r) + v0;
        if (flags & tc::F_O_VEC) {
          bf16* dst = reinterpret_cast<bf16*>(o.ptr) + off;
          tc::st8(dst, 0, x);
          tc::st8(dst, 8, x + 8);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) st_io(o.ptr, off + j, x[j], SCA2_BF16);
        }
      }
    });
  }
  // after a timeout: bounded waits for what is still in flight before TMEM and shared memory go
  if (inflight >= 0) umma::mbar_wait(mbar, (uint32_t)inflight);
  if (tma_pending) umma::mbar_wait(vbar, 0);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 128);
}

}  // namespace pcp

// Whether the chunk-parallel forward takes a training call: phase flavour, bf16 values,
// K = V = 64, a 16-byte aligned chunk-state buffer, and few (batch, head) sequences.  The
// sequential tensor-core forward runs one CTA per sequence at about 7 us per chunk whatever
// the sequence count, so it leaves SMs idle below one sequence per SM; the chunk-parallel
// kernels cost time in proportion to the chunks.  Measured forward on one B200 at T = 4096,
// H = 16 (chunk-parallel / sequential, ms): 16 sequences 0.19 / 0.52, 32: 0.27 / 0.54,
// 64: 0.42 / 0.57, 96: 0.62 / 0.61, 128: 0.77 / 0.65.  Up to SCA2_PCP_MAX_SEQ sequences go
// chunk-parallel.
#ifndef SCA2_PCP_MAX_SEQ
#define SCA2_PCP_MAX_SEQ 80
#endif
constexpr int PCP_MAX_SEQ = SCA2_PCP_MAX_SEQ;
bool pcp_covers(const sca2_scan_args& p, const float* cstates) {
  return p.flavor == SCA2_FLAVOR_PHASE && p.io_dtype == SCA2_BF16 && p.K == pcp::KD && p.V == pcp::VD &&
         cstates && ((uintptr_t)cstates & 15u) == 0 && p.T > 0 && (int64_t)p.B * p.H <= PCP_MAX_SEQ;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link against
// the driver library); nullptr where the driver does not provide it
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of the value tile (tc::tma_value_tile): v bf16, V = 64, 16-byte aligned rows, T % 8 == 0
// and rows of consecutive batches contiguous (sb == T st), so row = b T + t addresses every token.
// Used by the chunk-parallel kernels here and by the tensor-core chunk walk (scan_tc.cu).
// false (cp.async copies instead) where these do not hold or the encoder refuses the map.
bool value_tile_map(const sca2_scan_args& p, CUtensorMap* map) {
  const sca2_tok& v = p.v;
  if (p.V != pcp::VD || p.io_dtype != SCA2_BF16) return false;
  if (p.T % 8 || v.sb != (int64_t)p.T * v.st || v.st % 8 || v.sh % 8 || ((uintptr_t)v.ptr & 15u)) return false;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[5] = {8, 8, pcp::VD / 8, (cuuint64_t)p.B * p.T / 8, (cuuint64_t)p.H};
  const cuuint64_t strides[4] = {(cuuint64_t)v.st * 2, 16, (cuuint64_t)v.st * 16, (cuuint64_t)v.sh * 2};
  const cuuint32_t box[5] = {8, 8, pcp::VD / 8, tc::C / 8, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(v.ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// flags: tc::F_PH_VEC / F_V_VEC / F_O_VEC as computed for the tensor-core forward
cudaError_t pcp_scan_fwd(const sca2_scan_args& p, const sca2_out& o, float* S_final, float* cstates, int NS,
                         int flags, const PhaseProj& pp, cudaStream_t st) {
  const int NC = (p.T + tc::C - 1) / tc::C;
  const int BH = p.B * p.H;
  alignas(64) CUtensorMap vmap;
  memset(&vmap, 0, sizeof(vmap));
  const int use_tma = value_tile_map(p, &vmap) ? 1 : 0;
  cudaError_t e = cudaFuncSetAttribute(pcp::pcp_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, pcp::PrepL::TOTAL);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pcp::pcp_out, cudaFuncAttributeMaxDynamicSharedMemorySize, pcp::OutL::TOTAL);
  if (e != cudaSuccess) return e;
  pcp::pcp_prep<<<dim3(NC, BH), tc::NT, pcp::PrepL::TOTAL, st>>>(p, cstates, NS, flags, pp, vmap, use_tma);
  e = cudaFuncSetAttribute(pcp::pcp_state, cudaFuncAttributeMaxDynamicSharedMemorySize, pcp::StateL::TOTAL);
  if (e != cudaSuccess) return e;
  pcp::pcp_state<<<dim3(BH, pcp::VD / pcp::VBS), pcp::NTS, pcp::StateL::TOTAL, st>>>(p, cstates, NS, S_final);
  pcp::pcp_out<<<dim3(NC, BH), tc::NT, pcp::OutL::TOTAL, st>>>(p, o, cstates, NS, flags, pp, vmap, use_tma);
  return cudaGetLastError();
}

// Tensor map of the tensor-core backward's dO tiles (phase flavour, R = 2): dO (B, T, H, 2, V) bf16
// with the read column r next to the head (sh == 2 sr), batches' rows contiguous, T % 8 == 0 and
// 16-byte aligned rows; dims (value % 8, token % 8, value / 8, row / 8, 2 h + r), so the 64-token
// x 64-value tile of one (b, h, r) at coordinates (0, 0, vb0 / 8, (b T + t0) / 8, 2 h + r) lands in
// the K-major, no-swizzle operand layout, exactly as the value tiles above.  false (cp.async
// copies instead) where these do not hold or the encoder refuses the map.
bool dO_tile_map(const sca2_scan_args& p, const sca2_out& dO, CUtensorMap* map) {
  if (p.flavor != SCA2_FLAVOR_PHASE || p.io_dtype != SCA2_BF16 || p.V % 64 || p.T % 8) return false;
  if (dO.sb != (int64_t)p.T * dO.st || dO.sh != 2 * dO.sr || dO.st % 8 || dO.sr % 8 || ((uintptr_t)dO.ptr & 15u))
    return false;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[5] = {8, 8, (cuuint64_t)p.V / 8, (cuuint64_t)p.B * p.T / 8, (cuuint64_t)p.H * 2};
  const cuuint64_t strides[4] = {(cuuint64_t)dO.st * 2, 16, (cuuint64_t)dO.st * 16, (cuuint64_t)dO.sr * 2};
  const cuuint32_t box[5] = {8, 8, 8, tc::C / 8, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, dO.ptr, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// whether a training forward of these arguments runs chunk-parallel with its value tiles by TMA
bool pcp_value_tma(const sca2_scan_args& p, const float* cstates) {
  alignas(64) CUtensorMap map;
  return pcp_covers(p, cstates) && value_tile_map(p, &map);
}

// read and clear the device fault word of the chunk-parallel phase kernels (synchronous)
cudaError_t pcp_read_faults(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, pcp::g_fault_pcp, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(pcp::g_fault_pcp, &zero, sizeof(unsigned int));
}

}  // namespace sca2
