// Tensor-core (tcgen05 / TMEM) forward scan for bf16 inputs on sm_100a.
//
// One CTA per (batch*head, block of VB value columns), 64-token chunks walked in order.
// Per chunk (same algebra as the fp32 path and the oracle's forward_chunked):
//
//   state-independent   G   = KR KW^T                  (tcgen05, fp32 accumulate)
//                       P   = QR KW^T                  (codes split hi + lo)
//                       T   = (I + diag(beta) Gr)^{-1} (fp32, blocked, CUDA cores)
//                       U^T = V'^T T^T                 (tcgen05)
//                       Wk  = T Z^T, Z = beta a k e^{-lam i}/kappa
//   state chain         X^T = (d1 .* S)^T Wk^T
//   (S^T fp32 in regs)  Os  = QR (d1 .* S)
//                       E^T = U^T - X^T
//                       Op  = P E                      (P, E split hi + lo)
//                       O   = (a / kappa) .* Os + Op
//                       Su^T = E^T (KW diag(w))        (E split hi + lo)
//                       S   = dCm1 .* (a_last d1 .* S + Su)
//
// All MMA operands are bf16 in shared memory (K-major, no swizzle, see umma.cuh); every
// accumulator is fp32 in TMEM and the state itself stays fp32 in registers.  The products
// whose results feed other products are oriented so that each thread's accumulator row is a
// contiguous run of the next operand, and operands are written with 16-byte stores.  Where a
// bf16 operand alone would miss the bf16 parity bar (the intra-chunk read kernel P and the
// corrected values E) it is carried as a hi + lo pair (three products hi*hi + hi*lo + lo*hi),
// which keeps about 16 mantissa bits.  The next chunk's values are copied in while the current
// chunk runs, straight into the operand layout: by one TMA tensor copy per full chunk (phase
// flavour, V = 64, bf16 rows the tensor map can address; completion on an mbarrier whose wait is
// bounded), else by 16-byte cp.async copies; its phases (keys) and gates are loaded into
// registers meanwhile.  The MMAs of a batch are issued by two threads (warps 0 and
// 1, independent accumulators: a thread issues one instruction in about 50 cycles, about what
// an M = 128, N = 64 instruction takes on the tensor core) and complete on an mbarrier whose
// wait is bounded: on a timeout the CTA records a fault bit, waits (bounded) once more for its
// MMAs, frees its TMEM and returns.  Os only needs the state entering the chunk, so it is
// issued with P; when T is read back (training), U^T and Wk are issued right behind Os and
// complete on a second mbarrier, so they run during the P epilogue and only X^T (then Op,
// Su^T) waits on the state chain.
//
// Training runs save, per 64-token chunk c of the (B,H,slots,K,V) buffer: the state entering
// the chunk in slot 2c (fp32) and, in slot 2c+1, T (bf16 C x C, operand layout) followed by
// E^T (bf16, 64 x C per block of 64 value columns, operand layout; the hi part of the split).
// The backward reads them back instead of recomputing the inversion and the corrected values.
#include <cstring>

#include "tc_common.cuh"

namespace sca2 {
namespace tc {

__device__ unsigned int g_fault;  // bit 0: a bounded mbarrier wait timed out

// byte offsets of the shared-memory carve-up (operands 1024-byte aligned).  The lo halves of
// the split codes are only read by the P product and the fp32 inversion scratch is only used
// after that product has completed, so the two share one region.
template <int KD, int VB, int R>
struct FwdLayout {
  static constexpr int al(int x) { return (x + 1023) & ~1023; }
  static constexpr int mx(int a, int b) { return a > b ? a : b; }
  static constexpr int KR = 0;                                  // C x KD
  static constexpr int KW = KR + al(C * KD * 2);                // C x KD (hi)
  static constexpr int QR = KW + al(C * KD * 2);                // R*C x KD (hi)
  static constexpr int ZA = QR + al(R * C * KD * 2);            // C x KD  beta a kr / kappa [i][m]
  static constexpr int VA = ZA + al(C * KD * 2);                // C x VB  values [j][v]
  static constexpr int KWW = VA + al(VB * C * 2);               // C x KD  w kw [i][m]
  static constexpr int TB = KWW + al(KD * C * 2);               // C x C
  static constexpr int PB = TB + al(C * C * 2);                 // R*C x C (hi)
  static constexpr int PBL = PB + al(R * C * C * 2);            // R*C x C (lo)
  static constexpr int WK = PBL + al(R * C * C * 2);            // C x KD
  static constexpr int SB = WK + al(C * KD * 2);                // VB x KD: (d1 .* S)^T
  static constexpr int EB = SB + al(VB * KD * 2);               // VB x C (hi): E^T
  static constexpr int EBL = EB + al(VB * C * 2);               // VB x C (lo)
  static constexpr int A0 = EBL + al(VB * C * 2);               // shared region
  static constexpr int KWL = A0;                                //   C x KD (lo)
  static constexpr int QRL = KWL + al(C * KD * 2);              //   R*C x KD (lo)
  static constexpr int LS = A0;                                 //   fp32 C x LDF
  static constexpr int TS = LS + al(C * LDF * 4);               //   fp32 C x LDF
  static constexpr int WS = TS + al(C * LDF * 4);               //   fp32 1024
  static constexpr int A0_END = mx(QRL + al(R * C * KD * 2), WS + al(1024 * 4));
  // scalars (floats): two sets of gates beta[C], Gc[C], a[C], w[C] (this chunk, next chunk),
  // d1[KD], dCm1[KD], lam[KD], wr[KD], wi[KD], a of the previous chunk [C], the column factors
  // of the decay mask [C]; phase flavour (R = 2): the head's theta and omega [KD / 2 each]
  static constexpr int SC_FLOATS = 10 * C + 5 * KD + (R == 2 ? KD : 0);
  // fp32 KD x VB staging of the state to save [m][v], where it fits the 227 KB opt-in limit
  static constexpr bool STAGE = A0_END + al(KD * VB * 4) + al(SC_FLOATS * 4) + 64 <= 227 * 1024;
  static constexpr int ST = A0_END;
  static constexpr int SC = ST + (STAGE ? al(KD * VB * 4) : 0);
  static constexpr int MBAR = SC + al(SC_FLOATS * 4);
  // mbarrier (8 B), TMEM base (4 B), error flag (4 B), U^T / Wk mbarrier (8 B), value-tile mbarrier (8 B)
  static constexpr int TOTAL = MBAR + 64;
};

// TMEM columns: [0,64) Op ; [64,128) P ; [128,192) G, later U^T, later X^T ; [192, 192+KD) Wk,
// later Su^T ; then Os (two buffers when the outputs are deferred)
template <int KD, int VB>
struct Cols {
  // With VB = 64 the outputs of a chunk are formed while the next chunk's first MMA batch runs,
  // so Os is double-buffered (chunk c in OS + (c & 1) VB) and nothing in that batch writes Op.
  static constexpr bool DEFER = VB == 64;
  static constexpr int G = 128, P = 64, OP = 0, UT = 128, XT = 128, WK = 192, SUT = 192, OS = 192 + KD;
  static constexpr int NEED = OS + (DEFER ? 2 : 1) * VB;
  static constexpr int ALLOC = NEED <= 256 ? 256 : 512;
  static_assert(NEED <= 512, "TMEM columns");
};

// 16-byte copy of an operand from shared to global memory (both 16-byte aligned)
__device__ __forceinline__ void copy_out(uint8_t* dst, const bf16* src, int nbytes) {
  const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
  for (int u = threadIdx.x * 16; u < nbytes; u += NT * 16)
    *reinterpret_cast<uint4*>(dst + u) = *reinterpret_cast<const uint4*>(s + u);
}

// HG: a per-token scalar decay (p.g) is present; PJ: phases formed from projections (PhaseProj::on,
// phase flavour).  Both are compile-time variants, so a kernel carries only the code its inputs use.
template <int FL, int KD, int VB, int R, bool HG, bool PJ>
__global__ void __launch_bounds__(NT, 1) scan_fwd_tc(sca2_scan_args p, sca2_out o, float* S_final,
                                                    float* cstates, int NCS, int flags, PhaseProj pp_in,
                                                    TSlots ts, const __grid_constant__ CUtensorMap vmap,
                                                    int use_tma) {
  PhaseProj pp = pp_in;
  pp.on = PJ;
  using L = FwdLayout<KD, VB, R>;
  using CO = Cols<KD, VB>;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int vb0 = blockIdx.y * VB;
  const int V = p.V;
  constexpr bool has_g = HG;  // a per-token scalar decay (p.g) is present
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)(KD / 2) : 1.f;
  const float ik = 1.f / kappa;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  // gates of chunk c in set c & 1: the next chunk's are formed while this one runs
  auto gset = [&](int k) -> Gates {
    float* g0 = sc + 4 * C * (k & 1);
    return Gates{g0, g0 + C, g0 + 2 * C, g0 + 3 * C};
  };
  float* s_d1 = sc + 8 * C;
  float* s_dCm1 = s_d1 + KD;
  float* s_lam = s_dCm1 + KD;
  float* s_wr = s_lam + KD;
  float* s_wi = s_wr + KD;
  float* s_aprev = s_wi + KD;
  float* s_fdec = s_aprev + C;  // column factors of the decay mask (decay_block)
  float* s_th = R == 2 ? s_fdec + C : nullptr;  // theta, omega of the head (phases from projections)
  float* s_om = R == 2 ? s_fdec + C + KD / 2 : nullptr;
  float* LS = reinterpret_cast<float*>(sm + L::LS);
  float* TS = reinterpret_cast<float*>(sm + L::TS);
  float* WS = reinterpret_cast<float*>(sm + L::WS);
  bf16* VA = reinterpret_cast<bf16*>(sm + L::VA);
  bf16* TB = reinterpret_cast<bf16*>(sm + L::TB);
  bf16* PB = reinterpret_cast<bf16*>(sm + L::PB);
  bf16* PBL = reinterpret_cast<bf16*>(sm + L::PBL);
  bf16* WK = reinterpret_cast<bf16*>(sm + L::WK);
  bf16* SB = reinterpret_cast<bf16*>(sm + L::SB);
  bf16* EB = reinterpret_cast<bf16*>(sm + L::EB);
  bf16* EBL = reinterpret_cast<bf16*>(sm + L::EBL);
  CodeOps<FL, KD, R> cops{reinterpret_cast<bf16*>(sm + L::KR), reinterpret_cast<bf16*>(sm + L::KW),
                          reinterpret_cast<bf16*>(sm + L::KWL), reinterpret_cast<bf16*>(sm + L::QR),
                          reinterpret_cast<bf16*>(sm + L::QRL), reinterpret_cast<bf16*>(sm + L::ZA),
                          reinterpret_cast<bf16*>(sm + L::KWW)};
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  volatile int* s_err = reinterpret_cast<volatile int*>(sm + L::MBAR + 12);
  uint64_t* mbar2 = reinterpret_cast<uint64_t*>(sm + L::MBAR + 16);  // U^T / Wk batch (training)
  // value tiles of full chunks by one TMA copy (issued by thread 0, completion on vbar, waited by
  // every thread at the top of the chunk); the ragged last chunk takes 16-byte cp.async copies
  uint64_t* vbar = reinterpret_cast<uint64_t*>(sm + L::MBAR + 24);
  uint32_t vph = 0;
  bool vpend = false;  // a value tile is in flight (uniform over the CTA)
  float* ST = reinterpret_cast<float*>(sm + L::ST);
  // MMA issuers: thread 0 and thread 32 (warps 0 and 1) issue independent products in parallel;
  // each mbar phase takes one arrival from each (a commit, or a plain arrive when it has none)
  constexpr int NISS = 2;
  const bool issuer = (tid & 31) == 0 && warp < NISS;
  // the next chunk's gates: loaded and formed by the last warp, which issues no products
  constexpr int GW = NT / 32 - 1;

  // ---- set-up: per-head constants, mbarrier, TMEM
  constexpr int KH = FL == SCA2_FLAVOR_PHASE ? KD / 2 : KD;
  for (int m = tid; m < KD; m += NT) {
    const float l = p.lam ? p.lam[h * KH + (m % KH)] : 0.f;
    s_lam[m] = l;
    s_d1[m] = expf(-l);
    s_wr[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wr[h * KH + m] : 0.f;
    s_wi[m] = (FL == SCA2_FLAVOR_PHASE && m < KH) ? p.wi[h * KH + m] : 0.f;
    if (R == 2 && pp.on && m < KD / 2) {
      s_th[m] = pp.theta[h * (KD / 2) + m];
      s_om[m] = pp.omega[h * (KD / 2) + m];
    }
  }
  if (tid == 0) {
    umma::mbar_init(mbar, NISS);
    umma::mbar_init(mbar2, 1);
    umma::mbar_init(vbar, 1);
    umma::fence_mbar_init();
    *s_err = 0;
  }
  if (tid < 32) umma::tmem_alloc(s_tmem, CO::ALLOC);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  uint32_t phase = 0, phase2 = 0;
  bool pending2 = false;  // a U^T / Wk batch was committed to mbar2 and not yet waited for

  // ---- state S^T: fp32 registers in the layout of the Su^T accumulator (M = VB, N = KD).  With
  // VB = 64 that is the all-lane layout of for_frag16 (element k at row s_v(k), column s_m(k));
  // with VB = 128 the 32x32b one (lane row srow, columns frag_col0 + j).
  constexpr bool W16 = VB == 64;
  constexpr int NS = W16 ? KD / 4 : KD / 2;
  float Sreg[NS];
  const int srow = frag_row<VB>();
  const bool sown = W16 || owns_rows<VB>();
  const int sv0 = 16 * (warp & 3) + (tid & 31) / 4, sm0 = (warp >> 2) * (KD / 2) + 2 * (tid & 3);
  auto s_v = [&](int k) { return W16 ? sv0 + 8 * ((k >> 1) & 1) : srow; };
  auto s_m = [&](int k) { return W16 ? sm0 + 8 * (k >> 2) + (k & 1) : frag_col0<VB, KD>(k / 16) + (k & 15); };
  const int64_t bhKV = ((int64_t)b * p.H + h) * KD * (int64_t)V;
  if constexpr (W16) {
#pragma unroll
    for (int g = 0; g < NS / 4; ++g) {
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = 4 * g + e, m = s_m(k);
        const float s = p.S0 ? p.S0[bhKV + vb0 + s_v(k) + (int64_t)m * V] : 0.f;
        Sreg[k] = s;
        x[e] = s * s_d1[m];
        if (L::STAGE && cstates && (flags & F_CS16)) ST[m * VB + s_v(k)] = s;
      }
      st2(SB, umma::kmaj(sv0, sm0 + 8 * g, KD), x[0], x[1]);
      st2(SB, umma::kmaj(sv0 + 8, sm0 + 8 * g, KD), x[2], x[3]);
    }
  } else {
    const int64_t sbase = bhKV + vb0 + srow;
#pragma unroll
    for (int q = 0; q < KD / 32; ++q) {
      float x[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = frag_col0<VB, KD>(q) + j;
        const float s = (sown && p.S0) ? p.S0[sbase + (int64_t)m * V] : 0.f;
        Sreg[16 * q + j] = s;
        x[j] = s * s_d1[m];
      }
      if (sown) {
        st8(SB, umma::kmaj(srow, frag_col0<VB, KD>(q), KD), x);
        st8(SB, umma::kmaj(srow, frag_col0<VB, KD>(q) + 8, KD), x + 8);
        if (L::STAGE && cstates && (flags & F_CS16))
#pragma unroll
          for (int j = 0; j < 16; ++j) ST[(frag_col0<VB, KD>(q) + j) * VB + srow] = Sreg[16 * q + j];
      }
    }
  }
  // The state entering each chunk goes to slot 2c.  Staged: in ST (fp32 [m][v]), written with
  // bulk copies (one for the whole block when VB == V, else one per row m) issued at the top of
  // the chunk; the copies have read ST before the chunk's state update rewrites it.  Otherwise
  // (no room for ST) with plain stores from the state registers.
  const bool st_one = VB == V;
  const bool stage = L::STAGE && cstates && (flags & F_CS16);
  const bool st_issuer = stage && (st_one ? tid == 0 : tid < KD);
  publish_smem();
  float Ureg[W16 ? C / 4 : C / 2];  // U^T in the Su^T / X^T accumulator layout

  auto wait_mma = [&]() -> bool {
    if (!umma::mbar_wait(mbar, phase)) *s_err = 1;
    phase ^= 1u;
    __syncthreads();
    umma::fence_after_sync();
    return *s_err == 0;
  };
  auto wait_mma2 = [&]() -> bool {  // on a timeout the phase stays pending for the drain
    if (!umma::mbar_wait(mbar2, phase2)) *s_err = 1;
    __syncthreads();
    umma::fence_after_sync();
    if (*s_err != 0) return false;
    phase2 ^= 1u;
    pending2 = false;
    return true;
  };

  // ---- outputs O = (a / kappa) .* Os + Op of chunk cc (both accumulators share one row layout)
  auto emit_out = [&](int cc, uint32_t os_col, const float* av) {
    constexpr int M = R * 64;
    const int t0o = cc * C, Clo = min(C, p.T - t0o);
    const int sub = (tid >> 5) & 3;
    const bool own = owns_rows<M>();
    const int row = frag_row<M>(), r = row >> 6, i = row & 63;
    uint32_t ra[VB / 32][16], rx[VB / 32][16];
#pragma unroll
    for (int q = 0; q < VB / 32; ++q) {
      umma::ld16_issue(umma::taddr(os_col, 32 * sub, frag_col0<M, VB>(q)), ra[q]);
      umma::ld16_issue(umma::taddr(tb + CO::OP, 32 * sub, frag_col0<M, VB>(q)), rx[q]);
    }
    umma::ld_wait();
#pragma unroll
    for (int q = 0; q < VB / 32; ++q) {
      const int v0 = frag_col0<M, VB>(q);
      float a[16], x[16];
      umma::take<16>(ra[q], a);
      umma::take<16>(rx[q], x);
      if (own && i < Clo) {
        const float fa = av[i] * ik;
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = fa * a[j] + x[j];
        const int64_t off = out_off(o, b, t0o + i, h, r) + vb0 + v0;
        if (flags & F_O_VEC) {
          bf16* dst = reinterpret_cast<bf16*>(o.ptr) + off;
          st8(dst, 0, y);
          st8(dst, 8, y + 8);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (vb0 + v0 + j < V) st_io(o.ptr, off + j, y[j], p.io_dtype);
        }
      }
    }
  };

  const int NC = (p.T + C - 1) / C;
  const bool code_vec = flags & (FL == SCA2_FLAVOR_PHASE ? F_PH_VEC : F_K_VEC);
  // chunk 0's values (cp.async), codes and gates (registers); later chunks are prefetched while
  // the previous one runs
  CodeRegs<FL, KD> creg;
  GateRegs greg;
  // prep: T of every chunk is read from ts (training: slot 2c + 1; inference: the work buffer)
  const bool prep = (flags & F_PREP) && ts.base;
  // training: each chunk's P (hi part, operand layout) goes to slot 2 NC + c for the backward,
  // one bulk copy issued by thread 32 (plain 16-byte stores when the buffer is not aligned)
  const bool p_save = prep && cstates && blockIdx.y == 0;
  const bool p_issuer = p_save && (flags & F_CS16) && tid == 32;
  auto saved_at = [&](int cc) -> uint8_t* {
    return reinterpret_cast<uint8_t*>(cstates + (((int64_t)b * p.H + h) * NCS + 2 * cc + 1) * KD * (int64_t)V);
  };
  auto t_at = [&](int cc) -> const uint8_t* {
    return ts.base + ((int64_t)b * p.H + h) * ts.bh_stride + (int64_t)cc * ts.c_stride;
  };
  {
    const int Cl0 = min(C, p.T);
    if (use_tma && Cl0 == C) {
      if (tid == 0) tma_value_tile<VB>(VA, &vmap, b * p.T, h, vbar);
      vpend = true;
    } else {
      pf_values<VB>(p, VA, flags & F_V_VEC, b, h, 0, Cl0, vb0);
    }
    if (prep)
      for (int u = tid * 16; u < C * C * 2; u += NT * 16) cp16(reinterpret_cast<uint8_t*>(TB) + u, t_at(0) + u, true);
    cp_commit();
    load_code_regs<FL, KD>(p, creg, code_vec, b, h, 0, Cl0, pp);
    if (warp == 0) {
      load_gate_regs(p, greg, b, h, 0, Cl0);
      gates_from_regs(greg, gset(0), Cl0);
    }
    __syncthreads();
    finish_code_regs<FL, KD>(creg, pp, h, 0, Cl0, s_th, s_om);
    build_codes<FL, KD, R>(creg, cops, gset(0), s_lam, s_wr, s_wi, p.q_scale, Cl0, ik, !prep);
  }
  // Per chunk c: the codes of chunk c (but KWW) and its gates were formed while chunk c - 1's
  // last MMA batches ran (nothing in flight then reads them); KWW = w KW is formed at the top.
  bool ok = true;
  for (int c = 0; c < NC && ok; ++c) {
    const int t0 = c * C, Cl = min(C, p.T - t0);
    // saved for the backward in slot 2c+1: T (bf16 [i][j]) then E^T (bf16 [v][j]) per value block
    uint8_t* saved = cstates ? saved_at(c) : nullptr;
    if (st_issuer) {
      // state entering chunk c (staged in ST) -> slot 2c of the (B,H,NCS,K,V) buffer
      float* cb = cstates + (((int64_t)b * p.H + h) * NCS + 2 * c) * KD * (int64_t)V + vb0;
      if (st_one)
        bulk_store(cb, ST, KD * VB * 4);
      else
        bulk_store(cb + (int64_t)tid * V, ST + tid * VB, VB * 4);
      bulk_commit();
    }
    if (!stage && cstates && sown) {
      const int64_t cb = (((int64_t)b * p.H + h) * NCS + 2 * c) * KD * (int64_t)V + vb0;
#pragma unroll
      for (int k = 0; k < NS; ++k) cstates[cb + s_v(k) + (int64_t)s_m(k) * V] = Sreg[k];
    }
    // ---- operands of the chunk
    const Gates gates = gset(c);
    cp_wait_all();
    if (vpend) {  // this chunk's value tile (TMA)
      if (!umma::mbar_wait(vbar, vph)) *s_err = 1;
      vph ^= 1u;
      vpend = false;
    }
    for (int m = tid; m < KD; m += NT) s_dCm1[m] = expf(-s_lam[m] * (float)(Cl - 1));
    if (has_g) decay_factors(gates.Gc, s_fdec);
    kww_from_kw<FL, KD, R>(cops, gates);
    if (p.v_times_beta) {
      __syncthreads();  // every thread's value copies have landed
      scale_values<VB>(VA, gates.beta);
    }
    publish_smem();
    if (issuer) {
      if (warp == 0) {
        if (!prep) umma::gemm(tb + CO::G, sm + L::KR, sm + L::KW, 64, 64, KD, false);
        umma::gemm(tb + CO::P, sm + L::QR, sm + L::KW, R * 64, 64, KD, false);
        umma::gemm(tb + CO::P, sm + L::QR, sm + L::KWL, R * 64, 64, KD, true);
        umma::gemm(tb + CO::P, sm + L::QRL, sm + L::KW, R * 64, 64, KD, true);
        umma::commit(mbar);
      } else {
        umma::gemm(tb + CO::OS + (CO::DEFER ? (c & 1) * VB : 0), sm + L::QR, sm + L::SB, R * 64, VB, KD, false);
        umma::commit(mbar);
        if (prep) {  // T is already in place: U^T and Wk run while the P epilogue does
          umma::gemm_t(tb + CO::UT, VA, true, TB, false, VB, C, C, false);
          umma::gemm_t(tb + CO::WK, TB, false, sm + L::ZA, true, 64, KD, C, false);
          umma::commit(mbar2);
        }
      }
    }
    pending2 = prep;
    if (c + 1 < NC) {  // next chunk's codes and gates into registers
      const int t1 = t0 + C, Cl1 = min(C, p.T - t1);
      load_code_regs<FL, KD>(p, creg, code_vec, b, h, t1, Cl1, pp);
      if (warp == GW) load_gate_regs(p, greg, b, h, t1, Cl1);
    }
    // the previous chunk's outputs while this chunk's first batch runs
    if (CO::DEFER && c > 0) emit_out(c - 1, tb + CO::OS + ((c - 1) & 1) * VB, s_aprev);
    if (p_issuer) bulk_wait_read();  // the P epilogue below rewrites PB
    if (!(ok = wait_mma())) break;
    // ---- L = beta Gr (fp32) and P (hi + lo), masked and decayed
    if (!prep) for_frag<64, 64>(tb + CO::G, [&](int i, int j0, int, const float* x) {
      const float bi = gates.beta[i] * ik;
      float dg[16];
      if (has_g) decay_block(gates.Gc, s_fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
    });
    {
      auto p_epi = [&](int row, int j0, int, const float* x) {
        const int i = row & 63;
        float y[16], dg[16];
        if (has_g) decay_block(gates.Gc, s_fdec, i, j0, dg);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          y[j] = jj <= i ? x[j] * ik * (has_g ? dg[j] : 1.f) : 0.f;
        }
        st8_split(PB, PBL, umma::kmaj(row, j0, C), y);
        st8_split(PB, PBL, umma::kmaj(row, j0 + 8, C), y + 8);
      };
      for_frag<R * 64, 64>(tb + CO::P, p_epi);
    }
    if (!prep) {
      __syncthreads();
      invert_unit_lower(LS, TS, WS);
      store_T<false>(TS, TB);
      publish_smem();
      if (cstates && blockIdx.y == 0) copy_out(saved, TB, C * C * 2);
      if (issuer) {
        if (warp == 0)
          umma::gemm_t(tb + CO::UT, VA, true, TB, false, VB, C, C, false);
        else
          umma::gemm_t(tb + CO::WK, TB, false, sm + L::ZA, true, 64, KD, C, false);
        umma::commit(mbar);
      }
      if (!(ok = wait_mma())) break;
    } else {
      // (the P stores reach the async proxy with the publish before the product that reads them)
      if (!(ok = wait_mma2())) break;
    }
    if (c + 1 < NC) {  // VA and TB are free: next chunk's values (and T)
      const int t1 = t0 + C, Cl1 = min(C, p.T - t1);
      if (use_tma && Cl1 == C) {
        if (tid == 0) tma_value_tile<VB>(VA, &vmap, b * p.T + t1, h, vbar);
        vpend = true;
      } else {
        pf_values<VB>(p, VA, flags & F_V_VEC, b, h, t1, Cl1, vb0);
      }
      if (prep)
        for (int u = tid * 16; u < C * C * 2; u += NT * 16)
          cp16(reinterpret_cast<uint8_t*>(TB) + u, t_at(c + 1) + u, true);
      cp_commit();
    }
    if constexpr (W16) {
      for_frag16<C>(tb + CO::UT, [&](int g, int, int, const float* x) {
#pragma unroll
        for (int e = 0; e < 4; ++e) Ureg[4 * g + e] = x[e];
      });
    } else {
      for_frag<VB, C>(tb + CO::UT, [&](int, int, int q, const float* x) {
#pragma unroll
        for (int j = 0; j < 16; ++j) Ureg[16 * q + j] = x[j];
      });
    }
    for_frag16<KD>(tb + CO::WK, [&](int, int i0, int m, const float* x) {
      st2(WK, umma::kmaj(i0, m, KD), x[0], x[1]);
      st2(WK, umma::kmaj(i0 + 8, m, KD), x[2], x[3]);
    });
    publish_smem();
    if (p_save) {
      float* dst = cstates + (((int64_t)b * p.H + h) * NCS + 2 * NC + c) * KD * (int64_t)V;
      if (flags & F_CS16) {
        if (p_issuer) {
          bulk_store(dst, PB, R * C * C * 2);
          bulk_commit();
        }
      } else {
        copy_out(reinterpret_cast<uint8_t*>(dst), PB, R * C * C * 2);
      }
    }
    if (issuer) {
      if (warp == 0) {
        umma::gemm(tb + CO::XT, sm + L::SB, sm + L::WK, VB, C, KD, false);
        umma::commit(mbar);
      } else {
        umma::mbar_arrive(mbar);
      }
    }
    if (warp == GW && c + 1 < NC) gates_from_regs(greg, gset(c + 1), min(C, p.T - t0 - C));
    if (!(ok = wait_mma())) break;
    if constexpr (W16) {
      for_frag16<C>(tb + CO::XT, [&](int g, int v0, int i, const float* x) {
        st2_split(EB, EBL, umma::kmaj(v0, i, C), Ureg[4 * g] - x[0], Ureg[4 * g + 1] - x[1]);
        st2_split(EB, EBL, umma::kmaj(v0 + 8, i, C), Ureg[4 * g + 2] - x[2], Ureg[4 * g + 3] - x[3]);
      });
    } else {
      for_frag<VB, C>(tb + CO::XT, [&](int v, int i0, int q, const float* x) {
        float e[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) e[j] = Ureg[16 * q + j] - x[j];
        st8_split(EB, EBL, umma::kmaj(v, i0, C), e);
        st8_split(EB, EBL, umma::kmaj(v, i0 + 8, C), e + 8);
      });
    }
    publish_smem();
    if (cstates) copy_out(saved + C * C * 2 + blockIdx.y * (VB * C * 2), EB, VB * C * 2);
    if (issuer) {
      if (warp == 0) {
        umma::gemm(tb + CO::OP, sm + L::PB, sm + L::EB, R * 64, VB, C, false);
        umma::gemm(tb + CO::OP, sm + L::PB, sm + L::EBL, R * 64, VB, C, true);
        umma::gemm(tb + CO::OP, sm + L::PBL, sm + L::EB, R * 64, VB, C, true);
      } else {
        umma::gemm_t(tb + CO::SUT, EB, false, sm + L::KWW, true, VB, KD, C, false);
        umma::gemm_t(tb + CO::SUT, EBL, false, sm + L::KWW, true, VB, KD, C, true);
      }
      umma::commit(mbar);
    }
    if (st_issuer) bulk_wait_read();  // ST is rewritten by the state update below
    // the next chunk's codes (their buffers are free: only KWW is read by this batch)
    if (c + 1 < NC) {
      finish_code_regs<FL, KD>(creg, pp, h, t0 + C, min(C, p.T - t0 - C), s_th, s_om);
      build_codes<FL, KD, R>(creg, cops, gset(c + 1), s_lam, s_wr, s_wi, p.q_scale, min(C, p.T - t0 - C), ik,
                             !prep);
    }
    if (!(ok = wait_mma())) break;
    // ---- state update
    if (CO::DEFER && tid < C) s_aprev[tid] = gates.a[tid];
    const float aC = gates.a[Cl - 1];
    if constexpr (W16) {
      // ST [m][v] rows are VB = 64 floats apart (bank = v % 32): each staging store takes row v0
      // on lanes with (lane & 1) == 0 and row v0 + 8 on the others, 16 banks per instruction
      const bool odd = tid & 1;
      for_frag16<KD>(tb + CO::SUT, [&](int g, int v0, int m, const float* x) {
        float y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * g + e, mm = m + (e & 1);
          const float s = s_dCm1[mm] * (aC * s_d1[mm] * Sreg[k] + x[e]);
          Sreg[k] = s;
          y[e] = s * s_d1[mm];
        }
        st2(SB, umma::kmaj(v0, m, KD), y[0], y[1]);
        st2(SB, umma::kmaj(v0 + 8, m, KD), y[2], y[3]);
        if (stage && c + 1 < NC) {
          const int va = odd ? v0 + 8 : v0, vb = odd ? v0 : v0 + 8;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const float sa = Sreg[4 * g + cc], sb = Sreg[4 * g + 2 + cc];
            ST[(m + cc) * VB + va] = odd ? sb : sa;
            ST[(m + cc) * VB + vb] = odd ? sa : sb;
          }
        }
      });
    } else {
      for_frag<VB, KD>(tb + CO::SUT, [&](int v, int m0, int q, const float* x) {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + j;
          const float s = s_dCm1[m] * (aC * s_d1[m] * Sreg[16 * q + j] + x[j]);
          Sreg[16 * q + j] = s;
          y[j] = s * s_d1[m];
        }
        st8(SB, umma::kmaj(v, m0, KD), y);
        st8(SB, umma::kmaj(v, m0 + 8, KD), y + 8);
        if (stage && c + 1 < NC)
#pragma unroll
          for (int j = 0; j < 16; ++j) ST[(m0 + j) * VB + v] = Sreg[16 * q + j];
      });
    }
    if (!CO::DEFER) emit_out(c, tb + CO::OS, gates.a);
    publish_smem();
  }
  if (CO::DEFER && ok && NC > 0) emit_out(NC - 1, tb + CO::OS + ((NC - 1) & 1) * VB, s_aprev);
  cp_wait_all();
  if (st_issuer || p_issuer) bulk_wait_all();
  if (ok && S_final && sown) {
#pragma unroll
    for (int k = 0; k < NS; ++k) S_final[bhKV + vb0 + s_v(k) + (int64_t)s_m(k) * V] = Sreg[k];
  }
  if (!ok) {
    if (tid == 0) atomicOr(&g_fault, 1u);
    // bounded: let any MMA still in flight drain
    umma::mbar_wait(mbar, phase ^ 1u);
    if (pending2) umma::mbar_wait(mbar2, phase2);
  }
  if (vpend) umma::mbar_wait(vbar, vph);  // bounded: a value tile still in flight lands first
  umma::fence_before_sync();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tb, CO::ALLOC);
}

template <int FL, int KD, int VB, int R, bool HG>
auto fwd_kernel(bool pj) {
  if constexpr (FL == SCA2_FLAVOR_PHASE)
    return pj ? scan_fwd_tc<FL, KD, VB, R, HG, true> : scan_fwd_tc<FL, KD, VB, R, HG, false>;
  else
    return scan_fwd_tc<FL, KD, VB, R, HG, false>;
}

template <int FL, int KD, int VB, int R>
cudaError_t launch_fwd(const sca2_scan_args& p, const sca2_out& o, float* S_final, float* cstates,
                       int NCS, int flags, const PhaseProj& pp, const TSlots& ts, const CUtensorMap& vmap,
                       int use_tma, cudaStream_t st) {
  const bool pj = pp.on != 0;
  auto k = p.g.ptr ? fwd_kernel<FL, KD, VB, R, true>(pj) : fwd_kernel<FL, KD, VB, R, false>(pj);
  const int smem = FwdLayout<KD, VB, R>::TOTAL;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, p.V / VB);
  k<<<grid, NT, smem, st>>>(p, o, S_final, cstates, NCS, flags, pp, ts, vmap, use_tma);
  return cudaGetLastError();
}

}  // namespace tc

int tc_fwd_smem(int K, int VB, int R) {
#define SCA2_TC_SMEM(KD_, VB_, R_) \
  if (K == KD_ && VB == VB_ && R == R_) return tc::FwdLayout<KD_, VB_, R_>::TOTAL;
  SCA2_TC_SMEM(64, 64, 1) SCA2_TC_SMEM(64, 64, 2) SCA2_TC_SMEM(64, 128, 1) SCA2_TC_SMEM(64, 128, 2)
  SCA2_TC_SMEM(128, 64, 1)
#undef SCA2_TC_SMEM
  return 1 << 30;
}

// Value block of the tensor-core forward for this shape, or 0 when the shape is not covered:
// K in {64, 128} and the value block in {64, 128} (every MMA has M = 64 or 128), V a multiple
// of the block, shared memory within the device's opt-in limit.
int tc_fwd_vb(int K, int V, int R, int max_smem) {
  if (!(K == 64 || K == 128)) return 0;
  const int cand[2] = {64, 128};
  for (int i = 0; i < 2; ++i)
    if (V % cand[i] == 0 && tc_fwd_smem(K, cand[i], R) <= max_smem) return cand[i];
  return 0;
}

static int tc_flags(const sca2_scan_args& p, const sca2_out& o) {
  int f = 0;
  auto a16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
  if (p.flavor == SCA2_FLAVOR_PHASE && a16(p.phw.ptr) && a16(p.phq.ptr) && p.phw.sb % 4 == 0 &&
      p.phw.st % 4 == 0 && p.phw.sh % 4 == 0 && p.phq.sb % 4 == 0 && p.phq.st % 4 == 0 && p.phq.sh % 4 == 0)
    f |= tc::F_PH_VEC;
  if (p.flavor == SCA2_FLAVOR_KEY && a16(p.phw.ptr) && a16(p.phq.ptr) && p.phw.sb % 8 == 0 &&
      p.phw.st % 8 == 0 && p.phw.sh % 8 == 0 && p.phq.sb % 8 == 0 && p.phq.st % 8 == 0 && p.phq.sh % 8 == 0)
    f |= tc::F_K_VEC;
  if (a16(p.v.ptr) && p.v.sb % 8 == 0 && p.v.st % 8 == 0 && p.v.sh % 8 == 0 && p.V % 8 == 0) f |= tc::F_V_VEC;
  if (a16(o.ptr) && o.sb % 8 == 0 && o.st % 8 == 0 && o.sh % 8 == 0 && o.sr % 8 == 0 && p.V % 8 == 0)
    f |= tc::F_O_VEC;
  return f;
}

cudaError_t tc_scan_prep(const sca2_scan_args& p, const tc::TSlots& ts, int vec, const PhaseProj& pp,
                         cudaStream_t st);

// Bytes of the inference work buffer (T of every chunk, bf16 C x C each) for a K = 64 forward on
// the tensor cores; the preparation kernel covers K = 64 only.
int64_t tc_infer_work_bytes(const sca2_scan_args& p) {
  if (p.K != 64 || p.T <= 0) return 0;
  return (int64_t)p.B * p.H * ((p.T + tc::C - 1) / tc::C) * (tc::C * tc::C * 2);
}
// phase_cp.cu: the chunk-parallel training forward of the phase flavour at K = V = 64, and the
// tensor map of a chunk's value tile (bf16, V = 64)
bool pcp_covers(const sca2_scan_args& p, const float* cstates);
bool value_tile_map(const sca2_scan_args& p, CUtensorMap* map);
cudaError_t pcp_scan_fwd(const sca2_scan_args& p, const sca2_out& o, float* S_final, float* cstates, int NS,
                         int flags, const PhaseProj& pp, cudaStream_t st);

// work: inference only (cstates == nullptr), nullptr or tc_infer_work_bytes(p) bytes, 16-byte
// aligned: T of every chunk is computed chunk-parallel into it first and the walk reads it instead
// of inverting inside its sequential loop (the training forward does the same through slot 2c + 1)
cudaError_t tc_scan_fwd(const sca2_scan_args& p, int VB, const sca2_out& o, float* S_final,
                        float* cstates, int NCS, cudaStream_t st, const PhaseProj& pp, void* work) {
  const bool ph = p.flavor == SCA2_FLAVOR_PHASE;
  int fl = tc_flags(p, o);
  // training of the phase flavour at K = V = 64: chunk-parallel, its saved data in the layout the
  // tensor-core backward reads
  if (pcp_covers(p, cstates)) return pcp_scan_fwd(p, o, S_final, cstates, NCS, fl, pp, st);
  if (cstates && ((uintptr_t)cstates & 15u) == 0) fl |= tc::F_CS16;
  tc::TSlots ts{nullptr, 0, 0};
  if (cstates && p.K == 64) {  // training: T of every chunk in slot 2c + 1
    const int64_t slot = (int64_t)p.K * p.V * 4;
    ts = tc::TSlots{reinterpret_cast<uint8_t*>(cstates) + slot, NCS * slot, 2 * slot};
  } else if (!cstates && work && tc_infer_work_bytes(p) > 0 && ((uintptr_t)work & 15u) == 0) {
    const int64_t tb = tc::C * tc::C * 2;  // inference: compact, chunk after chunk
    ts = tc::TSlots{static_cast<uint8_t*>(work), ((p.T + tc::C - 1) / tc::C) * tb, tb};
  }
  if (ts.base) {  // T of every chunk from the chunk-parallel kernel
    cudaError_t e = tc_scan_prep(p, ts, fl & (ph ? tc::F_PH_VEC : tc::F_K_VEC), pp, st);
    if (e != cudaSuccess) return e;
    fl |= tc::F_PREP;
  }
  // the phase flavour at K = V = 64 (one value block): value tiles of full chunks by TMA
  alignas(64) CUtensorMap vmap;
  memset(&vmap, 0, sizeof(vmap));
  const int use_tma = (ph && p.K == 64 && VB == 64 && p.V == 64 && value_tile_map(p, &vmap)) ? 1 : 0;
#define SCA2_TC_FWD(KD_, VB_)                                                                             \
  if (p.K == KD_ && VB == VB_)                                                                            \
    return ph ? tc::launch_fwd<SCA2_FLAVOR_PHASE, KD_, VB_, 2>(p, o, S_final, cstates, NCS, fl, pp, ts, vmap,    \
                                                              use_tma, st)                                     \
              : tc::launch_fwd<SCA2_FLAVOR_KEY, KD_, VB_, 1>(p, o, S_final, cstates, NCS, fl, pp, ts, vmap, 0, st);
  SCA2_TC_FWD(64, 64) SCA2_TC_FWD(64, 128)
#undef SCA2_TC_FWD
  if (p.K == 128 && VB == 64 && !ph)
    return tc::launch_fwd<SCA2_FLAVOR_KEY, 128, 64, 1>(p, o, S_final, cstates, NCS, fl, pp, ts, vmap, 0, st);
  return cudaErrorInvalidValue;
}

// read and clear the device fault word of the tensor-core kernels (synchronous)
cudaError_t tc_read_faults(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, tc::g_fault, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(tc::g_fault, &zero, sizeof(unsigned int));
}

}  // namespace sca2
