// Chunk-parallel preparation for the tensor-core scan (sm_100a): for every 64-token chunk of
// every (b, h), the inverse
//
//     T = (I + diag(beta) Gr)^{-1},   Gr = (kr kw^T / kappa) .* Dg, strictly lower
//
// (the delta-rule solve of the chunk, independent of the state) is computed once and written,
// bf16 in the tcgen05 operand layout: in training to slot 2c+1 of the saved-state buffer, where
// the forward and the backward copy it from; in inference to a compact work buffer the forward
// copies it from.  Neither walk then inverts inside its sequential chunk loop.
//
// One CTA (8 warps) per chunk and about 60 KB of shared memory, so several chunks run per SM:
// codes from the phases (keys), G = KR KW^T on the tensor cores (bounded mbarrier wait), the
// fp32 blocked inversion of the unit lower-triangular matrix, a 16-byte copy out.
#include "tc_common.cuh"

namespace sca2 {
namespace tc {

// bit 0: a bounded mbarrier wait of the preparation kernel timed out
__device__ unsigned int g_fault_prep;

// The codes are dead once G has been computed, so T (bf16) and the inversion's scratch WS
// reuse their region; about 52 KB in all, four CTAs per SM.
template <int KD>
struct PrepLayout {
  static constexpr int al(int x) { return (x + 1023) & ~1023; }
  static constexpr int KR = 0;                     // C x KD  kr [i][m]
  static constexpr int KW = KR + al(C * KD * 2);   // C x KD  kw [i][m]
  static constexpr int TB = 0;                     // C x C   T  [i][j]       (after G)
  static constexpr int WS = TB + al(C * C * 2);    // fp32 1024               (after G)
  static constexpr int LS = KW + al(C * KD * 2);   // fp32 C x LDF
  static constexpr int TS = LS + al(C * LDF * 4);  // fp32 C x LDF
  static constexpr int SC = TS + al(C * LDF * 4);  // beta, Gc, a, w [C] + lam [KD] + decay factors [C]
  static constexpr int MBAR = SC + ((5 * C + KD) * 4 + 15) / 16 * 16;
  static constexpr int TOTAL = MBAR + 16;
  static_assert(WS + 1024 * 4 <= LS, "T and WS fit the code region");
};

template <int FL, int KD, bool HG>
__global__ void __launch_bounds__(NT, 4) scan_prep_tc(sca2_scan_args p, TSlots ts, int vec,
                                                     PhaseProj pp) {
  using L = PrepLayout<KD>;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  constexpr bool has_g = HG;  // a per-token scalar decay (p.g) is present
  constexpr int KH = FL == SCA2_FLAVOR_PHASE ? KD / 2 : KD;
  const float ik = FL == SCA2_FLAVOR_PHASE ? 1.f / (float)(KD / 2) : 1.f;
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  Gates gates{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* s_lam = sc + 4 * C;
  float* s_fdec = s_lam + KD;  // column factors of the decay mask (decay_block)
  bf16* KR = reinterpret_cast<bf16*>(sm + L::KR);
  bf16* KW = reinterpret_cast<bf16*>(sm + L::KW);
  bf16* TB = reinterpret_cast<bf16*>(sm + L::TB);
  float* LS = reinterpret_cast<float*>(sm + L::LS);
  float* TS = reinterpret_cast<float*>(sm + L::TS);
  float* WS = reinterpret_cast<float*>(sm + L::WS);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);

  for (int m = tid; m < KD; m += NT) s_lam[m] = p.lam ? p.lam[h * KH + (m % KH)] : 0.f;
  if (warp == 0) {
    GateRegs gr;
    load_gate_regs(p, gr, b, h, t0, Cl);
    gates_from_regs(gr, gates, Cl);
  }
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 64);
  CodeRegs<FL, KD> cr;
  load_code_regs<FL, KD>(p, cr, vec != 0, b, h, t0, Cl, pp);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem;
  if (has_g) decay_factors(gates.Gc, s_fdec);  // visible after the barrier past the Gram product
  finish_code_regs<FL, KD>(cr, pp, h, t0, Cl);
  // ---- codes kr, kw (bf16, [i][m])
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2;
    int i, m0;
    code_unit<KD / 16>(tid, i, m0);
    const float fi = (float)i;
    float kc[8], ks[8], wc[8], ws[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float s = 0.f, co = 0.f;
      if (i < Cl) sincos_big(cr.w[0][k], &s, &co);
      const float l = s_lam[m0 + k];
      const float ell = __expf(-l * fi), elli = __expf(l * fi);
      kc[k] = co * ell; ks[k] = s * ell; wc[k] = co * elli; ws[k] = s * elli;
    }
    st8(KR, umma::kmaj(i, m0, KD), kc);
    st8(KR, umma::kmaj(i, Mh + m0, KD), ks);
    st8(KW, umma::kmaj(i, m0, KD), wc);
    st8(KW, umma::kmaj(i, Mh + m0, KD), ws);
  } else {
    constexpr int MB = KD / 8;
#pragma unroll
    for (int u = 0; u < CodeRegs<FL, KD>::NU; ++u) {
      int i, m0;
      code_unit<MB>(tid + u * NT, i, m0);
      const float fi = (float)i;
      float kc[8], wc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float l = s_lam[m0 + k];
        kc[k] = cr.w[u][k] * __expf(-l * fi);
        wc[k] = cr.w[u][k] * __expf(l * fi);
      }
      st8(KR, umma::kmaj(i, m0, KD), kc);
      st8(KW, umma::kmaj(i, m0, KD), wc);
    }
  }
  publish_smem();
  if (tid == 0) {
    umma::gemm(tb, KR, KW, 64, 64, KD, false);
    umma::commit(mbar);
  }
  const bool ok = umma::mbar_wait(mbar, 0);
  __syncthreads();
  umma::fence_after_sync();
  if (ok) {
    // L = beta Gr (fp32, strictly lower), then T
    for_frag<64, 64>(tb, [&](int i, int j0, int, const float* x) {
      const float bi = gates.beta[i] * ik;
      float dg[16];
      if (has_g) decay_block(gates.Gc, s_fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
    });
    __syncthreads();
    invert_unit_lower(LS, TS, WS);
    store_T<false>(TS, TB);
    __syncthreads();
    uint8_t* dst = ts.base + (int64_t)bh * ts.bh_stride + (int64_t)c * ts.c_stride;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(TB);
    for (int u = tid * 16; u < C * C * 2; u += NT * 16)
      *reinterpret_cast<uint4*>(dst + u) = *reinterpret_cast<const uint4*>(src + u);
  } else {
    if (tid == 0) atomicOr(&g_fault_prep, 1u);
    umma::mbar_wait(mbar, 0);  // bounded: let the MMA drain before the columns are freed
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 64);
}

}  // namespace tc

// T of every chunk where ts says (K = 64); vec: 16-byte loads of the phases / keys
cudaError_t tc_scan_prep(const sca2_scan_args& p, const tc::TSlots& ts, int vec, const PhaseProj& pp,
                         cudaStream_t st) {
  const int NC = (p.T + tc::C - 1) / tc::C;
  if (NC == 0) return cudaSuccess;
  const int smem = tc::PrepLayout<64>::TOTAL;
  dim3 grid(NC, p.B * p.H);
  if (p.flavor == SCA2_FLAVOR_PHASE) {
    auto k = p.g.ptr ? tc::scan_prep_tc<SCA2_FLAVOR_PHASE, 64, true> : tc::scan_prep_tc<SCA2_FLAVOR_PHASE, 64, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k<<<grid, tc::NT, smem, st>>>(p, ts, vec, pp);
  } else {
    auto k = p.g.ptr ? tc::scan_prep_tc<SCA2_FLAVOR_KEY, 64, true> : tc::scan_prep_tc<SCA2_FLAVOR_KEY, 64, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k<<<grid, tc::NT, smem, st>>>(p, ts, vec, pp);
  }
  return cudaGetLastError();
}

// read and clear the preparation kernel's device fault word (synchronous)
cudaError_t tc_read_faults_prep(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, tc::g_fault_prep, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(tc::g_fault_prep, &zero, sizeof(unsigned int));
}

}  // namespace sca2
