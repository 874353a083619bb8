// Chunk-parallel training scan of the explicit-key delta rule (gated-delta-rule form) for
// K = V = 128, bf16 inputs, fp32 state (sm_100a).
//
// With few (batch, head) sequences and long T (B = 4, H = 8, T = 8192: 32 sequences of 128
// chunks), a walk of one CTA per sequence would leave most SMs idle.  Here the state-independent
// work of every chunk runs chunk-parallel on the tensor cores and only the two K x V recurrences
// are sequential:
//
//   chunk c (tokens i, j < 64; Gc = cumsum g, a = e^Gc, w = e^{Gc_last - Gc},
//            Dg_ij = e^{min(Gc_i - Gc_j, 0)}, v_eff = beta v (write-gated form) or v):
//     T  = (I + diag(beta) (k k^T .* Dg)_strict)^{-1}            delta solve, fp32
//     W  = T diag(beta a) k,   U = T v_eff                         (so E = U - W S)
//   sequential over c (per 32 value columns; state in fp32, products on the tensor cores):
//     E_c = U_c - W_c S_c,   S_{c+1} = a_last S_c + (w .* k)^T E_c
//   chunk-parallel again:
//     O = q_scale ((a .* q) S_c + ((q k^T) .* Dg) E_c)
//
// Backward (dS' = adjoint of the state leaving chunk c, P = q_scale (q k^T) .* Dg):
//     Yo = T^T P^T dO,   Mt = T^T diag(w) k                        chunk-parallel
//     dY_c = Yo_c + Mt_c dS',   dS = a_last dS' + q_scale (a .* q)^T dO - (beta a .* k)^T dY_c
//                                                                  sequential
//     every per-token gradient of chunk c from (S_c, E_c, dY_c, dS')   chunk-parallel
//
// This is the algebra of the reference's chunk closed form (lapa/layer.py:298-366 with the
// scalar-decay mask of sca2/arch_gatedc.py:136-139; fla 0.5.1 naive_chunk_gated_delta_rule as
// called at lapa/benchmarks/baselines.py:111-120), regrouped so that the sequential part is
// two small products per chunk.  Tensor-core operands are single bf16 (the state chain itself
// stays fp32); the saved per-chunk data live in the four slots of each chunk:
//   slot 4c    S_c as hi | lo (K x V bf16 each, operand layout)
//   slot 4c+1  E_c (64 x V bf16, operand layout) | backward: sum(S_c .* dS') per block of 32 value
//              columns (fp32, from the fp32 adjoint and the hi + lo state) | T (64 x 64 fp32, zeros
//              above the diagonal)
//   slot 4c+2  W | w .* k (64 x K bf16 each, operand layout) | U (64 x V fp32)
//              backward: Mt (64 x K bf16, operand layout) | Yo, then dY (64 x V fp32)
//   slot 4c+3  backward: dS' (K x V bf16, operand layout) | [q_scale a .* q ; -beta a .* k] (128 x K
//              bf16, operand layout)
// The backward overwrites only what it recomputes (W, U by Mt, Yo; nothing the forward saved for
// it), so it can run more than once on one forward's data.
// The two recurrences also run on the tensor cores: per chunk one product into TMEM for the
// token rows (E or dY, M = 64) and one for the state rows (M = 128); the state and its adjoint
// stay in fp32 registers (16 columns of a key row per thread) and enter the products as hi + lo
// bf16 pairs.
#include "tc_common.cuh"

namespace sca2 {
namespace cp {

using tc::C;
using tc::NT;
using tc::LDF;
using tc::Gates;
using tc::bf16;

constexpr int KD = 128, VD = 128, KV = KD * VD;
constexpr int VB = 32;  // value columns per CTA of the sequential passes
constexpr int VBP = VB + 4;  // fp32 staging row stride (rows 16-byte aligned, 4 banks apart)
constexpr int VBR = VB + 8;  // bf16 staging row stride (rows 16-byte aligned, 20 banks apart)
constexpr int OFF_T = C * VD, OFF_U = C * KD;
constexpr int OFF_KW = C * KD / 2;  // floats: w .* k (bf16) after W (bf16) in slot 4c+2
constexpr int OFF_A2 = KD * VD / 2; // floats: the stacked backward operand in slot 4c+3, after dS'
constexpr int OFF_LO = KD * VD / 2; // floats: the state's lo part in slot 4c
constexpr int OFF_P = C * VD / 2;   // floats: the S .* dS' partial sums in slot 4c+1, after E

// bit 0: a bounded mbarrier wait of a chunk-parallel kernel timed out
__device__ unsigned int g_fault_cp;

__host__ __device__ constexpr int al(int x) { return (x + 1023) & ~1023; }

__device__ __forceinline__ float* slot(float* cs, int bh, int NS, int c, int s) {
  return cs + ((int64_t)bh * NS + 4 * c + s) * KV;
}

// 64 token rows of a 128-wide bf16 per-token tensor into a K-major operand (zeros past Cl)
__device__ __forceinline__ void load_rows(bf16* dst, const bf16* base, int64_t sb, int64_t st, int64_t sh, int b,
                                          int t0, int h, int Cl, bool vec) {
  for (int u = threadIdx.x; u < C * 16; u += NT) {
    const int i = (u & 7) + 8 * (u >> 7), c0 = ((u >> 3) & 15) * 8;
    const bool live = i < Cl;
    const bf16* src = base + (live ? (int64_t)b * sb + (int64_t)(t0 + i) * st + (int64_t)h * sh + c0 : 0);
    bf16* d = dst + umma::kmaj(i, c0, 128);
    if (vec) {
      tc::cp16(d, src, live);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) d[k] = live ? src[k] : __float2bfloat16_rn(0.f);
    }
  }
}

// M = 64 accumulators read together: NA bases, N columns; f(row, col0, v[NA][16]) on lanes < 16
template <int N, int NA, class F>
__device__ __forceinline__ void frag_multi(const uint32_t* tb, F f) {
  const int warp = threadIdx.x >> 5, sub = warp & 3;
  const bool own = (threadIdx.x & 31) < 16;
  const int row = 16 * sub + (threadIdx.x & 31);
#pragma unroll
  for (int q = 0; q < N / 32; ++q) {
    const int col0 = (threadIdx.x >> 7) * (N / 2) + 16 * q;
    uint32_t r[NA][16];
#pragma unroll
    for (int a = 0; a < NA; ++a) umma::ld16_issue(umma::taddr(tb[a], 32 * sub, col0), r[a]);
    umma::ld_wait();
    float v[NA][16];
#pragma unroll
    for (int a = 0; a < NA; ++a) umma::take<16>(r[a], v[a]);
    if (own) f(row, col0, v);
  }
}

// nbytes (a multiple of 16 * NTHR) from global to shared, 16-byte async copies
template <int NTHR>
__device__ __forceinline__ void flat_copy(void* dst, const void* src, int nbytes) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  const uint4* g = reinterpret_cast<const uint4*>(src);
  for (int u = threadIdx.x; u < nbytes / 16; u += NTHR) tc::cp16(d + u, g + u, true);
}

__device__ __forceinline__ void unpack8(const bf16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) { x[2 * k] = __low2float(h2[k]); x[2 * k + 1] = __high2float(h2[k]); }
}

// one bulk copy global -> shared (16-byte aligned, size a multiple of 16) completing on `bar`;
// the issuing thread first announces the bytes with bulk_expect
__device__ __forceinline__ void bulk_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(umma::smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(umma::smem_u32(dst)), "l"(src), "r"(bytes), "r"(umma::smem_u32(bar))
               : "memory");
}

// bounded wait on the batch mbarrier; on timeout the fault word is set and false returned
// (the result is the same in every thread of the CTA)
__device__ __forceinline__ bool batch_wait(uint64_t* mbar, uint32_t parity) {
  const bool ok = umma::mbar_wait(mbar, parity);
  const bool bad = __syncthreads_or(!ok) != 0;
  umma::fence_after_sync();
  if (bad && threadIdx.x == 0) atomicOr(&g_fault_cp, 1u);
  return !bad;
}

// (warp 0) and, with a decay, the column factors of the decay mask (tc::decay_factors) in fdec
__device__ __forceinline__ void load_gates(const sca2_scan_args& p, const Gates& g, int b, int h, int t0, int Cl,
                                           float* fdec) {
  if ((threadIdx.x >> 5) == 0) {
    tc::GateRegs gr;
    tc::load_gate_regs(p, gr, b, h, t0, Cl);
    tc::gates_from_regs(gr, g, Cl);
    if (p.g.ptr) tc::decay_factors_warp(g.Gc, fdec);
  }
}

// ======================================================================================
//  F1: T, W = T diag(beta a) k, U = T v_eff per chunk
// ======================================================================================
// 75 KB of shared memory and 128 TMEM columns: three CTAs per SM.  T's two scaled operand
// copies reuse the region of L (dead after the inversion); W and U take turns in TMEM.
struct PrepL {
  static constexpr int KB = 0, VBUF = KB + al(C * KD * 2), LS = VBUF + al(C * VD * 2), TW = LS, TV = TW + C * C * 2,
                       TS = LS + al(C * LDF * 4), WS = TS + al(C * LDF * 4), SC = WS + 4096, MBAR = SC + 5 * C * 4,
                       TOTAL = MBAR + 16;
  static_assert(2 * C * C * 2 <= C * LDF * 4, "T's operand copies fit the region of L");
};

__global__ void __launch_bounds__(NT, 3) cp_prep(sca2_scan_args p, float* cs, int NS, int vec) {
  using L = PrepL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  bf16* KBf = reinterpret_cast<bf16*>(sm + L::KB);
  bf16* VBf = reinterpret_cast<bf16*>(sm + L::VBUF);
  bf16* TW = reinterpret_cast<bf16*>(sm + L::TW);
  bf16* TV = reinterpret_cast<bf16*>(sm + L::TV);
  float* LS = reinterpret_cast<float*>(sm + L::LS);
  float* TS = reinterpret_cast<float*>(sm + L::TS);
  float* WS = reinterpret_cast<float*>(sm + L::WS);
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* fdec = sc + 4 * C;  // decay-mask column factors (tc::decay_block)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;

  load_gates(p, gt, b, h, t0, Cl, fdec);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 128);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  load_rows(VBf, reinterpret_cast<const bf16*>(p.v.ptr), p.v.sb, p.v.st, p.v.sh, b, t0, h, Cl, vec);
  tc::cp_commit();
  tc::cp_wait_all();
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
  if (tid == 0) {
    umma::gemm(tb, KBf, KBf, 64, 64, KD, false);
    umma::commit(mbar);
  }
  bool ok = batch_wait(mbar, 0);
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int i, int j0, int, const float* x) {
      const float bi = gt.beta[i];
      float dg[16];
      if (has_g) tc::decay_block(gt.Gc, fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
    });
    umma::fence_before_sync();
    __syncthreads();
    tc::invert_unit_lower(LS, TS, WS);
    // T out (fp32, zeros above the diagonal) and the two scaled operand copies
    float* Tg = slot(cs, bh, NS, c, 1) + OFF_T;
    for (int u = tid; u < C * C / 4; u += NT) {
      const int i = u >> 4, j0 = (u & 15) * 4;
      float4 x;
      x.x = j0 <= i ? TS[i * LDF + j0] : 0.f;
      x.y = j0 + 1 <= i ? TS[i * LDF + j0 + 1] : 0.f;
      x.z = j0 + 2 <= i ? TS[i * LDF + j0 + 2] : 0.f;
      x.w = j0 + 3 <= i ? TS[i * LDF + j0 + 3] : 0.f;
      *reinterpret_cast<float4*>(Tg + i * C + j0) = x;
    }
    const bool vtb = p.v_times_beta != 0;
    for (int u = tid; u < C * C / 8; u += NT) {
      const int i = (u & 7) + 8 * (u >> 6), j0 = ((u >> 3) & 7) * 8;
      float xw[8], xv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int j = j0 + k;
        const float t = j <= i ? TS[i * LDF + j] : 0.f;
        xw[k] = t * gt.beta[j] * gt.a[j];
        xv[k] = vtb ? t * gt.beta[j] : t;
      }
      tc::st8(TW, umma::kmaj(i, j0, C), xw);
      tc::st8(TV, umma::kmaj(i, j0, C), xv);
    }
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, TW, false, KBf, true, 64, KD, C, false);         // W = (T beta a) k
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      float* Wg = slot(cs, bh, NS, c, 2);
      bf16* Wb = reinterpret_cast<bf16*>(Wg);
      bf16* KWg = reinterpret_cast<bf16*>(Wg + OFF_KW);
      tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
        tc::st8(Wb, umma::kmaj(i, j0, KD), x);
        tc::st8(Wb, umma::kmaj(i, j0 + 8, KD), x + 8);
      });
      for (int u = tid; u < C * KD / 8; u += NT) {  // w .* k, same layout
        const int i = u >> 4, m0 = (u & 15) * 8;
        float x[8];
        unpack8(KBf + umma::kmaj(i, m0, KD), x);
        const float wi = gt.w[i];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] *= wi;
        tc::st8(KWg, umma::kmaj(i, m0, KD), x);
      }
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
      if (tid == 0) {
        umma::gemm_t(tb, TV, false, VBf, true, 64, VD, C, false);  // U = (T [beta]) v
        umma::commit(mbar);
      }
      ok = batch_wait(mbar, 0);
      if (ok)
        tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
          float4* d = reinterpret_cast<float4*>(Wg + OFF_U + i * VD + j0);
#pragma unroll
          for (int k = 0; k < 4; ++k) d[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
        });
    }
  }
  if (!ok) umma::mbar_wait(mbar, 0), umma::mbar_wait(mbar, 1);  // bounded: let the MMAs drain
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 128);
}

// ======================================================================================
//  F2: the forward state recurrence (sequential over chunks, 32 value columns per CTA, fp32)
// ======================================================================================
__device__ __forceinline__ void cp4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(umma::smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}

// per-chunk gate inputs g (and beta) into smem (zeros past Cl), 4-byte async copies
__device__ __forceinline__ void prefetch_gates(const sca2_scan_args& p, float* gbuf, float* bbuf, int b, int h,
                                               int t0, int Cl) {
  const int i = threadIdx.x;
  if (i < C) {
    const float* gp = reinterpret_cast<const float*>(p.g.ptr);
    const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
    const bool lg = gp && i < Cl, lb = bp && i < Cl;
    const float* any = reinterpret_cast<const float*>(p.v.ptr);  // a valid address for zero-size copies
    cp4(gbuf + i, lg ? gp + tok_off(p.g, b, t0 + i, h) : any, lg);
    if (bbuf) cp4(bbuf + i, lb ? bp + tok_off(p.beta, b, t0 + i, h) : any, lb);
  }
}

// warp 0: Gc, a, w and a_last of a chunk from g in smem (g = 0 past Cl)
__device__ __forceinline__ void gates_from_g(const float* gbuf, float* Gc, float* a, float* w, float* aL, int Cl) {
  if ((threadIdx.x >> 5) != 0) return;
  const int l = threadIdx.x & 31;
  const float s0 = warp_incl_scan(gbuf[l]);
  const float tot0 = __shfl_sync(0xffffffffu, s0, 31);
  const float s1 = warp_incl_scan(gbuf[l + 32]) + tot0;
  const float sel = (Cl - 1) < 32 ? s0 : s1;
  const float Gl = __shfl_sync(0xffffffffu, sel, (Cl - 1) & 31);
  Gc[l] = s0;
  Gc[l + 32] = s1;
  a[l] = expf(s0);
  a[l + 32] = expf(s1);
  w[l] = l < Cl ? exp_le0(Gl - s0) : 0.f;
  w[l + 32] = l + 32 < Cl ? exp_le0(Gl - s1) : 0.f;
  if (l == 0) *aL = expf(Gl);
}

// The state recurrence on the tensor cores, one CTA of 8 warps per (b, h, 32 value columns):
//   E = U - W (S_hi + S_lo)         M = 64 tokens, N = 32, K = 128 keys
//   S' = a_last S + (w .* k)^T E    M = 128 keys, N = 32, K = 64 tokens
// A thread keeps 16 columns of one key row of S in fp32 registers.  The next chunk's W, w .* k
// (bulk copies), U and g (cp.async) are prefetched while the current chunk runs.
struct StateFL {
  static constexpr int WB = 0, KW = WB + 2 * C * KD * 2, U = KW + 2 * C * KD * 2, SH = U + 2 * C * VBP * 4,
                       SL = SH + KD * VB * 2, EB = SL + KD * VB * 2, G = EB + C * VB * 2, SC = G + 2 * C * 4,
                       MBAR = SC + 16, LBAR = MBAR + 16, TOTAL = LBAR + 16;
};

// warp 0: exp of the chunk's summed log-decay (g = 0 past the chunk's end)
__device__ __forceinline__ void chunk_decay(const float* gbuf, float* aL) {
  if ((threadIdx.x >> 5) != 0) return;
  const int l = threadIdx.x & 31;
  const float s = warp_sum(gbuf[l] + gbuf[l + 32]);
  if (l == 0) *aL = expf(s);
}

// 32 fp32 columns of an M = 128 accumulator row (thread t = row t; warps 0-3)
__device__ __forceinline__ void ld_row32(uint32_t tbase, float* v) {
  const int w = threadIdx.x >> 5;
  uint32_t r[2][16];
  umma::ld16_issue(umma::taddr(tbase, 32 * w, 0), r[0]);
  umma::ld16_issue(umma::taddr(tbase, 32 * w, 16), r[1]);
  umma::ld_wait();
  umma::take<16>(r[0], v);
  umma::take<16>(r[1], v + 16);
}

// 8 warps (both recurrences): warp w reads TMEM sub-partition w % 4 and owns value columns
// 16 (w / 4) .. + 15 of its rows, so each epilogue handles 16 columns per thread.
constexpr int NQF = 256;
__global__ void __launch_bounds__(NQF, 1) cp_state_fwd(sca2_scan_args p, float* cs, int NS, float* S_final) {
  using L = StateFL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, sub = warp & 3, c0 = (warp >> 2) * 16;
  const int m = 32 * sub + lane;  // key row of this thread's state columns
  const int vb = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C, n_base = vb * VB;
  bf16* WB = reinterpret_cast<bf16*>(sm + L::WB);
  bf16* KWB = reinterpret_cast<bf16*>(sm + L::KW);
  float* Ub = reinterpret_cast<float*>(sm + L::U);
  bf16* SH = reinterpret_cast<bf16*>(sm + L::SH);
  bf16* SL = reinterpret_cast<bf16*>(sm + L::SL);
  bf16* EB = reinterpret_cast<bf16*>(sm + L::EB);
  float* Gb = reinterpret_cast<float*>(sm + L::G);
  float* aL = reinterpret_cast<float*>(sm + L::SC);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  uint64_t* lbar = reinterpret_cast<uint64_t*>(sm + L::LBAR);  // bulk loads of W, w .* k per buffer

  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::mbar_init(lbar, 1);
    umma::mbar_init(lbar + 1, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 64);
  // 16 columns of key row m of the incoming state, and their hi / lo operand copy
  float S[16];
  {
    const float* src = p.S0 ? p.S0 + (int64_t)bh * KV + m * VD + n_base + c0 : nullptr;
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 x = src ? *reinterpret_cast<const float4*>(src + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      S[k] = x.x; S[k + 1] = x.y; S[k + 2] = x.z; S[k + 3] = x.w;
    }
#pragma unroll
    for (int k = 0; k < 16; k += 8) tc::st8_split(SH, SL, umma::kmaj(m, c0 + k, VB), S + k);
  }
  uint32_t pend = 0;  // buffers with a bulk load not yet waited for
  auto prefetch = [&](int c) {
    const int buf = c & 1, t0 = c * C, Cl = min(C, p.T - t0);
    const float* Wg = slot(cs, bh, NS, c, 2);
    pend |= 1u << buf;
    if (tid == 0) {  // W and w .* k: two contiguous 16 KB operand tiles
      bulk_expect(lbar + buf, 2 * C * KD * 2);
      bulk_load(WB + buf * C * KD, Wg, C * KD * 2, lbar + buf);
      bulk_load(KWB + buf * C * KD, Wg + OFF_KW, C * KD * 2, lbar + buf);
    }
    float* ud = Ub + buf * C * VBP;
    for (int u = tid; u < C * VB / 4; u += NQF) {
      const int i = u >> 3, n = (u & 7) * 4;
      tc::cp16(ud + i * VBP + n, Wg + OFF_U + i * VD + n_base + n, true);
    }
    prefetch_gates(p, Gb + buf * C, nullptr, b, h, t0, Cl);
    tc::cp_commit();
  };
  prefetch(0);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem, tE = tb, tS = tb + 32;
  uint32_t ph = 0, lph = 0;
  bool ok = true;
  for (int c = 0; c < NC && ok; ++c) {
    const int buf = c & 1;
    tc::cp_wait_all();
    ok = batch_wait(lbar + buf, (lph >> buf) & 1);
    lph ^= 1u << buf;
    pend &= ~(1u << buf);
    if (!ok) break;
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tE, WB + buf * C * KD, false, SH, true, 64, VB, KD, false);
      umma::gemm_t(tE, WB + buf * C * KD, false, SL, true, 64, VB, KD, true);
      umma::commit(mbar);
    }
    if (c + 1 < NC) prefetch(c + 1);
    chunk_decay(Gb + buf * C, aL);
    {  // the state entering chunk c: hi (the operand of q S and dY S^T) and lo, operand layout
      bf16* Sg = reinterpret_cast<bf16*>(slot(cs, bh, NS, c, 0));
#pragma unroll
      for (int k = 0; k < 16; k += 8) tc::st8_split(Sg, Sg + 2 * OFF_LO, umma::kmaj(m, n_base + c0 + k, VD), S + k);
    }
    ok = batch_wait(mbar, ph);
    ph ^= 1;
    if (!ok) break;
    {  // E rows: lanes 0-15 of warp w hold tokens 16 (w % 4) .. + 15 (the loads are warp-wide)
      uint32_t r[16];
      umma::ld16_issue(umma::taddr(tE, 32 * sub, c0), r);
      umma::ld_wait();
      float e[16];
      umma::take<16>(r, e);
      const int i = 16 * sub + (lane & 15);
      const float4* ur = reinterpret_cast<const float4*>(Ub + buf * C * VBP + i * VBP + c0);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 u4 = ur[k];
        e[4 * k] = u4.x - e[4 * k]; e[4 * k + 1] = u4.y - e[4 * k + 1];
        e[4 * k + 2] = u4.z - e[4 * k + 2]; e[4 * k + 3] = u4.w - e[4 * k + 3];
      }
      bf16* Eg = reinterpret_cast<bf16*>(slot(cs, bh, NS, c, 1));
      if (lane < 16) {
#pragma unroll
        for (int k = 0; k < 16; k += 8) {
          tc::st8(Eg, umma::kmaj(i, n_base + c0 + k, VD), e + k);
          tc::st8(EB, umma::kmaj(i, c0 + k, VB), e + k);
        }
      }
    }
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tS, KWB + buf * C * KD, true, EB, true, 128, VB, C, false);
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, ph);
    ph ^= 1;
    if (!ok) break;
    uint32_t r[16];
    umma::ld16_issue(umma::taddr(tS, 32 * sub, c0), r);
    umma::ld_wait();
    float acc[16];
    umma::take<16>(r, acc);
    const float al_ = *aL;
#pragma unroll
    for (int k = 0; k < 16; ++k) S[k] = fmaf(al_, S[k], acc[k]);
#pragma unroll
    for (int k = 0; k < 16; k += 8) tc::st8_split(SH, SL, umma::kmaj(m, c0 + k, VB), S + k);
  }
  if (ok && S_final) {
    float* dst = S_final + (int64_t)bh * KV + m * VD + n_base + c0;
#pragma unroll
    for (int k = 0; k < 16; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(S[k], S[k + 1], S[k + 2], S[k + 3]);
  }
  tc::cp_wait_all();
  for (int q = 0; q < 2; ++q)  // after a fault: let issued bulk loads land before the CTA exits (bounded)
    if ((pend >> q) & 1) umma::mbar_wait(lbar + q, (lph >> q) & 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 64);
}

// ======================================================================================
//  F3: outputs O = q_scale (a .* (q S_c) + ((q k^T) .* Dg) E_c)
// ======================================================================================
// 73 KB of shared memory (E is fetched into k's place once q k^T is done) and 128 TMEM columns:
// three CTAs per SM.  The decay a enters as a row scale of q, so q S and P E share one
// accumulator.
struct OutL {
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), EB = KB, SB = KB + al(C * KD * 2),
                       PB = SB + al(KD * VD * 2), SC = PB + al(C * C * 2), MBAR = SC + 5 * C * 4,
                       TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 3) cp_out(sca2_scan_args p, sca2_out o, const float* cs_, int NS, int vec,
                                                int ovec) {
  using L = OutL;
  extern __shared__ __align__(1024) uint8_t sm[];
  float* cs = const_cast<float*>(cs_);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  bf16* QB = reinterpret_cast<bf16*>(sm + L::QB);
  bf16* KBf = reinterpret_cast<bf16*>(sm + L::KB);
  bf16* SB = reinterpret_cast<bf16*>(sm + L::SB);
  bf16* EB = reinterpret_cast<bf16*>(sm + L::EB);
  bf16* PB = reinterpret_cast<bf16*>(sm + L::PB);
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* fdec = sc + 4 * C;  // decay-mask column factors (tc::decay_block)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;
  const float qs = p.q_scale;

  load_gates(p, gt, b, h, t0, Cl, fdec);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 128);
  load_rows(QB, reinterpret_cast<const bf16*>(p.phq.ptr), p.phq.sb, p.phq.st, p.phq.sh, b, t0, h, Cl, vec);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  flat_copy<NT>(SB, slot(cs, bh, NS, c, 0), KD * VD * 2);
  tc::cp_commit();
  tc::cp_wait_all();
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
  if (tid == 0) {
    umma::gemm(tb, QB, KBf, 64, 64, KD, false);  // q k^T
    umma::commit(mbar);
  }
  bool ok = batch_wait(mbar, 0);
  if (ok) {
    flat_copy<NT>(EB, slot(cs, bh, NS, c, 1), C * VD * 2);  // over k (read by the product)
    tc::cp_commit();
    tc::for_frag<64, 64>(tb, [&](int i, int j0, int, const float* x) {
      float y[16], dg[16];
      if (has_g) tc::decay_block(gt.Gc, fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        y[j] = jj <= i ? x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
      tc::st8(PB, umma::kmaj(i, j0, C), y);
      tc::st8(PB, umma::kmaj(i, j0 + 8, C), y + 8);
    });
    for (int u = tid; u < C * KD / 8; u += NT) {  // q -> a .* q in place
      const int r = ((u >> 7) << 3) + (u & 7);
      float xv[8];
      unpack8(QB + 8 * u, xv);
      const float f = gt.a[r];
#pragma unroll
      for (int k = 0; k < 8; ++k) xv[k] *= f;
      tc::st8(QB, 8 * u, xv);
    }
    tc::cp_wait_all();
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, QB, false, SB, true, 64, VD, KD, false);  // (a .* q) S
      umma::gemm_t(tb, PB, false, EB, true, 64, VD, C, true);    // + P E
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      bf16* ob = reinterpret_cast<bf16*>(o.ptr);
      tc::for_frag<64, 128>(tb, [&](int i, int col0, int, const float* v) {
        if (i >= Cl) return;
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = qs * v[j];
        bf16* dst = ob + out_off(o, b, t0 + i, h, 0) + col0;
        if (ovec) {
          uint4 u0, u1;
          u0.x = tc::pack2(y[0], y[1]); u0.y = tc::pack2(y[2], y[3]); u0.z = tc::pack2(y[4], y[5]); u0.w = tc::pack2(y[6], y[7]);
          u1.x = tc::pack2(y[8], y[9]); u1.y = tc::pack2(y[10], y[11]); u1.z = tc::pack2(y[12], y[13]); u1.w = tc::pack2(y[14], y[15]);
          reinterpret_cast<uint4*>(dst)[0] = u0;
          reinterpret_cast<uint4*>(dst)[1] = u1;
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) dst[j] = __float2bfloat16_rn(y[j]);
        }
      });
    }
  }
  if (!ok) umma::mbar_wait(mbar, 0), umma::mbar_wait(mbar, 1);
  tc::cp_wait_all();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 128);
}

// ======================================================================================
//  B1: Yo = T^T P^T dO and Mt = T^T diag(w) k per chunk
// ======================================================================================
// 73 KB of shared memory (P^T dO takes the place of dO once formed) and 128 TMEM columns, the
// products one after another: three CTAs per SM.
struct BPrepL {
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), DOB = KB + al(C * KD * 2), PB = DOB + al(C * VD * 2),
                       TB = PB + al(C * C * 2), TWB = TB + al(C * C * 2), Z1 = DOB,
                       SC = TWB + al(C * C * 2), MBAR = SC + 5 * C * 4, TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 3) cp_bprep(sca2_scan_args p, sca2_out dO, float* cs, int NS, int vec,
                                                  int dvec) {
  using L = BPrepL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  bf16* QB = reinterpret_cast<bf16*>(sm + L::QB);
  bf16* KBf = reinterpret_cast<bf16*>(sm + L::KB);
  bf16* DOB = reinterpret_cast<bf16*>(sm + L::DOB);
  bf16* PB = reinterpret_cast<bf16*>(sm + L::PB);
  bf16* TB = reinterpret_cast<bf16*>(sm + L::TB);
  bf16* TWB = reinterpret_cast<bf16*>(sm + L::TWB);
  bf16* Z1 = reinterpret_cast<bf16*>(sm + L::Z1);
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* fdec = sc + 4 * C;  // decay-mask column factors (tc::decay_block)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;
  const float qs = p.q_scale;

  load_gates(p, gt, b, h, t0, Cl, fdec);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 128);
  load_rows(QB, reinterpret_cast<const bf16*>(p.phq.ptr), p.phq.sb, p.phq.st, p.phq.sh, b, t0, h, Cl, vec);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  load_rows(DOB, reinterpret_cast<const bf16*>(dO.ptr), dO.sb, dO.st, dO.sh, b, t0, h, Cl, dvec);
  tc::cp_commit();
  tc::publish_smem();  // gates
  {
    const float* Tg = slot(cs, bh, NS, c, 1) + OFF_T;
    for (int u = tid; u < C * C / 8; u += NT) {
      const int i = (u & 7) + 8 * (u >> 6), j0 = ((u >> 3) & 7) * 8;
      const float4 x0 = *reinterpret_cast<const float4*>(Tg + i * C + j0);
      const float4 x1 = *reinterpret_cast<const float4*>(Tg + i * C + j0 + 4);
      float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      tc::st8(TB, umma::kmaj(i, j0, C), x);
      const float wi = gt.w[i];
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] *= wi;
      tc::st8(TWB, umma::kmaj(i, j0, C), x);
    }
  }
  tc::cp_wait_all();
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
  if (tid == 0) {
    umma::gemm(tb, QB, KBf, 64, 64, KD, false);  // q k^T
    umma::commit(mbar);
  }
  bool ok = batch_wait(mbar, 0);
  if (ok) {
    tc::for_frag<64, 64>(tb, [&](int i, int j0, int, const float* x) {
      float y[16], dg[16];
      if (has_g) tc::decay_block(gt.Gc, fdec, i, j0, dg);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        y[j] = jj <= i ? qs * x[j] * (has_g ? dg[j] : 1.f) : 0.f;
      }
      tc::st8(PB, umma::kmaj(i, j0, C), y);
      tc::st8(PB, umma::kmaj(i, j0 + 8, C), y + 8);
    });
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, PB, true, DOB, true, 64, VD, C, false);         // P^T dO
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      float* Mg = slot(cs, bh, NS, c, 2);
      bf16* Mb = reinterpret_cast<bf16*>(Mg);
      tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {  // over dO (read by the product)
        tc::st8(Z1, umma::kmaj(i, j0, VD), x);
        tc::st8(Z1, umma::kmaj(i, j0 + 8, VD), x + 8);
      });
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
      if (tid == 0) {
        umma::gemm_t(tb, TWB, true, KBf, true, 64, KD, C, false);  // (diag(w) T)^T k
        umma::commit(mbar);
      }
      ok = batch_wait(mbar, 0);
      if (ok)
        tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
          tc::st8(Mb, umma::kmaj(i, j0, KD), x);
          tc::st8(Mb, umma::kmaj(i, j0 + 8, KD), x + 8);
        });
      // [q_scale a .* q ; -beta a .* k]
      bf16* A2 = reinterpret_cast<bf16*>(slot(cs, bh, NS, c, 3) + OFF_A2);
      for (int u = tid; u < 2 * C * KD / 8; u += NT) {
        const int r = u >> 4, m0 = (u & 15) * 8, i = r & (C - 1);
        float x[8];
        unpack8((r < C ? QB : KBf) + umma::kmaj(i, m0, KD), x);
        const float f = r < C ? qs * gt.a[i] : -gt.beta[i] * gt.a[i];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] *= f;
        tc::st8(A2, umma::kmaj(r, m0, KD), x);
      }
      tc::publish_smem();
      if (ok && tid == 0) {
        umma::gemm_t(tb, TB, true, Z1, true, 64, VD, C, false);  // Yo = T^T (P^T dO)
        umma::commit(mbar);
      }
      if (ok) ok = batch_wait(mbar, 1);
      if (ok)
        tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
          float4* d = reinterpret_cast<float4*>(Mg + OFF_U + i * VD + j0);
#pragma unroll
          for (int k = 0; k < 4; ++k) d[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
        });
    }
  }
  if (!ok) umma::mbar_wait(mbar, 0), umma::mbar_wait(mbar, 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 128);
}

// ======================================================================================
//  B2: the adjoint state recurrence on the tensor cores (reverse over chunks)
// ======================================================================================
//   dY = Yo + Mt (dS'_hi + dS'_lo)                                 M = 64, N = 32, K = 128
//   dS = a_last dS' + [q_scale a .* q ; -beta a .* k]^T [dO ; dY]  M = 128, N = 32, K = 128
//        (+ the dY lo part over the second 64 rows)
struct StateBL {
  static constexpr int MB = 0, A2 = MB + 2 * C * KD * 2, Y = A2 + 2 * 2 * C * KD * 2, BS = Y + 2 * C * VBP * 4,
                       YL = BS + 2 * 2 * C * VB * 2, DH = YL + C * VB * 2, DL = DH + KD * VB * 2,
                       SR = DL + KD * VB * 2, G = SR + 2 * 2 * KD * VBR * 2, SC = G + 2 * C * 4, MBAR = SC + 48,
                       LBAR = MBAR + 16, TOTAL = LBAR + 16;
};

__global__ void __launch_bounds__(NQF, 1) cp_state_bwd(sca2_scan_args p, sca2_out dO, const float* dS_final,
                                                      float* cs, int NS, float* dS0, int dvec) {
  using L = StateBL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, sub = warp & 3, c0 = (warp >> 2) * 16;
  const int m = 32 * sub + lane;  // key row of this thread's adjoint columns
  const int vb = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C, n_base = vb * VB;
  bf16* MB = reinterpret_cast<bf16*>(sm + L::MB);
  bf16* A2 = reinterpret_cast<bf16*>(sm + L::A2);
  float* Yb = reinterpret_cast<float*>(sm + L::Y);
  bf16* BS = reinterpret_cast<bf16*>(sm + L::BS);  // [dO ; dY_hi] (128 x 32), two buffers
  bf16* YL = reinterpret_cast<bf16*>(sm + L::YL);
  bf16* DH = reinterpret_cast<bf16*>(sm + L::DH);
  bf16* DL = reinterpret_cast<bf16*>(sm + L::DL);
  bf16* SR = reinterpret_cast<bf16*>(sm + L::SR);  // [buf][hi, lo][key row][32] of the state entering the chunk
  float* Gb = reinterpret_cast<float*>(sm + L::G);
  float* aL = reinterpret_cast<float*>(sm + L::SC);
  float* red = aL + 1;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  uint64_t* lbar = reinterpret_cast<uint64_t*>(sm + L::LBAR);  // bulk loads of Mt and the stacked operand

  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::mbar_init(lbar, 1);
    umma::mbar_init(lbar + 1, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 64);
  float D[16];  // 16 columns of key row m of the adjoint state
  {
    const float* src = dS_final ? dS_final + (int64_t)bh * KV + m * VD + n_base + c0 : nullptr;
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 x = src ? *reinterpret_cast<const float4*>(src + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      D[k] = x.x; D[k + 1] = x.y; D[k + 2] = x.z; D[k + 3] = x.w;
    }
#pragma unroll
    for (int k = 0; k < 16; k += 8) tc::st8_split(DH, DL, umma::kmaj(m, c0 + k, VB), D + k);
  }
  uint32_t pend = 0;  // buffers with a bulk load not yet waited for
  auto prefetch = [&](int c) {
    const int buf = c & 1, t0 = c * C, Cl = min(C, p.T - t0);
    const float* Mg = slot(cs, bh, NS, c, 2);
    pend |= 1u << buf;
    if (tid == 0) {  // Mt (16 KB) and the stacked operand (32 KB), contiguous operand tiles
      bulk_expect(lbar + buf, 3 * C * KD * 2);
      bulk_load(MB + buf * C * KD, Mg, C * KD * 2, lbar + buf);
      bulk_load(A2 + buf * 2 * C * KD, slot(cs, bh, NS, c, 3) + OFF_A2, 2 * C * KD * 2, lbar + buf);
    }
    float* yd = Yb + buf * C * VBP;
    for (int u = tid; u < C * VB / 4; u += NQF) {
      const int i = u >> 3, n = (u & 7) * 4;
      tc::cp16(yd + i * VBP + n, Mg + OFF_U + i * VD + n_base + n, true);
    }
    bf16* dd = BS + buf * 2 * C * VB;
    const bf16* dg = reinterpret_cast<const bf16*>(dO.ptr);
    for (int u = tid; u < C * VB / 8; u += NQF) {
      const int i = u >> 2, n = (u & 3) * 8;
      const bool live = i < Cl;
      const bf16* src = dg + (live ? out_off(dO, b, t0 + i, h, 0) + n_base + n : 0);
      bf16* d = dd + umma::kmaj(i, n, VB);
      if (dvec) {
        tc::cp16(d, src, live);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) d[k] = live ? src[k] : __float2bfloat16_rn(0.f);
      }
    }
    {  // key row m of the state entering the chunk, this thread's 16 columns, hi and lo
      const bf16* sg = reinterpret_cast<const bf16*>(slot(cs, bh, NS, c, 0));
      bf16* sr = SR + buf * 2 * KD * VBR + m * VBR + c0;
#pragma unroll
      for (int k = 0; k < 16; k += 8) {
        tc::cp16(sr + k, sg + umma::kmaj(m, n_base + c0 + k, VD), true);
        tc::cp16(sr + KD * VBR + k, sg + 2 * OFF_LO + umma::kmaj(m, n_base + c0 + k, VD), true);
      }
    }
    prefetch_gates(p, Gb + buf * C, nullptr, b, h, t0, Cl);
    tc::cp_commit();
  };
  prefetch(NC - 1);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = *s_tmem, tY = tb, tD = tb + 32;
  uint32_t ph = 0, lph = 0;
  bool ok = true;
  for (int c = NC - 1; c >= 0 && ok; --c) {
    const int buf = c & 1;
    tc::cp_wait_all();
    ok = batch_wait(lbar + buf, (lph >> buf) & 1);
    lph ^= 1u << buf;
    pend &= ~(1u << buf);
    if (!ok) break;
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tY, MB + buf * C * KD, false, DH, true, 64, VB, KD, false);
      umma::gemm_t(tY, MB + buf * C * KD, false, DL, true, 64, VB, KD, true);
      umma::commit(mbar);
    }
    if (c > 0) prefetch(c - 1);
    chunk_decay(Gb + buf * C, aL);
    {  // the adjoint of the state leaving chunk c (bf16, operand layout), and sum(S_c .* dS')
      bf16* dSg = reinterpret_cast<bf16*>(slot(cs, bh, NS, c, 3));
#pragma unroll
      for (int k = 0; k < 16; k += 8) tc::st8(dSg, umma::kmaj(m, n_base + c0 + k, VD), D + k);
      const bf16* sr = SR + buf * 2 * KD * VBR + m * VBR + c0;
      float sd = 0.f;
#pragma unroll
      for (int k = 0; k < 16; k += 8) {
        float hi[8], lo[8];
        unpack8(sr + k, hi);
        unpack8(sr + KD * VBR + k, lo);
#pragma unroll
        for (int q = 0; q < 8; ++q) sd = fmaf(D[k + q], hi[q] + lo[q], sd);
      }
      sd = warp_sum(sd);
      if (lane == 0) red[warp] = sd;
    }
    ok = batch_wait(mbar, ph);
    ph ^= 1;
    if (!ok) break;
    if (tid == 0) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < NQF / 32; ++q) t += red[q];
      slot(cs, bh, NS, c, 1)[OFF_P + vb] = t;
    }
    {
      uint32_t r[16];
      umma::ld16_issue(umma::taddr(tY, 32 * sub, c0), r);
      umma::ld_wait();
      float y[16];
      umma::take<16>(r, y);
      const int i = 16 * sub + (lane & 15);
      const float4* yr = reinterpret_cast<const float4*>(Yb + buf * C * VBP + i * VBP + c0);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 y4 = yr[k];
        y[4 * k] += y4.x; y[4 * k + 1] += y4.y; y[4 * k + 2] += y4.z; y[4 * k + 3] += y4.w;
      }
      if (lane < 16) {
        float* Yg = slot(cs, bh, NS, c, 2) + OFF_U + i * VD + n_base + c0;
#pragma unroll
        for (int k = 0; k < 16; k += 4) *reinterpret_cast<float4*>(Yg + k) = make_float4(y[k], y[k + 1], y[k + 2], y[k + 3]);
#pragma unroll
        for (int k = 0; k < 16; k += 8) {  // dY hi below dO in the stacked operand, dY lo apart
          float hv[8], lv[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            hv[q] = __bfloat162float(__float2bfloat16_rn(y[k + q]));
            lv[q] = y[k + q] - hv[q];
          }
          tc::st8(BS + buf * 2 * C * VB, umma::kmaj(C + i, c0 + k, VB), hv);
          tc::st8(YL, umma::kmaj(i, c0 + k, VB), lv);
        }
      }
    }
    tc::publish_smem();
    if (tid == 0) {
      const bf16* a2 = A2 + buf * 2 * C * KD;
      umma::gemm_t(tD, a2, true, BS + buf * 2 * C * VB, true, 128, VB, 2 * C, false);
      umma::gemm_t(tD, a2 + umma::kmaj(C, 0, KD), true, YL, true, 128, VB, C, true);
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, ph);
    ph ^= 1;
    if (!ok) break;
    uint32_t r[16];
    umma::ld16_issue(umma::taddr(tD, 32 * sub, c0), r);
    umma::ld_wait();
    float acc[16];
    umma::take<16>(r, acc);
    const float al_ = *aL;
#pragma unroll
    for (int k = 0; k < 16; ++k) D[k] = fmaf(al_, D[k], acc[k]);
#pragma unroll
    for (int k = 0; k < 16; k += 8) tc::st8_split(DH, DL, umma::kmaj(m, c0 + k, VB), D + k);
  }
  if (ok && dS0) {
    float* dst = dS0 + (int64_t)bh * KV + m * VD + n_base + c0;
#pragma unroll
    for (int k = 0; k < 16; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(D[k], D[k + 1], D[k + 2], D[k + 3]);
  }
  tc::cp_wait_all();
  for (int q = 0; q < 2; ++q)  // after a fault: let issued bulk loads land before the CTA exits (bounded)
    if ((pend >> q) & 1) umma::mbar_wait(lbar + q, (lph >> q) & 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 64);
}

// ======================================================================================
//  B3: per-token gradients of every chunk
// ======================================================================================
struct GradL {
  static constexpr int DDP = C + 1, YFP = VD + 4;  // padded fp32 rows (dDg, dY)
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), DOB = KB + al(C * KD * 2), DYB = DOB + al(C * VD * 2),
                       EB = DYB + al(C * VD * 2), SB = EB + al(C * VD * 2), DSB = SB + al(KD * VD * 2),
                       DKK = DSB + al(KD * VD * 2), DQK = DKK + al(C * C * 2), DYF = DQK + al(C * C * 2),
                       DDG = DYF + C * YFP * 4, SC = DDG + C * DDP * 4, NSC = 4 * C + 12 * C + 16 + C, MBAR = SC + NSC * 4,
                       TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 1) cp_grads(sca2_scan_args p, sca2_out dO, const float* cs_, int NS,
                                                  sca2_scan_grads gr, int vec, int dvec) {
  using L = GradL;
  extern __shared__ __align__(1024) uint8_t sm[];
  float* cs = const_cast<float*>(cs_);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, Cl = min(C, p.T - t0);
  bf16* QB = reinterpret_cast<bf16*>(sm + L::QB);
  bf16* KBf = reinterpret_cast<bf16*>(sm + L::KB);
  bf16* DOB = reinterpret_cast<bf16*>(sm + L::DOB);
  bf16* DYB = reinterpret_cast<bf16*>(sm + L::DYB);
  bf16* EB = reinterpret_cast<bf16*>(sm + L::EB);
  bf16* SB = reinterpret_cast<bf16*>(sm + L::SB);
  bf16* DSB = reinterpret_cast<bf16*>(sm + L::DSB);
  bf16* DKK = reinterpret_cast<bf16*>(sm + L::DKK);
  bf16* DQK = reinterpret_cast<bf16*>(sm + L::DQK);
  float* DDG = reinterpret_cast<float*>(sm + L::DDG);
  float* DYF = reinterpret_cast<float*>(sm + L::DYF);
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* fdec = sc + 16 * C + 16;  // decay-mask column factors (tc::decay_block)
  float* rsum = sc + 4 * C;          // [2 halves][6 sums][C]: dbeta1, rowDg, rY, rE, rO, (spare)
  float* red = rsum + 12 * C;        // block reduction scratch (16)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr, has_beta = p.beta.ptr != nullptr;
  const bool vtb = p.v_times_beta != 0, ow = gr.overwrite != 0, gio = gr.grad_io_dtype != 0;
  const float qs = p.q_scale;
  enum { R_DB = 0, R_DG = 1, R_Y = 2, R_E = 3, R_O = 4 };
  auto rs = [&](int half, int which) { return rsum + (half * 6 + which) * C; };

  load_gates(p, gt, b, h, t0, Cl, fdec);
  for (int u = tid; u < 12 * C; u += NT) rsum[u] = 0.f;
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 512);
  load_rows(QB, reinterpret_cast<const bf16*>(p.phq.ptr), p.phq.sb, p.phq.st, p.phq.sh, b, t0, h, Cl, vec);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  load_rows(DOB, reinterpret_cast<const bf16*>(dO.ptr), dO.sb, dO.st, dO.sh, b, t0, h, Cl, dvec);
  flat_copy<NT>(SB, slot(cs, bh, NS, c, 0), KD * VD * 2);
  flat_copy<NT>(DSB, slot(cs, bh, NS, c, 3), KD * VD * 2);
  flat_copy<NT>(EB, slot(cs, bh, NS, c, 1), C * VD * 2);
  const float* Yg = slot(cs, bh, NS, c, 2) + OFF_U;
  for (int u = tid; u < C * VD / 4; u += NT) {  // dY (fp32) into padded rows
    const int i = u >> 5, n = (u & 31) * 4;
    tc::cp16(DYF + i * L::YFP + n, Yg + i * VD + n, true);
  }
  tc::cp_commit();
  tc::cp_wait_all();
  __syncthreads();
  // dY as an operand; the chunk's sum of S .* dS' (the gradient of a_last through the carry)
  auto dy_to_op = [&](auto scale) {
    for (int u = tid; u < C * 16; u += NT) {
      const int r = (u & 7) + 8 * (u >> 7), c0 = ((u >> 3) & 15) * 8;
      const float4 x0 = *reinterpret_cast<const float4*>(DYF + r * L::YFP + c0);
      const float4 x1 = *reinterpret_cast<const float4*>(DYF + r * L::YFP + c0 + 4);
      const float f = scale(r);
      float x[8] = {f * x0.x, f * x0.y, f * x0.z, f * x0.w, f * x1.x, f * x1.y, f * x1.z, f * x1.w};
      tc::st8(DYB, umma::kmaj(r, c0, VD), x);
    }
  };
  dy_to_op([](int) { return 1.f; });
  if (tid < VD / VB) red[tid] = slot(cs, bh, NS, c, 1)[OFF_P + tid];
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
  uint2 vreg[C / 8];
  if (tid == 0) {
    umma::gemm(tb, QB, KBf, 64, 64, KD, false);          // q k^T
    umma::gemm(tb + 64, KBf, KBf, 64, 64, KD, false);    // k k^T
    umma::gemm(tb + 128, DYB, EB, 64, 64, VD, false);    // dY E^T
    umma::gemm(tb + 192, DOB, EB, 64, 64, VD, false);    // dO E^T
    umma::gemm(tb + 256, DYB, SB, 64, KD, VD, false);    // dY S^T
    umma::gemm(tb + 384, EB, DSB, 64, KD, VD, false);    // E dS'^T
    umma::commit(mbar);
  }
  bool ok = batch_wait(mbar, 0);
  if (ok) {
    const int half = tid >> 7;
    // ---- C x C terms
    {
      const uint32_t bases[4] = {tb, tb + 64, tb + 128, tb + 192};
      frag_multi<64, 4>(bases, [&](int i, int j0, float (*v)[16]) {
        const float bi = gt.beta[i];
        float dkk[16], dqk[16], db1 = 0.f, rdg = 0.f, dgv[16];
        if (has_g) tc::decay_block(gt.Gc, fdec, i, j0, dgv);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          const bool incl = jj <= i, strict = jj < i;
          const float dg = incl ? (has_g ? dgv[j] : 1.f) : 0.f;
          const float qk = qs * v[0][j], gkk = v[1][j];
          const float dL = strict ? -v[2][j] : 0.f;
          const float dP = incl ? v[3][j] : 0.f;
          const float dGm = bi * dL;
          db1 = fmaf(dL, gkk * dg, db1);
          dkk[j] = dGm * dg;
          dqk[j] = qs * dP * dg;
          const float ddg = (dGm * gkk + dP * qk) * dg;
          rdg += ddg;
          DDG[i * L::DDP + jj] = ddg;
        }
        tc::st8(DKK, umma::kmaj(i, j0, C), dkk);
        tc::st8(DKK, umma::kmaj(i, j0 + 8, C), dkk + 8);
        tc::st8(DQK, umma::kmaj(i, j0, C), dqk);
        tc::st8(DQK, umma::kmaj(i, j0 + 8, C), dqk + 8);
        rs(half, R_DB)[i] += db1;
        rs(half, R_DG)[i] += rdg;
      });
    }
    // ---- row sums sum_m k_im (dY S^T)_im and sum_m k_im (E dS'^T)_im
    {
      const uint32_t bases[2] = {tb + 256, tb + 384};
      frag_multi<128, 2>(bases, [&](int i, int col0, float (*v)[16]) {
        float kx[16];
        unpack8(KBf + umma::kmaj(i, col0, KD), kx);
        unpack8(KBf + umma::kmaj(i, col0 + 8, KD), kx + 8);
        float ry = 0.f, re = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) { ry = fmaf(kx[j], v[0][j], ry); re = fmaf(kx[j], v[1][j], re); }
        rs(half, R_Y)[i] += ry;
        rs(half, R_E)[i] += re;
      });
    }
    umma::fence_before_sync();
    __syncthreads();
    // operands of the second batch: dY -> -beta a .* dY, E -> w .* E (in place)
    dy_to_op([&](int r) { return -gt.beta[r] * gt.a[r]; });
    for (int u = tid; u < C * VD / 8; u += NT) {
      const int r = ((u >> 7) << 3) + (u & 7);
      float x[8];
      unpack8(EB + 8 * u, x);
      const float f = gt.w[r];
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] *= f;
      tc::st8(EB, 8 * u, x);
    }
    tc::publish_smem();
    // the value rows for sum_v dY v, loaded while the second batch runs (one warp per 8 rows)
#pragma unroll
    for (int j = 0; j < C / 8; ++j) {
      const int i = warp + 8 * j;
      vreg[j] = i < Cl ? *reinterpret_cast<const uint2*>(reinterpret_cast<const bf16*>(p.v.ptr) +
                                                          tok_off(p.v, b, t0 + i, h) + 4 * lane)
                       : make_uint2(0u, 0u);
    }
    if (tid == 0) {
      umma::gemm_t(tb, DKK, false, KBf, true, 64, KD, C, false);   // dKK k
      umma::gemm_t(tb, DKK, true, KBf, true, 64, KD, C, true);     // dKK^T k
      umma::gemm_t(tb, DQK, true, QB, true, 64, KD, C, true);      // dQK^T q
      umma::gemm(tb, DYB, SB, 64, KD, VD, true);                   // (-beta a dY) S^T
      umma::gemm(tb, EB, DSB, 64, KD, VD, true);                   // (w E) dS'^T
      umma::gemm_t(tb + 128, DQK, false, KBf, true, 64, KD, C, false);  // dQK k
      umma::gemm(tb + 256, DOB, SB, 64, KD, VD, false);            // dO S^T
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      float* dk = reinterpret_cast<float*>(const_cast<void*>(gr.dphw.ptr));
      float* dq = reinterpret_cast<float*>(const_cast<void*>(gr.dphq.ptr));
      const uint32_t bases[3] = {tb, tb + 128, tb + 256};
      frag_multi<128, 3>(bases, [&](int i, int col0, float (*v)[16]) {
        float qx[16];
        unpack8(QB + umma::kmaj(i, col0, KD), qx);
        unpack8(QB + umma::kmaj(i, col0 + 8, KD), qx + 8);
        float ro = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) ro = fmaf(qx[j], v[2][j], ro);
        rs(half, R_O)[i] += qs * ro;
        if (i >= Cl) return;
        const float sa = qs * gt.a[i];
        if (gio) {  // io dtype (bf16), written
          float yk[16], yq[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) { yk[j] = v[0][j]; yq[j] = fmaf(sa, v[2][j], v[1][j]); }
          bf16* kb = reinterpret_cast<bf16*>(dk) + tok_off(gr.dphw, b, t0 + i, h) + col0;
          bf16* qb = reinterpret_cast<bf16*>(dq) + tok_off(gr.dphq, b, t0 + i, h) + col0;
          tc::st8(kb, 0, yk); tc::st8(kb, 8, yk + 8);
          tc::st8(qb, 0, yq); tc::st8(qb, 8, yq + 8);
          return;
        }
        float* kd = dk + tok_off(gr.dphw, b, t0 + i, h) + col0;
        float* qd = dq + tok_off(gr.dphq, b, t0 + i, h) + col0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float4 xk = make_float4(v[0][4 * k], v[0][4 * k + 1], v[0][4 * k + 2], v[0][4 * k + 3]);
          float4 xq = make_float4(fmaf(sa, v[2][4 * k], v[1][4 * k]), fmaf(sa, v[2][4 * k + 1], v[1][4 * k + 1]),
                                  fmaf(sa, v[2][4 * k + 2], v[1][4 * k + 2]), fmaf(sa, v[2][4 * k + 3], v[1][4 * k + 3]));
          if (!ow) {
            const float4 pk = reinterpret_cast<float4*>(kd)[k], pq = reinterpret_cast<float4*>(qd)[k];
            xk.x += pk.x; xk.y += pk.y; xk.z += pk.z; xk.w += pk.w;
            xq.x += pq.x; xq.y += pq.y; xq.z += pq.z; xq.w += pq.w;
          }
          reinterpret_cast<float4*>(kd)[k] = xk;
          reinterpret_cast<float4*>(qd)[k] = xq;
        }
      });
    }
  }
  if (!ok) umma::mbar_wait(mbar, 0), umma::mbar_wait(mbar, 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 512);
  // ---- dv = [beta] dY and sum_v dY v (one warp per token row)
  if (ok) {
    bf16* dvg = reinterpret_cast<bf16*>(const_cast<void*>(gr.dv.ptr));
#pragma unroll
    for (int j = 0; j < C / 8; ++j) {
      const int i = warp + 8 * j;
      if (i >= Cl) break;
      const float bi = gt.beta[i];
      const float4 y = *reinterpret_cast<const float4*>(DYF + i * L::YFP + 4 * lane);
      const float yv[4] = {y.x, y.y, y.z, y.w};
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vreg[j]);
      const float vv[4] = {__low2float(v2[0]), __high2float(v2[0]), __low2float(v2[1]), __high2float(v2[1])};
      float s = 0.f;
      bf16* dr = dvg + tok_off(gr.dv, b, t0 + i, h) + 4 * lane;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s = fmaf(yv[k], vv[k], s);
        dr[k] = __float2bfloat16_rn(vtb ? bi * yv[k] : yv[k]);
      }
      s = warp_sum(s);
      if (lane == 0) rsum[5 * C + i] = s;  // spare row of half 0
    }
  }
  __syncthreads();
  // ---- per-token scalars: dbeta, dg (reverse cumulative sum of dGc over the chunk)
  if (tid < C) {
    const int i = tid;
    auto both = [&](int w_) { return rs(0, w_)[i] + rs(1, w_)[i]; };
    float col = 0.f;
    for (int r = i; r < C; ++r) col += DDG[r * L::DDP + i];
    const float ai = gt.a[i], bi = gt.beta[i], wi = gt.w[i];
    const float rY = both(R_Y), rE = both(R_E), rO = both(R_O);
    const float da = (rO - bi * rY) * ai;
    const float dw = rE * wi;
    float dGc = both(R_DG) - col + da - dw;
    // the carry's a_last and w terms enter at the chunk's last token
    float dwsum = warp_sum(dw);
    if (C > 32) {
      __shared__ float part[2];
      if (lane == 0) part[warp] = dwsum;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      dwsum = part[0] + part[1];
    }
    float sdsum = 0.f;
#pragma unroll
    for (int k = 0; k < VD / VB; ++k) sdsum += red[k];
    if (i == Cl - 1) dGc += dwsum + gt.a[Cl - 1] * sdsum;
    if (i >= Cl) dGc = 0.f;
    // reverse inclusive scan over 64 tokens (two warps)
    const float x = __shfl_sync(0xffffffffu, dGc, 31 - lane);
    float s = warp_incl_scan(x);            // lane l holds sum over tokens (31-l .. 31) of this warp
    __shared__ float tot[2];
    const float wsum = __shfl_sync(0xffffffffu, s, 31);
    if (lane == 0) tot[warp] = wsum;
    asm volatile("bar.sync 1, 64;" ::: "memory");
    float rev = __shfl_sync(0xffffffffu, s, 31 - lane);  // sum over tokens i .. end of this warp
    if (warp == 0) rev += tot[1];
    if (i < Cl) {
      if (has_g) {
        float* dgp = reinterpret_cast<float*>(const_cast<void*>(gr.dg.ptr)) + tok_off(gr.dg, b, t0 + i, h);
        *dgp = ow ? rev : *dgp + rev;
      }
      if (has_beta) {
        const float dbt = both(R_DB) - ai * rY + (vtb ? rsum[5 * C + i] : 0.f);
        float* dbp = reinterpret_cast<float*>(const_cast<void*>(gr.dbeta.ptr)) + tok_off(gr.dbeta, b, t0 + i, h);
        *dbp = ow ? dbt : *dbp + dbt;
      }
    }
  }
}

}  // namespace cp

// Whether the chunk-parallel path covers the call: explicit keys, bf16, K = V = 128, no per-channel
// decay, 16-byte aligned rows of q, k and v.
bool cp_covers(const sca2_scan_args& p) {
  auto a16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
  auto rows = [&](const sca2_tok& t) { return a16(t.ptr) && t.sb % 8 == 0 && t.st % 8 == 0 && t.sh % 8 == 0; };
  return p.flavor == SCA2_FLAVOR_KEY && p.io_dtype == SCA2_BF16 && p.K == cp::KD && p.V == cp::VD &&
         p.lam == nullptr && rows(p.phw) && rows(p.phq) && rows(p.v);
}

static bool out_rows16(const sca2_out& o) {
  return ((uintptr_t)o.ptr & 15u) == 0 && o.sb % 8 == 0 && o.st % 8 == 0 && o.sh % 8 == 0;
}

template <class K>
static cudaError_t set_smem(K k, int bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

cudaError_t cp_scan_fwd(const sca2_scan_args& p, sca2_out o, float* S_final, float* cstates, int NS,
                        cudaStream_t st) {
  const int NC = (p.T + cp::C - 1) / cp::C;
  const dim3 gc(NC, p.B * p.H), gs(cp::VD / cp::VB, p.B * p.H);
  cudaError_t e;
  if ((e = set_smem(cp::cp_prep, cp::PrepL::TOTAL)) != cudaSuccess) return e;
  if ((e = set_smem(cp::cp_state_fwd, cp::StateFL::TOTAL)) != cudaSuccess) return e;
  if ((e = set_smem(cp::cp_out, cp::OutL::TOTAL)) != cudaSuccess) return e;
  cp::cp_prep<<<gc, cp::NT, cp::PrepL::TOTAL, st>>>(p, cstates, NS, 1);
  cp::cp_state_fwd<<<gs, cp::NQF, cp::StateFL::TOTAL, st>>>(p, cstates, NS, S_final);
  cp::cp_out<<<gc, cp::NT, cp::OutL::TOTAL, st>>>(p, o, cstates, NS, 1, out_rows16(o) ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t cp_scan_bwd(const sca2_scan_args& p, sca2_out dO, const float* dS_final, float* cstates,
                        const sca2_scan_grads& gr, int NS, cudaStream_t st) {
  const int NC = (p.T + cp::C - 1) / cp::C;
  const dim3 gc(NC, p.B * p.H), gs(cp::VD / cp::VB, p.B * p.H);
  const int dvec = out_rows16(dO) ? 1 : 0;
  cudaError_t e;
  if ((e = set_smem(cp::cp_bprep, cp::BPrepL::TOTAL)) != cudaSuccess) return e;
  if ((e = set_smem(cp::cp_state_bwd, cp::StateBL::TOTAL)) != cudaSuccess) return e;
  if ((e = set_smem(cp::cp_grads, cp::GradL::TOTAL)) != cudaSuccess) return e;
  cp::cp_bprep<<<gc, cp::NT, cp::BPrepL::TOTAL, st>>>(p, dO, cstates, NS, 1, dvec);
  cp::cp_state_bwd<<<gs, cp::NQF, cp::StateBL::TOTAL, st>>>(p, dO, dS_final, cstates, NS, gr.dS0, dvec);
  cp::cp_grads<<<gc, cp::NT, cp::GradL::TOTAL, st>>>(p, dO, cstates, NS, gr, 1, dvec);
  return cudaGetLastError();
}

// read and clear the chunk-parallel kernels' device fault word (synchronous)
cudaError_t cp_read_faults(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, cp::g_fault_cp, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(cp::g_fault_cp, &zero, sizeof(unsigned int));
}

}  // namespace sca2
