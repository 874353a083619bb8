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
//   sequential over c (per 32 value columns, fp32 on the CUDA cores):
//     E_c = U_c - W_c S_c,   S_{c+1} = a_last S_c + (w .* k)^T E_c
//   chunk-parallel again:
//     O = q_scale (a .* (q S_c) + ((q k^T) .* Dg) E_c)
//
// Backward (dS' = adjoint of the state leaving chunk c, P = q_scale (q k^T) .* Dg):
//     Yo = T^T P^T dO,   Mt = T^T diag(w) k                        chunk-parallel
//     dY_c = Yo_c + Mt_c dS',   dS = a_last dS' + q_scale (a .* q)^T dO - (beta a .* k)^T dY_c
//                                                                  sequential, fp32
//     every per-token gradient of chunk c from (S_c, E_c, dY_c, dS')   chunk-parallel
//
// This is the algebra of the reference's chunk closed form (lapa/layer.py:298-366 with the
// scalar-decay mask of sca2/arch_gatedc.py:136-139; fla 0.5.1 naive_chunk_gated_delta_rule as
// called at lapa/benchmarks/baselines.py:111-120), regrouped so that the sequential part is
// two small products per chunk.  Tensor-core operands are single bf16 (the state chain itself
// stays fp32); the saved per-chunk data live in the four slots of each chunk:
//   slot 4c    S_c (K x V)
//   slot 4c+1  E_c (64 x V) | T (64 x 64, zeros above the diagonal)
//   slot 4c+2  W (64 x K) | U (64 x V)        backward: Mt (64 x K) | Yo, then dY (64 x V)
//   slot 4c+3  backward: dS' (K x V)
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
constexpr int OFF_T = C * VD, OFF_U = C * KD;

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

// R x 128 fp32 rows (row-major, 16-byte aligned) into a K-major bf16 operand, rows scaled by
// scale(r); returns nothing
template <class F>
__device__ __forceinline__ void f32_rows_to_op(bf16* dst, const float* src, int R, F scale) {
  for (int u = threadIdx.x; u < R * 16; u += NT) {
    const int r = (u & 7) + 8 * (u >> 7), c0 = ((u >> 3) & 15) * 8;
    const float4 x0 = *reinterpret_cast<const float4*>(src + r * 128 + c0);
    const float4 x1 = *reinterpret_cast<const float4*>(src + r * 128 + c0 + 4);
    const float s = scale(r);
    float x[8] = {s * x0.x, s * x0.y, s * x0.z, s * x0.w, s * x1.x, s * x1.y, s * x1.z, s * x1.w};
    tc::st8(dst, umma::kmaj(r, c0, 128), x);
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

__device__ __forceinline__ void unpack8(const bf16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) { x[2 * k] = __low2float(h2[k]); x[2 * k + 1] = __high2float(h2[k]); }
}

// bounded wait on the batch mbarrier; on timeout the fault word is set and false returned
__device__ __forceinline__ bool batch_wait(uint64_t* mbar, uint32_t parity) {
  const bool ok = umma::mbar_wait(mbar, parity);
  __syncthreads();
  umma::fence_after_sync();
  if (!ok && threadIdx.x == 0) atomicOr(&g_fault_cp, 1u);
  return ok;
}

__device__ __forceinline__ void load_gates(const sca2_scan_args& p, const Gates& g, int b, int h, int t0, int Cl) {
  if ((threadIdx.x >> 5) == 0) {
    tc::GateRegs gr;
    tc::load_gate_regs(p, gr, b, h, t0, Cl);
    tc::gates_from_regs(gr, g, Cl);
  }
}

// ======================================================================================
//  F1: T, W = T diag(beta a) k, U = T v_eff per chunk
// ======================================================================================
struct PrepL {
  static constexpr int KB = 0, VBUF = KB + al(C * KD * 2), TW = VBUF + al(C * VD * 2), TV = TW + al(C * C * 2),
                       LS = TV + al(C * C * 2), TS = LS + al(C * LDF * 4), WS = TS + al(C * LDF * 4),
                       SC = WS + 4096, MBAR = SC + 4 * C * 4, TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 2) cp_prep(sca2_scan_args p, float* cs, int NS, int vec) {
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
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;

  load_gates(p, gt, b, h, t0, Cl);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 256);
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
      const float bi = gt.beta[i], gi = gt.Gc[i];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        const float dg = has_g ? __expf(fminf(gi - gt.Gc[jj], 0.f)) : 1.f;
        LS[i * LDF + jj] = jj < i ? bi * x[j] * dg : 0.f;
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
      umma::gemm_t(tb + 128, TV, false, VBf, true, 64, VD, C, false);   // U = (T [beta]) v
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      float* Wg = slot(cs, bh, NS, c, 2);
      tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
        float4* d = reinterpret_cast<float4*>(Wg + i * KD + j0);
#pragma unroll
        for (int k = 0; k < 4; ++k) d[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
      });
      tc::for_frag<64, 128>(tb + 128, [&](int i, int j0, int, const float* x) {
        float4* d = reinterpret_cast<float4*>(Wg + OFF_U + i * VD + j0);
#pragma unroll
        for (int k = 0; k < 4; ++k) d[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
      });
    }
  }
  if (!ok) umma::mbar_wait(mbar, 0), umma::mbar_wait(mbar, 1);  // bounded: let the MMAs drain
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 256);
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

struct StateFL {
  static constexpr int WP = KD + 4;   // W row stride (floats)
  static constexpr int SP = VB;       // S row stride
  static constexpr int EP = VB + 4;   // E row stride
  static constexpr int S = 0, E = S + KD * SP * 4, W = E + C * EP * 4, U = W + 2 * C * WP * 4,
                       K = U + 2 * C * VB * 4, G = K + 2 * C * KD * 2, SC = G + 2 * C * 4,
                       TOTAL = SC + (3 * C + 4) * 4;
};

__global__ void __launch_bounds__(NT, 1) cp_state_fwd(sca2_scan_args p, float* cs, int NS, float* S_final) {
  using L = StateFL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x;
  const int vb = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C, n_base = vb * VB;
  float* Ss = reinterpret_cast<float*>(sm + L::S);
  float* Es = reinterpret_cast<float*>(sm + L::E);
  float* Wb = reinterpret_cast<float*>(sm + L::W);
  float* Ub = reinterpret_cast<float*>(sm + L::U);
  bf16* Kb = reinterpret_cast<bf16*>(sm + L::K);
  float* Gb = reinterpret_cast<float*>(sm + L::G);
  float* Gc = reinterpret_cast<float*>(sm + L::SC);
  float* av = Gc + C;
  float* wv = av + C;
  float* aL = wv + C;

  // initial state
  for (int u = tid; u < KD * VB / 4; u += NT) {
    const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.S0) x = *reinterpret_cast<const float4*>(p.S0 + (int64_t)bh * KV + m * VD + n_base + n);
    *reinterpret_cast<float4*>(Ss + m * L::SP + n) = x;
  }
  auto prefetch = [&](int c) {
    const int buf = c & 1, t0 = c * C, Cl = min(C, p.T - t0);
    const float* Wg = slot(cs, bh, NS, c, 2);
    float* wd = Wb + buf * C * L::WP;
    for (int u = tid; u < C * KD / 4; u += NT) {
      const int i = u >> 5, m = (u & 31) * 4;
      tc::cp16(wd + i * L::WP + m, Wg + i * KD + m, true);
    }
    float* ud = Ub + buf * C * VB;
    for (int u = tid; u < C * VB / 4; u += NT) {
      const int i = u >> 3, n = (u & 7) * 4;
      tc::cp16(ud + i * VB + n, Wg + OFF_U + i * VD + n_base + n, true);
    }
    bf16* kd = Kb + buf * C * KD;
    const bf16* kg = reinterpret_cast<const bf16*>(p.phw.ptr);
    for (int u = tid; u < C * KD / 8; u += NT) {
      const int i = u >> 4, m = (u & 15) * 8;
      const bool live = i < Cl;
      tc::cp16(kd + i * KD + m, kg + (live ? tok_off(p.phw, b, t0 + i, h) + m : 0), live);
    }
    prefetch_gates(p, Gb + buf * C, nullptr, b, h, t0, Cl);
    tc::cp_commit();
  };
  prefetch(0);
  // thread tiles: E (64 x 32): row i = tid / 4, columns n0..n0+7 with n0 = 8 (tid % 4);
  //               S (128 x 32): rows m0, m0+1 with m0 = 2 (tid / 4), the same columns
  const int ti = tid >> 2, n0 = (tid & 3) * 8, m0 = 2 * (tid >> 2);
  for (int c = 0; c < NC; ++c) {
    const int buf = c & 1, Cl = min(C, p.T - c * C);
    tc::cp_wait_all();
    __syncthreads();
    if (c + 1 < NC) prefetch(c + 1);
    gates_from_g(Gb + buf * C, Gc, av, wv, aL, Cl);
    // the state entering chunk c
    float* Sg = slot(cs, bh, NS, c, 0);
    for (int u = tid; u < KD * VB / 4; u += NT) {
      const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
      *reinterpret_cast<float4*>(Sg + m * VD + n_base + n) = *reinterpret_cast<const float4*>(Ss + m * L::SP + n);
    }
    // E = U - W S
    {
      const float* Wr = Wb + buf * C * L::WP + ti * L::WP;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll 4
      for (int m = 0; m < KD; m += 4) {
        const float4 wq = *reinterpret_cast<const float4*>(Wr + m);
        const float wk[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 s0 = *reinterpret_cast<const float4*>(Ss + (m + q) * L::SP + n0);
          const float4 s1 = *reinterpret_cast<const float4*>(Ss + (m + q) * L::SP + n0 + 4);
          acc[0] = fmaf(wk[q], s0.x, acc[0]); acc[1] = fmaf(wk[q], s0.y, acc[1]);
          acc[2] = fmaf(wk[q], s0.z, acc[2]); acc[3] = fmaf(wk[q], s0.w, acc[3]);
          acc[4] = fmaf(wk[q], s1.x, acc[4]); acc[5] = fmaf(wk[q], s1.y, acc[5]);
          acc[6] = fmaf(wk[q], s1.z, acc[6]); acc[7] = fmaf(wk[q], s1.w, acc[7]);
        }
      }
      const float* Ur = Ub + buf * C * VB + ti * VB + n0;
      float e[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = Ur[k] - acc[k];
      *reinterpret_cast<float4*>(Es + ti * L::EP + n0) = make_float4(e[0], e[1], e[2], e[3]);
      *reinterpret_cast<float4*>(Es + ti * L::EP + n0 + 4) = make_float4(e[4], e[5], e[6], e[7]);
      float* Eg = slot(cs, bh, NS, c, 1) + ti * VD + n_base + n0;
      *reinterpret_cast<float4*>(Eg) = make_float4(e[0], e[1], e[2], e[3]);
      *reinterpret_cast<float4*>(Eg + 4) = make_float4(e[4], e[5], e[6], e[7]);
    }
    __syncthreads();
    // S' = a_last S + (w .* k)^T E
    {
      const bf16* kr = Kb + buf * C * KD + m0;
      float acc[2][8];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[r][k] = 0.f;
#pragma unroll 4
      for (int i = 0; i < C; ++i) {
        const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162*>(kr + i * KD);
        const float wi = wv[i];
        const float k0 = wi * __low2float(k2), k1 = wi * __high2float(k2);
        const float4 e0 = *reinterpret_cast<const float4*>(Es + i * L::EP + n0);
        const float4 e1 = *reinterpret_cast<const float4*>(Es + i * L::EP + n0 + 4);
        const float ev[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc[0][k] = fmaf(k0, ev[k], acc[0][k]);
          acc[1][k] = fmaf(k1, ev[k], acc[1][k]);
        }
      }
      const float al_ = *aL;
      __syncthreads();  // every thread has read S for E
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float* srow = Ss + (m0 + r) * L::SP + n0;
        float4 x0 = *reinterpret_cast<float4*>(srow), x1 = *reinterpret_cast<float4*>(srow + 4);
        x0.x = fmaf(al_, x0.x, acc[r][0]); x0.y = fmaf(al_, x0.y, acc[r][1]);
        x0.z = fmaf(al_, x0.z, acc[r][2]); x0.w = fmaf(al_, x0.w, acc[r][3]);
        x1.x = fmaf(al_, x1.x, acc[r][4]); x1.y = fmaf(al_, x1.y, acc[r][5]);
        x1.z = fmaf(al_, x1.z, acc[r][6]); x1.w = fmaf(al_, x1.w, acc[r][7]);
        *reinterpret_cast<float4*>(srow) = x0;
        *reinterpret_cast<float4*>(srow + 4) = x1;
      }
    }
  }
  __syncthreads();
  if (S_final)
    for (int u = tid; u < KD * VB / 4; u += NT) {
      const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
      *reinterpret_cast<float4*>(S_final + (int64_t)bh * KV + m * VD + n_base + n) =
          *reinterpret_cast<const float4*>(Ss + m * L::SP + n);
    }
}

// ======================================================================================
//  F3: outputs O = q_scale (a .* (q S_c) + ((q k^T) .* Dg) E_c)
// ======================================================================================
struct OutL {
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), SB = KB + al(C * KD * 2), EB = SB + al(KD * VD * 2),
                       PB = EB + al(C * VD * 2), SC = PB + al(C * C * 2), MBAR = SC + 4 * C * 4,
                       TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 2) cp_out(sca2_scan_args p, sca2_out o, const float* cs_, int NS, int vec,
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
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;
  const float qs = p.q_scale;

  load_gates(p, gt, b, h, t0, Cl);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 256);
  load_rows(QB, reinterpret_cast<const bf16*>(p.phq.ptr), p.phq.sb, p.phq.st, p.phq.sh, b, t0, h, Cl, vec);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  tc::cp_commit();
  f32_rows_to_op(SB, slot(cs, bh, NS, c, 0), KD, [](int) { return 1.f; });
  f32_rows_to_op(EB, slot(cs, bh, NS, c, 1), C, [](int) { return 1.f; });
  tc::cp_wait_all();
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
  if (tid == 0) {
    umma::gemm(tb + 128, QB, KBf, 64, 64, KD, false);            // q k^T
    umma::gemm_t(tb, QB, false, SB, true, 64, VD, KD, false);    // q S
    umma::commit(mbar);
  }
  bool ok = batch_wait(mbar, 0);
  if (ok) {
    tc::for_frag<64, 64>(tb + 128, [&](int i, int j0, int, const float* x) {
      const float gi = gt.Gc[i];
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        const float dg = has_g ? __expf(fminf(gi - gt.Gc[jj], 0.f)) : 1.f;
        y[j] = jj <= i ? x[j] * dg : 0.f;
      }
      tc::st8(PB, umma::kmaj(i, j0, C), y);
      tc::st8(PB, umma::kmaj(i, j0 + 8, C), y + 8);
    });
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb + 128, PB, false, EB, true, 64, VD, C, false);  // P E
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      const uint32_t bases[2] = {tb, tb + 128};
      bf16* ob = reinterpret_cast<bf16*>(o.ptr);
      frag_multi<128, 2>(bases, [&](int i, int col0, float (*v)[16]) {
        if (i >= Cl) return;
        const float ai = gt.a[i];
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = qs * fmaf(ai, v[0][j], v[1][j]);
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
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tb, 256);
}

// ======================================================================================
//  B1: Yo = T^T P^T dO and Mt = T^T diag(w) k per chunk
// ======================================================================================
struct BPrepL {
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), DOB = KB + al(C * KD * 2), PB = DOB + al(C * VD * 2),
                       TB = PB + al(C * C * 2), TWB = TB + al(C * C * 2), Z1 = TWB + al(C * C * 2),
                       SC = Z1 + al(C * VD * 2), MBAR = SC + 4 * C * 4, TOTAL = MBAR + 16;
};

__global__ void __launch_bounds__(NT, 2) cp_bprep(sca2_scan_args p, sca2_out dO, float* cs, int NS, int vec,
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
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr;
  const float qs = p.q_scale;

  load_gates(p, gt, b, h, t0, Cl);
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 256);
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
      const float gi = gt.Gc[i];
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = j0 + j;
        const float dg = has_g ? __expf(fminf(gi - gt.Gc[jj], 0.f)) : 1.f;
        y[j] = jj <= i ? qs * x[j] * dg : 0.f;
      }
      tc::st8(PB, umma::kmaj(i, j0, C), y);
      tc::st8(PB, umma::kmaj(i, j0 + 8, C), y + 8);
    });
    tc::publish_smem();
    if (tid == 0) {
      umma::gemm_t(tb, PB, true, DOB, true, 64, VD, C, false);         // P^T dO
      umma::gemm_t(tb + 128, TWB, true, KBf, true, 64, KD, C, false);  // (diag(w) T)^T k
      umma::commit(mbar);
    }
    ok = batch_wait(mbar, 1);
    if (ok) {
      float* Mg = slot(cs, bh, NS, c, 2);
      tc::for_frag<64, 128>(tb, [&](int i, int j0, int, const float* x) {
        tc::st8(Z1, umma::kmaj(i, j0, VD), x);
        tc::st8(Z1, umma::kmaj(i, j0 + 8, VD), x + 8);
      });
      tc::for_frag<64, 128>(tb + 128, [&](int i, int j0, int, const float* x) {
        float4* d = reinterpret_cast<float4*>(Mg + i * KD + j0);
#pragma unroll
        for (int k = 0; k < 4; ++k) d[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
      });
      tc::publish_smem();
      if (tid == 0) {
        umma::gemm_t(tb, TB, true, Z1, true, 64, VD, C, false);  // Yo = T^T (P^T dO)
        umma::commit(mbar);
      }
      ok = batch_wait(mbar, 0);
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
  if (warp == 0) umma::tmem_dealloc(tb, 256);
}

// ======================================================================================
//  B2: the adjoint state recurrence (reverse over chunks, 32 value columns per CTA, fp32)
// ======================================================================================
struct StateBL {
  static constexpr int MP = KD + 4, SP = VB, YP = VB + 4;
  static constexpr int DS = 0, DY = DS + KD * SP * 4, DOF = DY + C * YP * 4, M = DOF + C * YP * 4,
                       Y = M + 2 * C * MP * 4, Q = Y + 2 * C * VB * 4, K = Q + 2 * C * KD * 2,
                       DO = K + 2 * C * KD * 2, G = DO + 2 * C * VB * 2, BT = G + 2 * C * 4, SC = BT + 2 * C * 4,
                       TOTAL = SC + (5 * C + 4) * 4;
};

__global__ void __launch_bounds__(NT, 1) cp_state_bwd(sca2_scan_args p, sca2_out dO, const float* dS_final,
                                                      float* cs, int NS, float* dS0, int dvec) {
  using L = StateBL;
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x;
  const int vb = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int NC = (p.T + C - 1) / C, n_base = vb * VB;
  float* dSs = reinterpret_cast<float*>(sm + L::DS);
  float* dYs = reinterpret_cast<float*>(sm + L::DY);
  float* dOf = reinterpret_cast<float*>(sm + L::DOF);
  float* Mb = reinterpret_cast<float*>(sm + L::M);
  float* Yb = reinterpret_cast<float*>(sm + L::Y);
  bf16* Qb = reinterpret_cast<bf16*>(sm + L::Q);
  bf16* Kb = reinterpret_cast<bf16*>(sm + L::K);
  bf16* DOb = reinterpret_cast<bf16*>(sm + L::DO);
  float* Gb = reinterpret_cast<float*>(sm + L::G);
  float* Bb = reinterpret_cast<float*>(sm + L::BT);
  float* Gc = reinterpret_cast<float*>(sm + L::SC);
  float* av = Gc + C;
  float* wv = av + C;
  float* ca = wv + C;
  float* cb = ca + C;
  float* aL = cb + C;
  const float qs = p.q_scale;
  const bool has_beta = p.beta.ptr != nullptr;

  for (int u = tid; u < KD * VB / 4; u += NT) {
    const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (dS_final) x = *reinterpret_cast<const float4*>(dS_final + (int64_t)bh * KV + m * VD + n_base + n);
    *reinterpret_cast<float4*>(dSs + m * L::SP + n) = x;
  }
  auto prefetch = [&](int c) {
    const int buf = c & 1, t0 = c * C, Cl = min(C, p.T - t0);
    const float* Mg = slot(cs, bh, NS, c, 2);
    float* md = Mb + buf * C * L::MP;
    for (int u = tid; u < C * KD / 4; u += NT) {
      const int i = u >> 5, m = (u & 31) * 4;
      tc::cp16(md + i * L::MP + m, Mg + i * KD + m, true);
    }
    float* yd = Yb + buf * C * VB;
    for (int u = tid; u < C * VB / 4; u += NT) {
      const int i = u >> 3, n = (u & 7) * 4;
      tc::cp16(yd + i * VB + n, Mg + OFF_U + i * VD + n_base + n, true);
    }
    bf16* qd = Qb + buf * C * KD;
    bf16* kd = Kb + buf * C * KD;
    const bf16* qg = reinterpret_cast<const bf16*>(p.phq.ptr);
    const bf16* kg = reinterpret_cast<const bf16*>(p.phw.ptr);
    for (int u = tid; u < C * KD / 8; u += NT) {
      const int i = u >> 4, m = (u & 15) * 8;
      const bool live = i < Cl;
      tc::cp16(qd + i * KD + m, qg + (live ? tok_off(p.phq, b, t0 + i, h) + m : 0), live);
      tc::cp16(kd + i * KD + m, kg + (live ? tok_off(p.phw, b, t0 + i, h) + m : 0), live);
    }
    bf16* dd = DOb + buf * C * VB;
    const bf16* dg = reinterpret_cast<const bf16*>(dO.ptr);
    for (int u = tid; u < C * VB / 8; u += NT) {
      const int i = u >> 2, n = (u & 3) * 8;
      const bool live = i < Cl;
      const bf16* src = dg + (live ? out_off(dO, b, t0 + i, h, 0) + n_base + n : 0);
      if (dvec) {
        tc::cp16(dd + i * VB + n, src, live);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) dd[i * VB + n + k] = live ? src[k] : __float2bfloat16_rn(0.f);
      }
    }
    prefetch_gates(p, Gb + buf * C, Bb + buf * C, b, h, t0, Cl);
    tc::cp_commit();
  };
  prefetch(NC - 1);
  const int ti = tid >> 2, n0 = (tid & 3) * 8, m0 = 2 * (tid >> 2);
  for (int c = NC - 1; c >= 0; --c) {
    const int buf = c & 1, Cl = min(C, p.T - c * C);
    tc::cp_wait_all();
    __syncthreads();
    if (c > 0) prefetch(c - 1);
    gates_from_g(Gb + buf * C, Gc, av, wv, aL, Cl);
    // dO (bf16) of this block of value columns to fp32
    for (int u = tid; u < C * VB; u += NT) {
      const int i = u / VB, n = u % VB;
      dOf[i * L::YP + n] = __bfloat162float(DOb[buf * C * VB + i * VB + n]);
    }
    // the adjoint of the state leaving chunk c
    float* dSg = slot(cs, bh, NS, c, 3);
    for (int u = tid; u < KD * VB / 4; u += NT) {
      const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
      *reinterpret_cast<float4*>(dSg + m * VD + n_base + n) = *reinterpret_cast<const float4*>(dSs + m * L::SP + n);
    }
    __syncthreads();
    if (tid < C) {
      const float bt = has_beta ? Bb[buf * C + tid] : 0.f;
      ca[tid] = qs * av[tid];
      cb[tid] = -bt * av[tid];
    }
    // dY = Yo + Mt dS'
    {
      const float* Mr = Mb + buf * C * L::MP + ti * L::MP;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll 4
      for (int m = 0; m < KD; m += 4) {
        const float4 wq = *reinterpret_cast<const float4*>(Mr + m);
        const float wk[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 s0 = *reinterpret_cast<const float4*>(dSs + (m + q) * L::SP + n0);
          const float4 s1 = *reinterpret_cast<const float4*>(dSs + (m + q) * L::SP + n0 + 4);
          acc[0] = fmaf(wk[q], s0.x, acc[0]); acc[1] = fmaf(wk[q], s0.y, acc[1]);
          acc[2] = fmaf(wk[q], s0.z, acc[2]); acc[3] = fmaf(wk[q], s0.w, acc[3]);
          acc[4] = fmaf(wk[q], s1.x, acc[4]); acc[5] = fmaf(wk[q], s1.y, acc[5]);
          acc[6] = fmaf(wk[q], s1.z, acc[6]); acc[7] = fmaf(wk[q], s1.w, acc[7]);
        }
      }
      const float* Yr = Yb + buf * C * VB + ti * VB + n0;
      float y[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = Yr[k] + acc[k];
      *reinterpret_cast<float4*>(dYs + ti * L::YP + n0) = make_float4(y[0], y[1], y[2], y[3]);
      *reinterpret_cast<float4*>(dYs + ti * L::YP + n0 + 4) = make_float4(y[4], y[5], y[6], y[7]);
      float* Yg = slot(cs, bh, NS, c, 2) + OFF_U + ti * VD + n_base + n0;
      *reinterpret_cast<float4*>(Yg) = make_float4(y[0], y[1], y[2], y[3]);
      *reinterpret_cast<float4*>(Yg + 4) = make_float4(y[4], y[5], y[6], y[7]);
    }
    __syncthreads();
    // dS = a_last dS' + (q_scale a .* q)^T dO - (beta a .* k)^T dY
    {
      const bf16* qr = Qb + buf * C * KD + m0;
      const bf16* kr = Kb + buf * C * KD + m0;
      float acc[2][8];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[r][k] = 0.f;
#pragma unroll 2
      for (int i = 0; i < C; ++i) {
        const __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162*>(qr + i * KD);
        const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162*>(kr + i * KD);
        const float ci = ca[i], di = cb[i];
        const float q0 = ci * __low2float(q2), q1 = ci * __high2float(q2);
        const float k0 = di * __low2float(k2), k1 = di * __high2float(k2);
        const float4 o0 = *reinterpret_cast<const float4*>(dOf + i * L::YP + n0);
        const float4 o1 = *reinterpret_cast<const float4*>(dOf + i * L::YP + n0 + 4);
        const float4 y0 = *reinterpret_cast<const float4*>(dYs + i * L::YP + n0);
        const float4 y1 = *reinterpret_cast<const float4*>(dYs + i * L::YP + n0 + 4);
        const float ov[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        const float yv[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc[0][k] = fmaf(q0, ov[k], fmaf(k0, yv[k], acc[0][k]));
          acc[1][k] = fmaf(q1, ov[k], fmaf(k1, yv[k], acc[1][k]));
        }
      }
      const float al_ = *aL;
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float* srow = dSs + (m0 + r) * L::SP + n0;
        float4 x0 = *reinterpret_cast<float4*>(srow), x1 = *reinterpret_cast<float4*>(srow + 4);
        x0.x = fmaf(al_, x0.x, acc[r][0]); x0.y = fmaf(al_, x0.y, acc[r][1]);
        x0.z = fmaf(al_, x0.z, acc[r][2]); x0.w = fmaf(al_, x0.w, acc[r][3]);
        x1.x = fmaf(al_, x1.x, acc[r][4]); x1.y = fmaf(al_, x1.y, acc[r][5]);
        x1.z = fmaf(al_, x1.z, acc[r][6]); x1.w = fmaf(al_, x1.w, acc[r][7]);
        *reinterpret_cast<float4*>(srow) = x0;
        *reinterpret_cast<float4*>(srow + 4) = x1;
      }
    }
  }
  __syncthreads();
  if (dS0)
    for (int u = tid; u < KD * VB / 4; u += NT) {
      const int m = u / (VB / 4), n = (u % (VB / 4)) * 4;
      *reinterpret_cast<float4*>(dS0 + (int64_t)bh * KV + m * VD + n_base + n) =
          *reinterpret_cast<const float4*>(dSs + m * L::SP + n);
    }
}

// ======================================================================================
//  B3: per-token gradients of every chunk
// ======================================================================================
struct GradL {
  static constexpr int DDP = C + 1;
  static constexpr int QB = 0, KB = QB + al(C * KD * 2), DOB = KB + al(C * KD * 2), DYB = DOB + al(C * VD * 2),
                       EB = DYB + al(C * VD * 2), SB = EB + al(C * VD * 2), DSB = SB + al(KD * VD * 2),
                       DKK = DSB + al(KD * VD * 2), DQK = DKK + al(C * C * 2), DDG = DQK + al(C * C * 2),
                       SC = DDG + C * DDP * 4, NSC = 4 * C + 12 * C + 16, MBAR = SC + NSC * 4,
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
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  const Gates gt{sc, sc + C, sc + 2 * C, sc + 3 * C};
  float* rsum = sc + 4 * C;          // [2 halves][6 sums][C]: dbeta1, rowDg, rY, rE, rO, (spare)
  float* red = rsum + 12 * C;        // block reduction scratch (16)
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L::MBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::MBAR + 8);
  const bool has_g = p.g.ptr != nullptr, has_beta = p.beta.ptr != nullptr;
  const bool vtb = p.v_times_beta != 0, ow = gr.overwrite != 0;
  const float qs = p.q_scale;
  enum { R_DB = 0, R_DG = 1, R_Y = 2, R_E = 3, R_O = 4 };
  auto rs = [&](int half, int which) { return rsum + (half * 6 + which) * C; };

  load_gates(p, gt, b, h, t0, Cl);
  for (int u = tid; u < 12 * C; u += NT) rsum[u] = 0.f;
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
  }
  if (warp == 0) umma::tmem_alloc(s_tmem, 512);
  load_rows(QB, reinterpret_cast<const bf16*>(p.phq.ptr), p.phq.sb, p.phq.st, p.phq.sh, b, t0, h, Cl, vec);
  load_rows(KBf, reinterpret_cast<const bf16*>(p.phw.ptr), p.phw.sb, p.phw.st, p.phw.sh, b, t0, h, Cl, vec);
  load_rows(DOB, reinterpret_cast<const bf16*>(dO.ptr), dO.sb, dO.st, dO.sh, b, t0, h, Cl, dvec);
  tc::cp_commit();
  const float* Sg = slot(cs, bh, NS, c, 0);
  const float* Eg = slot(cs, bh, NS, c, 1);
  const float* Yg = slot(cs, bh, NS, c, 2) + OFF_U;
  const float* dSg = slot(cs, bh, NS, c, 3);
  f32_rows_to_op(DYB, Yg, C, [](int) { return 1.f; });
  f32_rows_to_op(EB, Eg, C, [](int) { return 1.f; });
  // S and dS' with the chunk's sum of S .* dS' (the gradient of a_last through the carry)
  float sds = 0.f;
  for (int u = tid; u < KD * 16; u += NT) {
    const int r = (u & 7) + 8 * (u >> 7), c0 = ((u >> 3) & 15) * 8;
    const float4 s0 = *reinterpret_cast<const float4*>(Sg + r * VD + c0);
    const float4 s1 = *reinterpret_cast<const float4*>(Sg + r * VD + c0 + 4);
    const float4 d0 = *reinterpret_cast<const float4*>(dSg + r * VD + c0);
    const float4 d1 = *reinterpret_cast<const float4*>(dSg + r * VD + c0 + 4);
    float xs[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float xd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) sds = fmaf(xs[k], xd[k], sds);
    tc::st8(SB, umma::kmaj(r, c0, VD), xs);
    tc::st8(DSB, umma::kmaj(r, c0, VD), xd);
  }
  sds = warp_sum(sds);
  if (lane == 0) red[warp] = sds;
  tc::cp_wait_all();
  tc::publish_smem();
  const uint32_t tb = *s_tmem;
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
        const float gi = gt.Gc[i], bi = gt.beta[i];
        float dkk[16], dqk[16], db1 = 0.f, rdg = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int jj = j0 + j;
          const bool incl = jj <= i, strict = jj < i;
          const float dg = incl ? (has_g ? __expf(fminf(gi - gt.Gc[jj], 0.f)) : 1.f) : 0.f;
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
    // operands of the second batch: dY -> -beta a .* dY, E -> w .* E (from the fp32 copies)
    f32_rows_to_op(DYB, Yg, C, [&](int r) { return -gt.beta[r] * gt.a[r]; });
    f32_rows_to_op(EB, Eg, C, [&](int r) { return gt.w[r]; });
    tc::publish_smem();
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
  {
    const bf16* vg = reinterpret_cast<const bf16*>(p.v.ptr);
    bf16* dvg = reinterpret_cast<bf16*>(const_cast<void*>(gr.dv.ptr));
    for (int i = warp; i < Cl; i += NT / 32) {
      const float bi = gt.beta[i];
      const float4 y = *reinterpret_cast<const float4*>(Yg + i * VD + 4 * lane);
      const bf16* vr = vg + tok_off(p.v, b, t0 + i, h) + 4 * lane;
      const float yv[4] = {y.x, y.y, y.z, y.w};
      float s = 0.f;
      bf16* dr = dvg + tok_off(gr.dv, b, t0 + i, h) + 4 * lane;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s = fmaf(yv[k], __bfloat162float(vr[k]), s);
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
    for (int k = 0; k < NT / 32; ++k) sdsum += red[k];
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
  cp::cp_state_fwd<<<gs, cp::NT, cp::StateFL::TOTAL, st>>>(p, cstates, NS, S_final);
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
  cp::cp_state_bwd<<<gs, cp::NT, cp::StateBL::TOTAL, st>>>(p, dO, dS_final, cstates, NS, gr.dS0, dvec);
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
