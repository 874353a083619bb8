// Short head (sm_100a): the exact L-tap window read of the LapA / SCA2 short head, forward
// (prefill and decode), backward, and the ring-buffer update.
//
//   phi_t = K(h_t) theta + ((pos + t) mod L) omega,   psi_t = K(z_t) theta + ((pos + t) mod L) omega
//   kappa(t, s) = (1/L) sum_m (wr + i wi)_m e^{i (phi_s - psi_t)}
//   o_t = [ sum_{s=t-L+1..t} Re kappa(t,s) e_s  |  sum Im kappa(t,s) e_s ]
//
// (lapa/layer.py:418-545 ShortHead._read/_banded/step; sca2/arch_short.py:45-158).  The
// L-1 previous writes come from the state (c = cos phi, s = sin phi, e = value, oldest
// first) and are prepended to the call's own writes ("extended" index x = s + L - 1).
//
// Everything is fp32 on the CUDA cores: the DFT grid's comb (sum over m of e^{i m 2pi k / L})
// cancels to zero at every lag k != 0 only to fp32 rounding, and bf16 tensor-core operands
// would turn that exact zero into a visible leak between lags.  The work is small (L (2L + 2dv)
// multiply-adds per token) and independent across tokens, so each CTA takes TT consecutive
// queries of one sequence and the L-1 keys before them; the codes (sin / cos of the phases,
// computed here from K(h), K(z), theta, omega and the position by the Cody-Waite reduction and
// the SFU, absolute error about 1e-6, so the comb's leak stays near L * 1e-6), kappa and the values sit in
// shared memory.  The inner products are register-blocked: a thread owns one token row and a
// group of 4 lags, 4 modes or 8 value columns, lanes of a warp walk consecutive rows, and the
// row strides (a multiple of 4 floats, = 4 mod 32 banks) make the 16-byte loads of 8
// consecutive rows hit distinct banks; kappa rows have an odd stride for the scalar loads.
// Values and output gradients are processed in slices of DS columns, so dv is unbounded.
#include "common.cuh"

namespace sca2 {
namespace shortk {

constexpr int NT = 256;
constexpr int DS = 32;      // value columns per slice
constexpr int ES = DS + 4;  // row stride of value / output-gradient slices (floats)

// row stride of the code arrays: L rounded up to 4 plus 4 (16-byte rows; 20 floats for L = 16)
__host__ __device__ constexpr int code_stride(int L) { return ((L + 3) & ~3) + 4; }
__host__ __device__ constexpr int lane_groups(int L) { return (L + 3) / 4; }

__device__ __forceinline__ int pmod(long long p, int L) {
  long long r = p % L;
  return (int)(r < 0 ? r + L : r);
}
// magic / qdiv (common.cuh): every use here has u < 2^16 with d < 2^16, or the phase position
// u < 2^27 with d = L <= 32
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

struct Geo {
  int L, n, dv, T, t0, tq;
  int pb;              // (pos mod L): token t >= 0 has phase position (pb + t) mod L
  uint32_t mL, mCS;    // magic(L), magic(code stride)
};
__device__ __forceinline__ Geo geo(const sca2_short_args& p, int TT) {
  Geo g;
  g.L = p.L;
  g.n = p.L - 1;
  g.dv = p.dv;
  g.T = p.T;
  g.t0 = blockIdx.x * TT;
  g.tq = min(TT, p.T - g.t0);
  g.pb = pmod(p.pos ? *p.pos : 0, p.L);
  g.mL = magic(p.L);
  g.mCS = magic(((p.L + 3) & ~3) + 4);
  return g;
}
// phase position (pos + t) mod L of token t >= 0 (pb + t < 2^27, checked on the host)
__device__ __forceinline__ float ppos(const Geo& g, int t) {
  const int a = g.pb + t;
  return (float)(a - qdiv(a, g.mL) * g.L);
}

// cos / sin of the write phase of token s (from the ring buffer for s < 0)
__device__ __forceinline__ void key_code(const sca2_short_args& p, const Geo& g, int b, int s, int l, float* c,
                                         float* sn) {
  if (s < 0) {
    const int64_t k = ((int64_t)b * g.n + g.n + s) * g.L + l;
    *c = p.c0 ? p.c0[k] : 1.f;
    *sn = p.s0 ? p.s0[k] : 0.f;
  } else {
    const float ph = p.kh[((int64_t)b * g.T + s) * g.L + l] * p.theta[l] + ppos(g, s) * p.omega[l];
    sincos_big(ph, sn, c);
  }
}
__device__ __forceinline__ float key_value(const sca2_short_args& p, const Geo& g, int b, int s, int j) {
  if (s < 0) return p.e0 ? p.e0[((int64_t)b * g.n + g.n + s) * g.dv + j] : 0.f;
  return p.v[((int64_t)b * g.T + s) * g.dv + j];
}

// key codes of rows x in [0, NX) (token t0 - n + x), zero in the padding columns
__device__ __forceinline__ void load_keys(const sca2_short_args& p, const Geo& g, int b, int NX, float* KC,
                                          float* KS) {
  const int CS = code_stride(g.L);
  for (int u = threadIdx.x; u < NX * CS; u += NT) {
    const int x = qdiv(u, g.mCS), l = u - x * CS;
    float c = 0.f, s = 0.f;
    if (l < g.L) key_code(p, g, b, g.t0 - g.n + x, l, &c, &s);
    KC[u] = c;
    KS[u] = s;
  }
}
// read codes c1, c2 (and cos / sin psi when CQ) of query rows y in [0, NY) (token t0 + y)
__device__ __forceinline__ void load_queries(const sca2_short_args& p, const Geo& g, int b, int NY, float* Q1,
                                             float* Q2, float* CQ, float* SQ) {
  const int CS = code_stride(g.L);
  for (int u = threadIdx.x; u < NY * CS; u += NT) {
    const int y = qdiv(u, g.mCS), l = u - y * CS, t = g.t0 + y;
    float c = 0.f, s = 0.f, wr = 0.f, wi = 0.f;
    if (l < g.L) {
      const float ph = p.kz[((int64_t)b * g.T + t) * g.L + l] * p.theta[l] + ppos(g, t) * p.omega[l];
      sincos_big(ph, &s, &c);
      wr = p.wr[l];
      wi = p.wi[l];
    }
    Q1[u] = wr * c + wi * s;
    Q2[u] = wr * s - wi * c;
    if (CQ) {
      CQ[u] = c;
      SQ[u] = s;
    }
  }
}

// kappa of the pairs (row y, lags 4 gq .. 4 gq + 3): key row x = y + n - lag, pairs with x >= NX
// are zero.  Lanes walk consecutive rows y.
__device__ __forceinline__ void kappa_pairs(const Geo& g, int NY, int NX, const float* KC, const float* KS,
                                            const float* Q1, const float* Q2, float* KR, float* KI) {
  const int L = g.L, n = g.n, CS = code_stride(L), KP = L + 1, NG = lane_groups(L);
  const float iL = 1.f / (float)L;
  const uint32_t mY = magic(NY);
  for (int u = threadIdx.x; u < NY * NG; u += NT) {
    const int gq = qdiv(u, mY), y = u - gq * NY;
    float kr[4] = {0.f, 0.f, 0.f, 0.f}, ki[4] = {0.f, 0.f, 0.f, 0.f};
    for (int l = 0; l < CS - 4; l += 4) {
      const float4 q1 = ld4(Q1 + y * CS + l), q2 = ld4(Q2 + y * CS + l);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int x = y + n - (4 * gq + k);
        if (4 * gq + k < L && x < NX) {
          const float4 kc = ld4(KC + x * CS + l), ks = ld4(KS + x * CS + l);
          kr[k] += dot4(kc, q1) + dot4(ks, q2);
          ki[k] += dot4(ks, q1) - dot4(kc, q2);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int lag = 4 * gq + k;
      if (lag < L) {
        KR[y * KP + lag] = kr[k] * iL;
        KI[y * KP + lag] = ki[k] * iL;
      }
    }
  }
}

// value slice [j0, j0 + DS) of key rows [0, NX) (zero beyond dv)
__device__ __forceinline__ void load_values(const sca2_short_args& p, const Geo& g, int b, int NX, int j0, float* E) {
  for (int u = threadIdx.x; u < NX * DS; u += NT) {
    const int x = u / DS, j = u - (u / DS) * DS;
    E[x * ES + j] = j0 + j < g.dv ? key_value(p, g, b, g.t0 - g.n + x, j0 + j) : 0.f;
  }
}
// output-gradient slice of query rows [0, NY): re part to GR, im part to GI
__device__ __forceinline__ void load_grads(const float* dO, const Geo& g, int b, int NY, int j0, float* GR, float* GI) {
  for (int u = threadIdx.x; u < NY * DS; u += NT) {
    const int y = u / DS, j = u - (u / DS) * DS;
    const float* row = dO + ((int64_t)b * g.T + g.t0 + y) * 2 * g.dv;
    GR[y * ES + j] = j0 + j < g.dv ? row[j0 + j] : 0.f;
    GI[y * ES + j] = j0 + j < g.dv ? row[g.dv + j0 + j] : 0.f;
  }
}

// dst += v summed over the CTA: lanes of a warp that hold the same dst (uniform) are reduced
// by shuffles first, so the shared-memory atomic is one per warp instead of one per lane
__device__ __forceinline__ void red_add(float* dst, float v, bool uniform) {
  if (uniform) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(dst, v);
  } else {
    atomicAdd(dst, v);
  }
}

size_t fwd_smem_floats(int L, int TT) {
  const int n = L - 1, CS = code_stride(L), KP = L + 1;
  return (size_t)(TT + n) * (2 * CS + ES) + (size_t)TT * (2 * CS + 2 * KP);
}
size_t bwd_smem_floats(int L, int TT) {
  const int n = L - 1, CS = code_stride(L), KP = L + 1, NX = TT + n;
  return (size_t)NX * (6 * CS + 4 * KP + 3 * ES) + 3 * L;
}

__global__ void __launch_bounds__(NT) short_fwd_kernel(sca2_short_args p, float* o, int TT) {
  extern __shared__ __align__(16) float sm[];
  const Geo g = geo(p, TT);
  const int tid = threadIdx.x, b = blockIdx.y, L = g.L, n = g.n, dv = g.dv;
  const int CS = code_stride(L), KP = L + 1, NX = g.tq + n;
  float* KC = sm;
  float* KS = KC + (TT + n) * CS;
  float* E = KS + (TT + n) * CS;
  float* Q1 = E + (TT + n) * ES;
  float* Q2 = Q1 + TT * CS;
  float* KR = Q2 + TT * CS;
  float* KI = KR + TT * KP;
  load_keys(p, g, b, NX, KC, KS);
  load_queries(p, g, b, g.tq, Q1, Q2, nullptr, nullptr);
  const uint32_t mQ = magic(g.tq);
  __syncthreads();
  kappa_pairs(g, g.tq, NX, KC, KS, Q1, Q2, KR, KI);
  for (int j0 = 0; j0 < dv; j0 += DS) {
    __syncthreads();  // kappa written / previous slice consumed
    load_values(p, g, b, NX, j0, E);
    __syncthreads();
    // row i, value columns jg*8 .. +7 of the slice
    for (int u = tid; u < g.tq * (DS / 8); u += NT) {
      const int jg = qdiv(u, mQ), i = u - jg * g.tq, jj = jg * 8;
      float ar[8], ai[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) ar[k] = ai[k] = 0.f;
      for (int lag = 0; lag < L; ++lag) {
        const float kr = KR[i * KP + lag], ki = KI[i * KP + lag];
        const float* e = E + (i + n - lag) * ES + jj;
        const float4 e0 = ld4(e), e1 = ld4(e + 4);
        const float ev[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          ar[k] = fmaf(kr, ev[k], ar[k]);
          ai[k] = fmaf(ki, ev[k], ai[k]);
        }
      }
      float* orow = o + ((int64_t)b * g.T + g.t0 + i) * 2 * dv + j0 + jj;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (j0 + jj + k < dv) {
          orow[k] = ar[k];
          orow[dv + k] = ai[k];
        }
    }
  }
}

// new ring buffer: entry k (0 <= k < n) is extended index T + k, i.e. token T - n + k
__global__ void __launch_bounds__(NT) short_state_kernel(sca2_short_args p, float* c1, float* s1, float* e1) {
  const int b = blockIdx.x, L = p.L, n = L - 1, dv = p.dv, T = p.T;
  const Geo g = geo(p, 0);
  for (int u = threadIdx.x; u < n * L; u += NT) {
    const int k = u / L, l = u - (u / L) * L;
    float c, s;
    key_code(p, g, b, T - n + k, l, &c, &s);
    c1[((int64_t)b * n + k) * L + l] = c;
    s1[((int64_t)b * n + k) * L + l] = s;
  }
  for (int u = threadIdx.x; u < n * dv; u += NT) {
    const int k = u / dv, j = u - (u / dv) * dv;
    e1[((int64_t)b * n + k) * dv + j] = key_value(p, g, b, T - n + k, j);
  }
}

// Backward of one CTA: queries [t0, t0 + tq) and the keys it owns, [t0, t0 + tq) plus the
// buffered keys [-n, 0) for the first CTA.  Key s is read by queries s .. s + n, so the CTA
// also loads the n queries after its own (up to T) and recomputes their kappa for the pairs
// that reach its keys.  Pairs are indexed (y, lag): query t = t0 + y, key s = t - lag,
// key row x = y + n - lag (< NX = tq + n for the pairs this CTA needs).
__global__ void __launch_bounds__(NT, 3) short_bwd_kernel(sca2_short_args p, const float* dO, const float* dc1,
                                                       const float* ds1, const float* de1, sca2_short_grads gr,
                                                       float* part, int TT) {
  extern __shared__ __align__(16) float sm[];
  const Geo g = geo(p, TT);
  const int tid = threadIdx.x, b = blockIdx.y, L = g.L, n = g.n, dv = g.dv, T = g.T;
  const int CS = code_stride(L), KP = L + 1, NG = lane_groups(L);
  const bool vec = (L & 3) == 0;           // 16-byte rows of the (B,T,L) tensors
  const int NX = g.tq + n;                 // key rows:   s = t0 - n + x
  const int NY = min(g.tq + n, T - g.t0);  // query rows: t = t0 + y
  const int R = TT + n;
  float* KC = sm;
  float* KS = KC + R * CS;
  float* Q1 = KS + R * CS;
  float* Q2 = Q1 + R * CS;
  float* CQ = Q2 + R * CS;
  float* SQ = CQ + R * CS;
  float* KR = SQ + R * CS;   // kappa and its gradient [y][lag]
  float* KI = KR + R * KP;
  float* DKR = KI + R * KP;
  float* DKI = DKR + R * KP;
  float* E = DKI + R * KP;   // value slice [x][j]
  float* GR = E + R * ES;    // output-gradient slice [y][j]
  float* GI = GR + R * ES;
  float* RED = GI + R * ES;  // dtheta, dwr, dwi partials of this CTA
  const float iL = 1.f / (float)L;
  const uint32_t mY = magic(NY), mQ = magic(g.tq);
  for (int u = tid; u < 3 * L; u += NT) RED[u] = 0.f;
  load_keys(p, g, b, NX, KC, KS);
  load_queries(p, g, b, NY, Q1, Q2, CQ, SQ);
  __syncthreads();
  kappa_pairs(g, NY, NX, KC, KS, Q1, Q2, KR, KI);
  // d kappa(t, s) = dO_t . e_s over the value slices; a thread keeps its pairs (row y, lags
  // 4 gq .. 4 gq + 3) in registers across the slices
  constexpr int MAXU = 3;  // NY * NG <= 3 * NT for the tile sizes used (checked on the host)
  float dr[MAXU][4], di[MAXU][4];
#pragma unroll
  for (int q = 0; q < MAXU; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k) dr[q][k] = di[q][k] = 0.f;
  for (int j0 = 0; j0 < dv; j0 += DS) {
    __syncthreads();
    load_values(p, g, b, NX, j0, E);
    load_grads(dO, g, b, NY, j0, GR, GI);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < MAXU; ++q) {
      const int u = tid + q * NT;
      if (u >= NY * NG) break;
      const int gq = qdiv(u, mY), y = u - gq * NY;
      for (int j = 0; j < DS; j += 4) {
        const float4 a = ld4(GR + y * ES + j), c = ld4(GI + y * ES + j);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int x = y + n - (4 * gq + k);
          if (4 * gq + k < L && x < NX) {
            const float4 e = ld4(E + x * ES + j);
            dr[q][k] += dot4(a, e);
            di[q][k] += dot4(c, e);
          }
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < MAXU; ++q) {
    const int u = tid + q * NT;
    if (u >= NY * NG) break;
    const int gq = qdiv(u, mY), y = u - gq * NY;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int lag = 4 * gq + k;
      if (lag < L) {
        const bool ok = y + n - lag < NX;
        DKR[y * KP + lag] = ok ? dr[q][k] : 0.f;
        DKI[y * KP + lag] = ok ? di[q][k] : 0.f;
      }
    }
  }
  __syncthreads();
  // queries (row y < tq, modes 4 gl .. 4 gl + 3): d c1, d c2 -> d psi -> d K(z); theta / wr /
  // wi partials.  With tq a multiple of 32 every warp holds one mode group.
  const bool quni = (g.tq & 31) == 0;
  for (int u = tid; u < g.tq * NG; u += NT) {
    const int lg = qdiv(u, mQ), y = u - lg * g.tq, l0 = 4 * lg, t = g.t0 + y;
    float a1[4] = {0.f, 0.f, 0.f, 0.f}, a2[4] = {0.f, 0.f, 0.f, 0.f};
    for (int lag = 0; lag < L; ++lag) {
      const int x = y + n - lag;
      const float r = DKR[y * KP + lag], i = DKI[y * KP + lag];
      const float4 kc = ld4(KC + x * CS + l0), ks = ld4(KS + x * CS + l0);
      const float c4[4] = {kc.x, kc.y, kc.z, kc.w}, s4[4] = {ks.x, ks.y, ks.z, ks.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        a1[k] = fmaf(r, c4[k], fmaf(i, s4[k], a1[k]));
        a2[k] = fmaf(r, s4[k], fmaf(-i, c4[k], a2[k]));
      }
    }
    const int64_t t0i = ((int64_t)b * T + t) * L + l0;
    float kz[4], dk[4];
    if (vec) {
      const float4 q = ld4(p.kz + t0i);
      kz[0] = q.x; kz[1] = q.y; kz[2] = q.z; kz[3] = q.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) kz[k] = l0 + k < L ? p.kz[t0i + k] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int l = l0 + k;
      if (l >= L) break;
      const float d1 = a1[k] * iL, d2 = a2[k] * iL;
      const float cq = CQ[y * CS + l], sq = SQ[y * CS + l], wr = p.wr[l], wi = p.wi[l];
      const float dcq = d1 * wr - d2 * wi, dsq = d1 * wi + d2 * wr;
      const float dpsi = -sq * dcq + cq * dsq;
      dk[k] = dpsi * p.theta[l];
      red_add(RED + l, dpsi * kz[k], quni);
      red_add(RED + L + l, d1 * cq + d2 * sq, quni);
      red_add(RED + 2 * L + l, d1 * sq - d2 * cq, quni);
    }
    if (vec) {
      *reinterpret_cast<float4*>(gr.dkz + t0i) = make_float4(dk[0], dk[1], dk[2], dk[3]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (l0 + k < L) gr.dkz[t0i + k] = dk[k];
    }
  }
  // owned keys: rows x in [x0, NX) (s = t0 .. t0 + tq - 1, and the buffer for the first CTA)
  const int x0 = g.t0 == 0 ? 0 : n;
  const int NO = NX - x0;
  const bool kuni = (NO & 31) == 0 && x0 == n;  // one mode group per warp, every key s >= 0
  const uint32_t mO = magic(NO);
  for (int u = tid; u < NO * NG; u += NT) {
    const int lg = qdiv(u, mO), x = x0 + u - lg * NO, l0 = 4 * lg, s = g.t0 - n + x;
    float cw[4] = {0.f, 0.f, 0.f, 0.f}, sw[4] = {0.f, 0.f, 0.f, 0.f};
    for (int lag = 0; lag < L; ++lag) {
      const int y = x - n + lag;
      if (y < 0 || y >= NY) continue;
      const float r = DKR[y * KP + lag], i = DKI[y * KP + lag];
      const float4 q1 = ld4(Q1 + y * CS + l0), q2 = ld4(Q2 + y * CS + l0);
      const float a4[4] = {q1.x, q1.y, q1.z, q1.w}, b4[4] = {q2.x, q2.y, q2.z, q2.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        cw[k] = fmaf(r, a4[k], fmaf(-i, b4[k], cw[k]));
        sw[k] = fmaf(r, b4[k], fmaf(i, a4[k], sw[k]));
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int l = l0 + k;
      if (l >= L) break;
      float dcw = cw[k] * iL, dsw = sw[k] * iL;
      if (s >= T - n) {  // the key is also in the new ring buffer
        const int64_t kk = ((int64_t)b * n + (s - (T - n))) * L + l;
        if (dc1) dcw += dc1[kk];
        if (ds1) dsw += ds1[kk];
      }
      if (s >= 0) {
        const float dphi = -KS[x * CS + l] * dcw + KC[x * CS + l] * dsw;
        const int64_t si = ((int64_t)b * T + s) * L + l;
        gr.dkh[si] = dphi * p.theta[l];
        red_add(RED + l, dphi * p.kh[si], kuni);
      } else {
        const int64_t kk = ((int64_t)b * n + n + s) * L + l;
        if (gr.dc0) gr.dc0[kk] = dcw;
        if (gr.ds0) gr.ds0[kk] = dsw;
      }
    }
  }
  // owned keys' values: d e_s = sum over the queries reading s of kappa . dO (8 columns a thread)
  for (int j0 = 0; j0 < dv; j0 += DS) {
    __syncthreads();
    load_grads(dO, g, b, NY, j0, GR, GI);
    __syncthreads();
    for (int u = tid; u < NO * (DS / 8); u += NT) {
      const int jg = qdiv(u, mO), x = x0 + u - jg * NO, jj = jg * 8, s = g.t0 - n + x;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      for (int lag = 0; lag < L; ++lag) {
        const int y = x - n + lag;
        if (y < 0 || y >= NY) continue;
        const float r = KR[y * KP + lag], i = KI[y * KP + lag];
        const float4 a0 = ld4(GR + y * ES + jj), a1 = ld4(GR + y * ES + jj + 4);
        const float4 c0 = ld4(GI + y * ES + jj), c1 = ld4(GI + y * ES + jj + 4);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = fmaf(r, av[k], fmaf(i, cv[k], acc[k]));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int j = j0 + jj + k;
        if (j >= dv) break;
        float a = acc[k];
        if (s >= T - n && de1) a += de1[((int64_t)b * n + (s - (T - n))) * dv + j];
        if (s >= 0)
          gr.dv[((int64_t)b * T + s) * dv + j] = a;
        else if (gr.de0)
          gr.de0[((int64_t)b * n + n + s) * dv + j] = a;
      }
    }
  }
  __syncthreads();
  float* dst = part + ((int64_t)b * gridDim.x + blockIdx.x) * 3 * L;
  for (int u = tid; u < 3 * L; u += NT) dst[u] = RED[u];
}

// dtheta, dwr, dwi: one block per output, a fixed-order tree over the per-CTA partials
__global__ void __launch_bounds__(256) short_reduce_kernel(const float* part, int nparts, int L, sca2_short_grads gr) {
  __shared__ float red[256];
  const int u = blockIdx.x;
  float acc = 0.f;
  for (int k = threadIdx.x; k < nparts; k += 256) acc += part[(int64_t)k * 3 * L + u];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float* out = u < L ? gr.dtheta : u < 2 * L ? gr.dwr : gr.dwi;
    out[u % L] = red[0];
  }
}

}  // namespace shortk

// Tokens per CTA: the largest of 64 / 32 / 16 whose shared memory lets two forward CTAs or
// three backward CTAs (its register bound) share an SM (16 whenever it fits at all), with the
// backward's pair groups within its register budget.
int short_tokens_per_cta(int L, bool bwd, int max_smem) {
  const int cand[3] = {64, 32, 16};
  const size_t lim = bwd ? 75u * 1024u : 112u * 1024u;
  for (int i = bwd ? 0 : 1; i < 3; ++i) {
    const int TT = cand[i];
    const size_t f = bwd ? shortk::bwd_smem_floats(L, TT) : shortk::fwd_smem_floats(L, TT);
    if (bwd && (TT + L - 1) * shortk::lane_groups(L) > 3 * shortk::NT) continue;
    if (f * sizeof(float) <= lim || (i == 2 && f * sizeof(float) <= (size_t)max_smem)) return TT;
  }
  return 0;
}

size_t short_work_floats(int B, int T, int L, int max_smem) {
  const int TT = short_tokens_per_cta(L, true, max_smem);
  if (TT == 0 || T < 1) return 0;
  return (size_t)B * ((T + TT - 1) / TT) * 3 * L;
}

cudaError_t short_fwd(const sca2_short_args& p, float* o, float* c1, float* s1, float* e1, int max_smem,
                      cudaStream_t st) {
  if (p.T > 0) {
    const int TT = short_tokens_per_cta(p.L, false, max_smem);
    const int smem = (int)(shortk::fwd_smem_floats(p.L, TT) * sizeof(float));
    cudaError_t e = cudaFuncSetAttribute(shortk::short_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.T + TT - 1) / TT, p.B);
    shortk::short_fwd_kernel<<<grid, shortk::NT, smem, st>>>(p, o, TT);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (p.L > 1 && (c1 || s1 || e1)) {
    shortk::short_state_kernel<<<p.B, shortk::NT, 0, st>>>(p, c1, s1, e1);
    return cudaGetLastError();
  }
  return cudaSuccess;
}

cudaError_t short_bwd(const sca2_short_args& p, const float* dO, const float* dc1, const float* ds1,
                      const float* de1, const sca2_short_grads& g, float* work, int max_smem, cudaStream_t st) {
  const int TT = short_tokens_per_cta(p.L, true, max_smem);
  const int smem = (int)(shortk::bwd_smem_floats(p.L, TT) * sizeof(float));
  cudaError_t e = cudaFuncSetAttribute(shortk::short_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int nch = (p.T + TT - 1) / TT;
  dim3 grid(nch, p.B);
  shortk::short_bwd_kernel<<<grid, shortk::NT, smem, st>>>(p, dO, dc1, ds1, de1, g, work, TT);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  shortk::short_reduce_kernel<<<3 * p.L, 256, 0, st>>>(work, p.B * nch, p.L, g);
  return cudaGetLastError();
}

}  // namespace sca2
