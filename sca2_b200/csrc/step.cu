// Single-token decode step: one CTA per (batch, head); the fp32 state is read once and
// written once (the kernel is HBM-bound: 2 * K * V * 4 bytes per (b, h)).
//
//   S~ = gamma .* S                        gamma[m] = exp(g) exp(-lam[m])
//   e  = v - beta (k^T S~) / kappa         (GDN form: v pre-scaled by beta)
//   o_r = (Q_r^T S~ + (Q_r . k) e) / kappa  == Q_r^T S_new / kappa
//   S_new = S~ + k e^T
// Follows lapa/layer.py:387-412 (LongHead.step), sca2/arch_gatedc.py:171-193
// (CHeadGated.step) and fla's recurrent GDN step.
#include "common.cuh"

namespace sca2 {
namespace step {

constexpr int NT = 256;
constexpr int MAXR = 32;  // largest number of state rows held in registers per thread

template <int FL, int VEC, int MAXR>
__global__ void __launch_bounds__(NT) step_kernel(sca2_scan_args p, const float* S_in,
                                                  float* S_out, sca2_out o) {
  extern __shared__ float sm[];
  constexpr int R = FL == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int bh = blockIdx.x, b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int K = p.K, V = p.V;
  const int slots = V / VEC;
  const int rg = max(1, min(NT / slots, K));
  const float kappa = FL == SCA2_FLAVOR_PHASE ? (float)(K / 2) : 1.f;
  const float ik = 1.f / kappa;
  float* kk = sm;                 // K
  float* Q = kk + K;              // R*K
  float* gam = Q + R * K;         // K
  float* vv = gam + K;            // V
  float* red = vv + V;            // (1+R) * rg * V
  float* ee = red + (1 + R) * rg * V;  // V
  float* scal = ee + V;           // 4

  // ---- prologue
  const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
  const float* gp = reinterpret_cast<const float*>(p.g.ptr);
  const float bt = bp ? bp[tok_off(p.beta, b, 0, h)] : 0.f;
  const float gdec = gp ? expf(gp[tok_off(p.g, b, 0, h)]) : 1.f;
  if (FL == SCA2_FLAVOR_PHASE) {
    const int Mh = K / 2;
    const float* phw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* phq = reinterpret_cast<const float*>(p.phq.ptr);
    for (int m = threadIdx.x; m < Mh; m += blockDim.x) {
      float s, c, sq, cq;
      sincosf(phw[tok_off(p.phw, b, 0, h) + m], &s, &c);
      sincosf(phq[tok_off(p.phq, b, 0, h) + m], &sq, &cq);
      const float wr = p.wr[h * Mh + m], wi = p.wi[h * Mh + m];
      const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
      kk[m] = c;
      kk[m + Mh] = s;
      Q[m] = c1;
      Q[m + Mh] = c2;
      Q[K + m] = -c2;
      Q[K + m + Mh] = c1;
      const float l = p.lam ? p.lam[h * Mh + m] : 0.f;
      gam[m] = gam[m + Mh] = gdec * expf(-l);
    }
  } else {
    for (int m = threadIdx.x; m < K; m += blockDim.x) {
      kk[m] = ld_io(p.phw.ptr, tok_off(p.phw, b, 0, h) + m, p.io_dtype);
      Q[m] = p.q_scale * ld_io(p.phq.ptr, tok_off(p.phq, b, 0, h) + m, p.io_dtype);
      const float l = p.lam ? p.lam[h * K + m] : 0.f;
      gam[m] = gdec * expf(-l);
    }
  }
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float x = ld_io(p.v.ptr, tok_off(p.v, b, 0, h) + j, p.io_dtype);
    if (p.v_times_beta) x *= bt;
    vv[j] = x;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // Q_r . k
    for (int r = 0; r < R; ++r) {
      float s = 0.f;
      for (int m = threadIdx.x; m < K; m += 32) s += Q[r * K + m] * kk[m];
      s = warp_sum(s);
      if (threadIdx.x == 0) scal[r] = s;
    }
  }

  // ---- pass over the state: decay, partial reductions over rows
  const int tx = threadIdx.x % slots, ty = threadIdx.x / slots;
  const bool active = threadIdx.x < slots * rg;
  const int64_t base = (int64_t)bh * K * V;
  float s_reg[MAXR][VEC];
  float pk[VEC], pq[R][VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
    pk[c] = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) pq[r][c] = 0.f;
  }
  if (active) {
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      const int m = ty + q * rg;
      if (m < K) {
        float x[VEC];
        if (VEC == 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(S_in + base + (int64_t)m * V + tx * 4);
          x[0] = t4.x; x[1] = t4.y; x[2] = t4.z; x[3] = t4.w;
        } else {
          x[0] = S_in[base + (int64_t)m * V + tx];
        }
        const float gm = gam[m], km = kk[m];
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
          const float s = gm * x[c];
          s_reg[q][c] = s;
          pk[c] = fmaf(km, s, pk[c]);
#pragma unroll
          for (int r = 0; r < R; ++r) pq[r][c] = fmaf(Q[r * K + m], s, pq[r][c]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const int j = tx * VEC + c;
      red[ty * V + j] = pk[c];
#pragma unroll
      for (int r = 0; r < R; ++r) red[((1 + r) * rg + ty) * V + j] = pq[r][c];
    }
  }
  __syncthreads();
  // ---- column reductions: e, o
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float sk = 0.f;
    for (int y = 0; y < rg; ++y) sk += red[y * V + j];
    const float e = vv[j] - bt * sk * ik;
    ee[j] = e;
    for (int r = 0; r < R; ++r) {
      float sq = 0.f;
      for (int y = 0; y < rg; ++y) sq += red[((1 + r) * rg + y) * V + j];
      st_io(o.ptr, out_off(o, b, 0, h, r) + j, (sq + scal[r] * e) * ik, p.io_dtype);
    }
  }
  __syncthreads();
  // ---- write the new state
  if (active) {
    float ev[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) ev[c] = ee[tx * VEC + c];
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      const int m = ty + q * rg;
      if (m < K) {
        const float km = kk[m];
        if (VEC == 4) {
          float4 t4;
          t4.x = fmaf(km, ev[0], s_reg[q][0]);
          t4.y = fmaf(km, ev[1], s_reg[q][1]);
          t4.z = fmaf(km, ev[2], s_reg[q][2]);
          t4.w = fmaf(km, ev[3], s_reg[q][3]);
          *reinterpret_cast<float4*>(S_out + base + (int64_t)m * V + tx * 4) = t4;
        } else {
          S_out[base + (int64_t)m * V + tx] = fmaf(km, ev[0], s_reg[q][0]);
        }
      }
    }
  }
}

// ---- persistent decode step -------------------------------------------------------------
// One CTA of 512 threads per SM walks (b, h) items.  Thread (tx, ty) holds columns 4tx..4tx+3
// of the state rows ty + RG q (q < RPT) in registers, and the next item's rows are loaded
// into a second register set while the current item is processed, so HBM reads stay in
// flight across items.  The token's codes (k, Q, gamma, v) for the next item are computed
// by warps 8..11 between the two barriers of the current item.
constexpr int PNT = 512;

template <int FL, int K, int V>
struct Pers {
  static constexpr int R = FL == SCA2_FLAVOR_PHASE ? 2 : 1;
  static constexpr int CQ = V / 4, RG = PNT / CQ, RPT = K / RG;
  static constexpr int NP = FL == SCA2_FLAVOR_PHASE ? K / 2 : K;  // code threads (modes | dims)
  static constexpr int NPW = (NP + 31) / 32;                        // their warps
  // params of one item: k[K], Q[R*K], gam[K], v[V], partial Q_r.k per code warp, beta
  static constexpr int PSZ = K + R * K + K + V + R * NPW + 4;
  static constexpr int SMEM = (2 * PSZ + (1 + R) * RG * V + V) * 4;
  static_assert(PNT % CQ == 0 && K % RG == 0 && RPT >= 1, "state tiling");
  static_assert(NP <= 128, "code threads live in warps 8..11");
};

template <int FL, int K, int V>
struct RawCode {  // raw per-token inputs of one item held by one code thread
  float a, b2, lam, wr, wi, v[(V + 127) / 128], beta, g;
};

template <int FL, int K, int V>
__device__ __forceinline__ void load_raw(const sca2_scan_args& p, RawCode<FL, K, V>& r, int item, int t) {
  using P = Pers<FL, K, V>;
  const int b = item / p.H, h = item - (item / p.H) * p.H;
  const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
  const float* gp = reinterpret_cast<const float*>(p.g.ptr);
  r.beta = bp ? bp[tok_off(p.beta, b, 0, h)] : 0.f;
  r.g = gp ? gp[tok_off(p.g, b, 0, h)] : 0.f;
  if (t < P::NP) {
    if (FL == SCA2_FLAVOR_PHASE) {
      r.a = reinterpret_cast<const float*>(p.phw.ptr)[tok_off(p.phw, b, 0, h) + t];
      r.b2 = reinterpret_cast<const float*>(p.phq.ptr)[tok_off(p.phq, b, 0, h) + t];
      r.wr = p.wr[h * P::NP + t];
      r.wi = p.wi[h * P::NP + t];
    } else {
      r.a = ld_io(p.phw.ptr, tok_off(p.phw, b, 0, h) + t, p.io_dtype);
      r.b2 = ld_io(p.phq.ptr, tok_off(p.phq, b, 0, h) + t, p.io_dtype);
    }
    r.lam = p.lam ? p.lam[h * P::NP + t] : 0.f;
  }
#pragma unroll
  for (int u = 0; u < (V + 127) / 128; ++u) {
    const int j = t + 128 * u;
    r.v[u] = j < V ? ld_io(p.v.ptr, tok_off(p.v, b, 0, h) + j, p.io_dtype) : 0.f;
  }
}

// code thread t (0..127) turns its raw inputs into the item's params
template <int FL, int K, int V>
__device__ __forceinline__ void make_params(const sca2_scan_args& p, const RawCode<FL, K, V>& r, float* prm, int t) {
  using P = Pers<FL, K, V>;
  constexpr int R = P::R;
  float* kk = prm;
  float* Q = kk + K;
  float* gam = Q + R * K;
  float* vv = gam + K;
  float* qk = vv + V;
  const float gdec = p.g.ptr ? expf(r.g) : 1.f;
  float part[R];
#pragma unroll
  for (int q = 0; q < R; ++q) part[q] = 0.f;
  if (t < P::NP) {
    if (FL == SCA2_FLAVOR_PHASE) {
      constexpr int Mh = K / 2;
      float s, c, sq, cq;
      sincosf(r.a, &s, &c);
      sincosf(r.b2, &sq, &cq);
      const float c1 = r.wr * cq + r.wi * sq, c2 = r.wr * sq - r.wi * cq;
      kk[t] = c;
      kk[t + Mh] = s;
      Q[t] = c1;
      Q[t + Mh] = c2;
      Q[K + t] = -c2;
      Q[K + t + Mh] = c1;
      gam[t] = gam[t + Mh] = gdec * expf(-r.lam);
      part[0] = c1 * c + c2 * s;
      if (R > 1) part[R - 1] = -c2 * c + c1 * s;
    } else {
      const float qv = p.q_scale * r.b2;
      kk[t] = r.a;
      Q[t] = qv;
      gam[t] = gdec * expf(-r.lam);
      part[0] = qv * r.a;
    }
  }
#pragma unroll
  for (int u = 0; u < (V + 127) / 128; ++u) {
    const int j = t + 128 * u;
    if (j < V) vv[j] = p.v_times_beta ? r.v[u] * r.beta : r.v[u];
  }
#pragma unroll
  for (int q = 0; q < R; ++q) {
    const float x = warp_sum(part[q]);
    if ((t & 31) == 0 && (t >> 5) < P::NPW) qk[q * P::NPW + (t >> 5)] = x;
  }
  if (t == 0) qk[R * P::NPW] = r.beta;
}

template <int FL, int K, int V>
__global__ void __launch_bounds__(PNT, 1) step_pers_kernel(sca2_scan_args p, const float* S_in, float* S_out,
                                                          sca2_out o, int items) {
  using P = Pers<FL, K, V>;
  constexpr int R = P::R, CQ = P::CQ, RG = P::RG, RPT = P::RPT, PSZ = P::PSZ;
  extern __shared__ float sm[];
  float* prm = sm;                  // [2][PSZ]
  float* red = prm + 2 * PSZ;       // [1 + R][RG][V]
  float* ee = red + (1 + R) * RG * V;
  const int tid = threadIdx.x, tx = tid % CQ, ty = tid / CQ;
  const bool coder = tid >= 256 && tid < 384;
  const int ct = tid - 256;
  const float ik = FL == SCA2_FLAVOR_PHASE ? 1.f / (float)(K / 2) : 1.f;
  const int first = blockIdx.x;
  if (first >= items) return;

  RawCode<FL, K, V> raw;
  if (coder) {
    load_raw<FL, K, V>(p, raw, first, ct);
    make_params<FL, K, V>(p, raw, prm, ct);
    if (first + (int)gridDim.x < items) load_raw<FL, K, V>(p, raw, first + gridDim.x, ct);
  }
  float4 nxt[RPT];
  {
    const float* src = S_in + (int64_t)first * K * V;
#pragma unroll
    for (int q = 0; q < RPT; ++q) nxt[q] = *reinterpret_cast<const float4*>(src + (int64_t)(ty + RG * q) * V + 4 * tx);
  }
  __syncthreads();
  int n = 0;
  for (int item = first; item < items; item += gridDim.x, ++n) {
    const float* pr = prm + (n & 1) * PSZ;
    const float* kk = pr;
    const float* Q = kk + K;
    const float* gam = Q + R * K;
    const float* vv = gam + K;
    const float* qk = vv + V;
    float4 cur[RPT];
#pragma unroll
    for (int q = 0; q < RPT; ++q) cur[q] = nxt[q];
    const int next = item + gridDim.x;
    if (next < items) {  // the next item's state, in flight while this one is processed
      const float* src = S_in + (int64_t)next * K * V;
#pragma unroll
      for (int q = 0; q < RPT; ++q) nxt[q] = *reinterpret_cast<const float4*>(src + (int64_t)(ty + RG * q) * V + 4 * tx);
    }
    // [A] decay and partial reductions over this thread's rows
    float pk[4] = {0.f, 0.f, 0.f, 0.f}, pq[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) pq[r][0] = pq[r][1] = pq[r][2] = pq[r][3] = 0.f;
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int m = ty + RG * q;
      const float gm = gam[m], km = kk[m];
      float* c = reinterpret_cast<float*>(&cur[q]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s = gm * c[j];
        c[j] = s;
        pk[j] = fmaf(km, s, pk[j]);
#pragma unroll
        for (int r = 0; r < R; ++r) pq[r][j] = fmaf(Q[r * K + m], s, pq[r][j]);
      }
    }
    *reinterpret_cast<float4*>(red + ty * V + 4 * tx) = make_float4(pk[0], pk[1], pk[2], pk[3]);
#pragma unroll
    for (int r = 0; r < R; ++r)
      *reinterpret_cast<float4*>(red + ((1 + r) * RG + ty) * V + 4 * tx) = make_float4(pq[r][0], pq[r][1], pq[r][2], pq[r][3]);
    __syncthreads();
    // [B] column reductions -> e, o; the code threads prepare the next item's params
    const int b = item / p.H, h = item - (item / p.H) * p.H;
    if (tid < V) {
      const int j = tid;
      float sk = 0.f;
#pragma unroll 4
      for (int y = 0; y < RG; ++y) sk += red[y * V + j];
      const float bt = qk[R * P::NPW];
      const float e = vv[j] - bt * sk * ik;
      ee[j] = e;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float sq = 0.f;
#pragma unroll 4
        for (int y = 0; y < RG; ++y) sq += red[((1 + r) * RG + y) * V + j];
        float qkr = 0.f;
#pragma unroll
        for (int w = 0; w < P::NPW; ++w) qkr += qk[r * P::NPW + w];
        st_io(o.ptr, out_off(o, b, 0, h, r) + j, (sq + qkr * e) * ik, p.io_dtype);
      }
    }
    if (coder && next < items) {
      make_params<FL, K, V>(p, raw, prm + ((n + 1) & 1) * PSZ, ct);
      if (next + (int)gridDim.x < items) load_raw<FL, K, V>(p, raw, next + gridDim.x, ct);
    }
    __syncthreads();
    // [C] new state
    {
      const float4 ev = *reinterpret_cast<const float4*>(ee + 4 * tx);
      float* dst = S_out + (int64_t)item * K * V;
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        const int m = ty + RG * q;
        const float km = kk[m];
        float4 t = cur[q];
        t.x = fmaf(km, ev.x, t.x);
        t.y = fmaf(km, ev.y, t.y);
        t.z = fmaf(km, ev.z, t.z);
        t.w = fmaf(km, ev.w, t.w);
        *reinterpret_cast<float4*>(dst + (int64_t)m * V + 4 * tx) = t;
      }
    }
  }
}

}  // namespace step

// persistent variant for the common state shapes (fp32 state 16-byte aligned)
static bool step_pers_covered(int K, int V) { return (K == 128 && V == 128) || (K == 64 && V == 64); }

template <int FL, int K, int V>
static cudaError_t launch_pers_t(const sca2_scan_args& p, const float* S_in, float* S_out, const sca2_out& o,
                                 cudaStream_t st) {
  auto k = step::step_pers_kernel<FL, K, V>;
  const int smem = step::Pers<FL, K, V>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = p.B * p.H;
  const int grid = items < sms ? items : sms;
  k<<<grid, step::PNT, smem, st>>>(p, S_in, S_out, o, items);
  return cudaGetLastError();
}

// Rows of state each thread must hold; the launcher rejects shapes needing more than MAXR.
int step_rows_per_thread(int K, int V, int vec) {
  const int slots = V / vec;
  if (slots > step::NT) return 1 << 30;
  const int rg = slots > 0 ? (step::NT / slots < K ? step::NT / slots : K) : 1;
  return (K + rg - 1) / (rg > 0 ? rg : 1);
}
int step_max_rows() { return step::MAXR; }  // rows per thread of the widest variant

size_t step_smem_bytes(int K, int V, int R, int vec) {
  const int slots = V / vec;
  int rg = step::NT / slots;
  if (rg > K) rg = K;
  if (rg < 1) rg = 1;
  return (size_t)(K + R * K + K + V + (1 + R) * rg * V + V + 4) * 4;
}

template <int FL, int VEC, int MR>
static void launch_step_t(const sca2_scan_args& p, const float* S_in, float* S_out,
                          const sca2_out& o, size_t smem, cudaStream_t st) {
  auto k = step::step_kernel<FL, VEC, MR>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k<<<dim3(p.B * p.H), step::NT, smem, st>>>(p, S_in, S_out, o);
}

template <int FL, int VEC>
static void launch_step_v(const sca2_scan_args& p, const float* S_in, float* S_out,
                          const sca2_out& o, size_t smem, int rows, cudaStream_t st) {
  if (rows <= 4)
    launch_step_t<FL, VEC, 4>(p, S_in, S_out, o, smem, st);
  else if (rows <= 16)
    launch_step_t<FL, VEC, 16>(p, S_in, S_out, o, smem, st);
  else
    launch_step_t<FL, VEC, 32>(p, S_in, S_out, o, smem, st);
}

cudaError_t launch_step(const sca2_scan_args& p, const float* S_in, float* S_out,
                        const sca2_out& o, int vec, cudaStream_t st) {
  if (vec == 4 && step_pers_covered(p.K, p.V)) {
    const bool ph = p.flavor == SCA2_FLAVOR_PHASE;
    if (p.K == 128) return ph ? launch_pers_t<SCA2_FLAVOR_PHASE, 128, 128>(p, S_in, S_out, o, st)
                              : launch_pers_t<SCA2_FLAVOR_KEY, 128, 128>(p, S_in, S_out, o, st);
    return ph ? launch_pers_t<SCA2_FLAVOR_PHASE, 64, 64>(p, S_in, S_out, o, st)
              : launch_pers_t<SCA2_FLAVOR_KEY, 64, 64>(p, S_in, S_out, o, st);
  }
  const int R = p.flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  const size_t smem = step_smem_bytes(p.K, p.V, R, vec);
  const int rows = step_rows_per_thread(p.K, p.V, vec);
  if (p.flavor == SCA2_FLAVOR_PHASE) {
    if (vec == 4) launch_step_v<SCA2_FLAVOR_PHASE, 4>(p, S_in, S_out, o, smem, rows, st);
    else launch_step_v<SCA2_FLAVOR_PHASE, 1>(p, S_in, S_out, o, smem, rows, st);
  } else {
    if (vec == 4) launch_step_v<SCA2_FLAVOR_KEY, 4>(p, S_in, S_out, o, smem, rows, st);
    else launch_step_v<SCA2_FLAVOR_KEY, 1>(p, S_in, S_out, o, smem, rows, st);
  }
  return cudaGetLastError();
}

// ---- RMS read-out ---------------------------------------------------------------------
namespace rms {
constexpr int NT = 256;
// one warp per row
__global__ void __launch_bounds__(NT) rms_fwd_kernel(const void* x, void* u, int64_t N, int D,
                                                     float eps, int dt) {
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const int64_t off = row * D;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    ss = fmaf(a, a, ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  for (int j = lane; j < D; j += 32) st_io(u, off + j, ld_io(x, off + j, dt) * r, dt);
}

__global__ void __launch_bounds__(NT) rms_bwd_kernel(const void* x, const void* du, void* dx,
                                                     int64_t N, int D, float eps, int dt) {
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const int64_t off = row * D;
  float ss = 0.f, sd = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    ss = fmaf(a, a, ss);
    sd = fmaf(a, ld_io(du, off + j, dt), sd);
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  const float r = rsqrtf(ss / (float)D + eps);
  const float c = r * r * sd / (float)D;  // mean(du * u) / r
  for (int j = lane; j < D; j += 32) {
    const float a = ld_io(x, off + j, dt);
    const float g = ld_io(du, off + j, dt);
    st_io(dx, off + j, r * (g - a * c), dt);
  }
}
}  // namespace rms

cudaError_t launch_rms_fwd(const void* x, void* u, int64_t N, int D, float eps, int dt,
                           cudaStream_t st) {
  const int64_t blocks = (N + rms::NT / 32 - 1) / (rms::NT / 32);
  rms::rms_fwd_kernel<<<(unsigned)blocks, rms::NT, 0, st>>>(x, u, N, D, eps, dt);
  return cudaGetLastError();
}
cudaError_t launch_rms_bwd(const void* x, const void* du, void* dx, int64_t N, int D, float eps,
                           int dt, cudaStream_t st) {
  const int64_t blocks = (N + rms::NT / 32 - 1) / (rms::NT / 32);
  rms::rms_bwd_kernel<<<(unsigned)blocks, rms::NT, 0, st>>>(x, du, dx, N, D, eps, dt);
  return cudaGetLastError();
}

}  // namespace sca2
