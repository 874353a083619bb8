// Separable D-head read-out and the bf16 hi / lo operand split of the heads' 16-bit
// projections (memory-bound row kernels on the CUDA cores).
//
// Read-out (sca2/arch_sepq.py:93-104, then the RMS read-out of sca2/ref.py:29-30): per row r
// (a token) and channel j < dv,
//     n_j = rsqrt(br_j^2 + bi_j^2 + eps_q),   pr = br_j n_j,   pi = bi_j n_j
//     u   = [ pr A_j + pi Bv_j | pr Bv_j - pi A_j ]              (2 dv values)
//     out = u * rsqrt(mean(u^2) + eps)
// with [A | Bv] the scan's contracted read.  One warp per row: a first pass forms u and its
// sum of squares, a second pass (the row's inputs are still in L1 / L2) writes out; the
// backward's first pass forms the row sums of u^2 and dout * u, its second pass the gradients
// of A, Bv, br and bi.  Loads and stores are coalesced along the channels (float4 when the
// widths and addresses allow).
//
// Split: hi = bf16(x), lo = bf16(x - hi), so hi + lo carries about 16 significant bits of x;
// a product chain hi*hi + hi*lo + lo*hi of two split operands then keeps 16-bit precision on
// bf16 tensor cores.  The kernel writes the column blocks of [hi | hi | lo]-style operands in
// one pass.
#include <algorithm>

#include "common.cuh"

namespace sca2 {
using bf16 = __nv_bfloat16;

namespace readout {

constexpr int NT = 256;        // 8 rows per CTA
constexpr int RPC = NT / 32;

struct RowIO {
  const float *ab, *br, *bi;
  int64_t ldq;
  float eps_q;
};

template <bool VEC>
__device__ __forceinline__ void load4(const float* p, int64_t i, float* x) {
  if (VEC) {
    const float4 v = *reinterpret_cast<const float4*>(p + i);
    x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = p[i + k];
  }
}
template <bool VEC>
__device__ __forceinline__ void store4(float* p, int64_t i, const float* x) {
  if (VEC) {
    *reinterpret_cast<float4*>(p + i) = make_float4(x[0], x[1], x[2], x[3]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) p[i + k] = x[k];
  }
}

// the row's values at channels j..j+3 (VEC) or j (scalar; the other three unused)
template <bool VEC>
struct Quad {
  float A[4], B[4], r[4], i[4], n[4], u1[4], u2[4];
  __device__ __forceinline__ int load(const RowIO& io, int64_t row, int dv, int j) {
    const int cnt = VEC ? 4 : 1;
    const float* a = io.ab + row * 2 * dv;
    if (VEC) {
      load4<true>(a, j, A);
      load4<true>(a, dv + j, B);
      load4<true>(io.br, row * io.ldq + j, r);
      load4<true>(io.bi, row * io.ldq + j, i);
    } else {
      A[0] = a[j], B[0] = a[dv + j], r[0] = io.br[row * io.ldq + j], i[0] = io.bi[row * io.ldq + j];
    }
#pragma unroll
    for (int k = 0; k < cnt; ++k) {
      n[k] = rsqrtf(fmaf(r[k], r[k], fmaf(i[k], i[k], io.eps_q)));
      const float pr = r[k] * n[k], pi = i[k] * n[k];
      u1[k] = fmaf(pr, A[k], pi * B[k]);
      u2[k] = fmaf(pr, B[k], -pi * A[k]);
    }
    return cnt;
  }
};

template <bool VEC>
__global__ void __launch_bounds__(NT) sepq_read_fwd_kernel(RowIO io, float* out, int64_t rows, int dv, float eps) {
  const int64_t row = (int64_t)blockIdx.x * RPC + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int STEP = VEC ? 128 : 32;
  const int j0 = VEC ? 4 * lane : lane;
  float ss = 0.f;
  for (int j = j0; j < dv; j += STEP) {
    Quad<VEC> q;
    const int cnt = q.load(io, row, dv, j);
    for (int k = 0; k < cnt; ++k) ss = fmaf(q.u1[k], q.u1[k], fmaf(q.u2[k], q.u2[k], ss));
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)(2 * dv) + eps);
  float* o = out + row * 2 * dv;
  for (int j = j0; j < dv; j += STEP) {
    Quad<VEC> q;
    q.load(io, row, dv, j);
    if (VEC) {
      float x1[4], x2[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) x1[k] = q.u1[k] * rs, x2[k] = q.u2[k] * rs;
      store4<true>(o, j, x1);
      store4<true>(o, dv + j, x2);
    } else {
      o[j] = q.u1[0] * rs;
      o[dv + j] = q.u2[0] * rs;
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(NT) sepq_read_bwd_kernel(RowIO io, const float* dout, float* dab, float* dbr,
                                                           float* dbi, int64_t lddq, int64_t rows, int dv,
                                                           float eps) {
  const int64_t row = (int64_t)blockIdx.x * RPC + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int STEP = VEC ? 128 : 32;
  const int j0 = VEC ? 4 * lane : lane;
  const float* g = dout + row * 2 * dv;
  float ss = 0.f, sd = 0.f;
  for (int j = j0; j < dv; j += STEP) {
    Quad<VEC> q;
    const int cnt = q.load(io, row, dv, j);
    float g1[4], g2[4];
    if (VEC) {
      load4<true>(g, j, g1);
      load4<true>(g, dv + j, g2);
    } else {
      g1[0] = g[j], g2[0] = g[dv + j];
    }
    for (int k = 0; k < cnt; ++k) {
      ss = fmaf(q.u1[k], q.u1[k], fmaf(q.u2[k], q.u2[k], ss));
      sd = fmaf(g1[k], q.u1[k], fmaf(g2[k], q.u2[k], sd));
    }
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  const float D = (float)(2 * dv);
  const float rs = rsqrtf(ss / D + eps);
  const float c = rs * rs * rs * sd / D;  // d out / d u = rs g - u rs^3 (g . u) / D
  float* da = dab + row * 2 * dv;
  for (int j = j0; j < dv; j += STEP) {
    Quad<VEC> q;
    const int cnt = q.load(io, row, dv, j);
    float g1[4], g2[4], oA[4], oB[4], oR[4], oI[4];
    if (VEC) {
      load4<true>(g, j, g1);
      load4<true>(g, dv + j, g2);
    } else {
      g1[0] = g[j], g2[0] = g[dv + j];
    }
    for (int k = 0; k < cnt; ++k) {
      const float d1 = fmaf(rs, g1[k], -c * q.u1[k]), d2 = fmaf(rs, g2[k], -c * q.u2[k]);
      const float pr = q.r[k] * q.n[k], pi = q.i[k] * q.n[k];
      oA[k] = fmaf(pr, d1, -pi * d2);
      oB[k] = fmaf(pi, d1, pr * d2);
      const float dpr = fmaf(q.A[k], d1, q.B[k] * d2), dpi = fmaf(q.B[k], d1, -q.A[k] * d2);
      const float n3s = q.n[k] * q.n[k] * q.n[k] * fmaf(q.r[k], dpr, q.i[k] * dpi);
      oR[k] = fmaf(q.n[k], dpr, -q.r[k] * n3s);
      oI[k] = fmaf(q.n[k], dpi, -q.i[k] * n3s);
    }
    if (VEC) {
      store4<true>(da, j, oA);
      store4<true>(da, dv + j, oB);
      store4<true>(dbr, row * lddq + j, oR);
      store4<true>(dbi, row * lddq + j, oI);
    } else {
      da[j] = oA[0], da[dv + j] = oB[0];
      dbr[row * lddq + j] = oR[0];
      dbi[row * lddq + j] = oI[0];
    }
  }
}

// ---- RMS read-out of a multi-head read (sca2/arch_gatedc.py:155-156, 168) ------------------
// x rows hold H heads of [re | im] halves of dvh values, (H, 2, dvh); out rows are
// [re of every head | im of every head], (2, H, dvh), times rsqrt(mean(x^2) + eps).  Four
// consecutive values (one head, one half; dvh % 4 == 0) per lane and step.
__device__ __forceinline__ void ld4_io(const void* p, int64_t i, int dt, float* x) {
  if (dt == SCA2_BF16) {
    const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    x[0] = __low2float(h[0]), x[1] = __high2float(h[0]), x[2] = __low2float(h[1]), x[3] = __high2float(h[1]);
  } else {
    load4<true>(reinterpret_cast<const float*>(p), i, x);
  }
}
__device__ __forceinline__ void st4_io(void* p, int64_t i, int dt, const float* x) {
  if (dt == SCA2_BF16) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<const uint32_t*>(&a);
    raw.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = raw;
  } else {
    store4<true>(reinterpret_cast<float*>(p), i, x);
  }
}
// output position of input position i (a multiple of 4) of a row
__device__ __forceinline__ int heads_out(int i, int H, int dvh) {
  const int hr = i / dvh, j = i - hr * dvh;  // hr = 2 h + r
  return ((hr & 1) * H + (hr >> 1)) * dvh + j;
}

__global__ void __launch_bounds__(NT) rms_heads_fwd_kernel(const void* x, int dt, float* out, int64_t rows, int H,
                                                           int dvh, float eps) {
  const int64_t row = (int64_t)blockIdx.x * RPC + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int D = 2 * H * dvh;
  const int64_t off = row * D;
  float ss = 0.f;
  for (int i = 4 * lane; i < D; i += 128) {
    float v[4];
    ld4_io(x, off + i, dt, v);
    ss = fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], fmaf(v[3], v[3], ss))));
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)D + eps);
  for (int i = 4 * lane; i < D; i += 128) {
    float v[4];
    ld4_io(x, off + i, dt, v);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= rs;
    store4<true>(out, off + heads_out(i, H, dvh), v);
  }
}

__global__ void __launch_bounds__(NT) rms_heads_bwd_kernel(const void* x, int dt, const float* dout, void* dx,
                                                           int64_t rows, int H, int dvh, float eps) {
  const int64_t row = (int64_t)blockIdx.x * RPC + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int D = 2 * H * dvh;
  const int64_t off = row * D;
  float ss = 0.f, sd = 0.f;
  for (int i = 4 * lane; i < D; i += 128) {
    float v[4], g[4];
    ld4_io(x, off + i, dt, v);
    load4<true>(dout, off + heads_out(i, H, dvh), g);
#pragma unroll
    for (int k = 0; k < 4; ++k) ss = fmaf(v[k], v[k], ss), sd = fmaf(v[k], g[k], sd);
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  const float rs = rsqrtf(ss / (float)D + eps);
  const float c = rs * rs * rs * sd / (float)D;
  for (int i = 4 * lane; i < D; i += 128) {
    float v[4], g[4], o[4];
    ld4_io(x, off + i, dt, v);
    load4<true>(dout, off + heads_out(i, H, dvh), g);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = fmaf(rs, g[k], -c * v[k]);
    st4_io(dx, off + i, dt, o);
  }
}

// ---- bf16 hi / lo split -------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool VEC>
__global__ void __launch_bounds__(NT) split_kernel(const float* x, int64_t rows, int cols, int64_t ldx, bf16* out,
                                                   int64_t ldo, int nblk, uint32_t lo_mask) {
  const int per = VEC ? 4 : 1;
  const int64_t cq = cols / per;
  const int64_t n = rows * cq;
  for (int64_t u = (int64_t)blockIdx.x * NT + threadIdx.x; u < n; u += (int64_t)gridDim.x * NT) {
    const int64_t r = u / cq;
    const int c = (int)(u - r * cq) * per;
    if (VEC) {
      float v[4], h[4], l[4];
      load4<true>(x, r * ldx + c, v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        h[k] = __bfloat162float(__float2bfloat16_rn(v[k]));
        l[k] = v[k] - h[k];
      }
      const uint2 ph = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
      const uint2 pl = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
      for (int b = 0; b < nblk; ++b)
        *reinterpret_cast<uint2*>(out + r * ldo + (int64_t)b * cols + c) = (lo_mask >> b) & 1u ? pl : ph;
    } else {
      const float v = x[r * ldx + c];
      const bf16 h = __float2bfloat16_rn(v);
      const bf16 l = __float2bfloat16_rn(v - __bfloat162float(h));
      for (int b = 0; b < nblk; ++b) out[r * ldo + (int64_t)b * cols + c] = (lo_mask >> b) & 1u ? l : h;
    }
  }
}

}  // namespace readout

namespace {
bool a16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
unsigned grid_rows(int64_t rows) { return (unsigned)((rows + readout::RPC - 1) / readout::RPC); }
}  // namespace

cudaError_t launch_sepq_read_fwd(const float* ab, const float* br, const float* bi, int64_t ldq, float* out,
                                 int64_t rows, int dv, float eps_q, float eps, cudaStream_t st) {
  const readout::RowIO io{ab, br, bi, ldq, eps_q};
  const bool vec = dv % 4 == 0 && ldq % 4 == 0 && a16(ab) && a16(br) && a16(bi) && a16(out);
  if (vec)
    readout::sepq_read_fwd_kernel<true><<<grid_rows(rows), readout::NT, 0, st>>>(io, out, rows, dv, eps);
  else
    readout::sepq_read_fwd_kernel<false><<<grid_rows(rows), readout::NT, 0, st>>>(io, out, rows, dv, eps);
  return cudaGetLastError();
}

cudaError_t launch_sepq_read_bwd(const float* ab, const float* br, const float* bi, int64_t ldq, const float* dout,
                                 float* dab, float* dbr, float* dbi, int64_t lddq, int64_t rows, int dv, float eps_q,
                                 float eps, cudaStream_t st) {
  const readout::RowIO io{ab, br, bi, ldq, eps_q};
  const bool vec = dv % 4 == 0 && ldq % 4 == 0 && lddq % 4 == 0 && a16(ab) && a16(br) && a16(bi) && a16(dout) &&
                   a16(dab) && a16(dbr) && a16(dbi);
  if (vec)
    readout::sepq_read_bwd_kernel<true>
        <<<grid_rows(rows), readout::NT, 0, st>>>(io, dout, dab, dbr, dbi, lddq, rows, dv, eps);
  else
    readout::sepq_read_bwd_kernel<false>
        <<<grid_rows(rows), readout::NT, 0, st>>>(io, dout, dab, dbr, dbi, lddq, rows, dv, eps);
  return cudaGetLastError();
}

cudaError_t launch_rms_heads_fwd(const void* x, int dt, float* out, int64_t rows, int H, int dvh, float eps,
                                 cudaStream_t st) {
  readout::rms_heads_fwd_kernel<<<grid_rows(rows), readout::NT, 0, st>>>(x, dt, out, rows, H, dvh, eps);
  return cudaGetLastError();
}
cudaError_t launch_rms_heads_bwd(const void* x, int dt, const float* dout, void* dx, int64_t rows, int H, int dvh,
                                 float eps, cudaStream_t st) {
  readout::rms_heads_bwd_kernel<<<grid_rows(rows), readout::NT, 0, st>>>(x, dt, dout, dx, rows, H, dvh, eps);
  return cudaGetLastError();
}

cudaError_t launch_split_bf16(const float* x, int64_t rows, int cols, int64_t ldx, void* out, int64_t ldo, int nblk,
                              uint32_t lo_mask, cudaStream_t st) {
  bf16* o = reinterpret_cast<bf16*>(out);
  const bool vec = cols % 4 == 0 && ldx % 4 == 0 && ldo % 4 == 0 && a16(x) && ((uintptr_t)out & 7u) == 0;
  const int64_t units = rows * (vec ? cols / 4 : cols);
  const unsigned grid = (unsigned)std::min<int64_t>((units + readout::NT - 1) / readout::NT, 148 * 16);
  if (grid == 0) return cudaSuccess;
  if (vec)
    readout::split_kernel<true><<<grid, readout::NT, 0, st>>>(x, rows, cols, ldx, o, ldo, nblk, lo_mask);
  else
    readout::split_kernel<false><<<grid, readout::NT, 0, st>>>(x, rows, cols, ldx, o, ldo, nblk, lo_mask);
  return cudaGetLastError();
}

}  // namespace sca2
