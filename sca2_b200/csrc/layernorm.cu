// LayerNorm forward and backward over rows of width d = 32 V (V a multiple of 4: d = 128 ...
// 1024), fp32 (the layers' pre-norms, torch.nn.LayerNorm semantics: biased variance, eps inside
// the root, affine weight and bias).
//
// One warp per row, V values per lane (float4 loads at 4 lane + 128 k), the row held in
// registers between its two reductions.  The backward also accumulates the weight and bias
// gradients of its rows in registers (the lane's columns are the same in every row), sums the
// warps of a CTA in shared memory and writes one partial row pair per CTA; a second kernel
// adds the partials column by column.
#include <algorithm>

#include "common.cuh"

namespace sca2 {
namespace ln {

constexpr int NT = 256;
constexpr int WPC = NT / 32;

template <int V>
__device__ __forceinline__ void load_row(const float* p, int lane, float* x) {
#pragma unroll
  for (int k = 0; k < V / 4; ++k) {
    const float4 q = *reinterpret_cast<const float4*>(p + 4 * lane + 128 * k);
    x[4 * k] = q.x, x[4 * k + 1] = q.y, x[4 * k + 2] = q.z, x[4 * k + 3] = q.w;
  }
}
template <int V>
__device__ __forceinline__ void store_row(float* p, int lane, const float* x) {
#pragma unroll
  for (int k = 0; k < V / 4; ++k)
    *reinterpret_cast<float4*>(p + 4 * lane + 128 * k) = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
}

template <int V>
__global__ void __launch_bounds__(NT) ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                    const float* __restrict__ b, float* __restrict__ y,
                                                    float* __restrict__ mean, float* __restrict__ rstd, int64_t rows,
                                                    float eps) {
  constexpr int D = 32 * V;
  const int lane = threadIdx.x & 31;
  float wr[V], br[V];
  load_row<V>(w, lane, wr);
  load_row<V>(b, lane, br);
  const int64_t nw = (int64_t)gridDim.x * WPC;
  for (int64_t row = (int64_t)blockIdx.x * WPC + (threadIdx.x >> 5); row < rows; row += nw) {
    float v[V];
    load_row<V>(x + row * D, lane, v);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) s += v[k];
    const float mu = warp_sum(s) * (1.f / D);
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float c = v[k] - mu;
      q = fmaf(c, c, q);
    }
    const float rs = rsqrtf(warp_sum(q) * (1.f / D) + eps);
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = fmaf((v[k] - mu) * rs, wr[k], br[k]);
    store_row<V>(y + row * D, lane, v);
    if (lane == 0) mean[row] = mu, rstd[row] = rs;
  }
}

template <int V>
__global__ void __launch_bounds__(NT) ln_bwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                    const float* __restrict__ mean, const float* __restrict__ rstd,
                                                    const float* __restrict__ dy, float* __restrict__ dx,
                                                    float* __restrict__ part, int64_t rows) {
  constexpr int D = 32 * V;
  __shared__ float sacc[2 * D];
  const int lane = threadIdx.x & 31;
  for (int u = threadIdx.x; u < 2 * D; u += NT) sacc[u] = 0.f;
  float wr[V], dw[V], db[V];
  load_row<V>(w, lane, wr);
#pragma unroll
  for (int k = 0; k < V; ++k) dw[k] = 0.f, db[k] = 0.f;
  const int64_t nw = (int64_t)gridDim.x * WPC;
  for (int64_t row = (int64_t)blockIdx.x * WPC + (threadIdx.x >> 5); row < rows; row += nw) {
    float v[V], g[V];
    load_row<V>(x + row * D, lane, v);
    load_row<V>(dy + row * D, lane, g);
    const float mu = mean[row], rs = rstd[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float xh = (v[k] - mu) * rs;
      dw[k] = fmaf(g[k], xh, dw[k]);
      db[k] += g[k];
      v[k] = xh;
      g[k] *= wr[k];
      s1 += g[k];
      s2 = fmaf(g[k], xh, s2);
    }
    s1 = warp_sum(s1) * (1.f / D);
    s2 = warp_sum(s2) * (1.f / D);
#pragma unroll
    for (int k = 0; k < V; ++k) g[k] = rs * (g[k] - s1 - v[k] * s2);
    store_row<V>(dx + row * D, lane, g);
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int c = 4 * lane + 128 * (k / 4) + (k & 3);
    atomicAdd(&sacc[c], dw[k]);
    atomicAdd(&sacc[D + c], db[k]);
  }
  __syncthreads();
  for (int u = threadIdx.x; u < 2 * D; u += NT) part[(int64_t)blockIdx.x * 2 * D + u] = sacc[u];
}

__global__ void __launch_bounds__(NT) ln_bwd_reduce(const float* __restrict__ part, int nparts, int D,
                                                    float* __restrict__ dw, float* __restrict__ db) {
  const int c = blockIdx.x * NT + threadIdx.x;
  if (c >= 2 * D) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += part[(int64_t)p * 2 * D + c];
  if (c < D) {
    if (dw) dw[c] = s;
  } else if (db) {
    db[c - D] = s;
  }
}

template <int V>
cudaError_t fwd_v(const float* x, const float* w, const float* b, float* y, float* mean, float* rstd, int64_t rows,
                  float eps, int grid, cudaStream_t st) {
  ln_fwd_kernel<V><<<grid, NT, 0, st>>>(x, w, b, y, mean, rstd, rows, eps);
  return cudaGetLastError();
}
template <int V>
cudaError_t bwd_v(const float* x, const float* w, const float* mean, const float* rstd, const float* dy, float* dx,
                  float* part, int64_t rows, int grid, cudaStream_t st) {
  ln_bwd_kernel<V><<<grid, NT, 0, st>>>(x, w, mean, rstd, dy, dx, part, rows);
  return cudaGetLastError();
}

}  // namespace ln

// widths with a kernel: d = 128 ... 1024 in steps of 128
bool ln_supported(int d) { return d >= 128 && d <= 1024 && d % 128 == 0; }

// CTAs of the backward (the partial rows it writes: 2 d floats each)
int ln_bwd_parts(int64_t rows) {
  const int64_t want = (rows + ln::WPC * 8 - 1) / (ln::WPC * 8);  // about 8 rows per warp
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, 148 * 4));
}

cudaError_t ln_fwd(const float* x, const float* w, const float* b, float* y, float* mean, float* rstd, int64_t rows,
                   int d, float eps, cudaStream_t st) {
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((rows + ln::WPC - 1) / ln::WPC, 148 * 8));
  switch (d / 32) {
    case 4: return ln::fwd_v<4>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 8: return ln::fwd_v<8>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 12: return ln::fwd_v<12>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 16: return ln::fwd_v<16>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 20: return ln::fwd_v<20>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 24: return ln::fwd_v<24>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 28: return ln::fwd_v<28>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    case 32: return ln::fwd_v<32>(x, w, b, y, mean, rstd, rows, eps, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t ln_bwd(const float* x, const float* w, const float* mean, const float* rstd, const float* dy, float* dx,
                   float* dw, float* db, float* part, int64_t rows, int d, cudaStream_t st) {
  const int grid = ln_bwd_parts(rows);
  cudaError_t e;
  switch (d / 32) {
    case 4: e = ln::bwd_v<4>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 8: e = ln::bwd_v<8>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 12: e = ln::bwd_v<12>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 16: e = ln::bwd_v<16>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 20: e = ln::bwd_v<20>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 24: e = ln::bwd_v<24>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 28: e = ln::bwd_v<28>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    case 32: e = ln::bwd_v<32>(x, w, mean, rstd, dy, dx, part, rows, grid, st); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  ln::ln_bwd_reduce<<<(2 * d + ln::NT - 1) / ln::NT, ln::NT, 0, st>>>(part, grid, d, dw, db);
  return cudaGetLastError();
}

}  // namespace sca2
