// Shared pieces of the tensor-core (tcgen05) scan kernels: operand stores, accumulator
// fragment iteration, the fp32 blocked inversion and the per-chunk operand prologue.
#pragma once

#include <cuda.h>  // CUtensorMap (the type only; the library does not link the driver library)

#include "common.cuh"
#include "umma.cuh"

namespace sca2 {
namespace tc {

constexpr int C = 64;     // chunk (tokens)
constexpr int NT = 256;   // 8 warps
constexpr int LDF = C + 4;  // fp32 row stride of the inversion scratch (rows 16-byte aligned)

using bf16 = __nv_bfloat16;

// launch flags (host-computed, uniform)
// F_PREP: T of every chunk was written by the preparation kernel (where TSlots says)
// F_CS16: the chunk-state buffer is 16-byte aligned (bulk copies may write it)
enum : int { F_PH_VEC = 1, F_O_VEC = 2, F_K_VEC = 4, F_V_VEC = 8, F_PREP = 16, F_CS16 = 32 };

// The value tile of a full chunk (64 tokens x VW bf16 values of one (b, h)) by one TMA load: the
// 5-D tensor map (value % 8, token % 8, value / 8, row / 8, head), row = b T + t, with strides
// (2 B, st, 16 B, 8 st, sh) traverses the tile in exactly the order of the K-major, no-swizzle
// tcgen05 operand layout (8 x 8 core matrices of 128 B), so the copy lands in operand layout.
// The map covers the value tensor of this GPU only and the box never leaves it; no cluster
// multicast.  Completion on `bar` (expect_tx of the tile's bytes, armed by the issuing thread).
// Arm `bar` for `bytes` of TMA data: one arrival (the issuing thread's) plus the expected bytes.
__device__ __forceinline__ void tma_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(umma::smem_u32(bar)), "r"(bytes)
               : "memory");
}
// One tile of a 5-D tensor map at coordinates (0, 0, x2, x3, x4) into shared memory, completing
// on `bar`.  The innermost coordinate is 0, so the copy starts on a 16-byte boundary.
__device__ __forceinline__ void tma_load5(void* dst, const CUtensorMap* map, int x2, int x3, int x4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      ::"r"(umma::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(0), "r"(x2), "r"(x3), "r"(x4),
        "r"(umma::smem_u32(bar))
      : "memory");
}
template <int VW>
__device__ __forceinline__ void tma_value_tile(void* dst, const CUtensorMap* map, int row0, int h, uint64_t* bar) {
  tma_expect(bar, (uint32_t)(C * VW * 2));
  tma_load5(dst, map, 0, row0 >> 3, h, bar);
}

// Where the preparation kernel puts each chunk's inverse T (bf16 C x C in operand layout, 8 KB):
// chunk c of sequence bh = b H + h at base + bh * bh_stride + c * c_stride (bytes, all multiples
// of 16).  Training: slot 2c + 1 of the chunk-state buffer, which the backward reads again;
// inference: a compact work buffer of the caller's (c_stride = 8 KB).
struct TSlots {
  uint8_t* base;
  int64_t bh_stride, c_stride;
};

// ---- bf16 vector stores -------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);  // .x (low address) = a
  return *reinterpret_cast<uint32_t*>(&t);
}
// 8 consecutive elements at element offset idx (a multiple of 8, so 16-byte aligned)
__device__ __forceinline__ void st8(bf16* base, int idx, const float* x) {
  uint4 u;
  u.x = pack2(x[0], x[1]);
  u.y = pack2(x[2], x[3]);
  u.z = pack2(x[4], x[5]);
  u.w = pack2(x[6], x[7]);
  *reinterpret_cast<uint4*>(base + idx) = u;
}
// x = hi + lo (hi = bf16(x), lo = bf16(x - hi)): about 16 mantissa bits through bf16 MMAs
__device__ __forceinline__ void st8_split(bf16* hi, bf16* lo, int idx, const float* x) {
  float h[8], l[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    h[k] = __bfloat162float(__float2bfloat16_rn(x[k]));
    l[k] = x[k] - h[k];
  }
  st8(hi, idx, h);
  st8(lo, idx, l);
}
__device__ __forceinline__ void st1(bf16* base, int idx, float x) { base[idx] = __float2bfloat16_rn(x); }
// 2 consecutive elements at element offset idx (even, so 4-byte aligned)
__device__ __forceinline__ void st2(bf16* base, int idx, float a, float b) {
  *reinterpret_cast<uint32_t*>(base + idx) = pack2(a, b);
}
// the same as a hi + lo pair (st8_split's rounding)
__device__ __forceinline__ void st2_split(bf16* hi, bf16* lo, int idx, float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  *reinterpret_cast<__nv_bfloat162*>(hi + idx) = h;
  *reinterpret_cast<uint32_t*>(lo + idx) = pack2(a - hf.x, b - hf.y);
}

// ---- accumulator fragments ----------------------------------------------------------------
// Accumulator with M rows (64 or 128) and N columns: warp w reads TMEM sub-partition w%4 and the
// column half w/4 in blocks of 16 columns.  For M = 128 the thread's row is 32*(w%4) + lane; for
// M = 64 it is 16*(w%4) + lane and only lanes < 16 hold rows.  f(row, col0, q, v[16]) gets the
// 16 values of columns col0..col0+15; q (compile-time after unrolling) numbers the thread's
// blocks, so a thread's values can live in registers indexed [16*q + j].
template <int M>
__device__ __forceinline__ bool owns_rows() { return M == 128 || (threadIdx.x & 31) < 16; }
template <int M>
__device__ __forceinline__ int frag_row() {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  return M == 128 ? 32 * (warp & 3) + lane : 16 * (warp & 3) + lane;
}
template <int M, int N>
__device__ __forceinline__ int frag_col0(int q) {
  return (threadIdx.x >> 7) * (N / 2) + 16 * q;  // warp >> 2 == threadIdx.x >> 7
}
template <int M, int N, class F>
__device__ __forceinline__ void for_frag(uint32_t tbase, F f) {
  const int warp = threadIdx.x >> 5;
  const int sub = warp & 3;
  const bool own = owns_rows<M>();
  const int row = frag_row<M>();
  uint32_t r[N / 32][16];
#pragma unroll
  for (int q = 0; q < N / 32; ++q) umma::ld16_issue(umma::taddr(tbase, 32 * sub, frag_col0<M, N>(q)), r[q]);
  umma::ld_wait();
#pragma unroll
  for (int q = 0; q < N / 32; ++q) {
    float v[16];
    umma::take<16>(r[q], v);
    if (own) f(row, frag_col0<M, N>(q), q, v);
  }
}
// 64-row accumulator over all 32 lanes (16x256b loads): warp w reads rows 16 (w%4) .. +15 and the
// column half w/4 in groups of 8 columns; lane t holds rows r0 = 16 (w%4) + t/4 and r0 + 8 and
// columns c = 2 (t%4), c + 1 of each group.  f(g, r0, col, v[4]) gets group g's values
// (r0, col), (r0, col + 1), (r0 + 8, col), (r0 + 8, col + 1); every lane takes part.
template <int N, class F>
__device__ __forceinline__ void for_frag16(uint32_t tbase, F f) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = warp & 3;
  const int r0 = 16 * sub + (lane >> 2), cb = (warp >> 2) * (N / 2);
  uint32_t r[N / 16][4];
#pragma unroll
  for (int g = 0; g < N / 16; ++g) umma::ld4_rows16_issue(umma::taddr(tbase, 32 * sub, cb + 8 * g), r[g]);
  umma::ld_wait();
#pragma unroll
  for (int g = 0; g < N / 16; ++g) {
    float v[4];
    umma::take<4>(r[g], v);
    f(g, r0, cb + 8 * g + 2 * (lane & 3), v);
  }
}

// ---- asynchronous global -> shared copies (16 bytes; zero-filled when !valid) ----------------
__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(umma::smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// wait until at most N of this thread's most recent commit groups are still pending
template <int N>
__device__ __forceinline__ void cp_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- bulk shared -> global copies (one thread; 16-byte aligned addresses, size a multiple of 16)
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t nbytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(umma::smem_u32(src)), "r"(nbytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the sources of this thread's bulk copies have been read (the shared memory may be rewritten)
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's bulk copies are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- warp transpose-reduce --------------------------------------------------------------------
// Every lane holds N values (N = 8 or 16); returns, in lane l, the sum over all 32 lanes of value
// number red_index<N>(l).  Lanes whose index bits below log2(32 / N) are zero hold distinct
// results.  Costs N shuffles instead of 5 N.
template <int N>
__device__ __forceinline__ float warp_transpose_sum(float* v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int half = N / 2, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
    const bool up = lane & bit;
#pragma unroll
    for (int k = 0; k < half; ++k) {
      const float send = up ? v[k] : v[k + half];
      const float keep = up ? v[k + half] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  float x = v[0];
#pragma unroll
  for (int bit = 32 / N / 2; bit >= 1; bit >>= 1) x += __shfl_xor_sync(0xffffffffu, x, bit);
  return x;
}
template <int N>
__device__ __forceinline__ int red_index(int lane) {
  // value k = sum of the selection bits, taken from lane bits 4, 3, ... (MSB first)
  int k = 0;
#pragma unroll
  for (int half = N / 2, bit = 16; half >= 1; half >>= 1, bit >>= 1)
    if (lane & bit) k += half;
  return k;
}

__device__ __forceinline__ void publish_smem() {
  umma::fence_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
}

// ---- inversion of the unit lower-triangular (I + L), L strictly lower, by recursive doubling --
// The eight 8x8 diagonal blocks are solved by forward substitution (one column per thread, zeros
// written above the diagonal), then pairs of inverted blocks of size N = 8, 16, 32 merge into
// blocks of 2N with the block formula of a lower-triangular inverse
//
//     [[A, 0], [B, D]]^{-1} = [[A^{-1}, 0], [-D^{-1} B A^{-1}, D^{-1}]]
//
// in two passes over all threads (W = B A^{-1}, then -D^{-1} W), each thread a 1 x 4 tile with
// float4 shared loads and paired fp32 FMAs.  The sums skip the zero triangles: A^{-1}[k][c] = 0 for k < c and
// D^{-1}[r][k] = 0 for k > r (beyond r's group of four the entries lie in the zero-written upper
// triangle of an 8x8 diagonal block).  All fp32; TS receives the lower triangle; WS holds 1024
// floats.
// c + a * (b.x, b.y) with one paired fp32 FMA (fma.rn.f32x2, sm_100): each lane rounds like fmaf
__device__ __forceinline__ float2 fma2_bcast(float a, float2 b, float2 c) {
  uint64_t d;
  const uint64_t aa = ((uint64_t)__float_as_uint(a) << 32) | __float_as_uint(a);
  const uint64_t bb = ((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x);
  const uint64_t cc = ((uint64_t)__float_as_uint(c.y) << 32) | __float_as_uint(c.x);
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(aa), "l"(bb), "l"(cc));
  return make_float2(__uint_as_float((uint32_t)d), __uint_as_float((uint32_t)(d >> 32)));
}
// acc (4 lanes as two pairs) += a * b
__device__ __forceinline__ void fma4_bcast(float a, const float4& b, float2& lo, float2& hi) {
  lo = fma2_bcast(a, make_float2(b.x, b.y), lo);
  hi = fma2_bcast(a, make_float2(b.z, b.w), hi);
}

template <int N>
__device__ __forceinline__ void merge_inverse_blocks(const float* LS, float* TS, float* WS) {
  constexpr int Q = N / 4, ITEMS = (64 / (2 * N)) * N * Q;
  for (int e = threadIdx.x; e < ITEMS; e += blockDim.x) {  // W = L21 T11
    const int pr = e / (N * Q), rem = e - pr * (N * Q), r = rem / Q, cq = (rem - r * Q) * 4;
    const int base = pr * 2 * N;
    const float* lrow = LS + (base + N + r) * LDF + base;
    float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
    for (int k = cq; k < N; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(lrow + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        fma4_bcast(av[q], *reinterpret_cast<const float4*>(TS + (base + k + q) * LDF + base + cq), lo, hi);
    }
    *reinterpret_cast<float4*>(WS + (pr * N + r) * N + cq) = make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ITEMS; e += blockDim.x) {  // T21 = -T22 W
    const int pr = e / (N * Q), rem = e - pr * (N * Q), r = rem / Q, cq = (rem - r * Q) * 4;
    const int base = pr * 2 * N;
    const float* trow = TS + (base + N + r) * LDF + base + N;
    float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
    for (int k = 0; k <= r; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(trow + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        fma4_bcast(av[q], *reinterpret_cast<const float4*>(WS + (pr * N + k + q) * N + cq), lo, hi);
    }
    *reinterpret_cast<float4*>(TS + (base + N + r) * LDF + base + cq) = make_float4(-lo.x, -lo.y, -hi.x, -hi.y);
  }
  __syncthreads();
}
__device__ inline void invert_unit_lower(const float* LS, float* TS, float* WS) {
  const int tid = threadIdx.x;
  if (tid < 64) {
    const int o = 8 * (tid >> 3), col = tid & 7;
    float x[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float acc = (r == col) ? 1.f : 0.f;
#pragma unroll
      for (int k = 0; k < r; ++k) acc = fmaf(-LS[(o + r) * LDF + o + k], x[k], acc);
      x[r] = (r < col) ? 0.f : acc;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) TS[(o + r) * LDF + o + col] = x[r];
  }
  __syncthreads();
  merge_inverse_blocks<8>(LS, TS, WS);
  merge_inverse_blocks<16>(LS, TS, WS);
  merge_inverse_blocks<32>(LS, TS, WS);
}

// TB (bf16, K-major rows i, K = j) <- lower triangle of TS; transposed = write T^T instead
template <bool TRANSPOSED>
__device__ __forceinline__ void store_T(const float* TS, bf16* TB) {
  for (int u = threadIdx.x; u < C * C / 8; u += NT) {
    const int i = (u & 7) + 8 * (u >> 6), j0 = ((u >> 3) & 7) * 8;  // conflict-free 16-byte stores
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + k;
      x[k] = TRANSPOSED ? (i <= j ? TS[j * LDF + i] : 0.f) : (j <= i ? TS[i * LDF + j] : 0.f);
    }
    st8(TB, umma::kmaj(i, j0, C), x);
  }
}

// ---- code units ---------------------------------------------------------------------------
// Code unit u = (token i, 8 consecutive modes / dims from m0), MB units per token: the 8 lanes of
// a quarter-warp take 8 consecutive tokens of the same 8 modes, so their 16-byte stores into a
// K-major operand (token rows 16 bytes apart within a core-matrix group) fill one 128-byte line
// instead of hitting one bank group 4 or 8 times.
template <int MB>
__device__ __forceinline__ void code_unit(int u, int& i, int& m0) {
  i = (u & 7) + 8 * (u / (8 * MB));
  m0 = ((u >> 3) % MB) * 8;
}

// ---- per-chunk gates ----------------------------------------------------------------------
// beta, cumulative log-decay Gc, a = exp(Gc), w = exp(Gc_last - Gc) for the chunk's 64 tokens
// (one warp); rows i >= Cl get beta = 0, g = 0, w = 0.
struct Gates {
  float *beta, *Gc, *a, *w;
};

// ---- the decay mask Dg(i, j) = exp(Gc_i - Gc_j), j <= i, of a chunk --------------------------
// Gc is non-increasing along the chunk.  Per 16-column block (last column jl) the column
// factors fdec[j] = exp(Gc_jl - Gc_j) <= 1 are formed once per chunk (threads 0..63); a block
// left of row i (jl < i) is then exp(Gc_i - Gc_jl) * fdec[j], both factors <= 1, so one
// exponential per row and block.  The row's own block is factored the same way (the row factor
// >= 1) unless that block decays by more than e^80, where it takes one exponential per element;
// blocks right of the row are zero.  Products are clamped at 1: min(e^x, 1) = e^min(x, 0), the
// mask's definition.
__device__ __forceinline__ void decay_factors(const float* Gc, float* fdec) {
  const int t = threadIdx.x;
  if (t < C) fdec[t] = __expf(Gc[t | 15] - Gc[t]);
}
// the same from the one warp that has just written Gc (two columns per lane)
__device__ __forceinline__ void decay_factors_warp(const float* Gc, float* fdec) {
  __syncwarp();
  const int l = threadIdx.x & 31;
  fdec[l] = __expf(Gc[l | 15] - Gc[l]);
  fdec[l + 32] = __expf(Gc[(l | 15) + 32] - Gc[l + 32]);
}
__device__ __forceinline__ void decay_block(const float* Gc, const float* fdec, int i, int j0, float* d) {
  const float gl = Gc[j0 + 15];
  if (j0 > i) {
#pragma unroll
    for (int j = 0; j < 16; ++j) d[j] = 0.f;
  } else if (j0 + 15 < i || Gc[j0] - gl <= 80.f) {
    const float r = __expf(Gc[i] - gl);
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 f = *reinterpret_cast<const float4*>(fdec + j0 + j);
      d[j] = fminf(r * f.x, 1.f), d[j + 1] = fminf(r * f.y, 1.f);
      d[j + 2] = fminf(r * f.z, 1.f), d[j + 3] = fminf(r * f.w, 1.f);
    }
  } else {
    const float gi = Gc[i];
#pragma unroll
    for (int j = 0; j < 16; ++j) d[j] = __expf(fminf(gi - Gc[j0 + j], 0.f));
  }
}
// ---- per-thread register prefetch of a chunk's code inputs and gates ----------------------------
// Codes: phase flavour, thread t holds (token t/4, modes 8(t%4)..+7) of phi and psi; key flavour,
// units t and t+256 of (token u/8, dims 8(u%8)..+7) of k and q.  vec: 16-byte loads are aligned.
template <int FL, int KD>
struct CodeRegs {
  // phase: one unit (phi, psi x 8 modes); key: NU units (k, q x 8 dims).  Phases from the
  // projections (PhaseProj::on): load_code_regs leaves the loaded K(h), K(z) bits in w, q (bf16:
  // 4 words each; fp32: 8 values) and the position offset in pos; finish_code_regs forms the
  // phases where the codes are built, so no thread waits for those loads in between.
  static constexpr int NU = FL == SCA2_FLAVOR_PHASE ? 1 : C * KD / 8 / NT;
  float w[NU][8], q[NU][8];
  float pos;
};

// 8 projection values of one token row (bf16 or fp32, 16-byte loads when vec)
__device__ __forceinline__ void load8(const void* base, int64_t off, int dtype, bool vec, float* x) {
  if (dtype == SCA2_BF16) {
    const bf16* q = reinterpret_cast<const bf16*>(base) + off;
    if (vec) {
      const uint4 u = *reinterpret_cast<const uint4*>(q);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) { x[2 * k] = __low2float(h2[k]); x[2 * k + 1] = __high2float(h2[k]); }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = __bfloat162float(q[k]);
    }
  } else {
    const float* q = reinterpret_cast<const float*>(base) + off;
    if (vec) {
      const float4 a = reinterpret_cast<const float4*>(q)[0], c = reinterpret_cast<const float4*>(q)[1];
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = q[k];
    }
  }
}

// 8 projection values of one token row as loaded: bf16 packed two per word in x[0..3], fp32 in
// x[0..7] (16-byte loads when vec; the registers are not read here)
__device__ __forceinline__ void raw8(const void* base, int64_t off, int dtype, bool vec, float* x) {
  if (dtype == SCA2_BF16) {
    const bf16* q = reinterpret_cast<const bf16*>(base) + off;
    uint4 u;
    if (vec) {
      u = *reinterpret_cast<const uint4*>(q);
    } else {
      const uint16_t* q16 = reinterpret_cast<const uint16_t*>(q);
      u.x = q16[0] | ((uint32_t)q16[1] << 16);
      u.y = q16[2] | ((uint32_t)q16[3] << 16);
      u.z = q16[4] | ((uint32_t)q16[5] << 16);
      u.w = q16[6] | ((uint32_t)q16[7] << 16);
    }
    x[0] = __uint_as_float(u.x), x[1] = __uint_as_float(u.y), x[2] = __uint_as_float(u.z), x[3] = __uint_as_float(u.w);
  } else {
    const float* q = reinterpret_cast<const float*>(base) + off;
    if (vec) {
      const float4 a = reinterpret_cast<const float4*>(q)[0], c = reinterpret_cast<const float4*>(q)[1];
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = q[k];
    }
  }
}

template <int FL, int KD>
__device__ __forceinline__ void load_code_regs(const sca2_scan_args& p, CodeRegs<FL, KD>& r, bool vec, int b, int h,
                                               int t0, int Cl, const PhaseProj& pp = PhaseProj{}) {
  const int tid = threadIdx.x;
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    int i, m0;
    code_unit<KD / 16>(tid, i, m0);
    if (pp.on) {  // projections K(h), K(z) as loaded (raw bits); the phases in finish_code_regs
#pragma unroll
      for (int k = 0; k < 8; ++k) { r.w[0][k] = 0.f; r.q[0][k] = 0.f; }
      r.pos = 0.f;
      if (i < Cl) {
        r.pos = pp.pos ? *pp.pos : 0.f;
        raw8(p.phw.ptr, tok_off(p.phw, b, t0 + i, h) + m0, pp.dtype, vec, r.w[0]);
        raw8(p.phq.ptr, tok_off(p.phq, b, t0 + i, h) + m0, pp.dtype, vec, r.q[0]);
      }
      return;
    }
    const float* pw = reinterpret_cast<const float*>(p.phw.ptr);
    const float* pq = reinterpret_cast<const float*>(p.phq.ptr);
    if (i < Cl) {
      const int64_t ow = tok_off(p.phw, b, t0 + i, h) + m0, oq = tok_off(p.phq, b, t0 + i, h) + m0;
      if (vec) {
        const float4 a0 = reinterpret_cast<const float4*>(pw + ow)[0], a1 = reinterpret_cast<const float4*>(pw + ow)[1];
        const float4 c0 = reinterpret_cast<const float4*>(pq + oq)[0], c1 = reinterpret_cast<const float4*>(pq + oq)[1];
        r.w[0][0] = a0.x; r.w[0][1] = a0.y; r.w[0][2] = a0.z; r.w[0][3] = a0.w;
        r.w[0][4] = a1.x; r.w[0][5] = a1.y; r.w[0][6] = a1.z; r.w[0][7] = a1.w;
        r.q[0][0] = c0.x; r.q[0][1] = c0.y; r.q[0][2] = c0.z; r.q[0][3] = c0.w;
        r.q[0][4] = c1.x; r.q[0][5] = c1.y; r.q[0][6] = c1.z; r.q[0][7] = c1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) { r.w[0][k] = pw[ow + k]; r.q[0][k] = pq[oq + k]; }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) { r.w[0][k] = 0.f; r.q[0][k] = 0.f; }
    }
  } else {
    constexpr int MB = KD / 8;
#pragma unroll
    for (int u = 0; u < CodeRegs<FL, KD>::NU; ++u) {
      int i, m0;
      code_unit<MB>(tid + u * NT, i, m0);
      if (i < Cl) {
        const int64_t ok = tok_off(p.phw, b, t0 + i, h) + m0, oq = tok_off(p.phq, b, t0 + i, h) + m0;
        if (vec) {
          const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.phw.ptr) + ok);
          const uint4 c = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.phq.ptr) + oq);
          const __nv_bfloat162* ap = reinterpret_cast<const __nv_bfloat162*>(&a);
          const __nv_bfloat162* cp = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            r.w[u][2 * k] = __low2float(ap[k]); r.w[u][2 * k + 1] = __high2float(ap[k]);
            r.q[u][2 * k] = __low2float(cp[k]); r.q[u][2 * k + 1] = __high2float(cp[k]);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            r.w[u][k] = ld_io(p.phw.ptr, ok + k, p.io_dtype);
            r.q[u][k] = ld_io(p.phq.ptr, oq + k, p.io_dtype);
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) { r.w[u][k] = 0.f; r.q[u][k] = 0.f; }
      }
    }
  }
}
// The phases of the projections (PhaseProj::on) in place of the loaded bits, with the rounding
// of each step as the reference forms them: phi = K(h) theta + (pos + t) omega and psi = K(z)
// theta + (pos + t) omega (rows i >= Cl stay zero).  A no-op for every other input.  Called where
// the codes are built, on the (t0, Cl) of the matching load_code_regs; s_th, s_om: the head's
// theta and omega staged in shared memory (else read from global memory).
template <int FL, int KD>
__device__ __forceinline__ void finish_code_regs(CodeRegs<FL, KD>& r, const PhaseProj& pp, int h, int t0, int Cl,
                                                 const float* s_th = nullptr, const float* s_om = nullptr) {
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    if (!pp.on) return;
    int i, m0;
    code_unit<KD / 16>(threadIdx.x, i, m0);
    if (i >= Cl) return;
    constexpr int Mh = KD / 2;
    float kh[8], kz[8];
    if (pp.dtype == SCA2_BF16) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t a = __float_as_uint(r.w[0][k]), c = __float_as_uint(r.q[0][k]);
        const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162*>(&c);
        kh[2 * k] = __low2float(a2), kh[2 * k + 1] = __high2float(a2);
        kz[2 * k] = __low2float(c2), kz[2 * k + 1] = __high2float(c2);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) kh[k] = r.w[0][k], kz[k] = r.q[0][k];
    }
    const float pt = __fadd_rn(r.pos, (float)(t0 + i));
    const float* th = (s_th ? s_th : pp.theta + h * Mh) + m0;
    const float* om = (s_om ? s_om : pp.omega + h * Mh) + m0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float po = __fmul_rn(pt, om[k]);
      r.w[0][k] = __fadd_rn(__fmul_rn(kh[k], th[k]), po);
      r.q[0][k] = __fadd_rn(__fmul_rn(kz[k], th[k]), po);
    }
  }
}

struct GateRegs {
  float bt[2], gg[2];
};
__device__ __forceinline__ void load_gate_regs(const sca2_scan_args& p, GateRegs& r, int b, int h, int t0, int Cl) {
  const int l = threadIdx.x & 31;
  const float* bp = reinterpret_cast<const float*>(p.beta.ptr);
  const float* gp = reinterpret_cast<const float*>(p.g.ptr);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = l + 32 * u;
    r.bt[u] = (bp && i < Cl) ? bp[tok_off(p.beta, b, t0 + i, h)] : 0.f;
    r.gg[u] = (gp && i < Cl) ? gp[tok_off(p.g, b, t0 + i, h)] : 0.f;
  }
}
// warp 0: beta, Gc (inclusive cumsum of g), a = e^Gc, w = e^{G_last - Gc} from the registers
__device__ __forceinline__ void gates_from_regs(const GateRegs& r, const Gates& s, int Cl) {
  const int l = threadIdx.x & 31;
  const float s0 = warp_incl_scan(r.gg[0]);
  const float tot0 = __shfl_sync(0xffffffffu, s0, 31);
  const float s1 = warp_incl_scan(r.gg[1]) + tot0;
  const float sel = (Cl - 1) < 32 ? s0 : s1;
  const float Glast = __shfl_sync(0xffffffffu, sel, (Cl - 1) & 31);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = l + 32 * u;
    const float G = u ? s1 : s0;
    s.beta[i] = r.bt[u];
    s.Gc[i] = G;
    s.a[i] = expf(G);
    s.w[i] = i < Cl ? exp_le0(Glast - G) : 0.f;
  }
}

// ---- code operands of one chunk (forward) -----------------------------------------------------
// From the prefetched code registers, for tokens i < 64 (zeros for i >= Cl):
//   KR[i][m] = k e^{-lam i}          KW|KWL[i][m] = k e^{+lam i} (hi|lo)
//   QR|QRL[(r,i)][m] = Q_r e^{-lam i} (hi|lo)
//   ZA[i][m] = beta a k e^{-lam i} / kappa     KWW[i][m] = w k e^{+lam i}
// all written with 16-byte stores; ZA and KWW are read through MN-major descriptors.
template <int FL, int KD, int R>
struct CodeOps {
  bf16 *KR, *KW, *KWL, *QR, *QRL, *ZA, *KWW;
};
// Codes of one chunk from its phases (keys) and gates: KR (when kr), KW + KWL, QR + QRL, ZA.
// KWW = w KW is formed separately (kww_from_kw), right before the chunk's first MMA batch.
template <int FL, int KD, int R>
__device__ void build_codes(const CodeRegs<FL, KD>& cr, const CodeOps<FL, KD, R>& op, const Gates& g, const float* s_lam,
                            const float* s_wr, const float* s_wi, float q_scale, int Cl, float ik, bool kr) {
  const int tid = threadIdx.x;
  if constexpr (FL == SCA2_FLAVOR_PHASE) {
    constexpr int Mh = KD / 2;
    static_assert(C * Mh / 8 == NT, "one (token, 8 modes) unit per thread");
    int i, m0;
    code_unit<KD / 16>(tid, i, m0);
    const bool live = i < Cl;
    const float fi = (float)i, zb = g.beta[i] * g.a[i] * ik;
    float kc[8], ks[8], wc[8], ws[8], q0a[8], q0b[8], q1a[8], q1b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int m = m0 + k;
      float c = 0.f, s = 0.f, cq = 0.f, sq = 0.f;
      if (live) {
        sincos_big(cr.w[0][k], &s, &c);
        sincos_big(cr.q[0][k], &sq, &cq);
      }
      const float l = s_lam[m];
      const float ell = __expf(-l * fi), elli = __expf(l * fi);
      const float wr = s_wr[m], wi = s_wi[m];
      const float c1 = wr * cq + wi * sq, c2 = wr * sq - wi * cq;
      kc[k] = c * ell; ks[k] = s * ell; wc[k] = c * elli; ws[k] = s * elli;
      q0a[k] = c1 * ell; q0b[k] = c2 * ell; q1a[k] = -c2 * ell; q1b[k] = c1 * ell;
    }
    if (kr) {
      st8(op.KR, umma::kmaj(i, m0, KD), kc);
      st8(op.KR, umma::kmaj(i, Mh + m0, KD), ks);
    }
    st8_split(op.KW, op.KWL, umma::kmaj(i, m0, KD), wc);
    st8_split(op.KW, op.KWL, umma::kmaj(i, Mh + m0, KD), ws);
    st8_split(op.QR, op.QRL, umma::kmaj(i, m0, KD), q0a);
    st8_split(op.QR, op.QRL, umma::kmaj(i, Mh + m0, KD), q0b);
    st8_split(op.QR, op.QRL, umma::kmaj(C + i, m0, KD), q1a);
    st8_split(op.QR, op.QRL, umma::kmaj(C + i, Mh + m0, KD), q1b);
    float t[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = zb * kc[k];
    st8(op.ZA, umma::kmaj(i, m0, KD), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = zb * ks[k];
    st8(op.ZA, umma::kmaj(i, Mh + m0, KD), t);
  } else {
    constexpr int MB = KD / 8, NU = CodeRegs<FL, KD>::NU;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      int i, m0;
      code_unit<MB>(tid + u * NT, i, m0);
      const float fi = (float)i, zb = g.beta[i] * g.a[i] * ik;
      float kc[8], wc[8], qc[8], t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float l = s_lam[m0 + k];
        const float ell = __expf(-l * fi), elli = __expf(l * fi);
        kc[k] = cr.w[u][k] * ell; wc[k] = cr.w[u][k] * elli; qc[k] = q_scale * cr.q[u][k] * ell;
      }
      if (kr) st8(op.KR, umma::kmaj(i, m0, KD), kc);
      st8_split(op.KW, op.KWL, umma::kmaj(i, m0, KD), wc);
      st8_split(op.QR, op.QRL, umma::kmaj(i, m0, KD), qc);
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = zb * kc[k];
      st8(op.ZA, umma::kmaj(i, m0, KD), t);
    }
  }
}

// KWW = w .* (KW + KWL) for the units this thread wrote in build_codes (same unit map, so no
// barrier is needed between the two)
__device__ __forceinline__ void ld8_bf16(const bf16* base, int idx, float* x) {
  const uint4 raw = *reinterpret_cast<const uint4*>(base + idx);
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    x[2 * k] = __low2float(h2[k]);
    x[2 * k + 1] = __high2float(h2[k]);
  }
}
template <int FL, int KD, int R>
__device__ void kww_from_kw(const CodeOps<FL, KD, R>& op, const Gates& g) {
  constexpr int MB = FL == SCA2_FLAVOR_PHASE ? KD / 16 : KD / 8;
  constexpr int NU = FL == SCA2_FLAVOR_PHASE ? 1 : CodeRegs<FL, KD>::NU;
  constexpr int NH = FL == SCA2_FLAVOR_PHASE ? 2 : 1;  // phase: cos and sin halves
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    int i, m0;
    code_unit<MB>(threadIdx.x + u * NT, i, m0);
    const float wv = g.w[i];
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      const int idx = umma::kmaj(i, hh * (KD / 2) + m0, KD);
      float a[8], l[8];
      ld8_bf16(op.KW, idx, a);
      ld8_bf16(op.KWL, idx, l);
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] = wv * (a[k] + l[k]);
      st8(op.KWW, idx, a);
    }
  }
}

// ---- value operand VA[j][v] (K-major over v: read MN-major as V'^T) ------------------------------
// 16-byte cp.async copies when vec (rows 16-byte aligned), else element loads; zero rows j >= Cl.
template <int VB>
__device__ __forceinline__ void pf_values(const sca2_scan_args& p, bf16* VA, bool vec, int b, int h, int t0, int Cl,
                                          int vb0) {
  for (int u = threadIdx.x; u < C * (VB / 8); u += NT) {
    // 8 consecutive rows of the same 8 columns per quarter-warp: conflict-free 16-byte writes
    const int j = (u & 7) + 8 * (u / VB), v0 = ((u >> 3) % (VB / 8)) * 8;
    const bool live = j < Cl && vb0 + v0 < p.V;
    const int64_t off = live ? tok_off(p.v, b, t0 + j, h) + vb0 + v0 : 0;
    bf16* dst = VA + umma::kmaj(j, v0, VB);
    if (vec) {
      cp16(dst, reinterpret_cast<const bf16*>(p.v.ptr) + off, live);
    } else {
      float x[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = (live && vb0 + v0 + k < p.V) ? ld_io(p.v.ptr, off + k, p.io_dtype) : 0.f;
      st8(dst, 0, x);
    }
  }
}
// V' = beta v for the GDN write: scale the rows of VA in place
template <int VB>
__device__ __forceinline__ void scale_values(bf16* VA, const float* s_beta) {
  for (int u = threadIdx.x; u < C * (VB / 8); u += NT) {
    const int j = (u & 7) + 8 * (u / VB), v0 = ((u >> 3) % (VB / 8)) * 8;
    bf16* q = VA + umma::kmaj(j, v0, VB);
    const uint4 raw = *reinterpret_cast<const uint4*>(q);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float x[8];
    const float bj = s_beta[j];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = bj * __low2float(h2[k]);
      x[2 * k + 1] = bj * __high2float(h2[k]);
    }
    st8(q, 0, x);
  }
}

}  // namespace tc
}  // namespace sca2
