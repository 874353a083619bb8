// tcgen05 (5th-generation tensor core) building blocks for sm_100a, written as inline PTX.
//
// Operand layout: every shared-memory MMA operand is bf16, K-major, no swizzle, in 8x8
// "core matrices" (8 rows x 16 bytes, 128 B each).  For an R x Kt operand, element (r, k)
// lives at element offset  ((r/8) * (Kt/8) + k/8) * 64 + (r%8) * 8 + k%8,  i.e. the core
// matrices of one 8-row group are contiguous along K (LBO = 128 B between K-adjacent core
// matrices) and 8-row groups are SBO = Kt/8 * 128 B apart.  One MMA instruction consumes
// K = 16 (two core matrices along K); the next K step starts 256 B further.
//
// Accumulators live in tensor memory (TMEM): for M = 128 row i is TMEM lane i; for M = 64
// row m is lane (m % 16) + 32 * (m / 16); column j is TMEM column base + j (fp32).  A warp
// may only read the 32-lane sub-partition (warp % 4).
//
// Every wait on an mbarrier is bounded: after kMaxSpin polls the caller gets `false`,
// records an error and leaves; nothing here can hang the GPU.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace sca2 {
namespace umma {

constexpr long long kMaxSpin = 1LL << 22;  // polls of mbarrier.try_wait (each may suspend briefly)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// element offset of (r, k) in a K-major no-swizzle operand with Kt columns
__device__ __forceinline__ int kmaj(int r, int k, int Kt) {
  return (((r >> 3) * (Kt >> 3) + (k >> 3)) << 6) + ((r & 7) << 3) + (k & 7);
}

// shared-memory matrix descriptor (sm100 format, SWIZZLE_NONE)
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm100
  return d;                // base offset 0, legacy LBO mode, layout type 0 = SWIZZLE_NONE
}

// descriptor of a K-major operand at smem address `base` with Kt columns, positioned at K step kk
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int Kt, int kk) {
  return sdesc(base + (uint32_t)kk * 256u, 128u, (uint32_t)(Kt >> 3) * 128u);
}

// descriptor of an MN-major operand at K step kk.  The buffer is the K-major layout of the
// operand's transpose: element (mn, k) of the operand sits at kmaj(k, mn, MNt), i.e. 16-byte
// runs along MN, 8-row groups along K are MNt * 16 bytes apart (LBO) and adjacent MN core
// matrices 128 bytes apart (SBO).  So one K-major buffer of X serves as X (K-major) in one
// product and as X^T (MN-major) in another.
__device__ __forceinline__ uint64_t mdesc(uint32_t base, int MNt, int kk) {
  return sdesc(base + (uint32_t)kk * 32u * (uint32_t)MNt, (uint32_t)MNt * 16u, 128u);
}

// instruction descriptor: kind::f16 with bf16 A/B, fp32 D, both operands K-major
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// same with the MN-major (transposed) flags for A (bit 15) and B (bit 16)
__host__ __device__ constexpr uint32_t idesc_bf16_t(int M, int N, bool a_mn, bool b_mn) {
  return idesc_bf16(M, N) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16);
}

// D[tmem] (+)= A * B^T for one K = 16 step; issued by ONE thread
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The descriptors of one operand differ between K steps only in the start-address field (low
// 14 bits, address >> 4; shared-memory addresses stay below 256 KB so the field never carries
// into LBO).  The issue loops therefore build the two 32-bit halves once per product and add
// the K-step stride to the low half: one integer add per operand and step instead of the
// 64-bit shifts and masks of sdesc, which kept the single issuing thread busy for tens of
// cycles per instruction.
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t desc_hi(uint32_t sbo_bytes) {
  return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14);  // bit 46 of the descriptor: sm100 version
}
__device__ __forceinline__ uint64_t desc_pack(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }

// D = A(M x Kt) * B(N x Kt)^T over all K steps; A, B K-major in smem; issued by ONE thread
__device__ __forceinline__ void gemm(uint32_t tmem_d, const void* A, const void* B, int M, int N, int Kt,
                                     bool accumulate) {
  const uint32_t id = idesc_bf16(M, N), hi = desc_hi((uint32_t)(Kt >> 3) * 128u);
  const uint32_t a = desc_lo(smem_u32(A), 128u), b = desc_lo(smem_u32(B), 128u);
#pragma unroll
  for (int kk = 0; kk < Kt / 16; ++kk)
    mma(tmem_d, desc_pack(a + 16u * kk, hi), desc_pack(b + 16u * kk, hi), id, (accumulate || kk > 0) ? 1u : 0u);
}

// D (+)= A * B^T where each operand is K-major (rows of its own K elements) or MN-major (the
// K-major buffer of its transpose, see mdesc).  M x Kt and N x Kt; issued by ONE thread.
__device__ __forceinline__ void gemm_t(uint32_t tmem_d, const void* A, bool a_mn, const void* B, bool b_mn, int M,
                                       int N, int Kt, bool accumulate) {
  const uint32_t id = idesc_bf16_t(M, N, a_mn, b_mn);
  const uint32_t ahi = a_mn ? desc_hi(128u) : desc_hi((uint32_t)(Kt >> 3) * 128u);
  const uint32_t bhi = b_mn ? desc_hi(128u) : desc_hi((uint32_t)(Kt >> 3) * 128u);
  const uint32_t a = a_mn ? desc_lo(smem_u32(A), (uint32_t)M * 16u) : desc_lo(smem_u32(A), 128u);
  const uint32_t b = b_mn ? desc_lo(smem_u32(B), (uint32_t)N * 16u) : desc_lo(smem_u32(B), 128u);
  const uint32_t as = a_mn ? 2u * (uint32_t)M : 16u, bs = b_mn ? 2u * (uint32_t)N : 16u;  // K-step strides >> 4
#pragma unroll
  for (int kk = 0; kk < Kt / 16; ++kk)
    mma(tmem_d, desc_pack(a + as * kk, ahi), desc_pack(b + bs * kk, bhi), id, (accumulate || kk > 0) ? 1u : 0u);
}

// arrive on `mbar` once every MMA issued so far by this thread has completed
__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(mbar)) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// bounded wait for the phase `parity` of `mbar` to complete; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity) {
  const uint32_t a = smem_u32(mbar);
  for (long long it = 0; it < kMaxSpin; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// plain arrive (one count) on `mbar`: an issuing thread with no MMAs in a batch signals with it
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" :: "r"(smem_u32(mbar)) : "memory");
}

// generic-proxy smem writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// TMEM allocation (one full warp); writes the base address to *dst
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(dst)), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 consecutive fp32 columns -> 16 registers per thread (thread t = lane base + t)
__device__ __forceinline__ void ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Split forms: issue several loads, wait once, then take the registers.  take() passes each
// register through an empty volatile asm that comes after the wait, so no use of a loaded
// value can be scheduled before the wait completes.
__device__ __forceinline__ void ld16_issue(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void ld8_issue(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
// 16 lanes x 8 columns (the 16 rows of an M = 64 accumulator in one sub-partition) spread over
// all 32 threads: thread t gets rows t/4 and t/4 + 8, columns 2(t%4) and 2(t%4) + 1, as
// r = {(t/4, 2(t%4)), (t/4, 2(t%4)+1), (t/4+8, 2(t%4)), (t/4+8, 2(t%4)+1)} (measured layout)
__device__ __forceinline__ void ld4_rows16_issue(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void take(uint32_t* r, float* v) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    asm volatile("" : "+r"(r[i]));
    v[i] = __uint_as_float(r[i]);
  }
}

// 32 lanes x 8 consecutive fp32 columns -> 8 registers per thread
__device__ __forceinline__ void ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// TMEM address of (lane, column)
__device__ __forceinline__ uint32_t taddr(uint32_t base, int lane, int col) {
  return base + ((uint32_t)lane << 16) + (uint32_t)col;
}

// lane holding row m of an M-row accumulator
__device__ __forceinline__ int row_lane(int m, int M) { return M == 128 ? m : (m & 15) + ((m >> 4) << 5); }

}  // namespace umma
}  // namespace sca2
