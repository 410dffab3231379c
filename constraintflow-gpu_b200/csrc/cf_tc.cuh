// sm_100a primitives: mbarriers with bounded waits, bulk (TMA-engine) copies, tcgen05
// tensor-memory allocation / MMA / loads, and the tf32 split.  Inline PTX only.
#pragma once
#include <stdint.h>

#include "cf_common.cuh"

namespace cf {
namespace tc {

// Every wait on an mbarrier gives up after this many polls (a kernel may pass a smaller limit) (each try_wait itself
// suspends for a while), records CF_ERR_TIMEOUT in the device error word and returns
// false so the caller can unwind instead of hanging the GPU.
constexpr uint32_t kMaxPolls = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  On timeout sets *err (if not already set) and returns false.  The error
// word (global memory: a volatile load is an L2 round trip of several hundred cycles, during
// which a barrier that completes is not seen) is read only every kErrPollInterval polls, so
// that the common short waits run at mbarrier latency.
constexpr uint32_t kErrPollInterval = 4096;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int site,
                                          uint32_t max_polls = kMaxPolls) {
  for (uint32_t i = 0; i < max_polls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & (kErrPollInterval - 1)) == kErrPollInterval - 1 && *(volatile int*)err != 0)
      return false;  // another role already gave up
  }
  atomicCAS(err, 0, site);
  return false;
}

// Bounded wait for work already in flight (bulk copies, MMAs) before the CTA releases what
// that work writes: unlike mbar_wait it does not give up when another role has recorded
// an error, only after kMaxPolls polls (then it records `site` if nothing was recorded).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err, int site,
                                                uint32_t max_polls = kMaxPolls) {
  for (uint32_t i = 0; i < max_polls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicCAS(err, 0, site);
  return false;
}

// Bulk copy global -> shared (TMA engine, contiguous bytes), completion on an mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tensor memory
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, fp32 accumulate, cta_group::1.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3)
      : "memory");
}

// Arrive on an mbarrier when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp gets lane (base+t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// ---- shared-memory matrix descriptor (K-major, 128-byte swizzle, 8-row x 128 B atoms)
// start address >> 4 in bits [0,14), leading offset 16 B (encoded 1) in [16,30),
// stride between 8-row groups 1024 B (encoded 64) in [32,46), descriptor version 1 in
// [46,48), swizzle mode 2 (128 B) in [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp32 accumulator, tf32 A and B, both K-major, M=128, N.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((N >> 3) << 17) | ((128u >> 4) << 24);
}

// Round-to-nearest tf32 (10-bit mantissa) kept in a 32-bit container.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// 3xTF32 operand split: hi = x rounded to the 10-bit tf32 mantissa (round half away
// from zero on the magnitude bits), lo = the tf32 rounding of the exact remainder x - hi.
__device__ __forceinline__ float tf32_round_bits(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = tf32_round_bits(x);
  lo = tf32_round_bits(x - hi);
}

// Byte offset of element (row, k) (k in [0,32), fp32) inside a K-major SW128 image whose
// rows are 128 B: 16-byte chunk (k/4) is stored at chunk position (k/4) ^ (row % 8).
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
  return row * 128u + ((((k >> 2) ^ (row & 7u)) & 7u) << 4) + (k & 3u) * 4u;
}

}  // namespace tc
}  // namespace cf
