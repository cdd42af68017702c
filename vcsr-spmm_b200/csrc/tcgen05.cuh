// tcgen05.cuh — device helpers shared by the tensor-core kernels (spmm_tc.cu,
// spmm_seg_tc.cu): bounded mbarrier waits, TMA and bulk copies into shared
// memory, shared-memory matrix descriptors, and tcgen05 TF32 MMA issue and
// commit.  Inline PTX for sm_100a; no multicast anywhere.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace vcsr {
namespace tc {

constexpr long long kPollLimit = 1ll << 22;
// The short limit of the one wait a test makes run out (TcView::inject).
constexpr long long kTestPollLimit = 1ll << 12;

// Where a bounded wait gave up (recorded in the plan's error word).
enum WaitSite : int {
  kWaitFull = 1, kWaitEmpty = 2, kWaitAccFull = 3, kWaitAccFree = 4, kWaitDrain = 5
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Adds to the transaction count of the current phase (no arrival).
__device__ __forceinline__ void mbar_add_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with the given parity; false when the poll
// limit ran out (the site is recorded) or another thread already reported a
// failure.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          volatile int *abort_flag, int site,
                                          long long limit = kPollLimit) {
  const uint32_t a = smem_u32(bar);
  for (long long i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 1023) == 1023 && *abort_flag) return false;
  }
  *abort_flag = site;
  return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Box {32, 16, 4} of the 3-D view: chunk-major, each chunk's 16 rows of 128
// bytes together, as four 2-D boxes placed 2 KB apart would be.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *tm, int x, int y,
                                            int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: start, leading and stride byte offsets
// (16-byte units), version 1, layout type (0 = no swizzle, 1 = 128-byte
// swizzle with 32-byte atoms).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// kind::tf32, D f32, A MN-major (bit 15), B K-major, N = 16, M = 128.
constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) |
                                ((16u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kInstrDesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

}  // namespace tc
}  // namespace vcsr
