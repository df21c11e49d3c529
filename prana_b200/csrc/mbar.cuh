// mbar.cuh -- mbarrier + bulk-copy (cp.async.bulk) primitives for sm_100a.
//
// A bulk copy moves a contiguous global range into the issuing CTA's own
// shared memory and completes on an mbarrier transaction count; one
// instruction replaces thousands of 16-byte loads.  Every copy reads this
// GPU's own memory.  Every wait is bounded: a wait that runs out reports
// failure and the caller raises the device error flag instead of spinning.
#pragma once
#include <stdint.h>

namespace prana {

enum : unsigned { ERR_NONE = 0, ERR_TIMEOUT = 1 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// make an initialized barrier visible to the bulk-copy (async) proxy
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// non-blocking: has the phase of the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// ~2^22 polls, each of which may itself suspend for a hardware-chosen time:
// far beyond any healthy copy.  Returns false on timeout.
constexpr uint32_t kMbarPolls = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t polls = kMbarPolls) {
  for (uint32_t i = 0; i < polls; i++)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}
// global -> this CTA's shared memory; src, dst 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

}  // namespace prana
