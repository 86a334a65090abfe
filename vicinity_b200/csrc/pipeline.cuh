// Shared-memory mbarrier and named-barrier helpers (inline PTX, sm_90+).
//
// Every wait in this file is bounded: after kWaitCycles of SM clock without
// progress the caller gets `false` and must leave through its role's abort
// path, so a protocol error surfaces as an error code instead of a hang.
#pragma once

#include <stdint.h>

namespace vg {

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.965 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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

// Wait until the phase with the given parity of *bar has completed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitCycles) return false;
  }
  return true;
}

// mbar_wait for waits that may last: each try_wait may suspend the thread
// until the phase completes or about `hint_ns` pass, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_sleep_for(uint64_t *bar, uint32_t parity, long long limit_cycles) {
  if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
  const long long start = clock64();
  while (!mbar_try_wait_hint(bar, parity, 20000u)) {
    if (clock64() - start > limit_cycles) return false;
  }
  return true;
}

__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity) {
  return mbar_wait_sleep_for(bar, parity, kWaitCycles);
}

// Add `bytes` of expected transaction count to the current phase of *bar.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on *bar.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Barrier among `count` threads (a multiple of 32) of the block; id 1..15.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace vg
