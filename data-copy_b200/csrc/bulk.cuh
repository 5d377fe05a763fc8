// Device helpers for the bulk-copy (TMA) engine on sm_100a: shared-memory
// addresses, mbarriers with bounded waits, and the untiled cp.async.bulk
// load / store / L2 prefetch.  None of these use cluster multicast; loads read
// the memory of the GPU the kernel runs on.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcopy {
namespace bulk {

// try_wait suspends for a hardware-defined time (about a microsecond) per call,
// so this many failed tries add up to seconds: the bound of every wait below.
constexpr uint32_t kWaitIters = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals));
}

// Makes an mbarrier initialised by this thread visible to the async proxy (the
// bulk-copy engine that completes its transactions) and to the other threads.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// False when the phase did not complete within kWaitIters tries.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  for (uint32_t it = 0; it < kWaitIters; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// One arrival on `bar` that also expects `bytes` of transactions, then the
// global -> shared copy that delivers them.  gsrc, smem_dst and bytes are
// multiples of 16.
__device__ __forceinline__ void load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                     uint64_t *bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// shared -> global copy in this thread's current bulk group (not committed).
__device__ __forceinline__ void store(void *gdst, const void *smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until this thread's committed bulk groups have completed (their writes
// are performed), so no copy outlives the CTA.
__device__ __forceinline__ void wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// L2 prefetch of [gsrc, gsrc + bytes): a hint that returns no data and does not
// order memory, so it may run before the dependent-launch wait.
__device__ __forceinline__ void prefetch_l2(const void *gsrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

}  // namespace bulk
}  // namespace dcopy
