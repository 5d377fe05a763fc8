// Kernel launch helpers: programmatic dependent launch and occupancy-sized grids.
//
// Every kernel of the library starts with pdl_trigger_at_entry(), may issue L2
// prefetches for its source, then calls pdl_wait() and pdl_launch_dependents().  Launched with programmatic stream serialization, a
// kernel may be scheduled while the previous kernel on the stream drains; its
// pdl_wait() returns only after that kernel has completed and its writes are
// visible, so stream order is kept for every caller.  Back-to-back copies on one
// stream thus overlap launch latency with the previous kernel's tail.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

#include "common.cuh"

#ifndef DCOPY_PDL
#define DCOPY_PDL 1
#endif

namespace dcopy {

__device__ __forceinline__ void pdl_wait() {
#if DCOPY_PDL
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

#ifndef DCOPY_EARLY_TRIGGER
// 1: a kernel lets its dependents launch as soon as it starts, before its own
// wait.  Safe: every dependent still blocks in pdl_wait() until this grid has
// completed, and a dependent can only launch once every CTA of this grid has
// started, so waiting CTAs never hold resources this grid still needs.
#define DCOPY_EARLY_TRIGGER 1
#endif

// Called first thing in a kernel; signals dependents only in early-trigger mode.
__device__ __forceinline__ void pdl_trigger_at_entry() {
#if DCOPY_PDL && DCOPY_EARLY_TRIGGER
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// Called right after pdl_wait().
__device__ __forceinline__ void pdl_launch_dependents() {
#if DCOPY_PDL && !DCOPY_EARLY_TRIGGER
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

template <typename... KArgs, typename... Args>
int launch_grid(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                const char *name, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
#if DCOPY_PDL
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 1;
#endif
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(DCOPY_ERR_CUDA, "launch of %s failed: %s (%s)", name, cudaGetErrorName(e),
                     cudaGetErrorString(e));
  }
  return DCOPY_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), unsigned grid, dim3 block, size_t smem, cudaStream_t s,
           const char *name, Args &&...args) {
  return launch_grid(kernel, dim3(grid), block, smem, s, name, std::forward<Args>(args)...);
}

// CTAs of `kernel` that fit on all SMs at once (cached per kernel and device).
template <typename K>
unsigned resident_ctas(K kernel, int threads, size_t smem) {
  static std::atomic<int> cache[128];
  const int dev = current_device();
  const int slot = (dev >= 0 && dev < 128) ? dev : 0;
  int per_sm = cache[slot].load(std::memory_order_relaxed);
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
            cudaSuccess ||
        per_sm <= 0) {
      (void)cudaGetLastError();
      per_sm = 1;
    }
    cache[slot].store(per_sm, std::memory_order_relaxed);
  }
  return (unsigned)per_sm * (unsigned)sm_count();
}

}  // namespace dcopy
