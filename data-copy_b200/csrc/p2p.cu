// Multi-GPU pieces: shard ranges, per-device launches, NVLink P2P copies, CUDA
// IPC mappings and bounded completion flags.
//
// The P2P copy picks its engine.  A push from this GPU to another GPU's memory
// goes to the copy engine (cudaMemcpyAsync on the caller's stream): in an
// exchange of 1 GiB per direction over NV18 it moves 766-775 GB/s, where every
// SM-issued write path measured settles at 689-715 (bulk-copy pipelines of 8-64
// KiB chunks, 2-8 stages, 1-4 CTAs per SM; 128-bit stores; half SM + half engine
// at 735), and it also wins at every shorter size measured (one way, GB/s, copy
// engine vs SM bulk push: 64 KiB 18.0 vs 10.4, 256 KiB 69.7 vs 51.9, 1 MiB 213 vs
// 176, 16 MiB 620 vs 591).  Pulls (launched on the receiving GPU, 786 GB/s one
// way) run the 128-bit load/store kernel.  With the SM engine forced
// (dcopy_set_p2p_engine) pushes run the SM bulk-copy pipeline: local loads into
// shared memory, bulk stores over NVLink.
// Completion flags use st.release.sys / ld.acquire.sys on a caller-owned word;
// the waiting kernel has a time bound and an iteration bound and reports a
// timeout through a caller-owned status word instead of hanging.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "copy.cuh"
#include "launch.cuh"

#ifndef DCOPY_P2P_BULK
#define DCOPY_P2P_BULK 1
#endif

namespace dcopy {
namespace {

std::atomic<int> g_p2p_engine{-1};  // -1: not read from the environment yet

// DCOPY_P2P_ENGINE = auto | sm | copy (or 0 | 1 | 2); unset or unknown: auto.
int initial_engine() {
  const char *e = std::getenv("DCOPY_P2P_ENGINE");
  if (!e) return DCOPY_P2P_ENGINE_AUTO;
  if (!std::strcmp(e, "sm") || !std::strcmp(e, "1")) return DCOPY_P2P_ENGINE_SM;
  if (!std::strcmp(e, "copy") || !std::strcmp(e, "2")) return DCOPY_P2P_ENGINE_COPY;
  return DCOPY_P2P_ENGINE_AUTO;
}

int p2p_engine() {
  int v = g_p2p_engine.load(std::memory_order_relaxed);
  if (v < 0) {
    int expected = -1;
    g_p2p_engine.compare_exchange_strong(expected, initial_engine());
    v = g_p2p_engine.load(std::memory_order_relaxed);
  }
  return v;
}

// RAII restore of the caller's current device.
struct DeviceGuard {
  int saved = -1;
  DeviceGuard() {
    if (cudaGetDevice(&saved) != cudaSuccess) saved = -1;
  }
  ~DeviceGuard() {
    if (saved >= 0) cudaSetDevice(saved);
  }
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void signal_kernel(uint32_t *flag, uint32_t value) {
  pdl_wait();
  asm volatile("fence.sc.sys;" ::: "memory");
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

// One thread.  Both bounds end the loop: time (globaltimer) and iterations
// (the host sizes max_iters so that it ends the loop even if the timer stalled).
__global__ void wait_signal_kernel(const uint32_t *flag, uint32_t value, uint64_t timeout_ns,
                                   uint64_t max_iters, uint32_t *status) {
  pdl_wait();
  const uint64_t start = global_ns();
  uint32_t result = 1;
  for (uint64_t it = 0; it < max_iters; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    // Sequence numbers: a signaller may already have moved the flag past `value`
    // (a ring neighbour one step ahead), which counts as arrived.  The signed
    // difference keeps the test right across 2^32 wrap-around.
    if ((int32_t)(v - value) >= 0) {
      result = 0;
      break;
    }
    if (global_ns() - start > timeout_ns) break;
    __nanosleep(256);
  }
  *status = result;
}

// ---- bulk-copy (TMA) push to another GPU ------------------------------------------
//
// One thread per CTA drives a kStages-deep pipeline of kChunk-byte chunks:
//   cp.async.bulk global(local) -> shared, completion on an mbarrier (complete_tx);
//   cp.async.bulk shared -> global(peer), bulk_group; the stage is refilled once
//   the store has read it (wait_group.read).
// Loads read this GPU's memory only; no multicast.  Every mbarrier wait is
// bounded; on a timeout the kernel records it in g_p2p_error, waits (bounded)
// for its own copies in flight and returns.
#ifndef DCOPY_P2P_STAGES
#define DCOPY_P2P_STAGES 4
#endif
#ifndef DCOPY_P2P_CHUNK_KIB
#define DCOPY_P2P_CHUNK_KIB 16
#endif
#ifndef DCOPY_P2P_CTAS_PER_SM
#define DCOPY_P2P_CTAS_PER_SM 3
#endif
constexpr int kStages = DCOPY_P2P_STAGES;
constexpr uint32_t kChunk = DCOPY_P2P_CHUNK_KIB * 1024;
constexpr uint32_t kWaitIters = 1u << 22;  // try_wait suspends ~us per call: seconds in total

__device__ uint32_t g_p2p_error;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
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

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  for (uint32_t it = 0; it < kWaitIters; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
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

__device__ __forceinline__ void bulk_store(void *gdst, const void *smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// bytes, src and dst are multiples of 16; chunk c of the copy is handled by
// CTA c mod gridDim.x.
__global__ void __launch_bounds__(32) p2p_bulk_push_kernel(uint8_t *__restrict__ dst,
                                                           const uint8_t *__restrict__ src,
                                                           uint64_t bytes) {
  extern __shared__ __align__(128) uint8_t stage_mem[];
  __shared__ __align__(8) uint64_t bars[kStages];
  pdl_trigger_at_entry();
  if (threadIdx.x != 0) return;
  for (int i = 0; i < kStages; ++i)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[i])));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  pdl_wait();
  pdl_launch_dependents();
  const uint64_t nchunks = (bytes + kChunk - 1) / kChunk;
  const uint64_t mine = blockIdx.x < nchunks ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  auto chunk_off = [&](uint64_t k) { return (blockIdx.x + k * gridDim.x) * (uint64_t)kChunk; };
  auto chunk_len = [&](uint64_t k) {
    const uint64_t off = chunk_off(k);
    return (uint32_t)(bytes - off < kChunk ? bytes - off : kChunk);
  };
  const uint64_t pro = mine < (uint64_t)kStages ? mine : (uint64_t)kStages;
  for (uint64_t k = 0; k < pro; ++k)
    bulk_load(stage_mem + k * kChunk, src + chunk_off(k), chunk_len(k), &bars[k]);
  uint64_t issued = pro, k = 0;
  bool ok = true;
  for (; k < mine; ++k) {
    const int st = (int)(k % kStages);
    if (!mbar_wait_bounded(&bars[st], (uint32_t)((k / kStages) & 1))) {
      ok = false;
      break;
    }
    bulk_store(dst + chunk_off(k), stage_mem + st * kChunk, chunk_len(k));
    if (issued < mine) {  // refill this stage once the store has read it
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      bulk_load(stage_mem + st * kChunk, src + chunk_off(issued), chunk_len(issued), &bars[st]);
      ++issued;
    }
  }
  if (!ok) {
    atomicExch(&g_p2p_error, 1u);
    // Drain every load still in flight (bounded), so no copy outlives the CTA.
    for (uint64_t j = k; j < issued; ++j)
      (void)mbar_wait_bounded(&bars[j % kStages], (uint32_t)((j / kStages) & 1));
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The route of one dcopy_p2p_copy.  The SM paths: a push of 16-byte granular
// buffers through the bulk-copy pipeline; anything else (pulls, odd sizes,
// local copies) through the load/store kernel.  (A bulk-copy pull from the peer
// measured 666 GB/s per direction in an exchange against 643 for the load
// kernel and 702 for the bulk push.)
int p2p_route(const void *dst, const void *src, uint64_t bytes) {
  const int engine = p2p_engine();
  const bool push = is_local_device_memory(src) && !is_local_device_memory(dst);
  if (engine == DCOPY_P2P_ENGINE_COPY || (engine == DCOPY_P2P_ENGINE_AUTO && push))
    return DCOPY_P2P_ROUTE_COPY_ENGINE;
  if (DCOPY_P2P_BULK && push && ((uintptr_t)dst | (uintptr_t)src | bytes) % 16 == 0)
    return DCOPY_P2P_ROUTE_SM_BULK_PUSH;
  return DCOPY_P2P_ROUTE_SM_LOAD_STORE;
}

int launch_bulk_push(void *dst, const void *src, uint64_t bytes, cudaStream_t s) {
  static std::atomic<bool> configured[128];
  const int dev = current_device();
  const size_t smem = (size_t)kStages * kChunk;
  if (dev >= 0 && dev < 128 && !configured[dev].load()) {
    cudaError_t e = cudaFuncSetAttribute(p2p_bulk_push_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    configured[dev] = true;
  }
  const uint64_t nchunks = (bytes + kChunk - 1) / kChunk;
  const uint64_t grid = std::min<uint64_t>(nchunks, (uint64_t)sm_count() * DCOPY_P2P_CTAS_PER_SM);
  return launch(p2p_bulk_push_kernel, (unsigned)grid, dim3(32), smem, s, "p2p_bulk_push_kernel",
                static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), bytes);
}

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_shard_range(uint64_t block_count, int32_t rank, int32_t world,
                                 uint64_t *begin, uint64_t *count) {
  DCOPY_API_BEGIN
  if (world <= 0 || rank < 0 || rank >= world || !begin || !count)
    return set_error(DCOPY_ERR_PARAM_INVALID, "shard_range: rank %d of world %d", rank, world);
  const uint64_t base = block_count / (uint64_t)world, extra = block_count % (uint64_t)world;
  const uint64_t r = (uint64_t)rank;
  *count = base + (r < extra ? 1 : 0);
  *begin = r * base + (r < extra ? r : extra);
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_copy_ext_multi(const DcopyDevCopy *copies, int32_t n) {
  DCOPY_API_BEGIN
  if (n < 0 || (n && !copies)) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_multi: n=%d", n);
  DeviceGuard guard;
  for (int32_t i = 0; i < n; ++i) {
    DCOPY_CUDA_TRY(cudaSetDevice(copies[i].device));
    const int rc = dcopy_copy_ext(copies[i].dst, copies[i].src, &copies[i].params,
                                  copies[i].stream);
    if (rc) return rc;
  }
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_enable_peer_access(int32_t device, int32_t peer) {
  DCOPY_API_BEGIN
  if (device == peer) return DCOPY_OK;
  int can = 0;
  DCOPY_CUDA_TRY(cudaDeviceCanAccessPeer(&can, device, peer));
  if (!can)
    return set_error(DCOPY_ERR_PARAM_INVALID, "device %d cannot access device %d", device, peer);
  DeviceGuard guard;
  DCOPY_CUDA_TRY(cudaSetDevice(device));
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return DCOPY_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_p2p_copy(void *dst, const void *src, uint64_t bytes, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!bytes) return DCOPY_OK;
  int rc = check_device_span(src, bytes, "p2p src");
  if (!rc) rc = check_device_span(dst, bytes, "p2p dst");
  if (!rc) rc = check_disjoint(src, bytes, dst, bytes, "p2p_copy");
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (p2p_route(dst, src, bytes)) {
    case DCOPY_P2P_ROUTE_COPY_ENGINE:
      DCOPY_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s));
      return DCOPY_OK;
    case DCOPY_P2P_ROUTE_SM_BULK_PUSH: return launch_bulk_push(dst, src, bytes, s);
    default: return copy_linear(dst, src, bytes, s);
  }
  DCOPY_API_END
}

extern "C" int dcopy_p2p_route(const void *dst, const void *src, uint64_t bytes,
                               int32_t *route) {
  DCOPY_API_BEGIN
  if (!route) return set_error(DCOPY_ERR_PARAM_INVALID, "p2p_route: route is NULL");
  *route = p2p_route(dst, src, bytes);
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_set_p2p_engine(int32_t engine, int32_t *previous) {
  DCOPY_API_BEGIN
  if (engine != DCOPY_P2P_ENGINE_AUTO && engine != DCOPY_P2P_ENGINE_SM &&
      engine != DCOPY_P2P_ENGINE_COPY)
    return set_error(DCOPY_ERR_PARAM_INVALID, "set_p2p_engine: engine %d", engine);
  const int was = p2p_engine();
  g_p2p_engine.store(engine);
  if (previous) *previous = was;
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_p2p_ring_shift(const int32_t *devices, void *const *src, void *const *dst,
                                    const dcopy_stream_t *streams, int32_t n, uint64_t bytes) {
  DCOPY_API_BEGIN
  if (n <= 0 || !devices || !src || !dst)
    return set_error(DCOPY_ERR_PARAM_INVALID, "ring_shift: n=%d", n);
  for (int32_t i = 0; i < n; ++i) {
    const int rc = dcopy_enable_peer_access(devices[i], devices[(i + 1) % n]);
    if (rc) return rc;
  }
  DeviceGuard guard;
  for (int32_t i = 0; i < n; ++i) {
    DCOPY_CUDA_TRY(cudaSetDevice(devices[i]));
    const int rc = dcopy_p2p_copy(dst[(i + 1) % n], src[i], bytes, streams ? streams[i] : nullptr);
    if (rc) return rc;
  }
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_ipc_get_handle(const void *dev_ptr, void *handle, uint64_t *offset) {
  DCOPY_API_BEGIN
  static_assert(sizeof(cudaIpcMemHandle_t) == DCOPY_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle || !offset)
    return set_error(DCOPY_ERR_PARAM_INVALID, "ipc_get_handle: NULL");
  const uint64_t base = allocation_base(dev_ptr);
  if (!base) return set_error(DCOPY_ERR_PARAM_INVALID, "ipc_get_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  DCOPY_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)));
  std::memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(uintptr_t)dev_ptr - base;
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_ipc_open_handle(const void *handle, void **dev_ptr) {
  DCOPY_API_BEGIN
  if (!handle || !dev_ptr) return set_error(DCOPY_ERR_PARAM_INVALID, "ipc_open_handle: NULL");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  DCOPY_CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  note_ipc_mapping(*dev_ptr, true);
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_ipc_close_handle(void *dev_ptr) {
  DCOPY_API_BEGIN
  if (!dev_ptr) return DCOPY_OK;
  DCOPY_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
  note_ipc_mapping(dev_ptr, false);
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_p2p_error(uint32_t *flag) {
  DCOPY_API_BEGIN
  if (!flag) return set_error(DCOPY_ERR_PARAM_INVALID, "p2p_error: NULL");
  uint32_t zero = 0;
  DCOPY_CUDA_TRY(cudaMemcpyFromSymbol(flag, g_p2p_error, sizeof(uint32_t)));
  DCOPY_CUDA_TRY(cudaMemcpyToSymbol(g_p2p_error, &zero, sizeof(uint32_t)));
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_signal(uint32_t *flag, uint32_t value, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  int rc = check_device_span(flag, sizeof(uint32_t), "flag");
  if (rc) return rc;
  if ((uintptr_t)flag % 4) return set_error(DCOPY_ERR_PARAM_INVALID, "flag must be 4-byte aligned");
  return launch(signal_kernel, 1, dim3(1), 0, reinterpret_cast<cudaStream_t>(stream),
                "signal_kernel", flag, value);
  DCOPY_API_END
}

extern "C" int dcopy_wait_signal(const uint32_t *flag, uint32_t value, uint64_t timeout_ns,
                                 uint32_t *status, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  int rc = check_device_span(flag, sizeof(uint32_t), "flag");
  if (!rc) rc = check_device_span(status, sizeof(uint32_t), "status");
  if (rc) return rc;
  if ((uintptr_t)flag % 4 || (uintptr_t)status % 4)
    return set_error(DCOPY_ERR_PARAM_INVALID, "flag and status must be 4-byte aligned");
  const uint64_t limit = 60ull * 1000 * 1000 * 1000;  // never wait more than a minute
  if (timeout_ns > limit) timeout_ns = limit;
  // Iteration bound for a __nanosleep that returns early: 32 ns per iteration.
  const uint64_t max_iters = timeout_ns / 32 + 4096;
  return launch(wait_signal_kernel, 1, dim3(1), 0, reinterpret_cast<cudaStream_t>(stream),
                "wait_signal_kernel", flag, value, timeout_ns, max_iters, status);
  DCOPY_API_END
}
