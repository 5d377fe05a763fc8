// Multi-GPU pieces: shard ranges, per-device launches, NVLink P2P copies, CUDA
// IPC mappings and bounded completion flags.
//
// The P2P copy pushes: each thread loads 16-byte units of the local source and
// stores them to the peer address (posted writes over NVLink); reads stay local.
// Completion flags use st.release.sys / ld.acquire.sys on a caller-owned word;
// the waiting kernel has a time bound and an iteration bound and reports a
// timeout through a caller-owned status word instead of hanging.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "copy.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

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
    if (v == value) {
      result = 0;
      break;
    }
    if (global_ns() - start > timeout_ns) break;
    __nanosleep(256);
  }
  *status = result;
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
  return copy_linear(dst, src, bytes, reinterpret_cast<cudaStream_t>(stream));
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
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_ipc_close_handle(void *dev_ptr) {
  DCOPY_API_BEGIN
  if (!dev_ptr) return DCOPY_OK;
  DCOPY_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
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
