// rtMemcpyAsyncWithCfg-shaped memcpy task on the library's copy kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "copy.cuh"

namespace dcopy {
namespace {

constexpr uint64_t kEngineBytes = 8ull << 20;  // host-side tasks from here on: copy engine
constexpr uint64_t kPieceBytes = 1ull << 30;

bool is_device_memory(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Memory a kernel can address: device (this GPU, a peer, managed) or pinned host.
bool gpu_addressable(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type != cudaMemoryTypeUnregistered;
}

int device_to_device(const DcopyMemcpyInfo *m, cudaStream_t s) {
  int rc = check_device_span(m->src, m->cnt, "memcpy src");
  if (!rc) rc = check_device_span(m->dst, m->cnt, "memcpy dst");
  if (!rc) rc = check_disjoint(m->src, m->cnt, m->dst, m->cnt, "memcpy");
  if (rc) return rc;
  return copy_linear(m->dst, m->src, m->cnt, s);
}

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_memcpy_async(const DcopyMemcpyInfo *info, int32_t kind,
                                  dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!info) return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy: info is NULL");
  if (info->cnt > info->destMax)
    return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy: count %llu exceeds destMax %llu",
                     (unsigned long long)info->cnt, (unsigned long long)info->destMax);
  if (info->cnt == 0) return DCOPY_OK;
  if (!info->dst || !info->src) return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy: NULL pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaMemcpyKind k;
  switch (kind) {
    case DCOPY_MEMCPY_DEVICE_TO_DEVICE: return device_to_device(info, s);
    case DCOPY_MEMCPY_DEFAULT:
      if (is_device_memory(info->dst) && is_device_memory(info->src))
        return device_to_device(info, s);
      k = cudaMemcpyDefault;
      break;
    case DCOPY_MEMCPY_HOST_TO_HOST: k = cudaMemcpyHostToHost; break;
    case DCOPY_MEMCPY_HOST_TO_DEVICE:
    case DCOPY_MEMCPY_HOST_TO_DEVICE_EX: k = cudaMemcpyHostToDevice; break;
    case DCOPY_MEMCPY_DEVICE_TO_HOST:
    case DCOPY_MEMCPY_DEVICE_TO_HOST_EX: k = cudaMemcpyDeviceToHost; break;
    case DCOPY_MEMCPY_MANAGED: k = cudaMemcpyDefault; break;
    case 5:
      return set_error(DCOPY_ERR_UNSUPPORTED,
                       "memcpy: RT_MEMCPY_ADDR_DEVICE_TO_DEVICE has no CUDA counterpart");
    default: return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy: unknown kind %d", kind);
  }
  DCOPY_CUDA_TRY(cudaMemcpyAsync(info->dst, info->src, info->cnt, k, s));
  return DCOPY_OK;
  DCOPY_API_END
}

// Tasks whose two buffers a kernel can address (device memory, or pinned host
// memory read and written over PCIe) and that are small enough for the launch
// cost to matter run as dcopy_copy_ext_batch launches: one launch for a run of
// such tasks instead of one copy call each.  Larger host-side transfers and
// pageable host memory take the copy engine, one cudaMemcpyAsync each.
//
// Task order is kept: the tasks of one launch run concurrently, so a run ends
// (its launch is issued) before a copy-engine task and before a task whose
// buffers overlap a buffer of a task already in the run.
namespace {

struct Span {
  uintptr_t lo, hi;  // [lo, hi)
  bool overlaps(const Span &o) const { return lo < o.hi && o.lo < hi; }
};

// Whether task m reads or writes memory that a task of the pending run writes,
// or writes memory that one of them reads.
bool conflicts(const std::vector<std::pair<Span, Span>> &run, const DcopyMemcpyInfo &m) {
  const Span d{(uintptr_t)m.dst, (uintptr_t)m.dst + m.cnt};
  const Span s{(uintptr_t)m.src, (uintptr_t)m.src + m.cnt};
  for (const auto &t : run)  // t.first: destination, t.second: source
    if (d.overlaps(t.first) || d.overlaps(t.second) || s.overlaps(t.first)) return true;
  return false;
}

}  // namespace

extern "C" int dcopy_memcpy_async_batch(const DcopyMemcpyInfo *infos, uint32_t count,
                                        int32_t kind, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!count) return DCOPY_OK;
  if (!infos) return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy_batch: infos is NULL");
  if (kind == 5)
    return set_error(DCOPY_ERR_UNSUPPORTED,
                     "memcpy_batch: RT_MEMCPY_ADDR_DEVICE_TO_DEVICE has no CUDA counterpart");
  if (kind < 0 || kind > 8)
    return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy_batch: unknown kind %d", kind);
  const bool host_side = kind != DCOPY_MEMCPY_DEVICE_TO_DEVICE;
  // Every task is checked before anything runs; `kernel` marks the tasks that
  // run on the batched copy kernel.
  std::vector<char> kernel(count, 0);
  for (uint32_t i = 0; i < count; ++i) {
    const DcopyMemcpyInfo &m = infos[i];
    if (m.cnt > m.destMax)
      return set_error(DCOPY_ERR_PARAM_INVALID,
                       "memcpy_batch: task %u: count %llu exceeds destMax %llu", i,
                       (unsigned long long)m.cnt, (unsigned long long)m.destMax);
    if (!m.cnt) continue;
    if (!m.dst || !m.src)
      return set_error(DCOPY_ERR_PARAM_INVALID, "memcpy_batch: task %u: NULL pointer", i);
    kernel[i] = kind != DCOPY_MEMCPY_HOST_TO_HOST && !(host_side && m.cnt >= kEngineBytes) &&
                gpu_addressable(m.dst) && gpu_addressable(m.src);
    if (kernel[i]) {
      int rc = check_device_span(m.src, m.cnt, "memcpy_batch src");
      if (!rc) rc = check_device_span(m.dst, m.cnt, "memcpy_batch dst");
      if (!rc) rc = check_disjoint(m.src, m.cnt, m.dst, m.cnt, "memcpy_batch");
      if (rc) return rc;
    }
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  std::vector<DcopyExtCopy> batch;
  std::vector<std::pair<Span, Span>> run;
  auto flush = [&]() -> int {
    if (batch.empty()) return DCOPY_OK;
    const int rc = dcopy_copy_ext_batch(batch.data(), (uint32_t)batch.size(), stream);
    batch.clear();
    run.clear();
    return rc;
  };
  for (uint32_t i = 0; i < count; ++i) {
    const DcopyMemcpyInfo &m = infos[i];
    if (!m.cnt) continue;
    if (!kernel[i] || conflicts(run, m)) {
      const int rc = flush();
      if (rc) return rc;
    }
    if (!kernel[i]) {
      cudaMemcpyKind k = cudaMemcpyDefault;
      if (kind == DCOPY_MEMCPY_HOST_TO_HOST) k = cudaMemcpyHostToHost;
      if (kind == DCOPY_MEMCPY_HOST_TO_DEVICE || kind == DCOPY_MEMCPY_HOST_TO_DEVICE_EX)
        k = cudaMemcpyHostToDevice;
      if (kind == DCOPY_MEMCPY_DEVICE_TO_HOST || kind == DCOPY_MEMCPY_DEVICE_TO_HOST_EX)
        k = cudaMemcpyDeviceToHost;
      DCOPY_CUDA_TRY(cudaMemcpyAsync(m.dst, m.src, m.cnt, k, s));
      continue;
    }
    run.push_back({Span{(uintptr_t)m.dst, (uintptr_t)m.dst + m.cnt},
                   Span{(uintptr_t)m.src, (uintptr_t)m.src + m.cnt}});
    // Contiguous pieces of at most 1 GiB (blockLen is 32-bit).
    for (uint64_t off = 0; off < m.cnt; off += kPieceBytes) {
      const uint64_t n = std::min<uint64_t>(kPieceBytes, m.cnt - off);
      batch.push_back(DcopyExtCopy{static_cast<uint8_t *>(m.dst) + off,
                                   static_cast<const uint8_t *>(m.src) + off,
                                   DcopyExtParams{1u, (uint32_t)n, 0, 0}});
    }
  }
  return flush();
  DCOPY_API_END
}
