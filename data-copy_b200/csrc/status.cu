// Status reporting, buffer checks and device queries shared by every entry point.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace dcopy {
namespace {

thread_local char g_message[1024] = {0};

typedef CUresult (*PfnPointerGetAttributes)(unsigned int, CUpointer_attribute *, void **,
                                            CUdeviceptr);

PfnPointerGetAttributes pointer_attrs_fn() {
  static PfnPointerGetAttributes fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuPointerGetAttributes", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnPointerGetAttributes>(p);
  });
  return fn;
}

bool checks_enabled() {
  static const bool enabled = [] {
    const char *v = std::getenv("DCOPY_CHECK_POINTERS");
    return !(v && v[0] == '0');
  }();
  return enabled;
}

}  // namespace

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_message[0] = 0; }

int cuda_fail(cudaError_t err, const char *what) {
  return set_error(DCOPY_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(err),
                   cudaGetErrorString(err));
}

int check_launch(const char *kernel) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(DCOPY_ERR_CUDA, "launch of %s failed: %s (%s)", kernel,
                     cudaGetErrorName(err), cudaGetErrorString(err));
  return DCOPY_OK;
}

int check_device_span(const void *ptr, uint64_t bytes, const char *name) {
  if (bytes == 0) return DCOPY_OK;
  if (!ptr) return set_error(DCOPY_ERR_PARAM_INVALID, "%s is NULL for %llu bytes", name,
                             (unsigned long long)bytes);
  if (!checks_enabled()) return DCOPY_OK;
  PfnPointerGetAttributes fn = pointer_attrs_fn();
  if (!fn) return DCOPY_OK;  // no driver entry point: cannot check, launch decides
  unsigned int mem_type = 0;
  CUdeviceptr start = 0;
  size_t size = 0;
  CUpointer_attribute attrs[3] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
                                  CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                  CU_POINTER_ATTRIBUTE_RANGE_SIZE};
  void *data[3] = {&mem_type, &start, &size};
  CUresult r = fn(3, attrs, data, (CUdeviceptr)(uintptr_t)ptr);
  if (r != CUDA_SUCCESS || mem_type == 0)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "%s (%p) is not memory the GPU can address (plain host memory?)", name, ptr);
  if (start != 0 && size != 0) {
    const uint64_t p = (uint64_t)(uintptr_t)ptr;
    if (p < start || p - start > size || bytes > size - (p - start))
      return set_error(DCOPY_ERR_PARAM_INVALID,
                       "%s: %llu bytes at %p run past its allocation [%p, +%llu)", name,
                       (unsigned long long)bytes, ptr, (void *)(uintptr_t)start,
                       (unsigned long long)size);
  }
  return DCOPY_OK;
}

namespace {
// CUDA IPC mappings opened through dcopy_ipc_open_handle: [base, base + size).
// The driver reports such a mapping as device memory of the device that opened
// it, so the ranges are kept here to tell them apart from local allocations.
// A base opened more than once (the driver may hand back the same mapping)
// is counted, and its record stays until the last close.
struct IpcRange {
  uint64_t base, size;
  int opens;
};
std::mutex g_ipc_mu;
std::vector<IpcRange> g_ipc_ranges;
std::atomic<int> g_ipc_open{0};
}  // namespace

void note_ipc_mapping(const void *base, bool opened) {
  const uint64_t b = (uint64_t)(uintptr_t)base;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  auto it = std::find_if(g_ipc_ranges.begin(), g_ipc_ranges.end(),
                         [b](const IpcRange &r) { return r.base == b; });
  if (opened) {
    if (it != g_ipc_ranges.end()) {
      ++it->opens;
    } else {
      uint64_t size = 1;  // the base alone when the size cannot be read
      PfnPointerGetAttributes fn = pointer_attrs_fn();
      size_t n = 0;
      CUpointer_attribute attr = CU_POINTER_ATTRIBUTE_RANGE_SIZE;
      void *data = &n;
      if (fn && fn(1, &attr, &data, (CUdeviceptr)b) == CUDA_SUCCESS && n) size = n;
      g_ipc_ranges.push_back({b, size, 1});
    }
  } else if (it != g_ipc_ranges.end() && --it->opens == 0) {
    g_ipc_ranges.erase(it);
  }
  g_ipc_open.store((int)g_ipc_ranges.size(), std::memory_order_release);
}

bool in_ipc_mapping(const void *ptr) {
  if (g_ipc_open.load(std::memory_order_acquire) == 0) return false;
  const uint64_t p = (uint64_t)(uintptr_t)ptr;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (const auto &r : g_ipc_ranges)
    if (p >= r.base && p - r.base < r.size) return true;
  return false;
}

bool is_local_device_memory(const void *ptr) {
  PfnPointerGetAttributes fn = pointer_attrs_fn();
  if (!fn || !ptr || in_ipc_mapping(ptr)) return false;
  unsigned int mem_type = 0;
  int ordinal = -1;
  CUpointer_attribute attrs[2] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
                                  CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL};
  void *data[2] = {&mem_type, &ordinal};
  if (fn(2, attrs, data, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS) return false;
  return mem_type == CU_MEMORYTYPE_DEVICE && ordinal == current_device();
}

uint64_t allocation_base(const void *ptr) {
  PfnPointerGetAttributes fn = pointer_attrs_fn();
  if (!fn || !ptr) return 0;
  CUdeviceptr start = 0;
  CUpointer_attribute attr = CU_POINTER_ATTRIBUTE_RANGE_START_ADDR;
  void *data = &start;
  if (fn(1, &attr, &data, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS) return 0;
  return (uint64_t)start;
}

int block_span(uint64_t count, uint64_t pitch, uint64_t len, uint64_t *span, const char *what) {
  const unsigned __int128 s = (unsigned __int128)(count ? count - 1 : 0) * pitch + len;
  if (s >= ((unsigned __int128)1 << 62))
    return set_error(DCOPY_ERR_PARAM_INVALID, "%s: the copy spans 2^62 bytes or more", what);
  *span = (uint64_t)s;
  return DCOPY_OK;
}

int check_disjoint(const void *a, uint64_t an, const void *b, uint64_t bn, const char *what) {
  if (!an || !bn) return DCOPY_OK;
  const uint64_t pa = (uint64_t)(uintptr_t)a, pb = (uint64_t)(uintptr_t)b;
  if (pa < pb + bn && pb < pa + an)
    return set_error(DCOPY_ERR_PARAM_INVALID, "%s: source and destination ranges overlap",
                     what);
  return DCOPY_OK;
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev;
}

int sm_count() {
  static std::atomic<int> cache[128];
  const int dev = current_device();
  if (dev < 0 || dev >= 128) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace dcopy

extern "C" {

const char *dcopy_last_error_message(void) { return dcopy::g_message; }

uint32_t dcopy_status_to_ge(int status) {
  switch (status) {
    case DCOPY_OK: return 0u;
    case DCOPY_ERR_PARAM_INVALID: return 145000u;
    case DCOPY_ERR_SHAPE_INVALID: return 145021u;
    case DCOPY_ERR_DATATYPE_INVALID: return 145022u;
    case DCOPY_ERR_FORMAT_INVALID: return 145020u;
    case DCOPY_ERR_CUDA: return 245002u;     // ACL_ERROR_GE_DEVICE_MEMORY_OPERATE_FAILED
    case DCOPY_ERR_TIMEOUT: return 545601u;  // ACL_ERROR_GE_MODEL_EXECUTE_TIMEOUT
    case DCOPY_ERR_FAILED: return 0xFFFFFFFFu;  // FAILED / GRAPH_FAILED
    default: return 545000u;                 // ACL_ERROR_GE_INTERNAL_ERROR
  }
}

int dcopy_version(void) { return 100; }

}  // extern "C"
