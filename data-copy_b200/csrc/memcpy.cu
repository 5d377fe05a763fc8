// rtMemcpyAsyncWithCfg-shaped memcpy task on the library's copy kernel.
#include <cuda_runtime.h>

#include "common.cuh"
#include "copy.cuh"

namespace dcopy {
namespace {

bool is_device_memory(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
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
