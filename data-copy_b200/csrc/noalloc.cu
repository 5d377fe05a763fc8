// dcopy_datacopy_pretranspose_noalloc: the pretranspose workflow for callers that
// cannot allocate device memory.
//
// The pretranspose mode of the standalone kernels needs a temporary device
// buffer B as large as the input: x is transposed into B, then B is copied to y.
// dcopy_datacopy_pretranspose / dcopy_datacopy_contiguous take B from the
// caller.  Some callers cannot provide it: code that runs under a framework
// which owns the whole device-memory budget (a model executor with a static
// memory plan, a plugin inside a host process whose allocator has reserved the
// device), or a latency-critical path where cudaMalloc/cudaFree would
// synchronise the device.  This entry point takes only x and y and keeps B in
// a fixed array in the library's own device memory, so it never allocates.
//
// Cost of that choice: every GPU that loads this part of the library holds the
// array (kStaticBytes) until the process exits, whether or not it is called.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "internal.cuh"

namespace dcopy {
namespace {

// Largest B the array holds: rows * cols * 4 <= 16 MiB (the reference's default
// 256 x 768 shape needs 768 KiB).  Larger shapes must use the entry points that
// take a caller buffer.
constexpr uint64_t kStaticBytes = 16ull << 20;

}  // namespace
}  // namespace dcopy

// The B buffer.  In host code this name is only a stand-in for the symbol, not
// a device address: it must be turned into one with cudaGetSymbolAddress, on
// each device, before a kernel can use it.
static __device__ __align__(256) unsigned char g_pretranspose_b[dcopy::kStaticBytes];

namespace dcopy {
namespace {

constexpr int kMaxDevices = 128;
std::mutex g_mutex;

// The array's address on one device, and the CUDA context it belongs to.  A
// device reset (or a primary context released and created again) reloads the
// module, which may place the array elsewhere: the address is then looked up
// again in the new context.
struct Slot {
  void *address = nullptr;
  unsigned long long context_id = 0;  // 0: not known
};
Slot g_slots[kMaxDevices];

}  // namespace

typedef int (*PfnCtxGetCurrent)(void **);
typedef int (*PfnCtxGetId)(void *, unsigned long long *);

bool current_context_id(unsigned long long *id) {
  static PfnCtxGetCurrent get_current = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PfnCtxGetId>(p);
  });
  void *ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx) return false;
  return get_id(ctx, id) == 0 && *id != 0;
}

namespace {

// Device address of g_pretranspose_b on the current device.  Set-up, once per
// device (and again after the device's context was replaced), with that device
// current: cudaGetSymbolAddress, whose return code is checked.
int b_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(DCOPY_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kMaxDevices);
  unsigned long long ctx = 0;
  bool known = current_context_id(&ctx);
  std::lock_guard<std::mutex> lock(g_mutex);
  Slot &slot = g_slots[dev];
  if (!slot.address || !known || slot.context_id != ctx) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pretranspose_b);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_pretranspose_b)");
    if (!p) return set_error(DCOPY_ERR_CUDA, "cudaGetSymbolAddress returned NULL");
    if (!known) known = current_context_id(&ctx);  // the look-up made the context current
    slot.address = p;
    slot.context_id = known ? ctx : 0;  // unknown: looked up again on the next call
  }
  *out = slot.address;
  return DCOPY_OK;
}

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_datacopy_pretranspose_noalloc(const void *x, void *y,
                                                   const DataCopyTiling *tiling,
                                                   dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  void *b = nullptr;
  const int rc = b_address(&b);
  if (rc) return rc;
  // Nothing in B needs clearing: the first kernel writes all rows*cols words of
  // it before the second reads them, so a previous call's contents never leak.
  return run_pretranspose_workflow(x, b, kStaticBytes, y, tiling, stream);
  DCOPY_API_END
}
