// Many independent DataCopyExt copies in one launch.
//
// An Ascend C kernel issues its DataCopy calls from the device, many per launch:
// the reference's standalone kernel moves every tile of a core with one call
// each (datacopy_data_collection.asc:16-62), and BASELINE's config 1 is 8 cores
// x 16 tiles.  Through a host C ABI each dcopy_copy_ext call is a launch with
// its own fixed cost (about a microsecond on B200), so a batch of copies goes
// to one kernel: copy k is cut into chunks of kChunk elements of its widest
// common width, CTA b finds the copy that owns chunk b by binary search over
// the chunk prefix sums, and moves that chunk with the strided element loop
// of the single-copy kernel.  The descriptors travel as one kernel parameter
// (up to kBatchMax copies, 16 KiB), so the batch needs no device allocation.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "copy.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;
constexpr int kU = 4;                            // elements in flight per thread
constexpr uint32_t kChunk = kThreads * kU;       // elements per CTA
constexpr uint32_t kBatchMax = 256;              // copies per launch
constexpr uint64_t kMaxBatchedElems = 1u << 30;  // larger copies launch on their own

struct BatchCopy {
  uint64_t dst, src;    // byte addresses
  uint64_t sp, dp;      // row pitches, bytes
  FastDiv epr;          // elements per row
  uint32_t elems;       // rows x elements per row
  uint32_t w;           // element width, bytes (16, 8, 4, 2 or 1)
  uint32_t first_chunk; // chunks of the copies before this one
};

struct BatchDesc {
  uint32_t n;
  BatchCopy c[kBatchMax];
};

template <typename T>
__device__ __forceinline__ void copy_chunk(const BatchCopy &c, uint32_t begin, uint32_t end) {
  const uint8_t *src = reinterpret_cast<const uint8_t *>(c.src);
  uint8_t *dst = reinterpret_cast<uint8_t *>(c.dst);
  for (uint32_t base = begin + threadIdx.x; base < end; base += kThreads * kU) {
    T v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t i = base + u * kThreads;
      if (i < end) {
        const uint32_t r = c.epr.div(i);
        v[u] = ld_stream(reinterpret_cast<const T *>(src + (uint64_t)r * c.sp) + (i - r * c.epr.d));
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t i = base + u * kThreads;
      if (i < end) {
        const uint32_t r = c.epr.div(i);
        *(reinterpret_cast<T *>(dst + (uint64_t)r * c.dp) + (i - r * c.epr.d)) = v[u];
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) batch_copy_kernel(const __grid_constant__ BatchDesc d) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t b = blockIdx.x;
  uint32_t lo = 0, hi = d.n;  // d.c[lo].first_chunk <= b < d.c[hi].first_chunk
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (d.c[mid].first_chunk <= b)
      lo = mid;
    else
      hi = mid;
  }
  const BatchCopy &c = d.c[lo];
  const uint32_t begin = (b - c.first_chunk) * kChunk;
  const uint32_t end = begin + kChunk < c.elems ? begin + kChunk : c.elems;
  switch (c.w) {
    case 16: copy_chunk<uint4>(c, begin, end); break;
    case 8: copy_chunk<uint2>(c, begin, end); break;
    case 4: copy_chunk<uint32_t>(c, begin, end); break;
    case 2: copy_chunk<uint16_t>(c, begin, end); break;
    default: copy_chunk<uint8_t>(c, begin, end); break;
  }
}

struct Span {
  uint64_t lo, hi;  // [lo, hi)
};

uint32_t widest_unit(uint64_t x) {
  uint32_t w = 16;
  while (w > 1 && x % w) w >>= 1;
  return w;
}

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_copy_ext_batch(const DcopyExtCopy *copies, uint32_t count,
                                    dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!count) return DCOPY_OK;
  if (!copies) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_batch: copies is NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Validation first, for every copy, as dcopy_copy_ext does; nothing launches
  // unless the whole batch is valid.
  std::vector<Span> dsts, srcs;
  dsts.reserve(count);
  srcs.reserve(count);
  for (uint32_t k = 0; k < count; ++k) {
    const DcopyExtCopy &c = copies[k];
    const uint64_t n = c.params.blockCount, len = c.params.blockLen;
    if (!n || !len) continue;
    if (c.params.srcStride > (1ull << 48) || c.params.dstStride > (1ull << 48))
      return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_batch: copy %u: stride beyond 2^48 bytes",
                       k);
    uint64_t src_span = 0, dst_span = 0;
    int rc = block_span(n, len + c.params.srcStride, len, &src_span, "copy_ext_batch src");
    if (!rc) rc = block_span(n, len + c.params.dstStride, len, &dst_span, "copy_ext_batch dst");
    if (!rc) rc = check_device_span(c.src, src_span, "copy_ext_batch src");
    if (!rc) rc = check_device_span(c.dst, dst_span, "copy_ext_batch dst");
    if (!rc) rc = check_disjoint(c.src, src_span, c.dst, dst_span, "copy_ext_batch");
    if (rc) return rc;
    dsts.push_back({(uint64_t)(uintptr_t)c.dst, (uint64_t)(uintptr_t)c.dst + dst_span});
    srcs.push_back({(uint64_t)(uintptr_t)c.src, (uint64_t)(uintptr_t)c.src + src_span});
  }
  // The copies run concurrently: no destination span may overlap another copy's
  // destination or source span (each copy's own pair was checked above).
  std::sort(dsts.begin(), dsts.end(), [](const Span &a, const Span &b) { return a.lo < b.lo; });
  for (size_t i = 1; i < dsts.size(); ++i)
    if (dsts[i].lo < dsts[i - 1].hi)
      return set_error(DCOPY_ERR_PARAM_INVALID,
                       "copy_ext_batch: two destinations overlap; copies run concurrently");
  std::sort(srcs.begin(), srcs.end(), [](const Span &a, const Span &b) { return a.lo < b.lo; });
  std::vector<uint64_t> max_hi(srcs.size());
  for (size_t i = 0; i < srcs.size(); ++i)
    max_hi[i] = std::max(srcs[i].hi, i ? max_hi[i - 1] : 0);
  for (const Span &d : dsts) {
    // Sources starting before d ends; the largest end among them decides.
    const size_t m = std::lower_bound(srcs.begin(), srcs.end(), d.hi,
                                      [](const Span &a, uint64_t v) { return a.lo < v; }) -
                     srcs.begin();
    if (m && max_hi[m - 1] > d.lo)
      return set_error(DCOPY_ERR_PARAM_INVALID,
                       "copy_ext_batch: a destination overlaps another copy's source");
  }

  BatchDesc desc;
  desc.n = 0;
  uint64_t chunks = 0;
  auto flush = [&]() -> int {
    if (!desc.n) return DCOPY_OK;
    const int rc = launch(batch_copy_kernel, (unsigned)chunks, dim3(kThreads), 0, s,
                          "batch_copy_kernel", desc);
    desc.n = 0;
    chunks = 0;
    return rc;
  };
  for (uint32_t k = 0; k < count; ++k) {
    const DcopyExtCopy &c = copies[k];
    uint64_t rows = c.params.blockCount, len = c.params.blockLen;
    if (!rows || !len) continue;
    uint64_t sp = len + c.params.srcStride, dp = len + c.params.dstStride;
    if (rows == 1 || (sp == len && dp == len)) {  // one contiguous run
      len *= rows;
      rows = 1;
      sp = dp = len;
    }
    const uint32_t w = widest_unit((uintptr_t)c.dst | (uintptr_t)c.src | len | sp | dp);
    const uint64_t elems = rows * (len / w);
    if (elems >= kMaxBatchedElems) {  // a large copy: its own launch (order is free)
      const int rc = copy2d(c.dst, c.src, rows, len, sp, dp, s);
      if (rc) return rc;
      continue;
    }
    BatchCopy &b = desc.c[desc.n++];
    b.dst = (uint64_t)(uintptr_t)c.dst;
    b.src = (uint64_t)(uintptr_t)c.src;
    b.sp = sp;
    b.dp = dp;
    b.epr = FastDiv((uint32_t)(len / w));
    b.elems = (uint32_t)elems;
    b.w = w;
    b.first_chunk = (uint32_t)chunks;
    chunks += (elems + kChunk - 1) / kChunk;
    if (desc.n == kBatchMax) {
      const int rc = flush();
      if (rc) return rc;
    }
  }
  return flush();
  DCOPY_API_END
}
