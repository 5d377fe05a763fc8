// DataCopyPad with the Unified-Buffer side conventions of DataCopyPadExtend.
//
// An Ascend C kernel moves a GM tile into its Unified Buffer (UB) and back with
// DataCopyPad; DataCopyPadExtend (ge/compiler/graph/optimize/autofuse/ascendc/
// api/datacopy.h:14-40, v35/ascendc/api_regbase/datacopy.h:14-72) fills its
// DataCopyExtParams so that the GM-side stride is a gap in bytes and the
// UB-side stride a gap in 32-byte blocks, and pads each GM->UB block in Normal
// mode to a 32-byte boundary with DataCopyPadExtParams{true, 0, 0, 0}.  On the
// GPU the "UB" is a device buffer laid out exactly as the UB would hold the
// tile, so a caller that ports such a kernel keeps its offsets.
//
// A GM -> UB transfer is the strided copy of the blocks into their slots
// (copy.cu picks the kernel) followed, when padding values are asked for, by
// pad_fill_kernel, which writes only the padding bytes of every slot.  A UB ->
// GM transfer is the strided copy alone.  Both are HBM-bound: the copy moves
// 2 x blockCount x blockLen bytes, the fill writes the padding bytes once.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "copy.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;

uint64_t round_up32(uint64_t x) { return (x + 31) / 32 * 32; }

// The padding bytes of every slot: slot i starts at ub + i*pitch and holds
// `lead` padding bytes, the block's `len` data bytes, then padding up to
// `slot` bytes.  Padding byte at slot offset o holds byte (o % eb) of value.
// Threads past count*per_slot write the `tail` bytes after the last slot
// (Compact mode rounds the whole transfer up to 32 bytes).
__global__ void __launch_bounds__(kThreads) pad_fill_kernel(uint8_t *__restrict__ ub,
                                                            uint32_t count, uint32_t pad_per_slot,
                                                            FastDiv per_slot, uint64_t pitch,
                                                            uint32_t lead, uint32_t len,
                                                            uint32_t slot, uint32_t tail,
                                                            uint64_t value, uint32_t eb) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  // pad_per_slot may be 0 (only the tail is written); per_slot divides by it
  // only for t < body, which is then empty.
  const uint64_t body = (uint64_t)count * pad_per_slot;
  const uint64_t total = body + tail;
  for (uint64_t t = (uint64_t)blockIdx.x * kThreads + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * kThreads) {
    uint64_t at;
    uint32_t o;
    if (t < body) {
      const uint32_t i = per_slot.div((uint32_t)t);
      const uint32_t k = (uint32_t)t - i * per_slot.d;
      o = k < lead ? k : k + len;
      at = (uint64_t)i * pitch + o;
    } else {
      at = (uint64_t)(count - 1) * pitch + slot + (t - body);
      o = (uint32_t)(at % eb);  // the slot base is element aligned
    }
    ub[at] = (uint8_t)(value >> (8 * (o % eb)));
  }
}

bool valid_eb(uint32_t eb) { return eb == 1 || eb == 2 || eb == 4 || eb == 8; }

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_copy_pad_gm_to_ub(void *ub, const void *gm, const DcopyExtParams *p,
                                       const DcopyPadParams *pad, int32_t mode,
                                       dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!p || !pad) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_gm_to_ub: params is NULL");
  if (mode != DCOPY_PAD_NORMAL && mode != DCOPY_PAD_COMPACT)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_gm_to_ub: mode %d", mode);
  const uint32_t eb = pad->elemBytes;
  if (!valid_eb(eb))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_gm_to_ub: elemBytes %u not 1, 2, 4 or 8",
                     eb);
  const uint64_t count = p->blockCount, len = p->blockLen;
  if (len % eb)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "copy_pad_gm_to_ub: blockLen %llu is not a whole number of %u-byte elements",
                     (unsigned long long)len, eb);
  const uint64_t lead = (uint64_t)pad->leftPadding * eb, trail = (uint64_t)pad->rightPadding * eb;
  if (lead > 32 || trail > 32)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "copy_pad_gm_to_ub: left/right padding of %llu/%llu bytes exceeds 32",
                     (unsigned long long)lead, (unsigned long long)trail);
  if (!count || !len) return DCOPY_OK;
  if (p->srcStride > (1ull << 48) || p->dstStride > (1ull << 43))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_gm_to_ub: stride beyond 2^48 bytes");
  const uint64_t used = lead + len + trail;
  const uint64_t slot = mode == DCOPY_PAD_NORMAL ? round_up32(used) : used;
  const uint64_t gm_pitch = len + p->srcStride, ub_pitch = slot + p->dstStride * 32;
  uint64_t gm_span = 0, ub_end = 0;
  int rc = block_span(count, gm_pitch, len, &gm_span, "copy_pad_gm_to_ub src");
  if (!rc) rc = block_span(count, ub_pitch, slot, &ub_end, "copy_pad_gm_to_ub dst");
  if (rc) return rc;
  const uint64_t ub_span = mode == DCOPY_PAD_NORMAL ? ub_end : round_up32(ub_end);
  rc = check_device_span(gm, gm_span, "copy_pad_gm_to_ub src");
  if (!rc) rc = check_device_span(ub, ub_span, "copy_pad_gm_to_ub dst");
  if (!rc) rc = check_disjoint(gm, gm_span, ub, ub_span, "copy_pad_gm_to_ub");
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = copy2d(static_cast<uint8_t *>(ub) + lead, gm, count, len, gm_pitch, ub_pitch, s);
  if (rc || !pad->isPad) return rc;
  const uint64_t per_slot = slot - len, tail = ub_span - ub_end;
  if (per_slot == 0 && tail == 0) return DCOPY_OK;
  if (count * per_slot >= (1ull << 32))
    return set_error(DCOPY_ERR_UNSUPPORTED, "copy_pad_gm_to_ub: %llu padding bytes",
                     (unsigned long long)(count * per_slot));
  const uint64_t total = count * per_slot + tail;
  const unsigned grid =
      (unsigned)std::min<uint64_t>((total + kThreads - 1) / kThreads, (uint64_t)sm_count() * 8);
  // With no padding per slot the divisor is unused (only tail threads run).
  const FastDiv div((uint32_t)(per_slot ? per_slot : 1));
  return launch(pad_fill_kernel, grid, dim3(kThreads), 0, s, "pad_fill_kernel",
                static_cast<uint8_t *>(ub), (uint32_t)count, (uint32_t)per_slot, div, ub_pitch,
                (uint32_t)lead, (uint32_t)len, (uint32_t)slot, (uint32_t)tail,
                pad->paddingValue, eb);
  DCOPY_API_END
}

extern "C" int dcopy_copy_pad_ub_to_gm(void *gm, const void *ub, const DcopyExtParams *p,
                                       int32_t mode, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!p) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_ub_to_gm: params is NULL");
  if (mode != DCOPY_PAD_NORMAL && mode != DCOPY_PAD_COMPACT)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_ub_to_gm: mode %d", mode);
  const uint64_t count = p->blockCount, len = p->blockLen;
  if (!count || !len) return DCOPY_OK;
  if (p->srcStride > (1ull << 43) || p->dstStride > (1ull << 48))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_pad_ub_to_gm: stride beyond 2^48 bytes");
  const uint64_t slot = mode == DCOPY_PAD_NORMAL ? round_up32(len) : len;
  const uint64_t ub_pitch = slot + p->srcStride * 32, gm_pitch = len + p->dstStride;
  uint64_t ub_span = 0, gm_span = 0;
  int rc = block_span(count, ub_pitch, len, &ub_span, "copy_pad_ub_to_gm src");
  if (!rc) rc = block_span(count, gm_pitch, len, &gm_span, "copy_pad_ub_to_gm dst");
  if (!rc) rc = check_device_span(ub, ub_span, "copy_pad_ub_to_gm src");
  if (!rc) rc = check_device_span(gm, gm_span, "copy_pad_ub_to_gm dst");
  if (!rc) rc = check_disjoint(ub, ub_span, gm, gm_span, "copy_pad_ub_to_gm");
  if (rc) return rc;
  return copy2d(gm, ub, count, len, ub_pitch, gm_pitch, reinterpret_cast<cudaStream_t>(stream));
  DCOPY_API_END
}

// DataCopyPadExtend's unit conversions (ascendc/api/datacopy.h:16-22, 31-37):
// lengths and GM strides are elements times sizeof(T); UB strides are elements
// divided (rounding down) by align_num = 32 / sizeof(T).
extern "C" int dcopy_datacopy_pad_extend_load(void *ub, const void *gm, uint32_t elem_bytes,
                                              uint32_t block_count, uint32_t block_len,
                                              uint32_t src_stride, uint32_t dst_stride,
                                              int32_t mode, dcopy_stream_t stream) {
  if (!valid_eb(elem_bytes) || (uint64_t)block_len * elem_bytes > 0xFFFFFFFFull) {
    clear_error();
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "datacopy_pad_extend: elem_bytes %u / block_len %u out of range", elem_bytes,
                     block_len);
  }
  const uint32_t align_num = 32 / elem_bytes;
  const DcopyExtParams p{block_count, block_len * elem_bytes, (uint64_t)src_stride * elem_bytes,
                         (uint64_t)(dst_stride / align_num)};
  const DcopyPadParams pad{1, 0, 0, 0, elem_bytes, 0};  // DataCopyPadExtParams{true, 0, 0, 0}
  return dcopy_copy_pad_gm_to_ub(ub, gm, &p, &pad, mode, stream);
}

extern "C" int dcopy_datacopy_pad_extend_store(void *gm, const void *ub, uint32_t elem_bytes,
                                               uint32_t block_count, uint32_t block_len,
                                               uint32_t src_stride, uint32_t dst_stride,
                                               int32_t mode, dcopy_stream_t stream) {
  if (!valid_eb(elem_bytes) || (uint64_t)block_len * elem_bytes > 0xFFFFFFFFull) {
    clear_error();
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "datacopy_pad_extend: elem_bytes %u / block_len %u out of range", elem_bytes,
                     block_len);
  }
  const uint32_t align_num = 32 / elem_bytes;
  const DcopyExtParams p{block_count, block_len * elem_bytes, (uint64_t)(src_stride / align_num),
                         (uint64_t)dst_stride * elem_bytes};
  return dcopy_copy_pad_ub_to_gm(gm, ub, &p, mode, stream);
}
