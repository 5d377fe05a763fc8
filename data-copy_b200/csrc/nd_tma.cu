// DataCopyNddma boxes through TMA tensor maps (cp.async.bulk.tensor) on sm_100a.
// Selected with dcopy_set_nd_tma (or DCOPY_ND_TMA=1); off by default, because on
// B200 the load/store row kernel measured as fast or faster on every box tried
// (TMA 3.3-5.9 TB/s against 3.4-6.4 TB/s).
//
// A 3- to 5-D box copy (v35/ascendc/api_regbase/datacopy_nddma.h:15-29) whose
// innermost axis is contiguous on both sides and whose other strides are
// 16-byte multiples is described by two tensor maps of the same shape: the
// source view and the destination view.  The box is cut into TMA boxes of at
// most 16 KiB (256 elements per axis at most); one thread per CTA drives a
// kStages-deep pipeline: a tensor load fills a shared-memory stage (completion
// on an mbarrier, transaction-counted), a tensor store drains it (bulk group),
// and the stage is refilled once that store has read it.  Edge boxes that run
// past the view are clipped by the hardware (loads fill, stores skip).
// Every x coordinate is a multiple of the box's x extent, whose byte size is a
// multiple of 16, as tiled tensor copies require.  No multicast; both views are
// this GPU's memory.  Every mbarrier wait is bounded; a give-up is recorded in
// a device word that dcopy_tma_error reads, after the kernel drains (bounded)
// the loads it issued.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

#ifndef DCOPY_TMA_STAGES
#define DCOPY_TMA_STAGES 4
#endif
#ifndef DCOPY_TMA_STAGE_KIB
#define DCOPY_TMA_STAGE_KIB 16
#endif
#ifndef DCOPY_TMA_CTAS_PER_SM
#define DCOPY_TMA_CTAS_PER_SM 3
#endif
#ifndef DCOPY_TMA_UNIT
#define DCOPY_TMA_UNIT 8  // TMA element: 0 the library element, 8 always 8-byte units
#endif
#ifndef DCOPY_TMA_SHORT_BURSTS
// 1: with the TMA paths selected, gapped 2-D bursts of 16 to 112 bytes (whole
// 16-byte granules) move as 2-D tensor copies.  Measured on B200 (256 MiB moved,
// against the load/store kernel): 32 B bursts with 4x / 16x gaps +5 % / +4 %,
// 32 B with 1x gaps and every 64 B point -4 to -6 %; so by default only the
// first kind takes it (DCOPY_TMA_SHORT_AUTO_MAX).
#define DCOPY_TMA_SHORT_BURSTS 1
#endif
#ifndef DCOPY_TMA_SHORT_AUTO_MAX
// Without the TMA paths selected, bursts of at most this many bytes whose source
// gap is at least 4x the burst still take the tensor copy: the points where it
// measured ahead.  bench.py's config 3 sweep (CUDA graph replay, 256 MiB moved,
// two runs each): 32 B / 4x 4008 vs 3832-3844 GB/s, 32 B / 16x 3505-3533 vs
// 3431-3458; every other point unchanged.  0: only with the paths selected.
#define DCOPY_TMA_SHORT_AUTO_MAX 32
#endif
#ifndef DCOPY_TMA_SHORT_PROMOTION
// L2 promotion of those loads: 64 (half lines).  No promotion measured 25-30 %
// slower on 32 B bursts with 4x / 16x gaps.
#define DCOPY_TMA_SHORT_PROMOTION 64
#endif
constexpr int kStages = DCOPY_TMA_STAGES;
constexpr uint32_t kStageBytes = DCOPY_TMA_STAGE_KIB * 1024;
constexpr uint32_t kWaitIters = 1u << 22;  // try_wait suspends ~us per call: seconds in total
constexpr int kMaxRank = 5;

__device__ uint32_t g_tma_error;

struct TmaGeom {
  uint32_t rank;                // 1..5, innermost first
  uint32_t box[kMaxRank];       // TMA box extents
  uint32_t nbox[kMaxRank];      // boxes per axis
  FastDiv f_nbox[kMaxRank];
  uint32_t box_bytes;
  uint64_t nboxes;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  for (uint32_t it = 0; it < kWaitIters; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

template <int R>
__device__ __forceinline__ void tma_load(void *smem, const CUtensorMap *map, const int32_t *c,
                                         uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  if constexpr (R == 1)
    asm volatile(
        "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2}], [%3];" ::"r"(smem_u32(smem)), "l"(m), "r"(c[0]), "r"(smem_u32(bar))
        : "memory");
  else if constexpr (R == 2)
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem)), "l"(m), "r"(c[0]), "r"(c[1]),
        "r"(smem_u32(bar))
        : "memory");
  else if constexpr (R == 3)
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem)), "l"(m), "r"(c[0]), "r"(c[1]),
        "r"(c[2]), "r"(smem_u32(bar))
        : "memory");
  else if constexpr (R == 4)
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem)), "l"(m), "r"(c[0]),
        "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(smem_u32(bar))
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(smem)), "l"(m), "r"(c[0]),
        "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(smem_u32(bar))
        : "memory");
}

template <int R>
__device__ __forceinline__ void tma_store(const CUtensorMap *map, const int32_t *c,
                                          const void *smem) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  if constexpr (R == 1)
    asm volatile("cp.async.bulk.tensor.1d.global.shared::cta.tile.bulk_group [%0, {%1}], [%2];" ::
                     "l"(m),
                 "r"(c[0]), "r"(smem_u32(smem))
                 : "memory");
  else if constexpr (R == 2)
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(m),
        "r"(c[0]), "r"(c[1]), "r"(smem_u32(smem))
        : "memory");
  else if constexpr (R == 3)
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::
            "l"(m),
        "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(smem_u32(smem))
        : "memory");
  else if constexpr (R == 4)
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::
            "l"(m),
        "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(smem_u32(smem))
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}],"
        " [%6];" ::"l"(m),
        "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(smem_u32(smem))
        : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Box k of this CTA -> its element coordinates (innermost first).
__device__ __forceinline__ void box_coords(const TmaGeom &g, uint64_t box, int32_t *c) {
  uint32_t rem = (uint32_t)box;  // nboxes < 2^31 (checked on the host)
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d < (int)g.rank) {
      const uint32_t q = g.f_nbox[d].div(rem);
      c[d] = (int32_t)((rem - q * g.nbox[d]) * g.box[d]);
      rem = q;
    } else {
      c[d] = 0;
    }
  }
}

template <int R>
__global__ void __launch_bounds__(32) nd_tma_kernel(const __grid_constant__ CUtensorMap src_map,
                                                    const __grid_constant__ CUtensorMap dst_map,
                                                    TmaGeom g) {
  extern __shared__ __align__(1024) uint8_t tma_stage[];
  __shared__ __align__(8) uint64_t bars[kStages];
  pdl_trigger_at_entry();
  if (threadIdx.x != 0) return;
  for (int i = 0; i < kStages; ++i)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[i])));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  pdl_wait();
  pdl_launch_dependents();
  const uint64_t mine =
      blockIdx.x < g.nboxes ? (g.nboxes - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  auto box_of = [&](uint64_t k) { return blockIdx.x + k * gridDim.x; };
  int32_t c[kMaxRank];
  const uint64_t pro = mine < (uint64_t)kStages ? mine : (uint64_t)kStages;
  for (uint64_t k = 0; k < pro; ++k) {
    box_coords(g, box_of(k), c);
    tma_load<R>(tma_stage + k * kStageBytes, &src_map, c, &bars[k], g.box_bytes);
  }
  uint64_t issued = pro, k = 0;
  bool ok = true;
  for (; k < mine; ++k) {
    const int st = (int)(k % kStages);
    if (!mbar_wait_bounded(&bars[st], (uint32_t)((k / kStages) & 1))) {
      ok = false;
      break;
    }
    box_coords(g, box_of(k), c);
    tma_store<R>(&dst_map, c, tma_stage + st * kStageBytes);
    // Refill the stage of box k-1 once its store has read it (at most the store
    // of box k may still be reading).
    if (k >= 1 && issued < mine) {
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      const int prev = (int)((k - 1) % kStages);
      box_coords(g, box_of(issued), c);
      tma_load<R>(tma_stage + prev * kStageBytes, &src_map, c, &bars[prev], g.box_bytes);
      ++issued;
    }
  }
  if (!ok) {
    atomicExch(&g_tma_error, 1u);
    for (uint64_t j = k; j < issued; ++j)  // drain the loads still in flight (bounded)
      (void)mbar_wait_bounded(&bars[j % kStages], (uint32_t)((j / kStages) & 1));
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

typedef CUresult (*PfnEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PfnEncodeTiled encode_fn() {
  static PfnEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnEncodeTiled>(p);
  });
  return fn;
}

template <int R>
int launch_rank(const CUtensorMap &sm, const CUtensorMap &dm, const TmaGeom &g, cudaStream_t s) {
  static std::atomic<bool> configured[128];
  const int dev = current_device();
  const size_t smem = (size_t)kStages * kStageBytes;
  if (dev >= 0 && dev < 128 && !configured[dev].load()) {
    const cudaError_t e = cudaFuncSetAttribute(nd_tma_kernel<R>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    configured[dev] = true;
  }
  const uint64_t grid =
      std::min<uint64_t>(g.nboxes, (uint64_t)sm_count() * DCOPY_TMA_CTAS_PER_SM);
  return launch(nd_tma_kernel<R>, (unsigned)std::max<uint64_t>(1, grid), dim3(32), smem, s,
                "nd_tma_kernel", sm, dm, g);
}

// Process-wide path selection: -1 until first read (then DCOPY_ND_TMA, default 0).
std::atomic<int> g_tma_selected{-1};

int initial_selection() {
  const char *e = std::getenv("DCOPY_ND_TMA");
  return e && std::atoi(e) != 0 ? 1 : 0;
}

bool tma_selected() {
  int v = g_tma_selected.load(std::memory_order_relaxed);
  if (v < 0) {
    int expected = -1;
    g_tma_selected.compare_exchange_strong(expected, initial_selection());
    v = g_tma_selected.load(std::memory_order_relaxed);
  }
  return v != 0;
}

}  // namespace

namespace {

// The tensor-copy path for one box whose views allow it (*taken = true), with
// the L2 promotion of short rows given by short_promotion.
int tma_box_copy(void *dst, const void *src, int ndim, const uint64_t *sizes,
                 const int64_t *src_strides, const int64_t *dst_strides, uint32_t eb,
                 dcopy_stream_t stream, CUtensorMapL2promotion short_promotion, bool *taken) {
  *taken = false;
  // Conditions of a tiled tensor copy on both views (checked, else the caller
  // takes its load/store kernels): 16-byte aligned bases, unit innermost stride,
  // 16-byte multiple strides, rows of whole 16-byte granules, local memory.
  if (ndim < 1 || ndim > kMaxRank) return DCOPY_OK;
  if (eb != 1 && eb != 2 && eb != 4 && eb != 8 && eb != 16) return DCOPY_OK;
  if (src_strides[ndim - 1] != 1 || dst_strides[ndim - 1] != 1) return DCOPY_OK;
  if (((uintptr_t)src | (uintptr_t)dst) % 16) return DCOPY_OK;
  // Rows must be whole 16-byte granules: a tensor store that ends inside a
  // granule writes the granule's remaining bytes too (measured: a row of 260
  // 2-byte elements also overwrote elements 260..263 of the destination pitch).
  if ((sizes[ndim - 1] * eb) % 16) return DCOPY_OK;
  for (int k = 0; k < ndim - 1; ++k)
    if (((uint64_t)src_strides[k] * eb) % 16 || ((uint64_t)dst_strides[k] * eb) % 16 ||
        (uint64_t)src_strides[k] * eb >= (1ull << 40) || (uint64_t)dst_strides[k] * eb >= (1ull << 40))
      return DCOPY_OK;
  for (int k = 0; k < ndim; ++k)
    if (sizes[k] == 0 || sizes[k] > 0x7FFFFFFFull) return DCOPY_OK;
  if (!is_local_device_memory(src) || !is_local_device_memory(dst)) return DCOPY_OK;
  PfnEncodeTiled encode = encode_fn();
  if (!encode) return DCOPY_OK;

  // TMA element: the library element, or 8-byte halves of a 16-byte element.
  // Rows are whole 16-byte granules, so 8-byte units always tile them.
  const uint32_t te = DCOPY_TMA_UNIT == 8 ? 8 : (eb == 16 ? 8 : eb);
  const CUtensorMapDataType dtype = te == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                    : te == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                    : te == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32
                                              : CU_TENSOR_MAP_DATA_TYPE_UINT64;
  const int R = ndim;
  cuuint64_t gdim[kMaxRank], sstride[kMaxRank], dstride[kMaxRank];
  cuuint32_t box[kMaxRank], estride[kMaxRank];
  TmaGeom g{};
  g.rank = (uint32_t)R;
  for (int d = 0; d < R; ++d) {  // d = 0 innermost
    const int k = ndim - 1 - d;
    gdim[d] = d == 0 ? sizes[k] * eb / te : sizes[k];
    if (d > 0) {
      sstride[d - 1] = (cuuint64_t)src_strides[k] * eb;
      dstride[d - 1] = (cuuint64_t)dst_strides[k] * eb;
    }
    estride[d] = 1;
  }
  // Box: x up to 256 elements (a multiple of 16 bytes), then the outer axes
  // while the box stays within one stage.
  const uint32_t align_elems = 16 / te;
  uint64_t bx = std::min<uint64_t>(gdim[0], 256);
  bx = bx / align_elems * align_elems;
  if (bx == 0) return DCOPY_OK;
  box[0] = (cuuint32_t)bx;
  uint64_t bytes = bx * te;
  for (int d = 1; d < R; ++d) {
    const uint64_t room = std::max<uint64_t>(1, kStageBytes / bytes);
    box[d] = (cuuint32_t)std::min<uint64_t>({gdim[d], 256, room});
    bytes *= box[d];
  }
  if (bytes > kStageBytes) return DCOPY_OK;
  uint64_t nboxes = 1;
  for (int d = 0; d < R; ++d) {
    g.box[d] = box[d];
    g.nbox[d] = (uint32_t)((gdim[d] + box[d] - 1) / box[d]);
    g.f_nbox[d] = FastDiv(g.nbox[d]);
    nboxes *= g.nbox[d];
  }
  if (nboxes >= (1ull << 31)) return DCOPY_OK;
  g.nboxes = nboxes;
  g.box_bytes = (uint32_t)bytes;
  // L2 sector promotion: rows shorter than a 128-byte line fill 64-byte half
  // lines (measured on B200: 64 B rows with 64 B gaps 3970 -> 5140 GB/s); longer
  // rows fill 256-byte spans.
  const CUtensorMapL2promotion kPromotion =
      sizes[ndim - 1] * eb < 128 ? short_promotion : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  CUtensorMap sm, dm;
  if (encode(&sm, dtype, (cuuint32_t)R, const_cast<void *>(src), gdim, sstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             kPromotion, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      encode(&dm, dtype, (cuuint32_t)R, dst, gdim, dstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             kPromotion, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DCOPY_OK;  // the driver refused the views: the load/store path copies them
  *taken = true;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (R) {
    case 1: return launch_rank<1>(sm, dm, g, s);
    case 2: return launch_rank<2>(sm, dm, g, s);
    case 3: return launch_rank<3>(sm, dm, g, s);
    case 4: return launch_rank<4>(sm, dm, g, s);
    default: return launch_rank<5>(sm, dm, g, s);
  }
}

}  // namespace

bool tma_paths_selected() { return tma_selected(); }

bool encode_tiled_map(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                      const uint64_t *dims, const uint64_t *strides, const uint32_t *box,
                      CUtensorMapL2promotion promotion) {
  PfnEncodeTiled encode = encode_fn();
  if (!encode || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], st[5];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  return encode(map, dtype, rank, base, d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, promotion,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int nd_copy_tma(void *dst, const void *src, int ndim, const uint64_t *sizes,
                const int64_t *src_strides, const int64_t *dst_strides, uint32_t eb,
                dcopy_stream_t stream, bool *taken) {
  *taken = false;
  if (!tma_selected()) return DCOPY_OK;
  return tma_box_copy(dst, src, ndim, sizes, src_strides, dst_strides, eb, stream,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_64B, taken);
}

int tma_short_bursts(void *dst, const void *src, uint64_t rows, uint64_t row_bytes,
                     uint64_t src_pitch, uint64_t dst_pitch, cudaStream_t s, bool *taken) {
  *taken = false;
  const bool automatic = row_bytes <= DCOPY_TMA_SHORT_AUTO_MAX && src_pitch >= 5 * row_bytes;
  if (!DCOPY_TMA_SHORT_BURSTS || !(tma_selected() || automatic) || row_bytes >= 128 ||
      row_bytes % 16 || src_pitch == row_bytes)
    return DCOPY_OK;
  if (rows < 2 || rows > 0x7FFFFFFFull) return DCOPY_OK;
  const uint64_t sizes[2] = {rows, row_bytes};
  const int64_t ss[2] = {(int64_t)src_pitch, 1}, ds[2] = {(int64_t)dst_pitch, 1};
  return tma_box_copy(dst, src, 2, sizes, ss, ds, 1, reinterpret_cast<dcopy_stream_t>(s),
                      DCOPY_TMA_SHORT_PROMOTION == 0 ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                                                     : CU_TENSOR_MAP_L2_PROMOTION_L2_64B,
                      taken);
}

}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_set_nd_tma(int enable, int *previous) {
  DCOPY_API_BEGIN
  const int was = tma_selected() ? 1 : 0;
  g_tma_selected.store(enable ? 1 : 0);
  if (previous) *previous = was;
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_tma_error(uint32_t *flag) {
  DCOPY_API_BEGIN
  if (!flag) return set_error(DCOPY_ERR_PARAM_INVALID, "tma_error: NULL");
  uint32_t zero = 0;
  DCOPY_CUDA_TRY(cudaMemcpyFromSymbol(flag, g_tma_error, sizeof(uint32_t)));
  DCOPY_CUDA_TRY(cudaMemcpyToSymbol(g_tma_error, &zero, sizeof(uint32_t)));
  const int rc = bulk_error_take(flag);
  return rc ? rc : fz_error_take(flag);
  DCOPY_API_END
}
