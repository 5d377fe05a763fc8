// DataCopyExt bursts through shared memory with the bulk-copy (TMA) engine.
//
// A 2-D strided copy whose bursts are whole 16-byte granules (both bases, the
// burst length and both pitches multiples of 16) moves as untiled bulk copies:
// a burst of blockLen bytes is one `cp.async.bulk` global -> shared and one
// shared -> global, cut into pieces of at most kMaxPiece bytes when longer.
// Each CTA is one warp and owns a run of consecutive pieces (kCtaBytes of
// shared memory in total); lane i issues pieces i, i + 32, ... .  All loads of
// the CTA complete on one mbarrier (one arrival per piece, each expecting its
// bytes); the lanes then issue the stores and wait for them.
//
// Design intent: the bytes in flight live in shared memory, not in registers,
// so a CTA needs 32 threads and a few registers, and a copy launch leaves most
// CTA slots of the GPU free.  Under programmatic dependent launch the next
// copy on the stream becomes resident in those slots while this one runs and
// prefetches its bursts into L2 (one bulk prefetch per piece) before it waits.
//
// Measured on B200 it loses to the load/store kernel (copy.cu): BASELINE
// config 2 (4096 bursts of 4 KiB, 16 per CUDA graph) 4736 against 5369 GB/s
// with 32 KiB per CTA (16 KiB: 4645, 64 KiB: 4239, no prefetch: 4048), and the
// 256 MiB sweep points from 512 B bursts equal or up to 5 % slower.  So it runs
// only with the TMA paths selected (dcopy_set_nd_tma), as the box kernel does.
//
// Loads read this GPU's memory only (the host checks both buffers); no
// multicast.  The mbarrier wait is bounded; a give-up is recorded in a device
// word (read through dcopy_tma_error), and the CTA then waits (bounded again)
// for the loads it issued before returning without storing.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "bulk.cuh"
#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

#ifndef DCOPY_BULK_BURSTS
#define DCOPY_BULK_BURSTS 1  // 0: never, even with the TMA paths selected
#endif
#ifndef DCOPY_BULK_CTA_KIB
#define DCOPY_BULK_CTA_KIB 32  // shared memory (bytes in flight) per CTA
#endif
#ifndef DCOPY_BULK_MIN_BURST
#define DCOPY_BULK_MIN_BURST 512  // shorter bursts keep the load/store kernels
#endif
#ifndef DCOPY_BULK_PREFETCH
#define DCOPY_BULK_PREFETCH 1
#endif

namespace dcopy {
namespace {

constexpr uint32_t kCtaBytes = DCOPY_BULK_CTA_KIB * 1024;
constexpr uint32_t kMaxPiece = 16 * 1024;

__device__ uint32_t g_bulk_error;

struct BurstPlan {
  uint64_t src_pitch, dst_pitch;  // bytes between burst starts
  uint32_t burst;                 // burst length in bytes (multiple of 16)
  uint32_t piece;                 // bytes per piece (multiple of 16); a burst's last piece may be shorter
  FastDiv per_burst;              // pieces per burst
  uint32_t total;                 // pieces in this launch
  uint32_t per_cta;               // pieces per CTA
};

// Piece j of the launch: its byte offsets in the source and destination, and
// its length.
__device__ __forceinline__ void piece_at(const BurstPlan &p, uint32_t j, uint64_t *so,
                                         uint64_t *dof, uint32_t *len) {
  const uint32_t b = p.per_burst.div(j);
  const uint32_t off = (j - b * p.per_burst.d) * p.piece;
  *so = (uint64_t)b * p.src_pitch + off;
  *dof = (uint64_t)b * p.dst_pitch + off;
  *len = min(p.piece, p.burst - off);
}

__global__ void __launch_bounds__(32) burst_bulk_kernel(uint8_t *__restrict__ dst,
                                                        const uint8_t *__restrict__ src,
                                                        BurstPlan p, bool prefetch) {
  extern __shared__ __align__(128) uint8_t stage[];
  __shared__ __align__(8) uint64_t bar;
  pdl_trigger_at_entry();
  const uint32_t lane = threadIdx.x;
  const uint32_t first = blockIdx.x * p.per_cta;
  const uint32_t n = min(p.per_cta, p.total - first);
  if (lane == 0) {
    bulk::mbar_init(&bar, n);
    bulk::mbar_init_fence();
  }
  if (DCOPY_BULK_PREFETCH && prefetch) {
    for (uint32_t i = lane; i < n; i += 32) {
      uint64_t so, dof;
      uint32_t len;
      piece_at(p, first + i, &so, &dof, &len);
      bulk::prefetch_l2(src + so, len);
    }
  }
  __syncwarp();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t i = lane; i < n; i += 32) {
    uint64_t so, dof;
    uint32_t len;
    piece_at(p, first + i, &so, &dof, &len);
    bulk::load(stage + (uint64_t)i * p.piece, src + so, len, &bar);
  }
  if (!bulk::mbar_wait_bounded(&bar, 0)) {
    if (lane == 0) atomicExch(&g_bulk_error, 1u);
    // Wait (bounded) for the loads still in flight before the CTA's shared
    // memory is released; nothing is stored.
    (void)bulk::mbar_wait_bounded(&bar, 0);
    return;
  }
  for (uint32_t i = lane; i < n; i += 32) {
    uint64_t so, dof;
    uint32_t len;
    piece_at(p, first + i, &so, &dof, &len);
    bulk::store(dst + dof, stage + (uint64_t)i * p.piece, len);
  }
  bulk::commit();
  bulk::wait_all();
}

int configure(size_t smem) {
  static std::atomic<bool> configured[128];
  const int dev = current_device();
  if (dev < 0 || dev >= 128 || configured[dev].load()) return DCOPY_OK;
  cudaError_t e =
      cudaFuncSetAttribute(burst_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(burst_bulk_kernel)");
  configured[dev] = true;
  return DCOPY_OK;
}

}  // namespace

int bulk_bursts(void *dst, const void *src, uint64_t rows, uint64_t row_bytes,
                uint64_t src_pitch, uint64_t dst_pitch, cudaStream_t s, bool *taken) {
  *taken = false;
  if (!DCOPY_BULK_BURSTS || !rows || !tma_paths_selected()) return DCOPY_OK;
  if (((uintptr_t)dst | (uintptr_t)src | row_bytes | src_pitch | dst_pitch) % 16) return DCOPY_OK;
  if (row_bytes < DCOPY_BULK_MIN_BURST || row_bytes >= (uint64_t(1) << 31)) return DCOPY_OK;
  // The engine reads and writes this GPU's memory here; peer and host buffers
  // take the load/store kernels.
  if (!is_local_device_memory(src) || !is_local_device_memory(dst)) return DCOPY_OK;
  // Bursts up to kMaxPiece are one piece; longer ones are cut into kMaxPiece
  // pieces and a shorter last one (every piece a multiple of 16 bytes).
  const uint64_t per_burst = (row_bytes + kMaxPiece - 1) / kMaxPiece;
  const uint64_t piece = std::min<uint64_t>(row_bytes, kMaxPiece);
  const uint64_t per_cta = std::max<uint64_t>(1, kCtaBytes / piece);
  const size_t smem = (size_t)(per_cta * piece);
  int rc = configure(kCtaBytes);  // smem <= kCtaBytes: per_cta * piece, piece <= kCtaBytes
  if (rc) return rc;
  *taken = true;
  // Keep every launch's piece index inside 32 bits.
  const uint64_t max_rows = std::max<uint64_t>(1, (uint64_t(1) << 31) / per_burst);
  const bool prefetch = true;  // both buffers are local (checked above)
  uint8_t *d = static_cast<uint8_t *>(dst);
  const uint8_t *sp = static_cast<const uint8_t *>(src);
  for (uint64_t r0 = 0; r0 < rows; r0 += max_rows) {
    const uint64_t nr = std::min(max_rows, rows - r0);
    BurstPlan p{};
    p.src_pitch = src_pitch;
    p.dst_pitch = dst_pitch;
    p.burst = (uint32_t)row_bytes;
    p.piece = (uint32_t)piece;
    p.per_burst = FastDiv((uint32_t)per_burst);
    p.total = (uint32_t)(nr * per_burst);
    p.per_cta = (uint32_t)per_cta;
    const unsigned grid = (unsigned)((p.total + per_cta - 1) / per_cta);
    rc = launch(burst_bulk_kernel, grid, dim3(32), smem, s, "burst_bulk_kernel",
                d + r0 * dst_pitch, sp + r0 * src_pitch, p, prefetch);
    if (rc) return rc;
  }
  return DCOPY_OK;
}

int bulk_error_take(uint32_t *flag) {
  uint32_t v = 0, zero = 0;
  DCOPY_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_bulk_error, sizeof(uint32_t)));
  DCOPY_CUDA_TRY(cudaMemcpyToSymbol(g_bulk_error, &zero, sizeof(uint32_t)));
  *flag |= v;
  return DCOPY_OK;
}

}  // namespace dcopy
