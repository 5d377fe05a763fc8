// DataCopyExt between host buffers through a device staging buffer.
//
// Every byte of an end-to-end copy whose source and destination live in host
// memory crosses PCIe twice.  Measured on B200 for BASELINE config 2 (16 MiB of
// 4 KiB bursts out of a 64 MiB source): the gather kernel reading and writing
// pinned host memory directly moves 56.8 GB/s (R+W); the copy engine gathering
// the bursts host -> device (a 2-D copy reads only the bursts) while the
// previous chunk goes back device -> host on a second stream moves 75-76 GB/s
// at 6 chunks, because the two PCIe directions then overlap.  This entry point
// runs that pipeline: chunk k is gathered into staging slot k % slots on the
// caller's stream, then written to the destination (with its gaps) on the
// library's per-device return stream, either by the copy kernel (writing
// pinned host memory) or by the copy engine; the caller's stream waits for the
// last write, so the call stays stream-ordered.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "copy.cuh"
#include "internal.cuh"

namespace dcopy {
namespace {

#ifndef DCOPY_STAGED_CHUNKS
// Pipeline depth when the staging buffer holds every chunk.  Measured on B200
// (config 2, copy-engine return, two interleaved rounds of three runs): 4
// chunks 73.6-74.5 GB/s, 6 chunks 74.8-75.6, 8 chunks 72.6-73.3, 16 chunks
// 52.8-54.2.  Each chunk costs about 14 us of device time beyond its bytes
// (host enqueue stays at 25-90 us per call against 445-635 us on the device),
// which outweighs the shorter pipeline fill past 6 chunks.
#define DCOPY_STAGED_CHUNKS 6
#endif

// One non-blocking return stream per device, created on first use.
cudaStream_t return_stream(int dev, int *rc) {
  static std::mutex mu;
  static cudaStream_t streams[128] = {};
  *rc = DCOPY_OK;
  if (dev < 0 || dev >= 128) {
    *rc = set_error(DCOPY_ERR_UNSUPPORTED, "staged copy: device %d", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!streams[dev]) {
    const cudaError_t e = cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      streams[dev] = nullptr;
      *rc = cuda_fail(e, "cudaStreamCreateWithFlags");
      return nullptr;
    }
  }
  return streams[dev];
}

#ifndef DCOPY_STAGED_EVENT_POOL
#define DCOPY_STAGED_EVENT_POOL 1  // 0: create and destroy a call's events every call
#endif

// The events a call enqueues with.  cudaStreamWaitEvent binds to the record of
// the event that precedes it, and a later cudaEventRecord does not change a wait
// already enqueued, so a call needs its events only while it enqueues: it takes
// them from its device's pool and puts them back before returning, and the next
// call (any thread) may re-record them while this call's copies still run.  A
// pool belongs to one CUDA context; after a device reset (a new context id) the
// old handles, which died with their context, are dropped.  Without a context
// id (a driver lacking cuCtxGetId) the events are created and destroyed per call.
struct EventPool {
  std::mutex mu;
  unsigned long long ctx = 0;
  std::vector<cudaEvent_t> idle;
};
EventPool g_event_pools[128];

class CallEvents {
 public:
  CallEvents() = default;
  CallEvents(const CallEvents &) = delete;
  CallEvents &operator=(const CallEvents &) = delete;
  ~CallEvents() {
    if (pool_) {
      std::lock_guard<std::mutex> lock(pool_->mu);
      if (pool_->ctx == ctx_) {
        pool_->idle.insert(pool_->idle.end(), ev_.begin(), ev_.end());
        return;
      }
    }
    for (cudaEvent_t e : ev_) cudaEventDestroy(e);
  }
  // n events of the current device into ev_ (pooled when the context is known).
  cudaError_t take(int dev, size_t n) {
    unsigned long long ctx = 0;
    if (DCOPY_STAGED_EVENT_POOL && dev >= 0 && dev < 128 && current_context_id(&ctx)) {
      EventPool &p = g_event_pools[dev];
      std::lock_guard<std::mutex> lock(p.mu);
      if (p.ctx != ctx) {
        p.idle.clear();
        p.ctx = ctx;
      }
      while (ev_.size() < n && !p.idle.empty()) {
        ev_.push_back(p.idle.back());
        p.idle.pop_back();
      }
      pool_ = &p;
      ctx_ = ctx;
    }
    while (ev_.size() < n) {
      cudaEvent_t e;
      const cudaError_t rc = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (rc != cudaSuccess) return rc;
      ev_.push_back(e);
    }
    return cudaSuccess;
  }
  cudaEvent_t operator[](size_t i) const { return ev_[i]; }

 private:
  std::vector<cudaEvent_t> ev_;
  EventPool *pool_ = nullptr;
  unsigned long long ctx_ = 0;
};

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_copy_ext_staged(void *dst, const void *src, const DcopyExtParams *p,
                                     void *staging, uint64_t staging_bytes, int32_t flags,
                                     dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!p) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_staged: params is NULL");
  if (flags & ~DCOPY_STAGED_COPY_ENGINE_RETURN)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_staged: unknown flags 0x%x", flags);
  const uint64_t rows = p->blockCount, len = p->blockLen;
  if (!rows || !len) return DCOPY_OK;
  if (p->srcStride > (1ull << 48) || p->dstStride > (1ull << 48))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_staged: stride beyond 2^48 bytes");
  if (!dst || !src || !staging)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_staged: NULL buffer");
  const uint64_t sp = len + p->srcStride, dp = len + p->dstStride;
  uint64_t src_span = 0, dst_span = 0;
  int rc = block_span(rows, sp, len, &src_span, "copy_ext_staged src");
  if (!rc) rc = block_span(rows, dp, len, &dst_span, "copy_ext_staged dst");
  if (rc) return rc;
  // The staging buffer is device memory of the current device; the destination
  // must be pinned for the kernel to write it (the copy engine takes any).
  rc = check_device_span(staging, std::min<uint64_t>(staging_bytes, rows * len),
                         "copy_ext_staged staging");
  if (rc) return rc;
  if (!is_local_device_memory(staging))
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "copy_ext_staged: staging must be device memory of the current device");
  const bool ce_return = (flags & DCOPY_STAGED_COPY_ENGINE_RETURN) != 0;
  if (!ce_return) {
    rc = check_device_span(dst, dst_span, "copy_ext_staged dst");
    if (rc) return rc;
  }
  rc = check_disjoint(src, src_span, dst, dst_span, "copy_ext_staged");
  if (rc) return rc;
  // Chunks: DCOPY_STAGED_CHUNKS when the staging buffer holds them all, else as
  // many rows per chunk as lets two slots alternate.
  uint64_t chunk_rows = (rows + DCOPY_STAGED_CHUNKS - 1) / DCOPY_STAGED_CHUNKS;
  uint64_t slots = staging_bytes / std::max<uint64_t>(1, chunk_rows * len);
  if (slots < DCOPY_STAGED_CHUNKS && slots < 2) {
    chunk_rows = staging_bytes / (2 * len);
    slots = 2;
  }
  if (chunk_rows == 0)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "copy_ext_staged: staging of %llu bytes holds fewer than two bursts of %llu",
                     (unsigned long long)staging_bytes, (unsigned long long)len);
  slots = std::min<uint64_t>(slots, (rows + chunk_rows - 1) / chunk_rows);
  const uint64_t nchunks = (rows + chunk_rows - 1) / chunk_rows;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaStream_t r = return_stream(current_device(), &rc);
  if (rc) return rc;
  // Event 0 hands one point of a stream to the other stream (each record is
  // waited on at once, so one event serves every hand-over); event 1 + j marks
  // slot j written back (free), waited on by the gather that reuses the slot.
  CallEvents ev;
  DCOPY_CUDA_TRY(ev.take(current_device(), 1 + slots));
  const cudaEvent_t handover = ev[0];
  // The return stream starts after everything already on the caller's stream.
  DCOPY_CUDA_TRY(cudaEventRecord(handover, s));
  DCOPY_CUDA_TRY(cudaStreamWaitEvent(r, handover, 0));
  const uint8_t *sb = static_cast<const uint8_t *>(src);
  uint8_t *db = static_cast<uint8_t *>(dst);
  uint8_t *stage = static_cast<uint8_t *>(staging);
  int err = DCOPY_OK;
  for (uint64_t k = 0; k < nchunks && !err; ++k) {
    const uint64_t r0 = k * chunk_rows, n = std::min(chunk_rows, rows - r0);
    uint8_t *slot = stage + (k % slots) * chunk_rows * len;
    const cudaEvent_t freed = ev[1 + k % slots];
    if (k >= slots) DCOPY_CUDA_TRY(cudaStreamWaitEvent(s, freed, 0));
    DCOPY_CUDA_TRY(cudaMemcpy2DAsync(slot, len, sb + r0 * sp, sp, len, n,
                                     cudaMemcpyHostToDevice, s));
    DCOPY_CUDA_TRY(cudaEventRecord(handover, s));
    DCOPY_CUDA_TRY(cudaStreamWaitEvent(r, handover, 0));
    if (ce_return) {
      DCOPY_CUDA_TRY(cudaMemcpy2DAsync(db + r0 * dp, dp, slot, len, len, n,
                                       cudaMemcpyDeviceToHost, r));
    } else {
      err = copy2d(db + r0 * dp, slot, n, len, len, dp, r);
    }
    if (!err) DCOPY_CUDA_TRY(cudaEventRecord(freed, r));
  }
  if (err) return err;
  // The caller's stream continues once the last chunk is back.
  DCOPY_CUDA_TRY(cudaEventRecord(handover, r));
  DCOPY_CUDA_TRY(cudaStreamWaitEvent(s, handover, 0));
  return DCOPY_OK;
  DCOPY_API_END
}
