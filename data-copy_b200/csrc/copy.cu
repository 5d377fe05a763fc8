// GM->GM copies: contiguous bursts, DataCopyExtParams strided bursts and the
// DataCopyNddma N-D box.
//
// Design (HBM-bound byte movement, no tensor cores):
//  * every thread keeps U independent loads in flight before its stores, and
//    the grid is a multiple of the SM count (8 CTAs of 256 threads per SM), so
//    each SM holds 2048 x U x 16 B of reads in flight -- well above the
//    bandwidth-latency product of one SM's share of HBM3e;
//  * the widest element (16, 8, 4, 2 or 1 bytes) that divides both base
//    addresses, the burst length and both pitches is chosen on the host, so
//    16-byte aligned bursts move as 128-bit loads/stores and anything else
//    still moves bit-exactly;
//  * a strided copy is a flat index over blockCount x elements-per-burst,
//    split with one multiply-high division (FastDiv) per element.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.cuh"
#include "copy.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 8;

#ifndef DCOPY_MIN_CTAS
#define DCOPY_MIN_CTAS 8  // linear copy: minimum CTAs per SM (caps registers at 32)
#endif
#ifndef DCOPY_MIN_CTAS_STRIDED
#define DCOPY_MIN_CTAS_STRIDED 8  // strided copy: <= 32 registers, 2048 threads per SM
#endif
#ifndef DCOPY_BALANCED
// 0: one chunk of kThreads*U elements per CTA (many CTAs).  1: one wave of
// resident CTAs with equal contiguous ranges.  Measured on B200: 0 streams at
// ~98 % of the copy peak, 1 at ~90 % (fewer, longer per-CTA streams).
#define DCOPY_BALANCED 0
#endif

#ifndef DCOPY_STRIDED_FILL
// 1: strided copies spread over every resident CTA slot when one chunk per CTA
// leaves part of the wave empty (config 2: 296 CTAs of 3552 elements instead of
// 256 of 4096).  Measured on B200 (bench.py headline, three runs each): 0.857-
// 0.858 of the copy peak against 0.860-0.861, so off.
#define DCOPY_STRIDED_FILL 0
#endif

#ifndef DCOPY_U16
#define DCOPY_U16 4  // 16-byte elements in flight per thread (linear copy)
#endif
#ifndef DCOPY_PREFETCH
#define DCOPY_PREFETCH 1  // L2-prefetch the source while waiting on the previous kernel
#endif
#ifndef DCOPY_COPY2D_SHIFT
#define DCOPY_COPY2D_SHIFT 1  // bursts of 1/2/4-byte units through the funnel-shift row kernel
#endif
#ifndef DCOPY_HALF_LINE_NO_PREFETCH
#define DCOPY_HALF_LINE_NO_PREFETCH 1
#endif
#ifndef DCOPY_STRIDED_U
#define DCOPY_STRIDED_U 4  // elements in flight per thread (strided copy)
#endif
#ifndef DCOPY_STRIDED_THREADS
// Threads per CTA of the strided copy over whole lines.  Measured on B200 (
// 16 gathers per CUDA graph): 1024 -> 5535 GB/s, 512 -> 5389, 256 -> 5372, 128 -> 5458; the
// 256 MiB sweep points unchanged.  Half-line copies (short gapped bursts) keep 256, where 1024
// cost 2 % on 64 B bursts.
#define DCOPY_STRIDED_THREADS 1024
#endif
template <bool kHalfLine>
struct StridedShape {
  static constexpr int threads = kHalfLine ? kThreads : DCOPY_STRIDED_THREADS;
};

template <typename T>
struct Unroll {
  static constexpr int value = sizeof(T) >= 16 ? DCOPY_U16 : 8;
  // Strided copies keep U 64-bit destination offsets live as well as the data.
  static constexpr int strided = DCOPY_STRIDED_U;
  static constexpr int strided_min_ctas = DCOPY_MIN_CTAS_STRIDED;
};

// Contiguous copy of `head` bytes, then `n` elements of T, then `tail` bytes.
// dst + head and src + head are aligned to sizeof(T).  CTA b copies elements
// [b*per_cta, min((b+1)*per_cta, n)).
template <typename T, int U>
__global__ void __launch_bounds__(kThreads, DCOPY_MIN_CTAS)
    linear_copy_kernel(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src, uint32_t head,
                       uint64_t n, uint32_t tail, uint64_t per_cta, bool prefetch) {
  pdl_trigger_at_entry();
  T *__restrict__ d = reinterpret_cast<T *>(dst + head);
  const T *__restrict__ s = reinterpret_cast<const T *>(src + head);
  const uint64_t begin = (uint64_t)blockIdx.x * per_cta;
  const uint64_t end = begin + per_cta < n ? begin + per_cta : n;
  if (DCOPY_PREFETCH && prefetch) {  // one per 128-byte line of this CTA's first chunk
    const uint64_t per_line = 128 / sizeof(T);
    const uint64_t i = begin + (uint64_t)threadIdx.x * per_line;
    if (threadIdx.x * per_line < (uint64_t)kThreads * U && i < end) prefetch_l2(s + i);
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint64_t base = begin + threadIdx.x; base < end; base += (uint64_t)kThreads * U) {
    T v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + (uint64_t)u * kThreads;
      if (i < end) v[u] = ld_stream(s + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + (uint64_t)u * kThreads;
      if (i < end) d[i] = v[u];
    }
  }
  if (blockIdx.x == 0) {
    if (threadIdx.x < head) dst[threadIdx.x] = src[threadIdx.x];
    if (threadIdx.x < tail) {
      const uint64_t o = head + n * sizeof(T) + threadIdx.x;
      dst[o] = src[o];
    }
  }
}

// Load-only pass over n elements of 16 bytes (plus bytes of head/tail): the
// loaded words are folded into a value stored only through `sink`, which the
// host passes as NULL, so every load stays in flight and nothing is written.
__global__ void __launch_bounds__(kThreads) linear_load_kernel(const uint8_t *__restrict__ src,
                                                               uint32_t head, uint64_t n,
                                                               uint32_t tail,
                                                               uint32_t *__restrict__ sink) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  const uint4 *s = reinterpret_cast<const uint4 *>(src + head);
  uint32_t acc = 0;
  const uint64_t tile = (uint64_t)kThreads * 4;
  for (uint64_t base = (uint64_t)blockIdx.x * tile + threadIdx.x; base < n;
       base += (uint64_t)gridDim.x * tile) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint64_t i = base + (uint64_t)u * kThreads;
      v[u] = make_uint4(0, 0, 0, 0);
      if (i < n) v[u] = ld_stream(s + i);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  if (blockIdx.x == 0) {
    if (threadIdx.x < head) acc ^= ld_stream(src + threadIdx.x);
    if (threadIdx.x < tail) acc ^= ld_stream(src + head + n * 16 + threadIdx.x);
  }
  // The host passes sink = NULL: the fold only keeps the loads alive.
  if (sink) sink[(uint64_t)blockIdx.x * kThreads + threadIdx.x] = acc;
}

// Strided copy: element i of the flat [rows x epr] index space moves from
// src + row*src_pitch + col*sizeof(T) to dst + row*dst_pitch + col*sizeof(T).
// CTA b handles elements [b*per_cta, min((b+1)*per_cta, total)).  kHalfLine:
// source loads fill 64-byte half lines of L2 (bursts that start or end inside a
// 128-byte line, with gaps between them).
template <typename T, int U, bool kHalfLine>
__global__ void __launch_bounds__(StridedShape<kHalfLine>::threads,
                      Unroll<T>::strided_min_ctas * kThreads / StridedShape<kHalfLine>::threads)
    strided_copy_kernel(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src,
                        uint32_t total, uint32_t per_cta, FastDiv epr, uint64_t src_pitch,
                        uint64_t dst_pitch, bool prefetch) {
  constexpr uint32_t kSThreads = StridedShape<kHalfLine>::threads;
  pdl_trigger_at_entry();
  const uint32_t begin = blockIdx.x * per_cta;
  const uint32_t end = begin + per_cta < total ? begin + per_cta : total;
  if (DCOPY_PREFETCH && prefetch) {  // first U elements, one prefetch per 128-byte line
    constexpr uint32_t per_line = 128 / sizeof(T) > 0 ? 128 / sizeof(T) : 1;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = begin + threadIdx.x + u * kSThreads;
      if (i < end && (threadIdx.x % per_line == 0 || i == begin)) {
        const uint32_t r = epr.div(i);
        prefetch_l2(reinterpret_cast<const T *>(src + (uint64_t)r * src_pitch) + (i - r * epr.d));
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t base = begin + threadIdx.x; base < end; base += kSThreads * U) {
    T v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * kSThreads;
      if (i < end) {
        const uint32_t r = epr.div(i);
        const T *p = reinterpret_cast<const T *>(src + (uint64_t)r * src_pitch) + (i - r * epr.d);
        if constexpr (kHalfLine)
          v[u] = ld_stream_half_line(p);
        else
          v[u] = ld_stream(p);
      }
    }
    // Destination addresses are recomputed (one multiply-high each) rather than
    // kept live, which holds the kernel at 32 registers: 8 CTAs per SM.
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * kSThreads;
      if (i < end) {
        const uint32_t r = epr.div(i);
        *(reinterpret_cast<T *>(dst + (uint64_t)r * dst_pitch) + (i - r * epr.d)) = v[u];
      }
    }
  }
}

// Grid and per-CTA range for `n` elements processed in chunks of kThreads*U.
// Balanced: one wave of resident CTAs with equal contiguous ranges (a multiple
// of kThreads elements, so warps stay aligned to 512-byte segments).
struct Split {
  unsigned grid;
  uint64_t per_cta;
};

template <typename K>
Split split_work(K kernel, uint64_t n, int U, int threads = kThreads) {
  const uint64_t chunk = (uint64_t)threads * U;
  uint64_t grid = (n + chunk - 1) / chunk;
#if DCOPY_BALANCED
  grid = std::min<uint64_t>(grid, resident_ctas(kernel, kThreads, 0));
#else
  grid = std::min<uint64_t>(grid, (uint64_t)sm_count() * kCtasPerSm * 64);
#endif
  grid = std::max<uint64_t>(grid, 1);
  uint64_t per = (n + grid - 1) / grid;
  per = (per + threads - 1) / threads * threads;
  grid = std::max<uint64_t>(1, (n + per - 1) / per);
  return {(unsigned)grid, per};
}

unsigned grid_for(uint64_t work_items, uint64_t items_per_cta) {
  const uint64_t need = (work_items + items_per_cta - 1) / items_per_cta;
  const uint64_t cap = (uint64_t)sm_count() * kCtasPerSm;
  return (unsigned)std::max<uint64_t>(1, std::min(need, cap));
}

uint32_t widest(uint64_t x) {
  if (x % 16 == 0) return 16;
  if (x % 8 == 0) return 8;
  if (x % 4 == 0) return 4;
  if (x % 2 == 0) return 2;
  return 1;
}

template <typename T>
int launch_linear(uint8_t *dst, const uint8_t *src, uint64_t bytes, cudaStream_t s) {
  constexpr int U = Unroll<T>::value;
  const uint64_t w = sizeof(T);
  uint64_t head = (w - ((uintptr_t)dst % w)) % w;
  if (head > bytes) head = bytes;
  const uint64_t n = (bytes - head) / w;
  const uint32_t tail = (uint32_t)(bytes - head - n * w);
  auto kernel = linear_copy_kernel<T, U>;
  const Split sp = split_work(kernel, std::max<uint64_t>(n, 1), U);
  return launch(kernel, sp.grid, dim3(kThreads), 0, s, "linear_copy_kernel", dst, src,
                (uint32_t)head, n, tail, sp.per_cta, is_local_device_memory(src));
}

template <typename T>
int launch_strided(uint8_t *dst, const uint8_t *src, uint64_t rows, uint64_t row_bytes,
                   uint64_t src_pitch, uint64_t dst_pitch, cudaStream_t s) {
  constexpr int U = Unroll<T>::strided;
  const uint64_t epr = row_bytes / sizeof(T);
  // Keep the flat index (and its grid-stride increments) inside 32 bits.
  const uint64_t max_rows = std::max<uint64_t>(1, (uint64_t(1) << 30) / epr);
  const FastDiv div((uint32_t)epr);
  const bool prefetch = is_local_device_memory(src);
  // Gapped bursts that do not cover whole 128-byte lines: half-line L2 fills,
  // and no L2 prefetch (a prefetch fills the whole line of every 8th element).
  const bool half_line =
      src_pitch != row_bytes && ((uintptr_t)src % 128 || row_bytes % 128 || src_pitch % 128);
  const bool prefetch_src = prefetch && !(half_line && DCOPY_HALF_LINE_NO_PREFETCH);
  for (uint64_t r0 = 0; r0 < rows; r0 += max_rows) {
    const uint64_t nr = std::min(max_rows, rows - r0);
    const uint32_t total = (uint32_t)(nr * epr);
    auto kernel = half_line ? strided_copy_kernel<T, U, true> : strided_copy_kernel<T, U, false>;
    const int threads = half_line ? StridedShape<true>::threads : StridedShape<false>::threads;
    Split sp = split_work(kernel, total, U, threads);
#if DCOPY_STRIDED_FILL
    // Spread the elements over every resident CTA slot (ranges of whole 128-byte
    // lines) when one chunk per CTA leaves part of the wave empty.
    {
      static std::atomic<int> per_sm_cache[2][128];
      const int dev = current_device();
      std::atomic<int> &cached = per_sm_cache[half_line ? 1 : 0][(dev >= 0 && dev < 128) ? dev : 0];
      int per_sm = cached.load(std::memory_order_relaxed);
      if (per_sm <= 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) !=
                cudaSuccess ||
            per_sm <= 0) {
          (void)cudaGetLastError();
          per_sm = 1;
        }
        cached.store(per_sm, std::memory_order_relaxed);
      }
      const uint64_t slots = (uint64_t)per_sm * (uint64_t)sm_count();
      if (slots > sp.grid && total > slots * 32) {
        uint64_t per = (total + slots - 1) / slots;
        per = (per + 31) / 32 * 32;
        sp.per_cta = per;
        sp.grid = (unsigned)std::max<uint64_t>(1, (total + per - 1) / per);
      }
    }
#endif
    int rc = launch(kernel, sp.grid, dim3(threads), 0, s, "strided_copy_kernel",
                    dst + r0 * dst_pitch, src + r0 * src_pitch, total, (uint32_t)sp.per_cta, div,
                    src_pitch, dst_pitch, prefetch_src);
    if (rc) return rc;
  }
  return DCOPY_OK;
}

}  // namespace

int copy_linear(void *dst, const void *src, uint64_t bytes, cudaStream_t s) {
  if (!bytes) return DCOPY_OK;
  uint8_t *d = static_cast<uint8_t *>(dst);
  const uint8_t *sp = static_cast<const uint8_t *>(src);
  const uint64_t delta = (uint64_t)((uintptr_t)d - (uintptr_t)sp);
  switch (widest(delta)) {
    case 16: return launch_linear<uint4>(d, sp, bytes, s);
    case 8: return launch_linear<uint2>(d, sp, bytes, s);
    case 4: return launch_linear<uint32_t>(d, sp, bytes, s);
    case 2: return launch_linear<uint16_t>(d, sp, bytes, s);
    default: return launch_linear<uint8_t>(d, sp, bytes, s);
  }
}

int load_linear(const void *src, uint64_t bytes, cudaStream_t s) {
  if (!bytes) return DCOPY_OK;
  const uint8_t *sp = static_cast<const uint8_t *>(src);
  uint64_t head = (16 - ((uintptr_t)sp % 16)) % 16;
  if (head > bytes) head = bytes;
  const uint64_t n = (bytes - head) / 16;
  const uint32_t tail = (uint32_t)(bytes - head - n * 16);
  uint32_t *no_sink = nullptr;
  return launch(linear_load_kernel, grid_for(std::max<uint64_t>(n, 1), (uint64_t)kThreads * 4),
                dim3(kThreads), 0, s, "linear_load_kernel", sp, (uint32_t)head, n, tail, no_sink);
}

int copy2d(void *dst, const void *src, uint64_t rows, uint64_t row_bytes, uint64_t src_pitch,
           uint64_t dst_pitch, cudaStream_t s) {
  if (!rows || !row_bytes) return DCOPY_OK;
  if (rows == 1 || (src_pitch == row_bytes && dst_pitch == row_bytes))
    return copy_linear(dst, src, rows * row_bytes, s);
  uint8_t *d = static_cast<uint8_t *>(dst);
  const uint8_t *sp = static_cast<const uint8_t *>(src);
  uint32_t w = widest((uintptr_t)d | (uintptr_t)sp | row_bytes | src_pitch | dst_pitch);
  if (row_bytes / w >= (uint64_t(1) << 30)) {  // gigantic bursts: one linear copy each
    for (uint64_t r = 0; r < rows; ++r) {
      int rc = copy_linear(d + r * dst_pitch, sp + r * src_pitch, row_bytes, s);
      if (rc) return rc;
    }
    return DCOPY_OK;
  }
  // Bursts of whole 16-byte granules from DCOPY_BULK_MIN_BURST bytes in this
  // GPU's memory: bulk copies through shared memory (bulk.cu).
  {
    bool taken = false;
    const int brc = bulk_bursts(dst, src, rows, row_bytes, src_pitch, dst_pitch, s, &taken);
    if (taken || brc) return brc;
    // Short gapped bursts (16 to 112 bytes): 2-D tensor copies (nd_tma.cu).
    const int trc = tma_short_bursts(dst, src, rows, row_bytes, src_pitch, dst_pitch, s, &taken);
    if (taken || trc) return trc;
  }
  // Bursts only 1- or 2-byte units tile, and long bursts of 4-byte units:
  // aligned 16-byte destination vectors assembled by funnel shifts (rows.cu;
  // the measured thresholds are in shift_rows_pay).
  if (DCOPY_COPY2D_SHIFT && shift_rows_pay(w, row_bytes, false) && row_bytes < (uint64_t(1) << 30) &&
      rows <= 0xFFFFFFFFull) {
    const uint64_t size[2] = {rows, row_bytes};
    const int64_t ss[2] = {(int64_t)src_pitch, 1}, ds[2] = {(int64_t)dst_pitch, 1};
    return rows_shift(dst, src, 2, size, ss, ds, 1, s);
  }
  switch (w) {
    case 16: return launch_strided<uint4>(d, sp, rows, row_bytes, src_pitch, dst_pitch, s);
    case 8: return launch_strided<uint2>(d, sp, rows, row_bytes, src_pitch, dst_pitch, s);
    case 4: return launch_strided<uint32_t>(d, sp, rows, row_bytes, src_pitch, dst_pitch, s);
    case 2: return launch_strided<uint16_t>(d, sp, rows, row_bytes, src_pitch, dst_pitch, s);
    default: return launch_strided<uint8_t>(d, sp, rows, row_bytes, src_pitch, dst_pitch, s);
  }
}

// ---- N-D box copy --------------------------------------------------------------

namespace {

constexpr int kMaxNd = 5;

struct NdDesc {
  int ndim;
  uint32_t size[kMaxNd];
  FastDiv div[kMaxNd];
  int64_t ss[kMaxNd];  // elements
  int64_t ds[kMaxNd];  // elements
};

template <typename T>
__global__ void __launch_bounds__(kThreads) nd_copy_kernel(uint8_t *__restrict__ dst,
                                                           const uint8_t *__restrict__ src,
                                                           uint32_t total, NdDesc d) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  const T *s = reinterpret_cast<const T *>(src);
  T *o = reinterpret_cast<T *>(dst);
  for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < total; i += gridDim.x * kThreads) {
    uint32_t rem = i;
    int64_t so = 0, dof = 0;
#pragma unroll
    for (int k = kMaxNd - 1; k >= 0; --k) {
      if (k < d.ndim) {
        const uint32_t q = d.div[k].div(rem);
        const uint32_t idx = rem - q * d.size[k];
        so += (int64_t)idx * d.ss[k];
        dof += (int64_t)idx * d.ds[k];
        rem = q;
      }
    }
    o[dof] = ld_stream(s + so);
  }
}

template <typename T>
int launch_nd(uint8_t *dst, const uint8_t *src, const NdDesc &desc0, cudaStream_t s) {
  // Chunk the outermost dimension so the flat index stays below 2^30.
  uint64_t inner = 1;
  for (int k = 1; k < desc0.ndim; ++k) inner *= desc0.size[k];
  if (inner >= (uint64_t(1) << 30))
    return set_error(DCOPY_ERR_UNSUPPORTED, "copy_nd: inner box of %llu elements is too large",
                     (unsigned long long)inner);
  const uint64_t chunk = std::max<uint64_t>(1, (uint64_t(1) << 30) / inner);
  for (uint64_t o0 = 0; o0 < desc0.size[0]; o0 += chunk) {
    NdDesc d = desc0;
    d.size[0] = (uint32_t)std::min<uint64_t>(chunk, desc0.size[0] - o0);
    d.div[0] = FastDiv(d.size[0]);
    const uint32_t total = (uint32_t)(d.size[0] * inner);
    int rc = launch(nd_copy_kernel<T>, grid_for(total, kThreads * 4), dim3(kThreads), 0, s,
                    "nd_copy_kernel", dst + (int64_t)o0 * desc0.ds[0] * (int64_t)sizeof(T),
                    src + (int64_t)o0 * desc0.ss[0] * (int64_t)sizeof(T), total, d);
    if (rc) return rc;
  }
  return DCOPY_OK;
}

}  // namespace

}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_copy_ext(void *dst, const void *src, const DcopyExtParams *p,
                              dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!p) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext: params is NULL");
  const uint64_t count = p->blockCount, len = p->blockLen;
  if (!count || !len) return DCOPY_OK;
  const uint64_t sp = len + p->srcStride, dp = len + p->dstStride;
  if (p->srcStride > (1ull << 48) || p->dstStride > (1ull << 48))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext: stride beyond 2^48 bytes");
  uint64_t src_span = 0, dst_span = 0;
  int rc = block_span(count, sp, len, &src_span, "copy_ext src");
  if (!rc) rc = block_span(count, dp, len, &dst_span, "copy_ext dst");
  if (!rc) rc = check_device_span(src, src_span, "copy_ext src");
  if (!rc) rc = check_device_span(dst, dst_span, "copy_ext dst");
  if (!rc) rc = check_disjoint(src, src_span, dst, dst_span, "copy_ext");
  if (rc) return rc;
  return copy2d(dst, src, count, len, sp, dp, reinterpret_cast<cudaStream_t>(stream));
  DCOPY_API_END
}

extern "C" int dcopy_copy_ext_32b(void *dst, const void *src, uint32_t blockCount,
                                  uint32_t blockLen32, uint32_t srcStride32, uint32_t dstStride32,
                                  dcopy_stream_t stream) {
  const uint64_t len = (uint64_t)blockLen32 * 32u;
  if (len > 0xFFFFFFFFull) {
    clear_error();
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_32b: blockLen %u x 32 B exceeds 4 GiB",
                     blockLen32);
  }
  DcopyExtParams p{blockCount, (uint32_t)len, (uint64_t)srcStride32 * 32u,
                   (uint64_t)dstStride32 * 32u};
  return dcopy_copy_ext(dst, src, &p, stream);
}

extern "C" int dcopy_copy_ext_loop(void *dst, const void *src, const DcopyExtParams *p,
                                   const DcopyLoopModeParams *loop, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (!p || !loop) return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_loop: params is NULL");
  if (p->srcStride > (1ull << 48) || p->dstStride > (1ull << 48) ||
      loop->loop1SrcStride > (1ull << 48) || loop->loop1DstStride > (1ull << 48) ||
      loop->loop2SrcStride > (1ull << 48) || loop->loop2DstStride > (1ull << 48))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_ext_loop: stride beyond 2^48 bytes");
  // [loop2][loop1][blockCount][blockLen] bytes; the box copy validates spans and
  // overlap and picks the kernel.
  const uint64_t sizes[4] = {loop->loop2Size, loop->loop1Size, p->blockCount, p->blockLen};
  const int64_t ss[4] = {(int64_t)loop->loop2SrcStride, (int64_t)loop->loop1SrcStride,
                         (int64_t)(p->blockLen + p->srcStride), 1};
  const int64_t ds[4] = {(int64_t)loop->loop2DstStride, (int64_t)loop->loop1DstStride,
                         (int64_t)(p->blockLen + p->dstStride), 1};
  return dcopy_copy_nd(dst, src, 4, sizes, ss, ds, 1, stream);
  DCOPY_API_END
}

extern "C" int dcopy_copy_nd(void *dst, const void *src, int ndim, const uint64_t *sizes,
                             const int64_t *src_strides, const int64_t *dst_strides,
                             uint32_t elem_bytes, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (ndim < 1 || ndim > kMaxNd || !sizes || !src_strides || !dst_strides)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_nd: ndim must be 1..%d with non-NULL arrays",
                     kMaxNd);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8 &&
      elem_bytes != 16)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "copy_nd: elem_bytes %u not in {1,2,4,8,16}",
                     elem_bytes);
  uint64_t total = 1;
  unsigned __int128 src_last = 0, dst_last = 0;  // element offset of the last element
  for (int k = 0; k < ndim; ++k) {
    if (src_strides[k] < 0 || dst_strides[k] < 0)
      return set_error(DCOPY_ERR_PARAM_INVALID, "copy_nd: negative stride in dim %d", k);
    if (dst_strides[k] == 0 && sizes[k] > 1)
      return set_error(DCOPY_ERR_PARAM_INVALID,
                       "copy_nd: dst stride 0 in dim %d would write one element twice", k);
    if (sizes[k] > 0xFFFFFFFFull)
      return set_error(DCOPY_ERR_UNSUPPORTED, "copy_nd: dim %d size beyond 2^32", k);
    total *= sizes[k];
    if (sizes[k]) {
      src_last += (unsigned __int128)(sizes[k] - 1) * (uint64_t)src_strides[k];
      dst_last += (unsigned __int128)(sizes[k] - 1) * (uint64_t)dst_strides[k];
    }
  }
  if (!total) return DCOPY_OK;
  // The kernels write every element of the box concurrently, so no two box
  // elements may share a destination.  Sorted by stride, each destination axis
  // must step past everything the axes below it cover (a layout that does not
  // interleave: dense, padded or permuted boxes).  Rarer injective interleavings
  // are refused as well.
  {
    int order[kMaxNd], m = 0;
    for (int k = 0; k < ndim; ++k)
      if (sizes[k] > 1) order[m++] = k;
    for (int j = 1; j < m; ++j)  // insertion sort by destination stride (m <= 5)
      for (int i = j; i > 0 && dst_strides[order[i]] < dst_strides[order[i - 1]]; --i)
        std::swap(order[i], order[i - 1]);
    unsigned __int128 covered = 1;  // elements from the first to the last offset so far
    for (int j = 0; j < m; ++j) {
      const int k = order[j];
      if ((unsigned __int128)(uint64_t)dst_strides[k] < covered)
        return set_error(DCOPY_ERR_PARAM_INVALID,
                         "copy_nd: dst stride %lld of dim %d is inside the %llu elements the "
                         "smaller-stride dims cover: destinations would repeat",
                         (long long)dst_strides[k], k, (unsigned long long)covered);
      covered += (unsigned __int128)(sizes[k] - 1) * (uint64_t)dst_strides[k];
    }
  }
  if ((src_last + 1) * elem_bytes >= ((unsigned __int128)1 << 62) ||
      (dst_last + 1) * elem_bytes >= ((unsigned __int128)1 << 62))
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_nd: the box spans 2^62 bytes or more");
  const uint64_t src_span = (uint64_t)((src_last + 1) * elem_bytes);
  const uint64_t dst_span = (uint64_t)((dst_last + 1) * elem_bytes);
  int rc = check_device_span(src, src_span, "copy_nd src");
  if (!rc) rc = check_device_span(dst, dst_span, "copy_nd dst");
  if (!rc) rc = check_disjoint(src, src_span, dst, dst_span, "copy_nd");
  if (rc) return rc;
  if (((uintptr_t)dst | (uintptr_t)src) % elem_bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "copy_nd: buffers not aligned to elem_bytes %u",
                     elem_bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The box is the same for any order of its axes: drop axes of size 1 and put
  // the destination's unit-stride axis last, so that the row and tile kernels
  // below see every box that has a unit-stride axis on each side.
  uint64_t cz[kMaxNd];
  int64_t cs[kMaxNd], cd[kMaxNd];
  int cn = 0;
  for (int k = 0; k < ndim; ++k)
    if (sizes[k] > 1) {
      cz[cn] = sizes[k];
      cs[cn] = src_strides[k];
      cd[cn] = dst_strides[k];
      ++cn;
    }
  if (cn == 0) {  // a single element
    cz[0] = 1;
    cs[0] = cd[0] = 1;
    cn = 1;
  }
  if (cd[cn - 1] != 1) {
    for (int k = cn - 2; k >= 0; --k)
      if (cd[k] == 1) {
        const uint64_t z = cz[k];
        const int64_t a = cs[k], b = cd[k];
        for (int j = k; j < cn - 1; ++j) {
          cz[j] = cz[j + 1];
          cs[j] = cs[j + 1];
          cd[j] = cd[j + 1];
        }
        cz[cn - 1] = z;
        cs[cn - 1] = a;
        cd[cn - 1] = b;
        break;
      }
  }
  // Merge neighbours whose strides chain on both sides (axis k steps over a
  // whole axis k+1): fewer axes, and packed boxes become plain copies.
  for (int k = cn - 2; k >= 0; --k) {
    const unsigned __int128 step_s = (unsigned __int128)(uint64_t)cs[k + 1] * cz[k + 1];
    const unsigned __int128 step_d = (unsigned __int128)(uint64_t)cd[k + 1] * cz[k + 1];
    if (step_s == (uint64_t)cs[k] && step_d == (uint64_t)cd[k] &&
        (unsigned __int128)cz[k] * cz[k + 1] <= 0xFFFFFFFFull) {
      cz[k + 1] *= cz[k];
      for (int j = k; j < cn - 1; ++j) {
        cz[j] = cz[j + 1];
        cs[j] = cs[j + 1];
        cd[j] = cd[j + 1];
      }
      --cn;
    }
  }
  ndim = cn;
  sizes = cz;
  src_strides = cs;
  dst_strides = cd;
  // Unit-stride innermost dim with <= 2 dims total: a burst copy.
  if (ndim <= 2 && src_strides[ndim - 1] == 1 && dst_strides[ndim - 1] == 1) {
    const uint64_t rows = ndim == 2 ? sizes[0] : 1;
    const uint64_t row_bytes = sizes[ndim - 1] * elem_bytes;
    const uint64_t sp = ndim == 2 ? (uint64_t)src_strides[0] * elem_bytes : row_bytes;
    const uint64_t dp = ndim == 2 ? (uint64_t)dst_strides[0] * elem_bytes : row_bytes;
    if (sp >= row_bytes && dp >= row_bytes)
      return copy2d(dst, src, rows, row_bytes, sp, dp, s);
  }
  // With the TMA path selected: 3- to 5-D boxes with 16-byte rows and strides
  // as TMA tensor copies (nd_tma.cu).
  if (ndim >= 3) {
    bool taken = false;
    const int trc = nd_copy_tma(dst, src, ndim, sizes, src_strides, dst_strides, elem_bytes,
                                stream, &taken);
    if (taken || trc) return trc;
  }
  // Other boxes with a contiguous innermost axis: rows in the widest unit that
  // divides the row length, both bases and every stride (permute.cu).
  {
    bool taken = false;
    const int rrc = rows_copy(dst, src, ndim, sizes, src_strides, dst_strides, (int)elem_bytes,
                              stream, &taken);
    if (taken || rrc) return rrc;
  }
  // A destination with contiguous rows read through a source whose unit-stride
  // axis is another one (an NCHW tensor read as an NHWC box): the Transpose tile
  // kernels, which take any destination strides but the innermost.
  {
    bool rows = dst_strides[ndim - 1] == 1, unit_src = false;
    for (int k = 0; k < ndim - 1; ++k) unit_src = unit_src || src_strides[k] == 1;
    for (int k = 0; k < ndim; ++k) rows = rows && sizes[k] <= 0x7FFFFFFFull;
    if (rows && unit_src && src_strides[ndim - 1] != 1)
      return permute_copy(dst, src, ndim, sizes, src_strides, dst_strides, (int)elem_bytes,
                          stream);
  }
  NdDesc d{};
  d.ndim = ndim;
  for (int k = 0; k < ndim; ++k) {
    d.size[k] = (uint32_t)sizes[k];
    d.div[k] = FastDiv(d.size[k]);
    d.ss[k] = src_strides[k];
    d.ds[k] = dst_strides[k];
  }
  uint8_t *o = static_cast<uint8_t *>(dst);
  const uint8_t *i = static_cast<const uint8_t *>(src);
  switch (elem_bytes) {
    case 16: return launch_nd<uint4>(o, i, d, s);
    case 8: return launch_nd<uint2>(o, i, d, s);
    case 4: return launch_nd<uint32_t>(o, i, d, s);
    case 2: return launch_nd<uint16_t>(o, i, d, s);
    default: return launch_nd<uint8_t>(o, i, d, s);
  }
  DCOPY_API_END
}
