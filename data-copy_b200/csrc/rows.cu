// Rows whose length, bases or strides are not 16-byte multiples (a DataCopyNddma
// box with a contiguous innermost axis of 55 fp16 elements, a Transpose that
// keeps an odd innermost axis): every destination row is written in aligned
// 16-byte vectors, each assembled with funnel shifts from the two aligned
// 16-byte source blocks that hold its bytes.  The element kernels would move
// such rows in 1- or 2-byte units.
//
// A thread moves a run of kRun consecutive aligned 16-byte vectors of one
// destination row (a row spans at most ceil(row_bytes / 16) + 1 vectors; runs
// past its end do nothing).  All vectors of a row share one shift against the
// source's aligned blocks, so a run loads kRun + 1 blocks for kRun vectors and
// computes the row's odometer once.  Bytes outside the row are neither read
// nor written: the vector at each end of a row is stored in aligned pieces, and
// a source block is only loaded when it holds a byte the run needs, so every
// load stays inside the page of a byte the caller owns.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;
constexpr int kRowDims = 4;  // row dims (outermost first) besides the row itself
constexpr int kRun = 4;  // destination vectors per thread (one row, consecutive)

struct ShiftGeom {
  uint32_t row_bytes;
  uint32_t slots;  // runs of kRun destination vectors per row
  FastDiv f_slots;
  uint32_t nd;
  uint32_t size[kRowDims];
  FastDiv f_size[kRowDims];
  uint64_t ss[kRowDims], ds[kRowDims];  // byte strides of the row dims
  uint32_t total;                       // slots of this launch (< 2^31)
};

// The 16 bytes at byte offset `s` (0..15) of the 32 bytes a || b.
__device__ __forceinline__ uint4 shift_pair(uint4 a, uint4 b, uint32_t s) {
  uint32_t w0 = a.x, w1 = a.y, w2 = a.z, w3 = a.w, w4 = b.x, w5 = b.y, w6 = b.z, w7 = b.w;
  if (s & 8) {
    w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
  }
  if (s & 4) {
    w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
  }
  const uint32_t r = (s & 3) * 8;
  return make_uint4(__funnelshift_r(w0, w1, r), __funnelshift_r(w1, w2, r),
                    __funnelshift_r(w2, w3, r), __funnelshift_r(w3, w4, r));
}

// Bytes [lo, hi) of the aligned 16-byte vector at v, in naturally aligned
// pieces: the span is cut at the 1-, 2-, 4- and 8-byte boundaries from both
// ends, so a partial vector takes at most 4 + 4 stores instead of 15.
__device__ __forceinline__ void store_partial(uint8_t *v, uint4 x, uint32_t lo, uint32_t hi) {
  const uint64_t q0 = ((uint64_t)x.y << 32) | x.x, q1 = ((uint64_t)x.w << 32) | x.z;
  auto piece = [&](uint32_t at, uint32_t bytes) {  // at % bytes == 0, at + bytes <= 16
    const uint64_t q = at < 8 ? q0 : q1;
    const uint64_t bits = q >> ((at & 7) * 8);
    if (bytes == 8) *reinterpret_cast<uint64_t *>(v + at) = bits;
    else if (bytes == 4) *reinterpret_cast<uint32_t *>(v + at) = (uint32_t)bits;
    else if (bytes == 2) *reinterpret_cast<uint16_t *>(v + at) = (uint16_t)bits;
    else v[at] = (uint8_t)bits;
  };
  uint32_t a = lo, b = hi;
#pragma unroll
  for (uint32_t w = 1; w <= 8; w <<= 1)  // grow from the left edge to alignment w*2
    if ((a & w) && a + w <= b) {
      piece(a, w);
      a += w;
    }
#pragma unroll
  for (uint32_t w = 8; w >= 1; w >>= 1)  // then whole aligned pieces, largest first
    if (a + w <= b && (a & (w - 1)) == 0 && (b - a) >= w) {
      piece(a, w);
      a += w;
    }
#pragma unroll
  for (uint32_t w = 4; w >= 1; w >>= 1)  // what remains on the right
    if (a + w <= b) {
      piece(a, w);
      a += w;
    }
}

// Source blocks of a run: neighbouring lanes read the two halves of a 32-byte
// sector one instruction apart, so these loads allocate in L1.
template <bool kHalfLine>
__device__ __forceinline__ uint4 load_block_l1(const uint8_t *p) {
  uint4 v;
  if constexpr (kHalfLine)
    asm("ld.global.nc.L2::64B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
  else
    asm("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
  return v;
}

template <bool kHalfLine>
__device__ __forceinline__ uint4 load_block(const uint8_t *p) {
  if constexpr (kHalfLine)
    return ld_stream_half_line(reinterpret_cast<const uint4 *>(p));
  else
    return ld_stream(reinterpret_cast<const uint4 *>(p));
}

template <bool kHalfLine>
__global__ void __launch_bounds__(kThreads) rows_shift_kernel(uint8_t *__restrict__ dst,
                                                              const uint8_t *__restrict__ src,
                                                              ShiftGeom g) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < g.total; i += gridDim.x * kThreads) {
    uint32_t r = g.f_slots.div(i);
    const uint32_t k0 = (i - r * g.slots) * kRun;
    uint64_t so = 0, dof = 0;
#pragma unroll
    for (int d = kRowDims - 1; d >= 0; --d) {
      if (d < (int)g.nd) {
        const uint32_t q = g.f_size[d].div(r);
        const uint64_t idx = r - q * g.size[d];
        so += idx * g.ss[d];
        dof += idx * g.ds[d];
        r = q;
      }
    }
    const uintptr_t drow = reinterpret_cast<uintptr_t>(dst) + dof;
    const uintptr_t drow_end = drow + g.row_bytes;
    const uintptr_t v0 = (drow & ~(uintptr_t)15) + 16u * k0;
    if (v0 >= drow_end) continue;
    // Source address of the run's first destination byte (which may precede the
    // row); every vector of the run has the same shift against the source blocks.
    const uintptr_t sa0 = reinterpret_cast<uintptr_t>(src) + so + (v0 - drow);
    const uintptr_t blk0 = sa0 & ~(uintptr_t)15;
    const uint32_t sh = (uint32_t)(sa0 & 15);
    const uintptr_t run_end = v0 + 16u * kRun < drow_end ? v0 + 16u * kRun : drow_end;
    const uintptr_t need_lo = sa0 + ((v0 > drow ? v0 : drow) - v0), need_hi = sa0 + (run_end - v0);
    uint4 blk[kRun + 1];
#pragma unroll
    for (int j = 0; j <= kRun; ++j) {  // only blocks that hold a byte the run needs
      const uintptr_t b = blk0 + 16u * j;
      blk[j] = make_uint4(0, 0, 0, 0);
      if (b < need_hi && b + 16 > need_lo)
        blk[j] = load_block_l1<kHalfLine>(reinterpret_cast<const uint8_t *>(b));
    }
#pragma unroll
    for (int j = 0; j < kRun; ++j) {
      const uintptr_t v = v0 + 16u * j;
      const uintptr_t b_lo = v > drow ? v : drow;
      const uintptr_t b_hi = v + 16 < drow_end ? v + 16 : drow_end;
      if (b_lo >= b_hi) continue;
      const uint4 out = shift_pair(blk[j], blk[j + 1], sh);
      const uint32_t lo = (uint32_t)(b_lo - v), hi = (uint32_t)(b_hi - v);
      if (lo == 0 && hi == 16)
        *reinterpret_cast<uint4 *>(v) = out;
      else
        store_partial(reinterpret_cast<uint8_t *>(v), out, lo, hi);
    }
  }
}

}  // namespace

int rows_shift(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
               const int64_t *ds, int eb, cudaStream_t s) {
  if (m < 1 || m > kRowDims + 1)
    return set_error(DCOPY_ERR_UNSUPPORTED, "rows: %d dims (at most %d)", m, kRowDims + 1);
  const uint64_t row_bytes = size[m - 1] * (uint64_t)eb;
  if (row_bytes == 0) return DCOPY_OK;
  if (row_bytes >= (1ull << 30))
    return set_error(DCOPY_ERR_UNSUPPORTED, "rows: rows of %llu bytes",
                     (unsigned long long)row_bytes);
  ShiftGeom g{};
  g.row_bytes = (uint32_t)row_bytes;
  g.slots = (uint32_t)(((row_bytes + 15) / 16 + 1 + kRun - 1) / kRun);
  g.f_slots = FastDiv(g.slots);
  g.nd = (uint32_t)(m - 1);
  // Destination byte strides: given, or those of a contiguous destination.
  uint64_t dense = row_bytes;
  for (int k = m - 2; k >= 0; --k) {
    g.ds[k] = ds ? (uint64_t)ds[k] * eb : dense;
    dense *= size[k];
    g.ss[k] = (uint64_t)ss[k] * eb;
    if (size[k] > 0xFFFFFFFFull)
      return set_error(DCOPY_ERR_UNSUPPORTED, "rows: dim of %llu elements",
                       (unsigned long long)size[k]);
    g.size[k] = (uint32_t)size[k];
    g.f_size[k] = FastDiv(g.size[k]);
  }
  // NDDMA rows whose source has gaps and does not cover whole 128-byte lines:
  // half-line fills (transposes read every line whole).
  bool half_line = false;
  if (ds && m >= 2 && g.ss[m - 2] != row_bytes) {
    uint64_t lines = row_bytes | (uintptr_t)src;
    for (int k = 0; k < m - 1; ++k) lines |= g.ss[k];
    half_line = lines % 128 != 0;
  }
  // Chunk the outermost row dim so that one launch holds fewer than 2^31 slots.
  uint64_t inner = g.slots;
  for (int k = 1; k < m - 1; ++k) inner *= size[k];
  if (inner >= (1ull << 31))
    return set_error(DCOPY_ERR_UNSUPPORTED, "rows: %llu vectors per outer index",
                     (unsigned long long)inner);
  const uint64_t outer = m >= 2 ? size[0] : 1;
  const uint64_t chunk = std::max<uint64_t>(1, ((1ull << 31) - 1) / inner);
  auto kernel = half_line ? rows_shift_kernel<true> : rows_shift_kernel<false>;
  for (uint64_t o0 = 0; o0 < outer; o0 += chunk) {
    ShiftGeom c = g;
    const uint64_t n = std::min<uint64_t>(chunk, outer - o0);
    if (m >= 2) {
      c.size[0] = (uint32_t)n;
      c.f_size[0] = FastDiv(c.size[0]);
    }
    c.total = (uint32_t)(n * inner);
    const uint64_t per_cta = (uint64_t)kThreads;
    const uint32_t grid = (uint32_t)std::max<uint64_t>(1, (c.total + per_cta - 1) / per_cta);
    const uint64_t s_off = m >= 2 ? o0 * g.ss[0] : 0, d_off = m >= 2 ? o0 * g.ds[0] : 0;
    const int rc = launch(kernel, grid, dim3(kThreads), 0, s, "rows_shift_kernel",
                          static_cast<uint8_t *>(dst) + d_off,
                          static_cast<const uint8_t *>(src) + s_off, c);
    if (rc) return rc;
  }
  return DCOPY_OK;
}

}  // namespace dcopy
