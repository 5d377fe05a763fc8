// The standalone_datacopy kernels (datacopy_data_collection.asc:16-71) on sm_100a.
//
// Reference semantics: all four kernels move int32 A[rows, cols] into the
// transposed layout B[cols, rows] (B[c, r] = A[r, c]) one UB tile of tile_cols
// columns at a time; small/large differ only in tile size, pretranspose always
// writes B to GM, and contiguous copies the already-transposed B linearly.
//
// B200 mapping: the UB tile becomes a CTA's shared-memory tile.  The reference's
// tile size is a UB budget, not a data-layout choice -- output bytes do not
// depend on it -- so the caller's tile_cols/ub_bytes are validated exactly as
// the reference would need them and the kernel uses its own CTA tile:
//   64 rows x 32 cols of A per CTA (8 KiB), 256 threads, 8 loads in flight per
//   thread; A rows are read as 128-byte warp segments (coalesced), staged in
//   shared memory as [col][row] with one word of padding per column (so both
//   the transposing write and the row-wise read are bank-conflict-free), and B
//   rows are written as 128-byte warp segments.
// The load-only modes (store == 0) read the whole input into registers and
// write nothing to global memory: the loaded words are folded into a value that
// is stored only through a sink pointer the host always passes as NULL, which
// keeps every load in flight without an observable write.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "copy.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

#ifndef DCOPY_TRANSPOSE_PREFETCH
// L2-prefetch the first tile while waiting on the previous kernel.  Off: on B200
// it cost the transpose 3 % (5.59 -> 5.42 TB/s at 64 MiB), unlike the copies.
#define DCOPY_TRANSPOSE_PREFETCH 0
#endif

constexpr int kTileRows = 64;  // rows of A per CTA tile
constexpr int kTileCols = 32;  // cols of A per CTA tile
constexpr int kThreadsX = 32;
constexpr int kThreadsY = 8;

template <bool kStore>
__global__ void __launch_bounds__(kThreadsX *kThreadsY)
    transpose_i32_kernel(const uint32_t *__restrict__ a, uint32_t *__restrict__ b, uint32_t rows,
                         uint32_t cols, uint32_t pitch, uint32_t col_tiles, uint32_t tiles,
                         uint32_t *__restrict__ sink) {
  __shared__ uint32_t tile[kTileCols][kTileRows + 1];
  pdl_trigger_at_entry();
  const uint32_t tx = threadIdx.x, ty = threadIdx.y;
  if (DCOPY_TRANSPOSE_PREFETCH && blockIdx.x < tiles && (tx == 0 || tx == kThreadsX - 1)) {
    // L2-prefetch both ends of this warp's A row segments of the first tile.
    const uint32_t rt = blockIdx.x / col_tiles, ct = blockIdx.x - rt * col_tiles;
    const uint32_t c = ct * kTileCols + tx;
#pragma unroll
    for (int k = 0; k < kTileRows / kThreadsY; ++k) {
      const uint32_t r = rt * kTileRows + ty + k * kThreadsY;
      if (r < rows && c < cols) prefetch_l2(a + (uint64_t)r * pitch + c);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const uint32_t rt = t / col_tiles, ct = t - rt * col_tiles;
    const uint32_t r0 = rt * kTileRows, c0 = ct * kTileCols;
    const uint32_t c = c0 + tx;
    uint32_t v[kTileRows / kThreadsY];
#pragma unroll
    for (int k = 0; k < kTileRows / kThreadsY; ++k) {
      const uint32_t r = r0 + ty + k * kThreadsY;
      v[k] = 0;
      if (r < rows && c < cols) v[k] = ld_stream(a + (uint64_t)r * pitch + c);
    }
    if constexpr (!kStore) {  // load-only: fold the tile into a value only a NULL sink receives
      uint32_t acc = 0;
#pragma unroll
      for (int k = 0; k < kTileRows / kThreadsY; ++k) acc ^= v[k];
      if (sink) sink[(uint64_t)t * 256 + ty * kThreadsX + tx] = acc;
    } else {
#pragma unroll
      for (int k = 0; k < kTileRows / kThreadsY; ++k) tile[tx][ty + k * kThreadsY] = v[k];
      __syncthreads();
      // B rows c0..c0+31, each 64 consecutive ints starting at r0.
#pragma unroll
      for (int k = 0; k < kTileCols / kThreadsY; ++k) {
        const uint32_t cc = ty + k * kThreadsY;
        const uint32_t bc = c0 + cc;
#pragma unroll
        for (int h = 0; h < kTileRows / kThreadsX; ++h) {
          const uint32_t rr = tx + h * kThreadsX;
          const uint32_t br = r0 + rr;
          if (bc < cols && br < rows) b[(uint64_t)bc * rows + br] = tile[cc][rr];
        }
      }
      __syncthreads();
    }
  }
}

// B = A^T for A = rows x cols int32 with row pitch `pitch` elements (cols of a
// wider A when a column range is run on its own).
int launch_transpose(const void *x, void *y, uint32_t rows, uint32_t cols, uint32_t pitch,
                     bool store, cudaStream_t s) {
  const uint32_t col_tiles = (cols + kTileCols - 1) / kTileCols;
  const uint32_t row_tiles = (rows + kTileRows - 1) / kTileRows;
  const uint32_t tiles = col_tiles * row_tiles;
  // One tile per CTA (at most 8,256 tiles for the 64 MiB maximum).
  const uint32_t grid = std::max(1u, tiles);
  dim3 block(kThreadsX, kThreadsY);
  const uint32_t *a = static_cast<const uint32_t *>(x);
  uint32_t *b = static_cast<uint32_t *>(y);
  uint32_t *no_sink = nullptr;
  if (store)
    return launch(transpose_i32_kernel<true>, grid, block, 0, s, "transpose_i32_kernel", a, b,
                  rows, cols, pitch, col_tiles, tiles, no_sink);
  return launch(transpose_i32_kernel<false>, grid, block, 0, s, "transpose_i32_kernel", a, b, rows,
                cols, pitch, col_tiles, tiles, no_sink);
}

// Fetches the caller's tiling (host or device pointer) and validates it the way
// RunTiles needs it: rows 8..4088 and %8, cols 1..65535, store 0/1,
// 1 <= tile_cols <= cols (tile_cols == 0 would never advance c0, asc:36),
// ub_bytes >= tile_cols*rows*4 (the UB tile must hold a full tile, asc:22-25),
// ub_bytes <= 240 KiB (the UB budget, asc:114) and rows*cols*4 <= 64 MiB (asc:122).
int fetch_tiling(const DataCopyTiling *p, cudaStream_t s, DataCopyTiling *t) {
  if (!p) return set_error(DCOPY_ERR_PARAM_INVALID, "tiling is NULL");
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    attr.type = cudaMemoryTypeUnregistered;
  }
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
    DCOPY_CUDA_TRY(cudaMemcpyAsync(t, p, sizeof(*t), cudaMemcpyDeviceToHost, s));
    DCOPY_CUDA_TRY(cudaStreamSynchronize(s));
  } else {
    *t = *p;
  }
  if (!t->rows || t->rows > 4095 || t->rows % 8 || !t->cols || t->cols > 65535 || t->store > 1)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "tiling: rows %u must be 8..4088 and a multiple of 8, cols %u 1..65535, "
                     "store %u 0/1",
                     t->rows, t->cols, t->store);
  if (!t->tile_cols || t->tile_cols > t->cols)
    return set_error(DCOPY_ERR_PARAM_INVALID, "tiling: tile_cols %u must be 1..cols (%u)",
                     t->tile_cols, t->cols);
  if ((uint64_t)t->tile_cols * t->rows * 4u > t->ub_bytes || t->ub_bytes > 240u * 1024u)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "tiling: ub_bytes %u must hold tile_cols*rows*4 = %llu and be <= 240 KiB",
                     t->ub_bytes, (unsigned long long)t->tile_cols * t->rows * 4u);
  if ((uint64_t)t->rows * t->cols * 4u > 64ull << 20)
    return set_error(DCOPY_ERR_PARAM_INVALID, "tiling: input %llu bytes exceeds 64 MiB",
                     (unsigned long long)t->rows * t->cols * 4u);
  return DCOPY_OK;
}

// phase 0 = small/large, 1 = pretranspose, 2 = contiguous (RunTiles<phase>),
// over the reference's tiles [tile_begin, tile_begin + tile_count) of
// tiling->tile_cols columns each (all tiles: 0, UINT32_MAX).
int run_tiles(int phase, const void *in, void *out, const DataCopyTiling *tp,
              dcopy_stream_t stream, uint32_t tile_begin = 0, uint32_t tile_count = 0xFFFFFFFFu) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  DataCopyTiling t;
  int rc = fetch_tiling(tp, s, &t);
  if (rc) return rc;
  const bool store = phase == 1 || t.store;
  const uint64_t bytes = (uint64_t)t.rows * t.cols * 4u;
  rc = check_device_span(in, bytes, phase == 2 ? "b" : "x");
  if (!rc && store) rc = check_device_span(out, bytes, phase == 1 ? "b" : "y");
  if (!rc && store) rc = check_disjoint(in, bytes, out, bytes, "datacopy");
  if (rc) return rc;
  if ((uintptr_t)in % 4 || (store && (uintptr_t)out % 4))
    return set_error(DCOPY_ERR_PARAM_INVALID, "datacopy: int32 buffers must be 4-byte aligned");
  // Columns of the requested tiles (asc:36: tile c0 covers [c0, min(c0 + tile_cols, cols))).
  const uint32_t ntiles = (t.cols + t.tile_cols - 1) / t.tile_cols;
  if (tile_begin > ntiles || (tile_count != 0xFFFFFFFFu && tile_count > ntiles - tile_begin))
    return set_error(DCOPY_ERR_PARAM_INVALID, "datacopy: tiles [%u, +%u) outside the %u tiles",
                     tile_begin, tile_count, ntiles);
  const uint32_t c_lo = std::min(t.cols, tile_begin * t.tile_cols);
  const uint32_t c_hi = tile_count == 0xFFFFFFFFu
                            ? t.cols
                            : (uint32_t)std::min<uint64_t>(
                                  t.cols, (uint64_t)(tile_begin + tile_count) * t.tile_cols);
  if (c_hi <= c_lo) return DCOPY_OK;
  const uint64_t off = (uint64_t)c_lo * t.rows * 4u, part = (uint64_t)(c_hi - c_lo) * t.rows * 4u;
  const uint8_t *ip = static_cast<const uint8_t *>(in);
  uint8_t *op = static_cast<uint8_t *>(out);
  if (phase == 2)  // B and y share the [cols, rows] layout: the tiles are one contiguous range
    return store ? copy_linear(op + off, ip + off, part, s) : load_linear(ip + off, part, s);
  return launch_transpose(ip + (uint64_t)c_lo * 4u, store ? op + off : nullptr, t.rows,
                          c_hi - c_lo, t.cols, store, s);
}

}  // namespace

int run_pretranspose_workflow(const void *x, void *scratch, uint64_t scratch_bytes, void *y,
                              const DataCopyTiling *tp, dcopy_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  DataCopyTiling t;
  int rc = fetch_tiling(tp, s, &t);
  if (rc) return rc;
  const uint64_t bytes = (uint64_t)t.rows * t.cols * 4u;
  if (bytes > scratch_bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "pretranspose workflow: rows*cols*4 = %llu bytes exceeds the %llu-byte "
                     "static B buffer",
                     (unsigned long long)bytes, (unsigned long long)scratch_bytes);
  rc = check_device_span(x, bytes, "x");
  if (!rc && t.store) rc = check_device_span(y, bytes, "y");
  if (!rc && t.store) rc = check_disjoint(x, bytes, y, bytes, "datacopy");
  if (rc) return rc;
  if ((uintptr_t)x % 4 || (t.store && (uintptr_t)y % 4))
    return set_error(DCOPY_ERR_PARAM_INVALID, "datacopy: int32 buffers must be 4-byte aligned");
  rc = launch_transpose(x, scratch, t.rows, t.cols, t.cols, true, s);  // RunTiles<1>: B written
  if (rc) return rc;
  return t.store ? copy_linear(y, scratch, bytes, s) : load_linear(scratch, bytes, s);
}

}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_plan_tiling(uint32_t rows, uint32_t cols, uint32_t tile_kib, uint32_t store,
                                 DataCopyTiling *out) {
  DCOPY_API_BEGIN
  if (!out) return set_error(DCOPY_ERR_PARAM_INVALID, "plan_tiling: out is NULL");
  // asc:115-118
  if (!rows || rows > 4095 || rows % 8 || !cols || cols > 65535 || !tile_kib || tile_kib > 240 ||
      store > 1)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "rows: 8..4088 multiple of 8; cols: 1..65535; tile: 1..240 KiB; store: 0/1");
  // asc:119-121
  const uint32_t tile_cols = std::min(cols, tile_kib * 1024u / (rows * 4u));
  if (!tile_cols)
    return set_error(DCOPY_ERR_PARAM_INVALID, "Tile budget must hold a complete transposed row");
  // asc:122-123
  if ((uint64_t)rows * cols * 4u > 64ull * 1024 * 1024)
    return set_error(DCOPY_ERR_PARAM_INVALID, "Experiment GM input limit: 64 MiB");
  out->rows = rows;
  out->cols = cols;
  out->tile_cols = tile_cols;
  out->ub_bytes = tile_cols * rows * 4u;
  out->store = store;
  return DCOPY_OK;
  DCOPY_API_END
}

extern "C" int dcopy_datacopy_small(const void *x, void *y, const DataCopyTiling *tiling,
                                    dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return run_tiles(0, x, y, tiling, stream);
  DCOPY_API_END
}

extern "C" int dcopy_datacopy_large(const void *x, void *y, const DataCopyTiling *tiling,
                                    dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return run_tiles(0, x, y, tiling, stream);
  DCOPY_API_END
}

extern "C" int dcopy_datacopy_pretranspose(const void *x, void *b, const DataCopyTiling *tiling,
                                           dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return run_tiles(1, x, b, tiling, stream);
  DCOPY_API_END
}

extern "C" int dcopy_datacopy_contiguous(const void *b, void *y, const DataCopyTiling *tiling,
                                         dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return run_tiles(2, b, y, tiling, stream);
  DCOPY_API_END
}

extern "C" int dcopy_datacopy_tiles(int32_t phase, const void *in, void *out,
                                    const DataCopyTiling *tiling, uint32_t tile_begin,
                                    uint32_t tile_count, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (phase < 0 || phase > 2)
    return set_error(DCOPY_ERR_PARAM_INVALID, "datacopy_tiles: phase %d is not 0, 1 or 2", phase);
  if (tile_count == 0xFFFFFFFFu)
    return set_error(DCOPY_ERR_PARAM_INVALID, "datacopy_tiles: tile_count out of range");
  return run_tiles(phase, in, out, tiling, stream, tile_begin, tile_count);
  DCOPY_API_END
}
