// ND <-> FRACTAL_NZ and ND <-> FRACTAL_ZZ TransData on sm_100a.
//
// Both formats cut the ND matrix [times, H, W] into blocks of BH rows x W0
// columns, zero-padded to whole blocks, each block stored row-major:
//   FRACTAL_NZ (format_transfer_fractal_nz.cc:131-298): [times, W1, H1, 16, W0],
//     BH = 16; the H1 blocks of one column slab (a panel) are adjacent.
//   FRACTAL_ZZ (format_transfer_fractal_zz.cc:140-334): [times, H1, W1, C0, C0],
//     BH = W0 = C0; the W1 blocks of one row band are adjacent.
// The tiled offset of ND element (h, w) of batch t is therefore
//   t*batch + (h / BH)*s_band + (w / W0)*s_panel + (h % BH)*W0 + w % W0,
// with (s_band, s_panel) = (BH*W0, H1*BH*W0) for NZ and (W1*BH*W0, BH*W0) for ZZ.
//
// Kernel design: bytes are moved in "units" of 16 (or fewer, for odd shapes)
// bytes; one block row of W0 elements is `upr` units.  A CTA tile covers one row
// band (BH rows) x PG consecutive column blocks (1024 units, e.g. 16 KiB), so
// within a tile the ND side is BH row segments of PG*W0 elements and the tiled
// side is PG contiguous BH-row fragments (for ZZ the whole tile is contiguous):
// both directions read and write whole 128-byte lines, and the threads of a warp
// walk the destination in address order.  Each thread keeps 4 units in flight.
// Out-of-range tiled units (H and W padding) are written as zero.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

#ifndef DCOPY_NZ_SMEM
#define DCOPY_NZ_SMEM 1
#endif
#ifndef DCOPY_PREFETCH
#define DCOPY_PREFETCH 1  // L2-prefetch the first tile while waiting on the previous kernel
#endif

constexpr int kThreads = 256;
constexpr int kTileUnits = 1024;  // 4 units per thread
constexpr int kNzRows = 16;       // H0 of FRACTAL_NZ

struct FracGeom {
  uint32_t H;           // ND rows
  uint32_t Wu;          // ND row length in units
  uint32_t upr;         // units per block row (W0 elements)
  uint32_t BH;          // rows per block
  uint32_t W1;          // column blocks
  uint32_t PG;          // column blocks per tile
  uint32_t hblocks;     // H1 (row bands)
  uint32_t pgroups;     // ceil(W1 / PG)
  uint32_t tile_units;  // BH * PG * upr
  FastDiv f_upr, f_bh, f_pgu, f_pgroups, f_hblocks;
  uint64_t nd_row;      // units between ND rows (Wu for a packed matrix)
  uint64_t nd_batch;    // units between ND batches (H * Wu for packed matrices)
  uint64_t fr_batch;    // units per tiled batch = H1 * W1 * BH * upr
  uint64_t s_band;      // units between row bands
  uint64_t s_panel;     // units between column blocks
  uint32_t times;       // batches
  uint32_t batch_fast;  // 1: consecutive tiles walk the batches first
  FastDiv f_times;
};

// Tile index -> (batch t, row band hb, column-block group pg).
__device__ __forceinline__ void frac_tile(const FracGeom &g, uint32_t tile, uint32_t &t,
                                          uint32_t &hb, uint32_t &pg) {
  if (g.batch_fast) {
    const uint32_t rest = g.f_times.div(tile);
    t = tile - rest * g.times;
    const uint32_t q = g.f_pgroups.div(rest);
    pg = rest - q * g.pgroups;
    hb = q;
  } else {
    const uint32_t q = g.f_pgroups.div(tile);
    pg = tile - q * g.pgroups;
    t = g.f_hblocks.div(q);
    hb = q - t * g.hblocks;
  }
}

template <typename T, bool kToFrac>
__global__ void __launch_bounds__(kThreads) nz_kernel(T *__restrict__ dst,
                                                      const T *__restrict__ src, FracGeom g,
                                                      uint32_t ntiles) {
  constexpr int U = kTileUnits / kThreads;
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    uint32_t t, hb, pg;
    frac_tile(g, tile, t, hb, pg);
    const uint32_t w1_0 = pg * g.PG, h_0 = hb * g.BH;
    const T *sb = src + (uint64_t)t * (kToFrac ? g.nd_batch : g.fr_batch);
    T *db = dst + (uint64_t)t * (kToFrac ? g.fr_batch : g.nd_batch);
    const uint64_t band = (uint64_t)hb * g.s_band;
    for (uint32_t jb = 0; jb < g.tile_units; jb += kTileUnits) {
      T v[U];
      uint64_t doff[U];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t j = jb + threadIdx.x + u * kThreads;
        ok[u] = false;
        if (j >= g.tile_units) continue;
        if (kToFrac) {
          // destination order inside the tile: [block][row][unit]
          const uint32_t r = g.f_upr.div(j);
          const uint32_t k = j - r * g.upr;
          const uint32_t pin = g.f_bh.div(r), hin = r - pin * g.BH;
          const uint32_t w1 = w1_0 + pin, hp = h_0 + hin;
          if (w1 >= g.W1) continue;
          const uint32_t col = w1 * g.upr + k;
          v[u] = T();
          if (hp < g.H && col < g.Wu) v[u] = ld_stream(sb + (uint64_t)hp * g.nd_row + col);
          doff[u] = band + (uint64_t)w1 * g.s_panel + (uint64_t)hin * g.upr + k;
          ok[u] = true;
        } else {
          // destination order inside the tile: [row][unit]
          const uint32_t hin = g.f_pgu.div(j);
          const uint32_t uin = j - hin * (g.PG * g.upr);
          const uint32_t h = h_0 + hin, col = w1_0 * g.upr + uin;
          if (h >= g.H || col >= g.Wu) continue;
          const uint32_t pin = g.f_upr.div(uin);
          const uint32_t k = uin - pin * g.upr;
          v[u] = ld_stream(sb + band + (uint64_t)(w1_0 + pin) * g.s_panel +
                           (uint64_t)hin * g.upr + k);
          doff[u] = (uint64_t)h * g.nd_row + col;
          ok[u] = true;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (ok[u]) db[doff[u]] = v[u];
    }
  }
}

// Shared-memory staged variant for power-of-two BH and `upr` with 16-byte units
// and BH * upr in [8, 1024]: the tile (BH rows x 1024/BH units) is read from
// global memory in source order (each warp 512 contiguous bytes), permuted
// through shared memory, and written in destination order (again 512
// contiguous bytes per warp).  Shared memory holds the tile in tiled order
// [block][row][unit]; the 16-byte unit index is XOR-swizzled with
// (block * upr) mod 8 so that the ND-order accesses (fixed row, consecutive
// blocks) and the tiled-order accesses (fixed block, consecutive rows) both hit
// 8 distinct 16-byte bank groups per 128-byte wavefront.
template <bool kToFrac>
__global__ void __launch_bounds__(kThreads) nz_smem_kernel(uint4 *__restrict__ dst,
                                                           const uint4 *__restrict__ src,
                                                           FracGeom g, uint32_t ntiles,
                                                           uint32_t upr_shift, uint32_t row_shift,
                                                           bool prefetch) {
  constexpr int U = kTileUnits / kThreads;
  __shared__ uint4 tile[kTileUnits];
  pdl_trigger_at_entry();
  // A tile row (ND order) is 1024 / BH = 2^row_shift units and a block fragment
  // (tiled order) is BH * upr = 2^panel_shift units.
  const uint32_t upr = g.upr;
  const uint32_t row_mask = (1u << row_shift) - 1;
  const uint32_t panel_shift = (10 - row_shift) + upr_shift;
  const uint32_t panel_units = 1u << panel_shift;
  if (DCOPY_PREFETCH && prefetch && blockIdx.x < ntiles) {
    // L2-prefetch the first tile's source, one prefetch per 128-byte line.
    uint32_t t, hb, pg;
    frac_tile(g, blockIdx.x, t, hb, pg);
    const uint4 *sb = src + (uint64_t)t * (kToFrac ? g.nd_batch : g.fr_batch);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      if (j % 8) continue;
      if (kToFrac) {
        const uint32_t h = hb * g.BH + (j >> row_shift), col = pg * g.PG * upr + (j & row_mask);
        if (h < g.H && col < g.Wu) prefetch_l2(sb + (uint64_t)h * g.nd_row + col);
      } else {
        const uint32_t pin = j >> panel_shift;
        if (pg * g.PG + pin < g.W1)
          prefetch_l2(sb + (uint64_t)hb * g.s_band + (uint64_t)(pg * g.PG + pin) * g.s_panel +
                      (j & (panel_units - 1)));
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t tile_id = blockIdx.x; tile_id < ntiles; tile_id += gridDim.x) {
    uint32_t t, hb, pg;
    frac_tile(g, tile_id, t, hb, pg);
    const uint32_t w1_0 = pg * g.PG, h_0 = hb * g.BH;
    const uint4 *sb = src + (uint64_t)t * (kToFrac ? g.nd_batch : g.fr_batch);
    uint4 *db = dst + (uint64_t)t * (kToFrac ? g.fr_batch : g.nd_batch);
    const uint64_t band = (uint64_t)hb * g.s_band;
    // ---- load: source order into swizzled tiled-order shared memory
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      v[u] = make_uint4(0, 0, 0, 0);
      if (kToFrac) {  // ND order [row][unit]
        const uint32_t hin = j >> row_shift, uin = j & row_mask;
        const uint32_t h = h_0 + hin, col = w1_0 * upr + uin;
        if (h < g.H && col < g.Wu) v[u] = ld_stream(sb + (uint64_t)h * g.nd_row + col);
      } else {  // tiled order [block][row][unit]
        const uint32_t pin = j >> panel_shift, rem = j & (panel_units - 1);
        if (w1_0 + pin < g.W1)
          v[u] = ld_stream(sb + band + (uint64_t)(w1_0 + pin) * g.s_panel + rem);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      uint32_t pin, rem;
      if (kToFrac) {
        const uint32_t hin = j >> row_shift, uin = j & row_mask;
        pin = uin >> upr_shift;
        rem = (hin << upr_shift) + (uin & (upr - 1));
      } else {
        pin = j >> panel_shift;
        rem = j & (panel_units - 1);
      }
      tile[pin * panel_units + (rem ^ ((pin << upr_shift) & 7))] = v[u];
    }
    __syncthreads();
    // ---- store: destination order out of shared memory
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      if (kToFrac) {  // tiled order
        const uint32_t pin = j >> panel_shift, rem = j & (panel_units - 1);
        if (w1_0 + pin < g.W1)
          db[band + (uint64_t)(w1_0 + pin) * g.s_panel + rem] =
              tile[pin * panel_units + (rem ^ ((pin << upr_shift) & 7))];
      } else {  // ND order
        const uint32_t hin = j >> row_shift, uin = j & row_mask;
        const uint32_t h = h_0 + hin, col = w1_0 * upr + uin;
        const uint32_t pin = uin >> upr_shift;
        const uint32_t rem = (hin << upr_shift) + (uin & (upr - 1));
        if (h < g.H && col < g.Wu)
          db[(uint64_t)h * g.nd_row + col] = tile[pin * panel_units + (rem ^ ((pin << upr_shift) & 7))];
      }
    }
    __syncthreads();
  }
}

}  // namespace

// Shape rules of TransShapeToFracNz (fractal_nz.cc:65-111), TransShapeToFracZz
// (fractal_zz.cc:74-118) and IsShapeValid (formats_trans_utils.cc:88-107).
constexpr int64_t kShapeItemNumMax = 1099511627776LL;

int64_t ge_ceil(int64_t n1, int64_t n2) {
  if (n1 == 0) return 0;
  return (n2 != 0) ? (((n1 - 1) / n2) + 1) : 0;
}

bool shape_valid(const int64_t *shape, int rank) {
  if (rank <= 0 || !shape) return false;
  int64_t num = 1;
  for (int i = 0; i < rank; ++i) {
    const int64_t dim = shape[i];
    if (dim < 0) return false;
    if (dim != 0 && (kShapeItemNumMax / dim) < num) return false;
    num *= dim;
  }
  return true;
}

int nz_shape(const int64_t *nd, int rank, int64_t w0, int64_t *nz, int *nz_rank, int64_t *hw) {
  int n = 0;
  if (rank == 1) {
    nz[n++] = ge_ceil(nd[0], w0);
    nz[n++] = 1;
    nz[n++] = kNzRows;
    nz[n++] = w0;
    hw[0] = 1;
    hw[1] = 1;
    hw[2] = nd[0];
  } else {
    int64_t times = 1;
    for (int i = 0; i < rank - 2; ++i) {
      nz[n++] = nd[i];
      times *= nd[i];
    }
    nz[n++] = ge_ceil(nd[rank - 1], w0);
    nz[n++] = ge_ceil(nd[rank - 2], kNzRows);
    nz[n++] = kNzRows;
    nz[n++] = w0;
    hw[0] = times;
    hw[1] = nd[rank - 2];
    hw[2] = nd[rank - 1];
  }
  *nz_rank = n;
  if (!shape_valid(nz, n))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_NZ shape for w0=%lld is invalid",
                     (long long)w0);
  return DCOPY_OK;
}

int zz_shape(const int64_t *nd, int rank, int64_t c0, int64_t *zz, int *zz_rank, int64_t *hw) {
  int n = 0;
  if (rank == 1) {  // one row: [1, W1, C0, C0]
    zz[n++] = 1;
    zz[n++] = ge_ceil(nd[0], c0);
    zz[n++] = c0;
    zz[n++] = c0;
    hw[0] = 1;
    hw[1] = 1;
    hw[2] = nd[0];
  } else {
    int64_t times = 1;
    for (int i = 0; i < rank - 2; ++i) {
      zz[n++] = nd[i];
      times *= nd[i];
    }
    zz[n++] = ge_ceil(nd[rank - 2], c0);
    zz[n++] = ge_ceil(nd[rank - 1], c0);
    zz[n++] = c0;
    zz[n++] = c0;
    hw[0] = times;
    hw[1] = nd[rank - 2];
    hw[2] = nd[rank - 1];
  }
  *zz_rank = n;
  if (!shape_valid(zz, n))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_ZZ shape for c0=%lld is invalid",
                     (long long)c0);
  return DCOPY_OK;
}

namespace {

uint32_t log2_exact(uint32_t v) {
  uint32_t s = 0;
  while ((1u << s) < v) ++s;
  return s;
}

template <typename T>
int launch_frac(void *dst, const void *src, const FracGeom &g, uint32_t ntiles, bool to_frac,
                cudaStream_t s) {
  // One tile per CTA: on B200 many short-lived CTAs stream better than a
  // persistent grid (the grid-stride loop only matters past 2^31 - 1 tiles).
  const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
  if (DCOPY_NZ_SMEM && sizeof(T) == 16 && g.tile_units == kTileUnits && g.BH * g.upr >= 8) {
    // tile_units == 1024 == BH * PG * upr: BH and upr are powers of two.
    const uint32_t upr_shift = log2_exact(g.upr), row_shift = 10 - log2_exact(g.BH);
    uint4 *d = static_cast<uint4 *>(dst);
    const uint4 *sp = static_cast<const uint4 *>(src);
    const bool pf = is_local_device_memory(src);
    if (to_frac)
      return launch(nz_smem_kernel<true>, grid, dim3(kThreads), 0, s, "nz_smem_kernel", d, sp, g,
                    ntiles, upr_shift, row_shift, pf);
    return launch(nz_smem_kernel<false>, grid, dim3(kThreads), 0, s, "nz_smem_kernel", d, sp, g,
                  ntiles, upr_shift, row_shift, pf);
  }
  T *d = static_cast<T *>(dst);
  const T *sp = static_cast<const T *>(src);
  if (to_frac)
    return launch(nz_kernel<T, true>, grid, dim3(kThreads), 0, s, "nz_kernel", d, sp, g, ntiles);
  return launch(nz_kernel<T, false>, grid, dim3(kThreads), 0, s, "nz_kernel", d, sp, g, ntiles);
}

}  // namespace

int frac_launch(const FracPlan &p, void *dst, const void *src, bool to_frac,
                dcopy_stream_t stream, const char *name) {
  const int eb = p.elem_bytes;
  // Unit: the widest power of two <= 16 bytes dividing every row, pitch and
  // stride on both sides and both base addresses.
  const uint64_t key = (uint64_t)(p.w0 * eb) | (uint64_t)(p.W * eb) | (uint64_t)(p.nd_row * eb) |
                       (uint64_t)(p.nd_batch * eb) | (uint64_t)(p.s_band * eb) |
                       (uint64_t)(p.s_panel * eb) | (uint64_t)(p.fr_batch * eb) |
                       (uintptr_t)dst | (uintptr_t)src;
  uint32_t us = 16;
  while (us > (uint32_t)eb && key % us) us >>= 1;
  if (key % us)
    return set_error(DCOPY_ERR_PARAM_INVALID, "buffers must be aligned to the element size");
  const uint64_t upr = (uint64_t)p.w0 * eb / us;
  const uint64_t Wu = (uint64_t)p.W * eb / us;
  if (p.times > 0xFFFFFFFFll || p.H1 * p.BH > (1ll << 30) || Wu > (1ull << 30) ||
      upr > (1ull << 20) || p.W1 > (1ll << 30) || (uint64_t)p.BH * upr > (1ull << 24))
    return set_error(DCOPY_ERR_UNSUPPORTED, "%s: shape beyond 32-bit tile indexing", name);
  FracGeom g{};
  g.H = (uint32_t)p.H;
  g.Wu = (uint32_t)Wu;
  g.upr = (uint32_t)upr;
  g.BH = (uint32_t)p.BH;
  g.W1 = (uint32_t)p.W1;
  g.PG = (uint32_t)std::max<uint64_t>(1, kTileUnits / ((uint64_t)p.BH * upr));
  g.hblocks = (uint32_t)p.H1;
  g.pgroups = (g.W1 + g.PG - 1) / g.PG;
  g.tile_units = g.BH * g.PG * g.upr;
  g.f_upr = FastDiv(g.upr);
  g.f_bh = FastDiv(g.BH);
  g.f_pgu = FastDiv(g.PG * g.upr);
  g.f_pgroups = FastDiv(std::max(1u, g.pgroups));
  g.f_hblocks = FastDiv(std::max(1u, g.hblocks));
  g.nd_row = (uint64_t)p.nd_row * eb / us;
  g.nd_batch = (uint64_t)p.nd_batch * eb / us;
  g.fr_batch = (uint64_t)p.fr_batch * eb / us;
  g.s_band = (uint64_t)p.s_band * eb / us;
  g.s_panel = (uint64_t)p.s_panel * eb / us;
  g.times = (uint32_t)p.times;
  g.batch_fast = p.batch_fast ? 1u : 0u;
  g.f_times = FastDiv(std::max(1u, g.times));
  const uint64_t ntiles = (uint64_t)p.times * g.hblocks * g.pgroups;
  if (ntiles == 0) return DCOPY_OK;
  if (ntiles > 0xFFFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "%s: %llu tiles exceed 32-bit indexing", name,
                     (unsigned long long)ntiles);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (us) {
    case 16: return launch_frac<uint4>(dst, src, g, (uint32_t)ntiles, to_frac, s);
    case 8: return launch_frac<uint2>(dst, src, g, (uint32_t)ntiles, to_frac, s);
    case 4: return launch_frac<uint32_t>(dst, src, g, (uint32_t)ntiles, to_frac, s);
    case 2: return launch_frac<uint16_t>(dst, src, g, (uint32_t)ntiles, to_frac, s);
    default: return launch_frac<uint8_t>(dst, src, g, (uint32_t)ntiles, to_frac, s);
  }
}

int frac_transfer(FracKind kind, void *dst, const void *src, const int64_t *nd_shape, int rank,
                  int elem_bytes, int64_t w0, bool to_frac, dcopy_stream_t stream) {
  const char *name = kind == FracKind::kNz ? "ND<->NZ" : "ND<->ZZ";
  if (elem_bytes <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d: data type size must be > 0",
                     elem_bytes);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8 &&
      elem_bytes != 16)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d not in {1,2,4,8,16}",
                     elem_bytes);
  if (rank <= 0 || rank > 30 || !shape_valid(nd_shape, rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "ND shape is invalid (rank %d)", rank);
  // The tiled -> ND direction divides by W0 (fractal_nz.cc:249, fractal_zz.cc:273).
  if (!to_frac && w0 <= 0)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 %lld must be positive", (long long)w0);
  int64_t fr[32], hw[3];
  int fr_rank = 0;
  int rc = kind == FracKind::kNz ? nz_shape(nd_shape, rank, w0, fr, &fr_rank, hw)
                                 : zz_shape(nd_shape, rank, w0, fr, &fr_rank, hw);
  if (rc) return rc;
  int64_t fr_items = 1, nd_items = 1;
  for (int i = 0; i < fr_rank; ++i) fr_items *= fr[i];
  for (int i = 0; i < rank; ++i) nd_items *= nd_shape[i];
  const uint64_t fr_bytes = (uint64_t)fr_items * elem_bytes;
  const uint64_t nd_bytes = (uint64_t)nd_items * elem_bytes;
  const uint64_t dst_bytes = to_frac ? fr_bytes : nd_bytes;
  if (dst_bytes == 0) return DCOPY_OK;  // the reference returns an empty result
  const uint64_t src_bytes = to_frac ? nd_bytes : fr_bytes;
  rc = check_device_span(src, src_bytes, "src");
  if (!rc) rc = check_device_span(dst, dst_bytes, "dst");
  if (!rc) rc = check_disjoint(src, src_bytes, dst, dst_bytes, to_frac ? "nd_to_frac" : "frac_to_nd");
  if (rc) return rc;

  FracPlan p{};
  p.elem_bytes = elem_bytes;
  p.times = hw[0];
  p.H = hw[1];
  p.W = hw[2];
  p.nd_row = p.W;
  p.nd_batch = p.H * p.W;
  p.w0 = w0;
  p.BH = fr[fr_rank - 2];
  p.W1 = kind == FracKind::kNz ? fr[fr_rank - 4] : fr[fr_rank - 3];
  p.H1 = kind == FracKind::kNz ? fr[fr_rank - 3] : fr[fr_rank - 4];
  const int64_t block = p.BH * w0;
  p.fr_batch = p.H1 * p.W1 * block;
  p.s_band = kind == FracKind::kNz ? block : p.W1 * block;
  p.s_panel = kind == FracKind::kNz ? p.H1 * block : block;
  return frac_launch(p, dst, src, to_frac, stream, name);
}

int nz_transfer(void *dst, const void *src, const int64_t *nd_shape, int rank, int elem_bytes,
                int64_t w0, bool to_nz, dcopy_stream_t stream) {
  return frac_transfer(FracKind::kNz, dst, src, nd_shape, rank, elem_bytes, w0, to_nz, stream);
}

}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_nz_shape(const int64_t *nd_shape, int rank, int64_t w0, int64_t *nz_shape_out,
                              int *nz_rank, int64_t *hw_shape) {
  DCOPY_API_BEGIN
  if (!nz_shape_out || !nz_rank)
    return set_error(DCOPY_ERR_PARAM_INVALID, "nz_shape: output pointers are NULL");
  if (rank <= 0 || rank > 30 || !nd_shape)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "nz_shape: rank %d", rank);
  int64_t hw[3];
  int rc = nz_shape(nd_shape, rank, w0, nz_shape_out, nz_rank, hw);
  if (hw_shape) {
    hw_shape[0] = hw[0];
    hw_shape[1] = hw[1];
    hw_shape[2] = hw[2];
  }
  return rc;
  DCOPY_API_END
}

extern "C" int dcopy_zz_shape(const int64_t *nd_shape, int rank, int64_t c0, int64_t *zz_shape_out,
                              int *zz_rank, int64_t *hw_shape) {
  DCOPY_API_BEGIN
  if (!zz_shape_out || !zz_rank)
    return set_error(DCOPY_ERR_PARAM_INVALID, "zz_shape: output pointers are NULL");
  if (rank <= 0 || rank > 30 || !nd_shape)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "zz_shape: rank %d", rank);
  int64_t hw[3];
  int rc = zz_shape(nd_shape, rank, c0, zz_shape_out, zz_rank, hw);
  if (hw_shape) {
    hw_shape[0] = hw[0];
    hw_shape[1] = hw[1];
    hw_shape[2] = hw[2];
  }
  return rc;
  DCOPY_API_END
}

extern "C" int dcopy_nd_to_zz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                              int elem_bytes, int64_t c0, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return frac_transfer(FracKind::kZz, dst, src, nd_shape, rank, elem_bytes, c0, true, stream);
  DCOPY_API_END
}

extern "C" int dcopy_zz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                              int elem_bytes, int64_t c0, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return frac_transfer(FracKind::kZz, dst, src, nd_shape, rank, elem_bytes, c0, false, stream);
  DCOPY_API_END
}

extern "C" int dcopy_nd_to_nz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                              int elem_bytes, int64_t w0, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return nz_transfer(dst, src, nd_shape, rank, elem_bytes, w0, true, stream);
  DCOPY_API_END
}

extern "C" int dcopy_nz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                              int elem_bytes, int64_t w0, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return nz_transfer(dst, src, nd_shape, rank, elem_bytes, w0, false, stream);
  DCOPY_API_END
}
