// ND <-> FRACTAL_NZ TransData on sm_100a.
//
// Layout (format_transfer_fractal_nz.cc:131-298): ND [times, H, W] and
// NZ [times, W1 = ceil(W/W0), H1 = ceil(H/16), 16, W0].  Panel w1 of batch t is
// the column slab [w1*W0, (w1+1)*W0) of the ND matrix stored row-major with
// rows of W0 elements and H padded to H1*16 rows; padding is zero.
//
// Kernel design: bytes are moved in "units" of 16 (or fewer, for odd shapes)
// bytes; one NZ row of W0 elements is `upr` units.  A CTA tile covers 16
// consecutive rows x PG consecutive panels (1024 units, e.g. 16 KiB for fp16),
// so within a tile the ND side is 16 row segments of PG*W0 elements (1 KiB for
// fp16) and the NZ side is PG contiguous 16-row fragments (512 B each): both
// directions read and write whole 128-byte lines, and the threads of a warp
// walk the destination in address order.  Each thread keeps 4 units in
// flight.  Out-of-range NZ units (H and W padding) are written as zero.
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
constexpr int kRowsPerTile = 16;  // H0

struct NzGeom {
  uint32_t H;        // ND rows
  uint32_t Hp;       // H1 * 16
  uint32_t Wu;       // ND row length in units
  uint32_t upr;      // units per NZ row (W0 elements)
  uint32_t W1;       // panels
  uint32_t PG;       // panels per tile
  uint32_t hblocks;  // Hp / 16
  uint32_t pgroups;  // ceil(W1 / PG)
  uint32_t tile_units;
  FastDiv f_upr, f_pgu, f_pgroups, f_hblocks;
  uint64_t nd_batch;  // units per ND batch = H * Wu
  uint64_t nz_batch;  // units per NZ batch = W1 * Hp * upr
  uint64_t panel;     // units per panel = Hp * upr
};

template <typename T, bool kToNz>
__global__ void __launch_bounds__(kThreads) nz_kernel(T *__restrict__ dst,
                                                      const T *__restrict__ src, NzGeom g,
                                                      uint32_t ntiles) {
  constexpr int U = kTileUnits / kThreads;
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const uint32_t q = g.f_pgroups.div(tile);
    const uint32_t pg = tile - q * g.pgroups;
    const uint32_t t = g.f_hblocks.div(q);
    const uint32_t hb = q - t * g.hblocks;
    const uint32_t w1_0 = pg * g.PG, h_0 = hb * kRowsPerTile;
    const T *sb = src + (uint64_t)t * (kToNz ? g.nd_batch : g.nz_batch);
    T *db = dst + (uint64_t)t * (kToNz ? g.nz_batch : g.nd_batch);
    for (uint32_t jb = 0; jb < g.tile_units; jb += kTileUnits) {
      T v[U];
      uint64_t doff[U];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t j = jb + threadIdx.x + u * kThreads;
        ok[u] = false;
        if (j >= g.tile_units) continue;
        if (kToNz) {
          // destination order inside the tile: [panel][row][unit]
          const uint32_t r = g.f_upr.div(j);
          const uint32_t k = j - r * g.upr;
          const uint32_t hin = r % kRowsPerTile, pin = r / kRowsPerTile;
          const uint32_t w1 = w1_0 + pin, hp = h_0 + hin;
          if (w1 >= g.W1) continue;
          const uint32_t col = w1 * g.upr + k;
          v[u] = T();
          if (hp < g.H && col < g.Wu) v[u] = ld_stream(sb + (uint64_t)hp * g.Wu + col);
          doff[u] = (uint64_t)w1 * g.panel + (uint64_t)hp * g.upr + k;
          ok[u] = true;
        } else {
          // destination order inside the tile: [row][unit]
          const uint32_t hin = g.f_pgu.div(j);
          const uint32_t uin = j - hin * (g.PG * g.upr);
          const uint32_t h = h_0 + hin, col = w1_0 * g.upr + uin;
          if (h >= g.H || col >= g.Wu) continue;
          const uint32_t pin = g.f_upr.div(uin);
          const uint32_t k = uin - pin * g.upr;
          v[u] = ld_stream(sb + (uint64_t)(w1_0 + pin) * g.panel + (uint64_t)h * g.upr + k);
          doff[u] = (uint64_t)h * g.Wu + col;
          ok[u] = true;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (ok[u]) db[doff[u]] = v[u];
    }
  }
}

// Shared-memory staged variant for a power-of-two `upr` with 16-byte units: the
// tile is read from global memory in source order (each warp 512 contiguous
// bytes), permuted through shared memory, and written in destination order
// (again 512 contiguous bytes per warp).  Shared memory holds the tile in NZ
// order [panel][row][unit]; the 16-byte unit index is XOR-swizzled with
// (panel * upr) mod 8 so that the ND-order accesses (fixed row, consecutive
// panels) and the NZ-order accesses (fixed panel, consecutive rows) both hit 8
// distinct 16-byte bank groups per 128-byte wavefront.
template <bool kToNz>
__global__ void __launch_bounds__(kThreads) nz_smem_kernel(uint4 *__restrict__ dst,
                                                           const uint4 *__restrict__ src,
                                                           NzGeom g, uint32_t ntiles,
                                                           uint32_t upr_shift, bool prefetch) {
  constexpr int U = kTileUnits / kThreads;
  __shared__ uint4 tile[kTileUnits];
  pdl_trigger_at_entry();
  // The tile is 16 rows x 64 units (1024 units), so a tile row (ND order) is 64
  // units and a panel fragment (NZ order) is 16 * upr units.
  const uint32_t upr = g.upr;
  constexpr uint32_t kRowShift = 6;  // log2(kTileUnits / kRowsPerTile)
  static_assert(kTileUnits / kRowsPerTile == 64, "tile row must be 64 units");
  const uint32_t panel_shift = 4 + upr_shift;
  const uint32_t panel_units = 1u << panel_shift;
  if (DCOPY_PREFETCH && prefetch && blockIdx.x < ntiles) {
    // L2-prefetch the first tile's source, one prefetch per 128-byte line.
    const uint32_t q = g.f_pgroups.div(blockIdx.x);
    const uint32_t pg = blockIdx.x - q * g.pgroups;
    const uint32_t t = g.f_hblocks.div(q);
    const uint32_t hb = q - t * g.hblocks;
    const uint4 *sb = src + (uint64_t)t * (kToNz ? g.nd_batch : g.nz_batch);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      if (j % 8) continue;
      if (kToNz) {
        const uint32_t h = hb * kRowsPerTile + (j >> kRowShift), col = pg * g.PG * upr + (j & 63);
        if (h < g.H && col < g.Wu) prefetch_l2(sb + (uint64_t)h * g.Wu + col);
      } else {
        const uint32_t pin = j >> panel_shift;
        if (pg * g.PG + pin < g.W1)
          prefetch_l2(sb + (uint64_t)(pg * g.PG + pin) * g.panel +
                      (uint64_t)hb * kRowsPerTile * upr + (j & (panel_units - 1)));
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t tile_id = blockIdx.x; tile_id < ntiles; tile_id += gridDim.x) {
    const uint32_t q = g.f_pgroups.div(tile_id);
    const uint32_t pg = tile_id - q * g.pgroups;
    const uint32_t t = g.f_hblocks.div(q);
    const uint32_t hb = q - t * g.hblocks;
    const uint32_t w1_0 = pg * g.PG, h_0 = hb * kRowsPerTile;
    const uint4 *sb = src + (uint64_t)t * (kToNz ? g.nd_batch : g.nz_batch);
    uint4 *db = dst + (uint64_t)t * (kToNz ? g.nz_batch : g.nd_batch);
    // ---- load: source order into swizzled NZ-order shared memory
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      v[u] = make_uint4(0, 0, 0, 0);
      if (kToNz) {  // ND order [row][unit]
        const uint32_t hin = j >> kRowShift, uin = j & 63;
        const uint32_t h = h_0 + hin, col = w1_0 * upr + uin;
        if (h < g.H && col < g.Wu) v[u] = ld_stream(sb + (uint64_t)h * g.Wu + col);
      } else {  // NZ order [panel][row][unit]
        const uint32_t pin = j >> panel_shift, rem = j & (panel_units - 1);
        if (w1_0 + pin < g.W1)
          v[u] = ld_stream(sb + (uint64_t)(w1_0 + pin) * g.panel + (uint64_t)h_0 * upr + rem);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = threadIdx.x + u * kThreads;
      uint32_t pin, rem;
      if (kToNz) {
        const uint32_t hin = j >> kRowShift, uin = j & 63;
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
      if (kToNz) {  // NZ order
        const uint32_t pin = j >> panel_shift, rem = j & (panel_units - 1);
        if (w1_0 + pin < g.W1)
          db[(uint64_t)(w1_0 + pin) * g.panel + (uint64_t)h_0 * upr + rem] =
              tile[pin * panel_units + (rem ^ ((pin << upr_shift) & 7))];
      } else {  // ND order
        const uint32_t hin = j >> kRowShift, uin = j & 63;
        const uint32_t h = h_0 + hin, col = w1_0 * upr + uin;
        const uint32_t pin = uin >> upr_shift;
        const uint32_t rem = (hin << upr_shift) + (uin & (upr - 1));
        if (h < g.H && col < g.Wu)
          db[(uint64_t)h * g.Wu + col] = tile[pin * panel_units + (rem ^ ((pin << upr_shift) & 7))];
      }
    }
    __syncthreads();
  }
}

}  // namespace

// Shape rules of TransShapeToFracNz (:65-111) and IsShapeValid
// (formats_trans_utils.cc:88-107).
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
    nz[n++] = kRowsPerTile;
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
    nz[n++] = ge_ceil(nd[rank - 2], kRowsPerTile);
    nz[n++] = kRowsPerTile;
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

namespace {


template <typename T>
int launch_nz(void *dst, const void *src, const NzGeom &g, uint32_t ntiles, bool to_nz,
              cudaStream_t s) {
  if (DCOPY_NZ_SMEM && sizeof(T) == 16 && g.tile_units == kTileUnits &&
      (g.upr & (g.upr - 1)) == 0 && g.upr <= 64) {
    uint32_t shift = 0;
    while ((1u << shift) < g.upr) ++shift;
    const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
    uint4 *d = static_cast<uint4 *>(dst);
    const uint4 *sp = static_cast<const uint4 *>(src);
    const bool pf = is_local_device_memory(src);
    if (to_nz)
      return launch(nz_smem_kernel<true>, grid, dim3(kThreads), 0, s, "nz_smem_kernel", d, sp, g,
                    ntiles, shift, pf);
    return launch(nz_smem_kernel<false>, grid, dim3(kThreads), 0, s, "nz_smem_kernel", d, sp, g,
                  ntiles, shift, pf);
  }
  // One tile per CTA: on B200 many short-lived CTAs stream better than a
  // persistent grid (the grid-stride loop only matters past 2^31 - 1 tiles).
  const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
  T *d = static_cast<T *>(dst);
  const T *sp = static_cast<const T *>(src);
  if (to_nz)
    return launch(nz_kernel<T, true>, grid, dim3(kThreads), 0, s, "nz_kernel", d, sp, g, ntiles);
  return launch(nz_kernel<T, false>, grid, dim3(kThreads), 0, s, "nz_kernel", d, sp, g, ntiles);
}

}  // namespace

int nz_transfer(void *dst, const void *src, const int64_t *nd_shape, int rank, int elem_bytes,
                int64_t w0, bool to_nz, dcopy_stream_t stream) {
  if (elem_bytes <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d: data type size must be > 0",
                     elem_bytes);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8 &&
      elem_bytes != 16)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d not in {1,2,4,8,16}",
                     elem_bytes);
  if (rank <= 0 || rank > 30 || !shape_valid(nd_shape, rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "ND shape is invalid (rank %d)", rank);
  if (!to_nz && w0 <= 0)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "w0 %lld must be positive", (long long)w0);
  int64_t nz[32], hw[3];
  int nz_rank = 0;
  int rc = nz_shape(nd_shape, rank, w0, nz, &nz_rank, hw);
  if (rc) return rc;
  int64_t nz_items = 1, nd_items = 1;
  for (int i = 0; i < nz_rank; ++i) nz_items *= nz[i];
  for (int i = 0; i < rank; ++i) nd_items *= nd_shape[i];
  const uint64_t nz_bytes = (uint64_t)nz_items * elem_bytes;
  const uint64_t nd_bytes = (uint64_t)nd_items * elem_bytes;
  const uint64_t dst_bytes = to_nz ? nz_bytes : nd_bytes;
  if (dst_bytes == 0) return DCOPY_OK;  // the reference returns an empty result (:134-137)
  const uint64_t src_bytes = to_nz ? nd_bytes : nz_bytes;
  rc = check_device_span(src, src_bytes, "src");
  if (!rc) rc = check_device_span(dst, dst_bytes, "dst");
  if (!rc) rc = check_disjoint(src, src_bytes, dst, dst_bytes, to_nz ? "nd_to_nz" : "nz_to_nd");
  if (rc) return rc;

  const int64_t times = hw[0], H = hw[1], W = hw[2];
  const int64_t W1 = nz[nz_rank - 4], Hp = nz[nz_rank - 3] * kRowsPerTile;
  // Unit: the widest power of two <= 16 bytes dividing the NZ row, the ND row
  // and both base addresses.
  uint64_t key = (uint64_t)w0 * elem_bytes | (uint64_t)W * elem_bytes | (uintptr_t)dst |
                 (uintptr_t)src;
  if (W == 0) key = (uint64_t)w0 * elem_bytes | (uintptr_t)dst | (uintptr_t)src;
  uint32_t us = 16;
  while (us > (uint32_t)elem_bytes && key % us) us >>= 1;
  if (key % us)
    return set_error(DCOPY_ERR_PARAM_INVALID, "buffers must be aligned to the element size");
  const uint64_t upr = (uint64_t)w0 * elem_bytes / us;
  const uint64_t Wu = (uint64_t)W * elem_bytes / us;
  if (times > 0xFFFFFFFFll || Hp > (1ll << 30) || Wu > (1ull << 30) || upr > (1ull << 20) ||
      W1 > (1ll << 30))
    return set_error(DCOPY_ERR_UNSUPPORTED, "ND<->NZ: shape beyond 32-bit tile indexing");
  NzGeom g{};
  g.H = (uint32_t)H;
  g.Hp = (uint32_t)Hp;
  g.Wu = (uint32_t)Wu;
  g.upr = (uint32_t)upr;
  g.W1 = (uint32_t)W1;
  g.PG = (uint32_t)std::max<uint64_t>(1, kTileUnits / (kRowsPerTile * upr));
  g.hblocks = (uint32_t)(Hp / kRowsPerTile);
  g.pgroups = (g.W1 + g.PG - 1) / g.PG;
  g.tile_units = kRowsPerTile * g.PG * g.upr;
  g.f_upr = FastDiv(g.upr);
  g.f_pgu = FastDiv(g.PG * g.upr);
  g.f_pgroups = FastDiv(std::max(1u, g.pgroups));
  g.f_hblocks = FastDiv(std::max(1u, g.hblocks));
  g.nd_batch = (uint64_t)H * Wu;
  g.panel = (uint64_t)Hp * upr;
  g.nz_batch = (uint64_t)W1 * g.panel;
  const uint64_t ntiles = (uint64_t)times * g.hblocks * g.pgroups;
  if (ntiles == 0) return DCOPY_OK;
  if (ntiles > 0xFFFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "ND<->NZ: %llu tiles exceed 32-bit indexing",
                     (unsigned long long)ntiles);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (us) {
    case 16: return launch_nz<uint4>(dst, src, g, (uint32_t)ntiles, to_nz, s);
    case 8: return launch_nz<uint2>(dst, src, g, (uint32_t)ntiles, to_nz, s);
    case 4: return launch_nz<uint32_t>(dst, src, g, (uint32_t)ntiles, to_nz, s);
    case 2: return launch_nz<uint16_t>(dst, src, g, (uint32_t)ntiles, to_nz, s);
    default: return launch_nz<uint8_t>(dst, src, g, (uint32_t)ntiles, to_nz, s);
  }
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
