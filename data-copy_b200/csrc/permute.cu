// Permuted copy into a contiguous destination (GE's Transpose after dimension
// merging): dst[i] = src[sum_k idx_k * src_stride_k] over the destination
// odometer, sizes and strides in elements, at most 5 dims, dst contiguous.
// The row kernel also serves strided destinations (rows_copy: NDDMA boxes).
//
// Two kernels, by where the source's contiguous axis lands:
//   * perm_rows_kernel: the innermost axis is contiguous on both sides, so the
//     copy is a set of rows of L elements whose source starts follow an up-to
//     4-D odometer.  Units of up to 16 bytes, 4 in flight per thread; the row
//     start is computed once per unit with invariant-divisor divisions.
//   * perm_tile_kernel: a true transpose of the destination's contiguous axis d
//     (source stride s_d) and the source's contiguous axis e (destination
//     stride t_e), batched over up to 3 further axes.  A tile of TD x TE elements
//     is read along e, staged in shared memory (rows of odd word pitch) and
//     written along d; with 16-byte aligned rows on both sides every global
//     access is a 16-byte vector of V = 16/eb consecutive elements, gathered
//     from or scattered to shared memory element by element.
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBatch = 3;
constexpr int kMaxRowDims = 4;
#ifndef DCOPY_PERM_PACKED
#define DCOPY_PERM_PACKED 1  // aligned tiles: packed [e][d] shared layout (0: element gather)
#endif
#ifndef DCOPY_ROWS_SHIFT
#define DCOPY_ROWS_SHIFT 1  // rows of narrow units through rows_shift (shift_rows_pay)
#endif
#ifndef DCOPY_PERM_MINB1
#define DCOPY_PERM_MINB1 7  // 1-byte packed tiles: resident CTAs per SM the registers must allow
                            // (measured: 59 registers, 4 CTAs/SM 4445-4780 GB/s; 32, 7 CTAs/SM
                            // 5578-5966 on B200)
#endif
#ifndef DCOPY_PERM_MINB
#define DCOPY_PERM_MINB 8  // wider packed tiles: resident CTAs per SM the registers must allow
#endif
#ifndef DCOPY_PERM_TD4
#define DCOPY_PERM_TD4 64  // 4-byte elements: tile rows (destination axis)
#endif
#ifndef DCOPY_PERM_TE4
#define DCOPY_PERM_TE4 64  // 4-byte elements: tile columns (source axis)
#endif
#ifndef DCOPY_PERM_TD2
#define DCOPY_PERM_TD2 64  // 2-byte elements: tile rows (destination axis)
#endif
#ifndef DCOPY_PERM_TE2
#define DCOPY_PERM_TE2 64  // 2-byte elements: tile columns (source axis)
#endif

// ---- rows ----------------------------------------------------------------------

struct PermRGeom {
  uint32_t vpr;               // units per row
  FastDiv f_vpr;
  uint32_t nd;                // row dims (outermost first), 0..4
  uint32_t size[kMaxRowDims];
  FastDiv f_size[kMaxRowDims];
  uint64_t ss[kMaxRowDims];   // source stride of each row dim, in units
  uint64_t ds[kMaxRowDims];   // destination stride of each row dim, in units (strided rows)
  uint64_t total;             // units (per launch below 2^31)
};

// kStridedDst: destination rows follow their own strides (NDDMA boxes); else the
// destination is contiguous and unit i lands at dst[i].  kHalfLine: source loads
// fill 64-byte half lines of L2 (gapped rows that do not cover whole lines).
template <typename T, bool kStridedDst, bool kHalfLine>
__global__ void __launch_bounds__(kThreads) perm_rows_kernel(T *__restrict__ dst,
                                                             const T *__restrict__ src,
                                                             PermRGeom g) {
  constexpr int U = 4;
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t total = (uint32_t)g.total;  // < 2^31 per launch (the host chunks)
  for (uint32_t base = blockIdx.x * kThreads * U + threadIdx.x; base < total;
       base += gridDim.x * kThreads * U) {
    T v[U];
    uint64_t at[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * kThreads;
      at[u] = ~0ull;
      if (i >= total) continue;
      uint32_t rem = g.f_vpr.div(i);
      const uint32_t col = i - rem * g.vpr;
      uint64_t so = col, dof = col;
#pragma unroll
      for (int k = kMaxRowDims - 1; k >= 0; --k) {
        if (k < (int)g.nd) {
          const uint32_t q = g.f_size[k].div(rem);
          const uint64_t idx = rem - q * g.size[k];
          so += idx * g.ss[k];
          if constexpr (kStridedDst) dof += idx * g.ds[k];
          rem = q;
        }
      }
      if constexpr (kHalfLine)
        v[u] = ld_stream_half_line(src + so);
      else
        v[u] = ld_stream(src + so);
      at[u] = kStridedDst ? dof : i;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (at[u] != ~0ull) dst[at[u]] = v[u];
  }
}

// ---- tiles ---------------------------------------------------------------------

struct PermTGeom {
  uint32_t D, E;              // extents of d (dst-contiguous) and e (src-contiguous)
  uint32_t TD, TE, P;         // tile extents, shared row pitch (elements)
  uint32_t dtiles, etiles;
  FastDiv f_dtiles, f_etiles;
  uint32_t nb;                // batch dims (outermost first)
  uint32_t bsize[kMaxBatch];
  FastDiv f_bsize[kMaxBatch];
  uint64_t bss[kMaxBatch], bds[kMaxBatch];  // batch strides, elements
  uint64_t s_d, t_e;          // source stride of d, destination stride of e
};

// Tile edge in elements: 64 for elements of up to 4 bytes, 32 for 8, 16 for 16.
template <typename T>
struct PermEdge {
  static constexpr uint32_t value = sizeof(T) <= 4 ? 64 : (sizeof(T) == 8 ? 32 : 16);
};

template <typename T, int V>
struct PermPack {
  using A = typename std::conditional<V == 1, T, uint4>::type;
  union U {
    A a;
    T e[V];
  };
};

template <typename T, int V>
__global__ void __launch_bounds__(kThreads) perm_tile_kernel(T *__restrict__ dst,
                                                             const T *__restrict__ src,
                                                             PermTGeom g, uint32_t ntiles) {
  using Pack = typename PermPack<T, V>::U;
  using A = typename PermPack<T, V>::A;
  extern __shared__ __align__(16) unsigned char perm_smem[];
  T *tile = reinterpret_cast<T *>(perm_smem);
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  constexpr uint32_t kEdge = PermEdge<T>::value;
  constexpr uint32_t ev = kEdge / V, dv = kEdge / V;  // vectors per tile row on each side
  for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint32_t q = g.f_etiles.div(t), et = t - q * g.etiles;
    uint32_t b = g.f_dtiles.div(q);
    const uint32_t dt = q - b * g.dtiles;
    uint64_t sb = 0, db = 0;
#pragma unroll
    for (int k = kMaxBatch - 1; k >= 0; --k) {
      if (k < (int)g.nb) {
        const uint32_t qq = g.f_bsize[k].div(b);
        const uint32_t idx = b - qq * g.bsize[k];
        sb += (uint64_t)idx * g.bss[k];
        db += (uint64_t)idx * g.bds[k];
        b = qq;
      }
    }
    const uint32_t d0 = dt * kEdge, e0 = et * kEdge;
    const uint32_t dw = min(kEdge, g.D - d0), ew = min(kEdge, g.E - e0);
    // ---- source rows (along e) -> shared memory [d][e]
    for (uint32_t u = threadIdx.x; u < dw * ev; u += kThreads) {
      const uint32_t r = u / ev, e = (u - r * ev) * V;
      if (e >= ew) continue;
      const T *sp = src + sb + (uint64_t)(d0 + r) * g.s_d + e0 + e;
      Pack x;
      if (e + V <= ew) {
        x.a = ld_stream(reinterpret_cast<const A *>(sp));
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) x.e[j] = e + j < ew ? sp[j] : T();
      }
      if (V * sizeof(T) == 16) {  // word-aligned: the pitch and e are multiples of 4 bytes
        uint32_t *w = reinterpret_cast<uint32_t *>(tile + r * g.P + e);
        const uint32_t *xw = reinterpret_cast<const uint32_t *>(&x);
        w[0] = xw[0];
        w[1] = xw[1];
        w[2] = xw[2];
        w[3] = xw[3];
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) tile[r * g.P + e + j] = x.e[j];
      }
    }
    __syncthreads();
    // ---- shared memory -> destination rows (along d)
    for (uint32_t u = threadIdx.x; u < ew * dv; u += kThreads) {
      const uint32_t c = u / dv, d = (u - c * dv) * V;
      if (d >= dw) continue;
      T *dp = dst + db + (uint64_t)(e0 + c) * g.t_e + d0 + d;
      Pack x;
#pragma unroll
      for (int j = 0; j < V; ++j) x.e[j] = tile[(d + j) * g.P + c];
      if (d + V <= dw) {
        *reinterpret_cast<A *>(dp) = x.a;
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j)
          if (d + j < dw) dp[j] = x.e[j];
      }
    }
    __syncthreads();
  }
}

// Aligned tiles: G = 4/eb source rows (eb <= 4) are read as 16-byte vectors
// along e and interleaved with byte permutes into 32-bit words, so shared memory
// holds the tile already transposed, [e][d] with d contiguous, and each 16-byte
// destination vector is one shared-memory load.  A warp reads 8 consecutive
// e-vectors (128 contiguous bytes) of 4 row groups; the 16-byte chunks of each
// shared row are XOR-swizzled with the row's e-vector index, so the word stores
// of those 32 lanes hit 32 distinct banks and the chunk loads stay conflict-free.
template <typename T, int V, int G, int TD, int TE>
__global__ void __launch_bounds__(kThreads, sizeof(T) == 1 ? DCOPY_PERM_MINB1 : DCOPY_PERM_MINB)
    perm_tile_packed_kernel(T *__restrict__ dst,
                                                                    const T *__restrict__ src,
                                                                    PermTGeom g,
                                                                    uint32_t ntiles) {
  static_assert(V * sizeof(T) == 16, "16-byte vectors");
  static_assert(G * sizeof(T) == 4 || G == 1, "a row group fills one 32-bit word");
  constexpr uint32_t kGroups = TD / G, kEv = TE / V, kDv = TD / V;
  static_assert(kEv % 8 == 0 && kGroups % 4 == 0 && (kDv & (kDv - 1)) == 0, "tile shape");
  union Vec {
    uint4 u;
    uint32_t w[4];
    T e[V];
  };
  extern __shared__ __align__(16) unsigned char perm_smem[];
  T *tile = reinterpret_cast<T *>(perm_smem);
  // Element offset of (row r of the [e][d] tile, column d): chunk-swizzled.
  auto at = [](uint32_t r, uint32_t d) {
    return r * TD + (((d / V) ^ ((r / V) & (kDv - 1))) * V) + d % V;
  };
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint32_t q = g.f_etiles.div(t), et = t - q * g.etiles;
    uint32_t b = g.f_dtiles.div(q);
    const uint32_t dt = q - b * g.dtiles;
    uint64_t sb = 0, db = 0;
#pragma unroll
    for (int k = kMaxBatch - 1; k >= 0; --k) {
      if (k < (int)g.nb) {
        const uint32_t qq = g.f_bsize[k].div(b);
        const uint32_t idx = b - qq * g.bsize[k];
        sb += (uint64_t)idx * g.bss[k];
        db += (uint64_t)idx * g.bds[k];
        b = qq;
      }
    }
    const uint32_t d0 = dt * TD, e0 = et * TE;
    const uint32_t dw = min((uint32_t)TD, g.D - d0), ew = min((uint32_t)TE, g.E - e0);
    // ---- G source rows x V elements -> V words (or elements) of the [e][d] tile
    for (uint32_t u = threadIdx.x; u < kGroups * kEv; u += kThreads) {
      const uint32_t lane = u & 31, wu = u >> 5;
      const uint32_t ev = (wu % (kEv / 8)) * 8 + (lane & 7);
      const uint32_t dg = (wu / (kEv / 8)) * 4 + (lane >> 3);
      const uint32_t e = ev * V, d = dg * G;
      if (e >= ew || d >= dw) continue;
      Vec x[G];
#pragma unroll
      for (int k = 0; k < G; ++k) {
        if (d + k < dw) {
          const T *sp = src + sb + (uint64_t)(d0 + d + k) * g.s_d + e0 + e;
          if (e + V <= ew) {
            x[k].u = ld_stream(reinterpret_cast<const uint4 *>(sp));
          } else {
#pragma unroll
            for (int j = 0; j < V; ++j) x[k].e[j] = e + j < ew ? sp[j] : T();
          }
        } else {
          x[k].u = make_uint4(0, 0, 0, 0);
        }
      }
      if (G == 1) {
#pragma unroll
        for (int j = 0; j < V; ++j) tile[at(e + j, d)] = x[0].e[j];
      } else if (G == 2) {  // 2-byte elements: word = (row d, row d+1) of column e+j
#pragma unroll
        for (int j = 0; j < V; ++j)
          *reinterpret_cast<uint32_t *>(tile + at(e + j, d)) =
              __byte_perm(x[0].w[j / 2], x[1].w[j / 2], (j & 1) ? 0x7632 : 0x5410);
      } else {  // 1-byte elements: word = byte j of rows d..d+3
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t lo01 = __byte_perm(x[0].w[i], x[1].w[i], 0x5140);
          const uint32_t hi01 = __byte_perm(x[0].w[i], x[1].w[i], 0x7362);
          const uint32_t lo23 = __byte_perm(x[2].w[i], x[3].w[i], 0x5140);
          const uint32_t hi23 = __byte_perm(x[2].w[i], x[3].w[i], 0x7362);
          const uint32_t r = e + 4 * i;
          *reinterpret_cast<uint32_t *>(tile + at(r, d)) = __byte_perm(lo01, lo23, 0x5410);
          *reinterpret_cast<uint32_t *>(tile + at(r + 1, d)) = __byte_perm(lo01, lo23, 0x7632);
          *reinterpret_cast<uint32_t *>(tile + at(r + 2, d)) = __byte_perm(hi01, hi23, 0x5410);
          *reinterpret_cast<uint32_t *>(tile + at(r + 3, d)) = __byte_perm(hi01, hi23, 0x7632);
        }
      }
    }
    __syncthreads();
    // ---- [e][d] tile -> destination rows along d, one 16-byte load per vector
    for (uint32_t u = threadIdx.x; u < TE * kDv; u += kThreads) {
      const uint32_t c = u / kDv, d = (u - c * kDv) * V;
      if (c >= ew || d >= dw) continue;
      Vec x;
      x.u = *reinterpret_cast<const uint4 *>(tile + at(c, d));
      T *dp = dst + db + (uint64_t)(e0 + c) * g.t_e + d0 + d;
      if (d + V <= dw) {
        *reinterpret_cast<uint4 *>(dp) = x.u;
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j)
          if (d + j < dw) dp[j] = x.e[j];
      }
    }
    __syncthreads();
  }
}

template <typename T, bool kStridedDst>
int launch_rows(void *dst, const void *src, const PermRGeom &g0, uint64_t outer_ss,
                uint64_t outer_ds, bool half_line, cudaStream_t s) {
  // Chunk the outermost row dim so that one launch covers fewer than 2^31 units.
  uint64_t inner_units = g0.vpr;
  for (uint32_t k = 1; k < g0.nd; ++k) inner_units *= g0.size[k];
  const uint64_t outer = g0.nd ? g0.size[0] : 1;
  if (inner_units >= (1ull << 31))
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: %llu units per outer index",
                     (unsigned long long)inner_units);
  const uint64_t chunk = std::max<uint64_t>(1, ((1ull << 31) - 1) / inner_units);
  for (uint64_t o0 = 0; o0 < outer; o0 += chunk) {
    PermRGeom g = g0;
    const uint64_t n = std::min<uint64_t>(chunk, outer - o0);
    if (g.nd) {
      g.size[0] = (uint32_t)n;
      g.f_size[0] = FastDiv(g.size[0]);
    }
    g.total = n * inner_units;
    const uint64_t per_cta = (uint64_t)kThreads * 4;
    const uint32_t grid = (uint32_t)std::max<uint64_t>(1, (g.total + per_cta - 1) / per_cta);
    auto kernel = half_line ? perm_rows_kernel<T, kStridedDst, true>
                            : perm_rows_kernel<T, kStridedDst, false>;
    const int rc = launch(kernel, grid, dim3(kThreads), 0, s, "perm_rows_kernel",
                          static_cast<T *>(dst) + o0 * (kStridedDst ? outer_ds : inner_units),
                          static_cast<const T *>(src) + o0 * outer_ss, g);
    if (rc) return rc;
  }
  return DCOPY_OK;
}

template <typename T, int V>
int launch_tiles(void *dst, const void *src, const PermTGeom &g, uint32_t ntiles, cudaStream_t s) {
  const size_t smem = (size_t)g.TD * g.P * sizeof(T);
  const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
  return launch(perm_tile_kernel<T, V>, grid, dim3(kThreads), smem, s, "perm_tile_kernel",
                static_cast<T *>(dst), static_cast<const T *>(src), g, ntiles);
}

// Widest unit (<= 16 bytes, power of two) dividing every value given.
uint32_t unit_for(uint64_t key, int eb) {
  uint32_t us = 16;
  while (us > (uint32_t)eb && key % us) us >>= 1;
  return us;
}

// Rows of size[m-1] elements; ds == NULL: contiguous destination.
int run_rows(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
             const int64_t *ds, int eb, cudaStream_t s) {
  const uint64_t L = size[m - 1];
  uint64_t key = L * eb | (uintptr_t)dst | (uintptr_t)src;
  for (int k = 0; k < m - 1; ++k) key |= (uint64_t)ss[k] * eb | (ds ? (uint64_t)ds[k] * eb : 0);
  const uint32_t us = unit_for(key, eb);
  if (DCOPY_ROWS_SHIFT && shift_rows_pay(us, L * eb, true))
    return rows_shift(dst, src, m, size, ss, ds, eb, s);
  PermRGeom g{};
  g.vpr = (uint32_t)(L * eb / us);
  if ((uint64_t)g.vpr != L * eb / us)
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: rows of %llu elements are too long",
                     (unsigned long long)L);
  g.f_vpr = FastDiv(g.vpr);
  g.nd = (uint32_t)(m - 1);
  uint64_t rows = 1;
  for (int k = 0; k < m - 1; ++k) {
    if (size[k] > 0xFFFFFFFFull)
      return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: dim of %llu elements",
                       (unsigned long long)size[k]);
    g.size[k] = (uint32_t)size[k];
    g.f_size[k] = FastDiv(g.size[k]);
    g.ss[k] = (uint64_t)ss[k] * eb / us;
    g.ds[k] = ds ? (uint64_t)ds[k] * eb / us : 0;
    rows *= size[k];
  }
  g.total = rows * g.vpr;
  if (g.total == 0) return DCOPY_OK;
  const uint64_t outer_ss = g.nd ? g.ss[0] : 0, outer_ds = g.nd ? g.ds[0] : 0;
  // NDDMA boxes whose source rows have gaps behind them and do not cover whole
  // 128-byte lines: half-line L2 fills (transposes read every line whole).
  bool half_line = false;
  if (ds && m >= 2 && (uint64_t)ss[m - 2] != L) {
    uint64_t lines = L * eb | (uintptr_t)src;
    for (int k = 0; k < m - 1; ++k) lines |= (uint64_t)ss[k] * eb;
    half_line = lines % 128 != 0;
  }
  if (ds) {
    switch (us) {
      case 16: return launch_rows<uint4, true>(dst, src, g, outer_ss, outer_ds, half_line, s);
      case 8: return launch_rows<uint2, true>(dst, src, g, outer_ss, outer_ds, half_line, s);
      case 4: return launch_rows<uint32_t, true>(dst, src, g, outer_ss, outer_ds, half_line, s);
      case 2: return launch_rows<uint16_t, true>(dst, src, g, outer_ss, outer_ds, half_line, s);
      default: return launch_rows<uint8_t, true>(dst, src, g, outer_ss, outer_ds, half_line, s);
    }
  }
  switch (us) {
    case 16: return launch_rows<uint4, false>(dst, src, g, outer_ss, 0, half_line, s);
    case 8: return launch_rows<uint2, false>(dst, src, g, outer_ss, 0, half_line, s);
    case 4: return launch_rows<uint32_t, false>(dst, src, g, outer_ss, 0, half_line, s);
    case 2: return launch_rows<uint16_t, false>(dst, src, g, outer_ss, 0, half_line, s);
    default: return launch_rows<uint8_t, false>(dst, src, g, outer_ss, 0, half_line, s);
  }
}

// Tile geometry shared by both tile kernels; *ntiles = 0 when there is nothing to do.
int tile_geometry(int m, const uint64_t *size, const int64_t *ss, const int64_t *ds, int e,
                  uint32_t TD, uint32_t TE, PermTGeom *g, uint64_t *ntiles) {
  const int d = m - 1;
  *g = PermTGeom{};
  if (size[d] > 0x7FFFFFFFull || size[e] > 0x7FFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: dims beyond 32-bit tile indexing");
  g->D = (uint32_t)size[d];
  g->E = (uint32_t)size[e];
  g->TD = TD;
  g->TE = TE;
  g->dtiles = (g->D + TD - 1) / TD;
  g->etiles = (g->E + TE - 1) / TE;
  g->f_dtiles = FastDiv(std::max(1u, g->dtiles));
  g->f_etiles = FastDiv(std::max(1u, g->etiles));
  g->s_d = (uint64_t)ss[d];
  g->t_e = (uint64_t)ds[e];
  uint64_t batches = 1;
  int nb = 0;
  for (int k = 0; k < m; ++k) {
    if (k == d || k == e) continue;
    if (size[k] > 0xFFFFFFFFull || nb == kMaxBatch)
      return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: too many or too large batch dims");
    g->bsize[nb] = (uint32_t)size[k];
    g->f_bsize[nb] = FastDiv(g->bsize[nb]);
    g->bss[nb] = (uint64_t)ss[k];
    g->bds[nb] = (uint64_t)ds[k];
    batches *= size[k];
    ++nb;
  }
  g->nb = (uint32_t)nb;
  *ntiles = batches * g->dtiles * g->etiles;
  if (*ntiles > 0xFFFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: %llu tiles exceed 32-bit indexing",
                     (unsigned long long)*ntiles);
  return DCOPY_OK;
}

// Element-access tiles (unaligned rows, 16-byte elements).
template <typename T>
int run_tiles_elem(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
                   const int64_t *ds, int e, cudaStream_t s) {
  constexpr int eb = sizeof(T);
  const uint32_t edge = PermEdge<T>::value;
  PermTGeom g;
  uint64_t ntiles = 0;
  int rc = tile_geometry(m, size, ss, ds, e, edge, edge, &g, &ntiles);
  if (rc || ntiles == 0) return rc;
  if (eb >= 4) {
    g.P = edge + 1;  // odd element pitch
  } else {           // odd word pitch, whole words per row
    int64_t words = ((int64_t)edge * eb + 3) / 4;
    if (words % 2 == 0) ++words;
    g.P = (uint32_t)(words * 4 / eb);
  }
  return launch_tiles<T, 1>(dst, src, g, (uint32_t)ntiles, s);
}

// 16-byte-vector tiles gathering element by element from shared memory.
template <typename T, int V>
int run_tiles_vec(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
                  const int64_t *ds, int e, cudaStream_t s) {
  constexpr int eb = sizeof(T);
  const uint32_t edge = PermEdge<T>::value;
  PermTGeom g;
  uint64_t ntiles = 0;
  int rc = tile_geometry(m, size, ss, ds, e, edge, edge, &g, &ntiles);
  if (rc || ntiles == 0) return rc;
  if (eb >= 4) {
    g.P = edge + 1;
  } else {
    int64_t words = ((int64_t)edge * eb + 3) / 4;
    if (words % 2 == 0) ++words;
    g.P = (uint32_t)(words * 4 / eb);
  }
  return launch_tiles<T, V>(dst, src, g, (uint32_t)ntiles, s);
}

// 16-byte-vector tiles with rows packed into words in shared memory.
template <typename T, int TD, int TE>
int run_tiles_packed(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
                     const int64_t *ds, int e, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  constexpr int G = sizeof(T) >= 4 ? 1 : 4 / sizeof(T);
  PermTGeom g;
  uint64_t ntiles = 0;
  int rc = tile_geometry(m, size, ss, ds, e, TD, TE, &g, &ntiles);
  if (rc || ntiles == 0) return rc;
  const size_t smem = (size_t)TD * TE * sizeof(T);
  const uint32_t grid = std::max(1u, std::min<uint32_t>((uint32_t)ntiles, 0x7FFFFFFFu));
  return launch(perm_tile_packed_kernel<T, V, G, TD, TE>, grid, dim3(kThreads), smem, s,
                "perm_tile_packed_kernel", static_cast<T *>(dst), static_cast<const T *>(src), g,
                (uint32_t)ntiles);
}

}  // namespace

int permute_copy(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
                 const int64_t *ds, int eb, dcopy_stream_t stream) {
  if (m < 1 || m > 5)
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: %d non-trivial dims (at most 5)", m);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (ss[m - 1] == 1) return run_rows(dst, src, m, size, ss, nullptr, eb, s);
  int e = -1;
  for (int k = 0; k < m - 1; ++k)
    if (ss[k] == 1) e = k;
  if (e < 0)  // a source without a unit-stride axis: not a permutation of a dense tensor
    return set_error(DCOPY_ERR_UNSUPPORTED, "transpose: no unit-stride source axis");
  // 16-byte vectors on both sides when every row start is 16-byte aligned.
  uint64_t key = (uintptr_t)dst | (uintptr_t)src | (uint64_t)ss[m - 1] * eb | (uint64_t)ds[e] * eb;
  for (int k = 0; k < m; ++k)
    if (k != m - 1 && k != e) key |= (uint64_t)ss[k] * eb | (uint64_t)ds[k] * eb;
  const bool vec = key % 16 == 0 && eb <= 16;
  if (!DCOPY_PERM_PACKED && vec) {
    switch (eb) {
      case 1: return run_tiles_vec<uint8_t, 16>(dst, src, m, size, ss, ds, e, s);
      case 2: return run_tiles_vec<uint16_t, 8>(dst, src, m, size, ss, ds, e, s);
      case 4: return run_tiles_vec<uint32_t, 4>(dst, src, m, size, ss, ds, e, s);
      case 8: return run_tiles_vec<uint2, 2>(dst, src, m, size, ss, ds, e, s);
      default: break;
    }
  }
  switch (eb) {
    case 1:
      return vec ? run_tiles_packed<uint8_t, 128, 128>(dst, src, m, size, ss, ds, e, s)
                 : run_tiles_elem<uint8_t>(dst, src, m, size, ss, ds, e, s);
    case 2:
      return vec ? run_tiles_packed<uint16_t, DCOPY_PERM_TD2, DCOPY_PERM_TE2>(dst, src, m, size,
                                                                             ss, ds, e, s)
                 : run_tiles_elem<uint16_t>(dst, src, m, size, ss, ds, e, s);
    case 4:
      return vec ? run_tiles_packed<uint32_t, DCOPY_PERM_TD4, DCOPY_PERM_TE4>(dst, src, m, size,
                                                                             ss, ds, e, s)
                 : run_tiles_elem<uint32_t>(dst, src, m, size, ss, ds, e, s);
    case 8:
      return vec ? run_tiles_packed<uint2, 32, 32>(dst, src, m, size, ss, ds, e, s)
                 : run_tiles_elem<uint2>(dst, src, m, size, ss, ds, e, s);
    case 16: return run_tiles_elem<uint4>(dst, src, m, size, ss, ds, e, s);
    default:
      return set_error(DCOPY_ERR_DATATYPE_INVALID, "transpose: element of %d bytes", eb);
  }
}

// Strided rows (dcopy_copy_nd boxes whose innermost axis is contiguous on both
// sides): m <= 5 dims, row dims outermost first.  *taken = false when the box
// does not fit the row kernel's 32-bit unit indexing.
int rows_copy(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
              const int64_t *ds, int eb, dcopy_stream_t stream, bool *taken) {
  *taken = false;
  if (m < 2 || m > kMaxRowDims + 1 || ss[m - 1] != 1 || ds[m - 1] != 1) return DCOPY_OK;
  uint64_t inner = size[m - 1];  // elements per outer index, bounded like launch_rows
  for (int k = 1; k < m - 1; ++k) inner *= size[k];
  if (inner >= (1ull << 31)) return DCOPY_OK;
  *taken = true;
  return run_rows(dst, src, m, size, ss, ds, eb, reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace dcopy
