// FRACTAL_Z (convolution weights) TransData on sm_100a.
//
// Layout (format_transfer_fractal_z.cc:41-537, fracz_{nchw,hwcn,nhwc}.cc):
// FRACTAL_Z is [C1*H*W, N1, 16, C0], i.e. [c1][h][w][n][c0] with N padded to
// N1*16 and C to C1*C0 (zeros): element (c1, h, w, n, c0) holds weight
// (n, c = c1*C0 + c0, h, w).  Three data paths, by where the weight's innermost
// axis lands:
//   * NHWC: C is innermost on both sides.  For each (h, w) the weight is an
//     [N rows x C cols] matrix (row pitch H*W*C) cut into 16 x C0 blocks: the
//     tiled-format kernels of the NZ/ZZ transfers do it with these strides.
//   * NCHW, HWCN and ND [C, N]: C0 is innermost in FRACTAL_Z but not in the
//     source, so every block is a transpose.  fz_transpose_kernel stages a tile
//     in shared memory: it reads rows of the source's contiguous axis (HW for
//     NCHW, N for HWCN) and writes rows along FRACTAL_Z's contiguous run
//     (n*C0 + c0), zero-filling the padding.
//   * HWCN with groups > 1 (fractal_z.cc:276-359): block-diagonal group layout,
//     gathered element by element (fz_groups_kernel).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "bulk.cuh"
#include "common.cuh"
#include "internal.cuh"
#include "launch.cuh"

namespace dcopy {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kNi = 16;  // kNiSize, formats_definitions.h:19
enum : int32_t { kNchw = 0, kNhwc = 1, kNd = 2, kHwcn = 16 };

// One transposed tile family: per batch (c1, b2) an R x K block where
//   source element  = nd_base + ra*s_ra + rb*s_rb + k   (R = ra*RB + rb),
//   FRACTAL_Z index = fz_base + k*dk + R,
// valid (else zero / skipped) when ra < ra_valid, c1*C0 + rb < C, k < k_valid.
struct FzTGeom {
  uint32_t RT, KT;        // full tile extents
  uint32_t R_ext, K_ext;  // extents per batch
  uint32_t rtiles, ktiles, B2;
  uint32_t RB, ra_valid, k_valid, C, C0;
  uint32_t rw_last, kw_last;
  FastDiv f_rb, f_ktiles, f_rtiles, f_b2, f_kw, f_kw_last, f_rw, f_rw_last;
  uint64_t s_ra, s_rb, nd_c1, nd_b2, dk, fz_c1, fz_b2;
};

template <typename T, bool kToFz>
__global__ void __launch_bounds__(kThreads) fz_transpose_kernel(T *__restrict__ dst,
                                                                const T *__restrict__ src,
                                                                FzTGeom g, uint32_t ntiles) {
  extern __shared__ __align__(16) unsigned char fz_smem[];
  T *tile = reinterpret_cast<T *>(fz_smem);
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint32_t q2 = g.f_ktiles.div(t), kt = t - q2 * g.ktiles;
    const uint32_t q = g.f_rtiles.div(q2), rt = q2 - q * g.rtiles;
    const uint32_t c1 = g.f_b2.div(q), b2 = q - c1 * g.B2;
    const bool klast = kt == g.ktiles - 1, rlast = rt == g.rtiles - 1;
    const uint32_t kw = klast ? g.kw_last : g.KT, rw = rlast ? g.rw_last : g.RT;
    const FastDiv fkw = klast ? g.f_kw_last : g.f_kw, frw = rlast ? g.f_rw_last : g.f_rw;
    const uint32_t pitch = kw | 1;  // odd row pitch: the R-fastest reads spread over banks
    const uint32_t R0 = rt * g.RT, K0 = kt * g.KT;
    const uint32_t rb_valid = min(g.C0, g.C - c1 * g.C0);
    const uint64_t nd_base = c1 * g.nd_c1 + b2 * g.nd_b2;
    const uint64_t fz_base = c1 * g.fz_c1 + b2 * g.fz_b2;
    const uint32_t n = rw * kw;
    if (kToFz) {
      for (uint32_t j = threadIdx.x; j < n; j += kThreads) {  // source order: k fastest
        const uint32_t r = fkw.div(j), k = j - r * kw;
        const uint32_t R = R0 + r, ra = g.f_rb.div(R), rb = R - ra * g.RB;
        T v = T();
        if (ra < g.ra_valid && rb < rb_valid && K0 + k < g.k_valid)
          v = ld_stream(src + nd_base + ra * g.s_ra + rb * g.s_rb + K0 + k);
        tile[r * pitch + k] = v;
      }
      __syncthreads();
      for (uint32_t j = threadIdx.x; j < n; j += kThreads) {  // FRACTAL_Z order: R fastest
        const uint32_t k = frw.div(j), r = j - k * rw;
        dst[fz_base + (uint64_t)(K0 + k) * g.dk + R0 + r] = tile[r * pitch + k];
      }
    } else {
      for (uint32_t j = threadIdx.x; j < n; j += kThreads) {
        const uint32_t k = frw.div(j), r = j - k * rw;
        tile[r * pitch + k] = ld_stream(src + fz_base + (uint64_t)(K0 + k) * g.dk + R0 + r);
      }
      __syncthreads();
      for (uint32_t j = threadIdx.x; j < n; j += kThreads) {
        const uint32_t r = fkw.div(j), k = j - r * kw;
        const uint32_t R = R0 + r, ra = g.f_rb.div(R), rb = R - ra * g.RB;
        if (ra < g.ra_valid && rb < rb_valid && K0 + k < g.k_valid)
          dst[nd_base + ra * g.s_ra + rb * g.s_rb + K0 + k] = tile[r * pitch + k];
      }
    }
    __syncthreads();
  }
}

// HWCN -> FRACTAL_Z with groups (fractal_z.cc:276-359), destination-linear:
// destination (gb, c1, hw, co, c0) holds group g = gb*e_mult + e's weight when
// channel dci = c1*k + c0 and output co both fall in slot e, else zero.
struct FzGGeom {
  uint64_t total;
  uint64_t k, cout_opt, hw, c1_dim, e_mult, groups, cin, cout, n;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) fz_groups_kernel(T *__restrict__ dst,
                                                             const T *__restrict__ src,
                                                             FzGGeom g) {
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint64_t i = blockIdx.x * (uint64_t)kThreads + threadIdx.x; i < g.total;
       i += (uint64_t)gridDim.x * kThreads) {
    uint64_t rest = i;
    const uint64_t c0 = rest % g.k;
    rest /= g.k;
    const uint64_t co = rest % g.cout_opt;
    rest /= g.cout_opt;
    const uint64_t hw = rest % g.hw;
    rest /= g.hw;
    const uint64_t c1 = rest % g.c1_dim;
    const uint64_t gb = rest / g.c1_dim;
    const uint64_t dci = c1 * g.k + c0, e = dci / g.cin;
    T v = T();
    if (e < g.e_mult && co / g.cout == e && gb * g.e_mult + e < g.groups) {
      const uint64_t c = dci - e * g.cin, nn = co - e * g.cout;
      v = ld_stream(src + (hw * g.cin + c) * g.n + (gb * g.e_mult + e) * g.cout + nn);
    }
    dst[i] = v;
  }
}

// Vectorised NCHW / HWCN / ND <-> FRACTAL_Z for 1-, 2- and 4-byte elements when
// C0 is a power of two and C0*eb a multiple of 16 bytes.  A tile is S source
// segments of L contiguous elements, moved between global and shared memory in
// 16-byte vectors:
//   NCHW: tile (c1, n block of NB): segment = weight n's C0 channels of block c1,
//         L = C0*HW; the FRACTAL_Z side is HW runs of NB*C0 elements (pitch N1*16*C0).
//   HWCN / ND: tile (c1, hw, n block of KT): segment = one input channel's KT
//         consecutive n, L = KT; the FRACTAL_Z side is one run of KT*C0 elements.
// The FRACTAL_Z side moves V = 16/eb consecutive c0 values per 16-byte vector,
// each gathered from (scattered into) shared memory at stride B.  Shared memory
// rows have an odd pitch in 4-byte words, so both the row-wise and the strided
// accesses spread over the banks.
template <int EB>
struct FzLane;
template <>
struct FzLane<1> {
  using T = uint8_t;
  static constexpr int V = 16;
};
template <>
struct FzLane<2> {
  using T = uint16_t;
  static constexpr int V = 8;
};
template <>
struct FzLane<4> {
  using T = uint32_t;
  static constexpr int V = 4;
};

struct FzSGeom {
  uint32_t S, L, P;      // segments per tile, segment length, shared row pitch (elements)
  uint32_t VPS;          // 16-byte vectors per segment
  FastDiv f_vps;
  uint32_t C, C0, lc0, N, N1N0, HW;
  uint32_t lrv;          // log2 of the 16-byte vectors per FRACTAL_Z run (NB*C0/V or C0/V)
  uint32_t C1, c1_fast;  // NCHW: channel blocks; 1 = tiles walk them first
  FastDiv f_c1;
  uint32_t NB, nblocks;  // NCHW: n per tile, n blocks
  uint32_t KT, ktiles;   // HWCN: n per tile, n tiles
  FastDiv f_nblocks, f_ktiles, f_hw;
  uint64_t seg_stride;   // global elements between segments
};

constexpr int kLoadBatch = 4;

template <int EB, bool kToFz, bool kNchw>
__global__ void __launch_bounds__(kThreads) fz_vec_kernel(unsigned char *__restrict__ dst_b,
                                                          const unsigned char *__restrict__ src_b,
                                                          FzSGeom g, uint32_t ntiles) {
  using T = typename FzLane<EB>::T;
  constexpr int V = FzLane<EB>::V;
  union Pack {
    uint4 u;
    T e[V];
  };
  extern __shared__ __align__(16) unsigned char fz_vsmem[];
  T *tile = reinterpret_cast<T *>(fz_vsmem);
  T *dst = reinterpret_cast<T *>(dst_b);
  const T *src = reinterpret_cast<const T *>(src_b);
  pdl_trigger_at_entry();
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    // ---- tile geometry
    uint32_t c1, s_valid, l_valid, k_out, r_vecs;
    uint64_t seg_base, fz_base, dk;
    uint32_t A, B;  // shared index of FRACTAL_Z element (R, k): (R >> lc0)*A + (R & (C0-1))*B + k
    if (kNchw) {
      uint32_t nb;
      if (g.c1_fast) {
        nb = g.f_c1.div(t);
        c1 = t - nb * g.C1;
      } else {
        c1 = g.f_nblocks.div(t);
        nb = t - c1 * g.nblocks;
      }
      const uint32_t n0 = nb * g.NB;
      const uint32_t rb_valid = min(g.C0, g.C - c1 * g.C0);
      s_valid = n0 < g.N ? min(g.NB, g.N - n0) : 0;
      l_valid = rb_valid * g.HW;
      seg_base = (uint64_t)n0 * g.seg_stride + (uint64_t)c1 * g.C0 * g.HW;
      fz_base = ((uint64_t)c1 * g.HW * g.N1N0 + n0) * g.C0;
      dk = (uint64_t)g.N1N0 * g.C0;
      k_out = g.HW;
      r_vecs = g.NB * g.C0 / V;
      A = g.P;
      B = g.HW;
    } else {
      const uint32_t q = g.f_ktiles.div(t), kt = t - q * g.ktiles;
      c1 = g.f_hw.div(q);
      const uint32_t hw = q - c1 * g.HW, n0 = kt * g.KT;
      s_valid = min(g.C0, g.C - c1 * g.C0);
      l_valid = n0 < g.N ? min(g.KT, g.N - n0) : 0;
      seg_base = ((uint64_t)hw * g.C + (uint64_t)c1 * g.C0) * g.N + n0;
      fz_base = (((uint64_t)c1 * g.HW + hw) * g.N1N0 + n0) * g.C0;
      dk = g.C0;
      k_out = min(g.KT, g.N1N0 - n0);
      r_vecs = g.C0 / V;
      A = 0;
      B = g.P;
    }
    const uint32_t n_seg_vec = g.S * g.VPS, n_fz_vec = k_out * r_vecs;
    if (kToFz) {
      // ---- weight -> shared memory, 16 bytes per step, zero past the valid range
      // kLoadBatch loads are issued before their shared-memory stores, so each
      // thread keeps that many 16-byte reads in flight.
      for (uint32_t ub = threadIdx.x; ub < n_seg_vec; ub += kLoadBatch * kThreads) {
        Pack x[kLoadBatch];
        uint32_t at[kLoadBatch];
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          const uint32_t u = ub + b * kThreads;
          at[b] = 0xFFFFFFFFu;
          if (u >= n_seg_vec) continue;
          const uint32_t sg = g.f_vps.div(u), f0 = (u - sg * g.VPS) * V;
          const uint32_t lv = sg < s_valid ? l_valid : 0;
          const T *sp = src + seg_base + (uint64_t)sg * g.seg_stride + f0;
          if (f0 + V <= lv) {
            x[b].u = ld_stream(reinterpret_cast<const uint4 *>(sp));
          } else {
#pragma unroll
            for (int j = 0; j < V; ++j) x[b].e[j] = f0 + j < lv ? sp[j] : T(0);
          }
          at[b] = sg * g.P + f0;
        }
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          if (at[b] == 0xFFFFFFFFu) continue;
          uint32_t *w = reinterpret_cast<uint32_t *>(tile + at[b]);
          w[0] = x[b].u.x;
          w[1] = x[b].u.y;
          w[2] = x[b].u.z;
          w[3] = x[b].u.w;
        }
      }
      __syncthreads();
      // ---- shared memory -> FRACTAL_Z, V consecutive c0 per 16-byte store
      for (uint32_t u = threadIdx.x; u < n_fz_vec; u += kThreads) {
        const uint32_t k = u >> g.lrv, r0 = (u & (r_vecs - 1)) * V;
        const uint32_t base = (r0 >> g.lc0) * A + (r0 & (g.C0 - 1)) * B + k;
        Pack x;
#pragma unroll
        for (int j = 0; j < V; ++j) x.e[j] = tile[base + j * B];
        *reinterpret_cast<uint4 *>(dst + fz_base + (uint64_t)k * dk + r0) = x.u;
      }
    } else {
      // ---- FRACTAL_Z -> shared memory, kLoadBatch reads in flight per thread
      for (uint32_t ub = threadIdx.x; ub < n_fz_vec; ub += kLoadBatch * kThreads) {
        Pack x[kLoadBatch];
        uint32_t at[kLoadBatch];
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          const uint32_t u = ub + b * kThreads;
          at[b] = 0xFFFFFFFFu;
          if (u >= n_fz_vec) continue;
          const uint32_t k = u >> g.lrv, r0 = (u & (r_vecs - 1)) * V;
          at[b] = (r0 >> g.lc0) * A + (r0 & (g.C0 - 1)) * B + k;
          x[b].u = ld_stream(reinterpret_cast<const uint4 *>(src + fz_base + (uint64_t)k * dk + r0));
        }
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          if (at[b] == 0xFFFFFFFFu) continue;
#pragma unroll
          for (int j = 0; j < V; ++j) tile[at[b] + j * B] = x[b].e[j];
        }
      }
      __syncthreads();
      // ---- shared memory -> weight, valid range only
      for (uint32_t u = threadIdx.x; u < n_seg_vec; u += kThreads) {
        const uint32_t sg = g.f_vps.div(u), f0 = (u - sg * g.VPS) * V;
        const uint32_t lv = sg < s_valid ? l_valid : 0;
        if (f0 >= lv) continue;
        const uint32_t *w = reinterpret_cast<const uint32_t *>(tile + sg * g.P + f0);
        Pack x;
        x.u = make_uint4(w[0], w[1], w[2], w[3]);
        T *dp = dst + seg_base + (uint64_t)sg * g.seg_stride + f0;
        if (f0 + V <= lv) {
          *reinterpret_cast<uint4 *>(dp) = x.u;
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j)
            if (f0 + j < lv) dp[j] = x.e[j];
        }
      }
    }
    __syncthreads();
  }
}

bool fz_dims(int32_t fmt, const int64_t *s, int rank, int64_t *n, int64_t *c, int64_t *h,
             int64_t *w) {
  if (!s) return false;
  switch (fmt) {
    case kNchw:
      if (rank != 4) return false;
      *n = s[0], *c = s[1], *h = s[2], *w = s[3];
      return true;
    case kNhwc:
      if (rank != 4) return false;
      *n = s[0], *h = s[1], *w = s[2], *c = s[3];
      return true;
    case kHwcn:
      if (rank != 4) return false;
      *h = s[0], *w = s[1], *c = s[2], *n = s[3];
      return true;
    case kNd:  // fractal_z_tbe.cc: a 2-D [C, N] weight, H = W = 1
      if (rank != 2) return false;
      *c = s[0], *n = s[1], *h = 1, *w = 1;
      return true;
    default:
      return false;
  }
}

int64_t ge_ceil(int64_t n1, int64_t n2) {  // Ceil, formats_trans_utils.h:69-75
  if (n1 == 0) return 0;
  return (n2 != 0) ? (((n1 - 1) / n2) + 1) : 0;
}

int64_t ge_gcd(int64_t x, int64_t y) {  // Measure, formats_trans_utils.h:76-88
  int64_t z = y;
  if (y == 0) return -1;
  while (x % y != 0) {
    z = x % y;
    x = y;
    y = z;
  }
  return z;
}

int64_t ge_lcm(int64_t a, int64_t b) {  // Lcm, formats_trans_utils.h:90-96
  if (b == 0) return -1;
  return (a * b) / ge_gcd(a, b);
}

struct GroupsLayout {
  int64_t e_mult, c1_dim, g_dim, cout_opt;
};

// fractal_z.cc:77-87 and :289-298.  cin, cout, k > 0.
GroupsLayout groups_layout(int64_t cin, int64_t cout, int64_t k, int64_t groups) {
  GroupsLayout l{};
  l.e_mult = std::min(ge_lcm(ge_lcm(cin, k) / cin, ge_lcm(cout, kNi) / cout), groups);
  l.c1_dim = ge_ceil(l.e_mult * cin, k) * k / k;
  l.g_dim = ge_ceil(groups, l.e_mult);
  l.cout_opt = ge_ceil(cout * l.e_mult, kNi) * kNi;
  return l;
}

template <typename T>
int launch_transpose(void *dst, const void *src, const FzTGeom &g, uint32_t ntiles, bool to_fz,
                     cudaStream_t s) {
  const size_t smem = (size_t)g.RT * (g.KT | 1) * sizeof(T);
  const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
  T *d = static_cast<T *>(dst);
  const T *sp = static_cast<const T *>(src);
  if (to_fz)
    return launch(fz_transpose_kernel<T, true>, grid, dim3(kThreads), smem, s,
                  "fz_transpose_kernel", d, sp, g, ntiles);
  return launch(fz_transpose_kernel<T, false>, grid, dim3(kThreads), smem, s,
                "fz_transpose_kernel", d, sp, g, ntiles);
}

template <typename T>
int launch_groups(void *dst, const void *src, const FzGGeom &g, cudaStream_t s) {
  const uint64_t blocks = (g.total + kThreads - 1) / kThreads;
  const uint32_t grid = (uint32_t)std::max<uint64_t>(
      1, std::min<uint64_t>(blocks, (uint64_t)sm_count() * 16));
  return launch(fz_groups_kernel<T>, grid, dim3(kThreads), 0, s, "fz_groups_kernel",
                static_cast<T *>(dst), static_cast<const T *>(src), g);
}

constexpr size_t kVecSmemMax = 96 * 1024;  // shared memory of one vectorised tile
#ifndef DCOPY_FZ_NCHW_NB
#define DCOPY_FZ_NCHW_NB 64  // largest n block of an NCHW tile (a multiple of 16)
#endif
#ifndef DCOPY_FZ_NHWC_BATCH_FAST
#define DCOPY_FZ_NHWC_BATCH_FAST 1  // NHWC tiles: walk (h, w) first
#endif
#ifndef DCOPY_FZ_C1_FAST
#define DCOPY_FZ_C1_FAST 1  // NCHW tiles: walk the channel blocks first
#endif
#ifndef DCOPY_FZ_HWCN_ELEMS
#define DCOPY_FZ_HWCN_ELEMS 8192  // elements of an HWCN tile (C0 rows x KT)
#endif

uint32_t log2_of(uint64_t v) {
  uint32_t l = 0;
  while ((1ull << l) < v) ++l;
  return l;
}

template <int EB>
int launch_vec(bool nchw, bool to_fz, void *dst, const void *src, const FzSGeom &g,
               uint32_t ntiles, size_t smem, cudaStream_t s) {
  static std::atomic<bool> raised[4][128];  // per kernel, per device: 48 KiB+ opt-in done
  const int dev = current_device();
  const int which = (nchw ? 2 : 0) + (to_fz ? 1 : 0);
  void (*k)(unsigned char *, const unsigned char *, FzSGeom, uint32_t) =
      nchw ? (to_fz ? fz_vec_kernel<EB, true, true> : fz_vec_kernel<EB, false, true>)
           : (to_fz ? fz_vec_kernel<EB, true, false> : fz_vec_kernel<EB, false, false>);
  if (smem > 48 * 1024 && dev >= 0 && dev < 128 && !raised[which][dev].load()) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVecSmemMax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    raised[which][dev] = true;
  }
  const uint32_t grid = std::max(1u, std::min<uint32_t>(ntiles, 0x7FFFFFFFu));
  return launch(k, grid, dim3(kThreads), smem, s, "fz_vec_kernel",
                static_cast<unsigned char *>(dst), static_cast<const unsigned char *>(src), g,
                ntiles);
}

// ---- NCHW -> FRACTAL_Z with bulk-copied, double-buffered tiles ----------------------
//
// A tile is NB weights (rows n) of one channel block c1: per row the C0*HW
// contiguous source elements (c0, hw) of that block.  The rows arrive by
// cp.async.bulk (one per row, this GPU's memory, no multicast) into one of two
// shared stages while the other stage is turned into FRACTAL_Z, so the loads of
// the next tile are in flight during the whole gather of this one and hold no
// registers.  Gather mapping (lane = hw lo 2 bits | c0 vector q | row nl): a
// warp builds the 16-byte FRACTAL_Z vectors (hw, n, q) of 4 consecutive hw x all
// C0/V vectors x NL = 32/(4 C0/V) rows, reading element (n, q*V + j, hw) at
// n*P + (q*V + j)*HW + hw.  The row pitch P (a multiple of 16 bytes, as bulk
// copies need) has the word residue 32/NL mod 32: for odd HW every gather of a
// warp then reads distinct banks (two lanes reading one word share it).  Each
// warp writes 4 whole 128-byte-aligned runs of NL*C0 elements.  Rows of padding
// weights (n >= N) are zero-filled by the threads.  The mbarrier waits are
// bounded; a give-up is recorded (read through dcopy_tma_error) and the CTA
// waits (bounded) for its own copies before returning.
struct FzBGeom {
  uint32_t N, HW, C0, NB, P, L;  // elements; L = C0*HW, P = row pitch
  uint32_t lq, lnl, lnnb;        // log2(C0/V), log2(NL), log2(NB/NL)
  uint32_t nblocks, ntiles, C1;
  FastDiv f_nblocks;
  uint64_t seg_stride, N1N0;     // global elements between weights; padded weight count
  // Tile order (fz_tile): groups of gn weight blocks; inside a group the weight
  // block varies fastest, then the channel block.  The last group holds gn_last
  // blocks.  gn = nblocks is one group: weight blocks fastest over the whole tensor.
  uint32_t gn, last_grp;
  FastDiv f_group_tiles, f_gn, f_gn_last;  // gn * C1; gn; gn_last
};

// Tile t -> channel block c1 and weight block nb under the grouped order.
__device__ __forceinline__ void fz_tile(const FzBGeom &g, uint32_t t, uint32_t *c1,
                                        uint32_t *nb) {
  const uint32_t grp = g.f_group_tiles.div(t);
  const uint32_t r = t - grp * g.f_group_tiles.d;
  const FastDiv &f = grp == g.last_grp ? g.f_gn_last : g.f_gn;
  const uint32_t q = f.div(r);
  *c1 = q;
  *nb = grp * g.gn + (r - q * f.d);
}

// One group over the whole tensor (the order the kernels had before grouping).
void fz_tile_groups(FzBGeom &g, uint32_t gn) {
  gn = std::max(1u, std::min(gn, g.nblocks));
  g.gn = gn;
  g.last_grp = (g.nblocks - 1) / gn;
  g.f_group_tiles = FastDiv(gn * g.C1);
  g.f_gn = FastDiv(gn);
  g.f_gn_last = FastDiv(g.nblocks - g.last_grp * gn);
}

__device__ uint32_t g_fz_error;

// kTensor: the whole tile arrives as one 2-D tensor copy (map: [N rows][C*HW],
// box [NB][P]) instead of one bulk copy per row; rows past N come zero-filled.
// kWordHW (1-byte elements, C0 = 32, H*W = kWordHW): the gather works on 32-bit
// words instead of single bytes.  A thread takes one weight n and one group of
// four channels: the group's 4*kWordHW bytes ([c0][hw]) are kWordHW words of the
// stage row; for each hw, two byte permutes pick the four channels' bytes and a
// third joins them into the FRACTAL_Z word (c0 4*grp .. 4*grp+3 of (hw, n)).
// Eight lanes write the 32 bytes of one (hw, n), a warp four consecutive n: a
// 128-byte segment per hw.  The row pitch is 8 words modulo 32, so a warp's
// word loads (rows n..n+3, word kWordHW*grp + m) hit 32 distinct banks for
// kWordHW 9 or 25.  Shared loads per output byte: 1/4 (the byte gather: 1).
template <int EB, bool kTensor, int kWordHW = 0>
__global__ void __launch_bounds__(kThreads) fz_nchw_bulk_kernel(unsigned char *__restrict__ dst_b,
                                                                const unsigned char *__restrict__ src_b,
                                                                FzBGeom g,
                                                                const __grid_constant__ CUtensorMap map) {
  using T = typename FzLane<EB>::T;
  constexpr int V = FzLane<EB>::V;
  union Pack {
    uint4 u;
    T e[V];
  };
  extern __shared__ __align__(128) unsigned char fzb_smem[];
  __shared__ __align__(8) uint64_t bars[2];
  T *dst = reinterpret_cast<T *>(dst_b);
  const T *src = reinterpret_cast<const T *>(src_b);
  const uint32_t stage_elems = g.NB * g.P;
  const uint32_t row_bytes = g.L * EB;
  pdl_trigger_at_entry();
  if (threadIdx.x == 0) {
    bulk::mbar_init(&bars[0], 1);
    bulk::mbar_init(&bars[1], 1);
    bulk::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  // Tile t: channel block c1 and weights n0 = nb * NB in the grouped order (fz_tile).
  auto issue = [&](uint32_t t, int st) {
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    const uint32_t valid = n0 < g.N ? min(g.NB, g.N - n0) : 0;
    T *stage = reinterpret_cast<T *>(fzb_smem) + st * stage_elems;
    if constexpr (kTensor) {
      if (threadIdx.x == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                         bulk::smem_u32(&bars[st])),
                     "r"(stage_elems * EB)
                     : "memory");
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3}], [%4];" ::"r"(bulk::smem_u32(stage)),
            "l"(reinterpret_cast<uint64_t>(&map)), "r"((int32_t)(c1 * g.L)), "r"((int32_t)n0),
            "r"(bulk::smem_u32(&bars[st]))
            : "memory");
      }
      return;
    }
    if (threadIdx.x < 32) {
      if (threadIdx.x == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                         bulk::smem_u32(&bars[st])),
                     "r"(valid * row_bytes)
                     : "memory");
      __syncwarp();
      const T *base = src + (uint64_t)n0 * g.seg_stride + (uint64_t)c1 * g.L;
      for (uint32_t r = threadIdx.x; r < valid; r += 32)
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
            "[%3];" ::"r"(bulk::smem_u32(stage + r * g.P)),
            "l"(base + (uint64_t)r * g.seg_stride), "r"(row_bytes), "r"(bulk::smem_u32(&bars[st]))
            : "memory");
    }
    // Padding weights: zero rows, written by the threads (read after the
    // __syncthreads that ends the current tile).
    for (uint32_t i = threadIdx.x; i < (g.NB - valid) * (g.L / V); i += kThreads) {
      const uint32_t r = valid + i / (g.L / V), f = (i % (g.L / V)) * V;
      *reinterpret_cast<uint4 *>(stage + r * g.P + f) = make_uint4(0, 0, 0, 0);
    }
  };
  uint32_t k = 0;  // tiles of this CTA so far
  if (blockIdx.x < g.ntiles) issue(blockIdx.x, 0);
  __syncthreads();  // the first tile's zero rows are visible to every thread
  bool ok = true, next_issued = false;
  for (uint32_t t = blockIdx.x; t < g.ntiles; t += gridDim.x, ++k) {
    const int st = (int)(k & 1);
    next_issued = t + gridDim.x < g.ntiles;
    if (next_issued) issue(t + gridDim.x, st ^ 1);
    // Every thread polls the barrier; the give-up decision is made for the
    // whole CTA, so no thread leaves the loop while others wait at a barrier.
    const bool arrived = bulk::mbar_wait_bounded(&bars[st], (k >> 1) & 1);
    if (__syncthreads_or(!arrived)) {
      ok = false;
      break;
    }
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    const T *stage = reinterpret_cast<const T *>(fzb_smem) + st * stage_elems;
    T *out = dst + ((uint64_t)c1 * g.HW * g.N1N0 + n0) * g.C0;
    if constexpr (kWordHW > 0) {
      static_assert(EB == 1 || EB == 2, "the word gather moves 1- or 2-byte elements");
      const uint64_t hw_words = (uint64_t)g.N1N0 * 8;  // 32-bit words between hw planes
      for (uint32_t u = threadIdx.x; u < g.NB * 8; u += kThreads) {
        // Group grp: the 4 / EB channels whose elements fill bytes 4*grp..4*grp+3
        // of a 32-byte FRACTAL_Z row; in the NCHW row they are 4*kWordHW bytes.
        const uint32_t n = u >> 3, grp = u & 7;
        const uint32_t *row =
            reinterpret_cast<const uint32_t *>(stage + n * g.P) + kWordHW * grp;
        uint32_t w[kWordHW];
#pragma unroll
        for (int m = 0; m < kWordHW; ++m) w[m] = row[m];
        uint32_t *o = reinterpret_cast<uint32_t *>(reinterpret_cast<unsigned char *>(out) + n * 32) +
                      grp;
#pragma unroll
        for (int hw = 0; hw < kWordHW; ++hw) {
          // Channel i of the group is element kWordHW * i + hw of the group.
          constexpr int k = kWordHW;
          uint32_t word;
          if constexpr (EB == 1) {
            const uint32_t lo = __byte_perm(w[hw >> 2], w[(k + hw) >> 2],
                                            (hw & 3) | ((4 + ((k + hw) & 3)) << 4));
            const uint32_t hi =
                __byte_perm(w[(2 * k + hw) >> 2], w[(3 * k + hw) >> 2],
                            ((2 * k + hw) & 3) | ((4 + ((3 * k + hw) & 3)) << 4));
            word = __byte_perm(lo, hi, 0x5410);
          } else {
            // Element e is half e & 1 of word e >> 1: bytes 2 * (e & 1) and the next.
            const uint32_t s0 = 2 * (hw & 1), s1 = 4 + 2 * ((k + hw) & 1);
            word = __byte_perm(w[hw >> 1], w[(k + hw) >> 1],
                               s0 | ((s0 + 1) << 4) | (s1 << 8) | ((s1 + 1) << 12));
          }
          o[(uint64_t)hw * hw_words] = word;
        }
      }
    } else {
      const uint32_t lane = threadIdx.x & 31, q = (lane >> 2) & ((1u << g.lq) - 1);
      const uint32_t units = ((g.HW + 3) >> 2) << g.lnnb;
      for (uint32_t un = threadIdx.x >> 5; un < units; un += kThreads / 32) {
        const uint32_t hw = ((un >> g.lnnb) << 2) + (lane & 3);
        if (hw >= g.HW) continue;
        const uint32_t n = ((un & ((1u << g.lnnb) - 1)) << g.lnl) + (lane >> (2 + g.lq));
        const uint32_t at = n * g.P + q * V * g.HW + hw;
        Pack x;
#pragma unroll
        for (int j = 0; j < V; ++j) x.e[j] = stage[at + j * g.HW];
        *reinterpret_cast<uint4 *>(out + (uint64_t)hw * g.N1N0 * g.C0 + n * g.C0 + q * V) = x.u;
      }
    }
    __syncthreads();  // every read of this stage is done before it is refilled
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(&g_fz_error, 1u);
    // Wait (bounded) for the copies still in flight into either stage before
    // the CTA's shared memory is released.
    (void)bulk::mbar_wait_bounded(&bars[k & 1], (k >> 1) & 1);
    if (next_issued) (void)bulk::mbar_wait_bounded(&bars[(k + 1) & 1], ((k + 1) >> 1) & 1);
  }
}

// ---- FRACTAL_Z -> NCHW, the mirror of fz_nchw_bulk_kernel -------------------------

#ifndef DCOPY_FZ_FROM_LSU_ROWS
// 1: the row stage of fz_to_nchw_bulk_kernel leaves by 16-byte stores of every
// thread instead of bulk stores issued by one warp, which the next tile had to
// wait for before reusing the stage.  Measured on B200 (dcopy_bench fz --replay
// 1, two rounds, GB/s, bulk stores vs 16-byte stores): int8 [2048,2048,3,3]
// 4087-4091 vs 5141, [4096,2048,3,3] 5097-5106 vs 5210-5212, [2048,1024,5,5]
// 4648-4650 vs 5067-5072; fp32 [2048,2048,3,3] 5141-5164 vs 5190-5196.
#define DCOPY_FZ_FROM_LSU_ROWS 1
#endif
#ifndef DCOPY_FZ_FROM_ROWS2
// 1: fz_to_nchw_bulk_kernel alternates two row stages, so a tile's scatter need
// not wait for the previous tile's row stores to read the stage.  Measured on
// B200 (dcopy_bench fz --replay 1, fp16 word scatter, GB/s, one stage vs two):
// [1024,2048,3,3] 4257-4291 vs 3773-3787, [2048,2048,3,3] 5327-5331 vs
// 4332-4334, [4096,2048,3,3] 5442-5452 vs 4831, [2048,1024,5,5] 5220-5239 vs
// 5553-5580; int8 3x3 4091 vs 3586-3597, fp32 3x3 5155 vs 4963-4972.  The
// second stage costs a resident CTA per SM; off.
#define DCOPY_FZ_FROM_ROWS2 0
#endif
//
// A tile is NB weights of one channel block.  Its FRACTAL_Z source is HW
// contiguous runs of NB*C0 elements (one per hw), bulk-copied into one of two
// "run" stages while the other is processed.  Each warp reads 16-byte FRACTAL_Z
// vectors (hw, n, q) from the run stage (4 consecutive hw x the C0/V vectors x
// NL rows: four 128-byte segments per warp read) and scatters their V elements
// into a row stage laid out as the NCHW rows (n, c0*HW + hw) with the bank-spread
// pitch of the other direction, so the scatter is conflict-free for odd HW.  The
// valid rows then leave by bulk stores (one per row); the row stage is reused
// once those stores have read it.  Waits are bounded as in the other direction.
// kWordHW (1-byte elements, C0 = 32, H*W = kWordHW): the scatter works on 32-bit
// words, the mirror of the word gather of fz_nchw_bulk_kernel.  A thread takes
// one weight n and one group of four channels, loads the group's FRACTAL_Z word
// for every hw (a warp: 32 consecutive words of a run), and writes the group's
// 4*kWordHW contiguous row bytes as kWordHW words, each joined from the bytes of
// up to four of those words with three byte permutes; the row pitch of 8 words
// modulo 32 keeps the warp's word stores conflict-free for kWordHW 9 or 25.
template <int EB, int kWordHW = 0>
__global__ void __launch_bounds__(kThreads) fz_to_nchw_bulk_kernel(unsigned char *__restrict__ dst_b,
                                                                   const unsigned char *__restrict__ src_b,
                                                                   FzBGeom g) {
  using T = typename FzLane<EB>::T;
  constexpr int V = FzLane<EB>::V;
  union Pack {
    uint4 u;
    T e[V];
  };
  extern __shared__ __align__(128) unsigned char fzr_smem[];
  __shared__ __align__(8) uint64_t bars[2];
  T *dst = reinterpret_cast<T *>(dst_b);
  const T *src = reinterpret_cast<const T *>(src_b);
  const uint32_t run = g.NB * g.C0;          // elements of one hw run
  const uint32_t run_stage = g.HW * run;     // elements of one run stage
  // NB x P row stage(s): with DCOPY_FZ_FROM_ROWS2 two, used by alternate tiles.
  T *const rows0 = reinterpret_cast<T *>(fzr_smem) + 2 * run_stage;
  pdl_trigger_at_entry();
  if (threadIdx.x == 0) {
    bulk::mbar_init(&bars[0], 1);
    bulk::mbar_init(&bars[1], 1);
    bulk::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  auto issue = [&](uint32_t t, int st) {
    if (threadIdx.x >= 32) return;
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    T *stage = reinterpret_cast<T *>(fzr_smem) + st * run_stage;
    if (threadIdx.x == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                       bulk::smem_u32(&bars[st])),
                   "r"(run_stage * EB)
                   : "memory");
    __syncwarp();
    const T *base = src + ((uint64_t)c1 * g.HW * g.N1N0 + n0) * g.C0;
    for (uint32_t hw = threadIdx.x; hw < g.HW; hw += 32)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(bulk::smem_u32(stage + hw * run)),
          "l"(base + (uint64_t)hw * g.N1N0 * g.C0), "r"(run * EB), "r"(bulk::smem_u32(&bars[st]))
          : "memory");
  };
  uint32_t k = 0;
  if (blockIdx.x < g.ntiles) issue(blockIdx.x, 0);
  bool ok = true, next_issued = false;
  for (uint32_t t = blockIdx.x; t < g.ntiles; t += gridDim.x, ++k) {
    const int st = (int)(k & 1);
    next_issued = t + gridDim.x < g.ntiles;
    if (next_issued) issue(t + gridDim.x, st ^ 1);
    const bool arrived = bulk::mbar_wait_bounded(&bars[st], (k >> 1) & 1);
    // The row stores that read this tile's row stage (the previous tile's, or with
    // two stages the one before it) must be done reading before it is overwritten;
    // warp 0 issued them, one bulk group per lane per tile.
    T *rows = rows0 + (DCOPY_FZ_FROM_ROWS2 ? (k & 1) * g.NB * g.P : 0);
    if (threadIdx.x < 32) {
      if (DCOPY_FZ_FROM_ROWS2)
        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      else
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    if (__syncthreads_or(!arrived)) {
      ok = false;
      break;
    }
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    const uint32_t valid = n0 < g.N ? min(g.NB, g.N - n0) : 0;
    const T *stage = reinterpret_cast<const T *>(fzr_smem) + st * run_stage;
    if constexpr (kWordHW > 0) {
      static_assert(EB == 1 || EB == 2, "the word scatter moves 1- or 2-byte elements");
      for (uint32_t u = threadIdx.x; u < valid * 8; u += kThreads) {
        const uint32_t n = u >> 3, grp = u & 7;
        uint32_t w[kWordHW];
#pragma unroll
        for (int hw = 0; hw < kWordHW; ++hw)
          w[hw] = *reinterpret_cast<const uint32_t *>(
              reinterpret_cast<const unsigned char *>(stage + hw * run) + n * 32 + 4 * grp);
        uint32_t *o = reinterpret_cast<uint32_t *>(rows + n * g.P) + kWordHW * grp;
#pragma unroll
        for (int m = 0; m < kWordHW; ++m) {
          constexpr int k = kWordHW;
          if constexpr (EB == 1) {
            // Row byte 4m+b of the group is channel (4m+b)/k at hw (4m+b)%k, i.e.
            // byte (4m+b)/k of FRACTAL_Z word (4m+b)%k.
            const uint32_t lo = __byte_perm(w[(4 * m) % k], w[(4 * m + 1) % k],
                                            ((4 * m) / k) | ((4 + (4 * m + 1) / k) << 4));
            const uint32_t hi = __byte_perm(w[(4 * m + 2) % k], w[(4 * m + 3) % k],
                                            ((4 * m + 2) / k) | ((4 + (4 * m + 3) / k) << 4));
            o[m] = __byte_perm(lo, hi, 0x5410);
          } else {
            // Row element 2m+b of the group is channel (2m+b)/k at hw (2m+b)%k, i.e.
            // half (2m+b)/k of FRACTAL_Z word (2m+b)%k.
            const uint32_t s0 = 2 * ((2 * m) / k), s1 = 4 + 2 * ((2 * m + 1) / k);
            o[m] = __byte_perm(w[(2 * m) % k], w[(2 * m + 1) % k],
                               s0 | ((s0 + 1) << 4) | (s1 << 8) | ((s1 + 1) << 12));
          }
        }
      }
    } else {
      const uint32_t lane = threadIdx.x & 31, q = (lane >> 2) & ((1u << g.lq) - 1);
      const uint32_t units = ((g.HW + 3) >> 2) << g.lnnb;
      for (uint32_t un = threadIdx.x >> 5; un < units; un += kThreads / 32) {
        const uint32_t hw = ((un >> g.lnnb) << 2) + (lane & 3);
        const uint32_t n = ((un & ((1u << g.lnnb) - 1)) << g.lnl) + (lane >> (2 + g.lq));
        if (hw >= g.HW || n >= valid) continue;
        Pack x;
        x.u = *reinterpret_cast<const uint4 *>(stage + hw * run + n * g.C0 + q * V);
        const uint32_t at = n * g.P + q * V * g.HW + hw;
#pragma unroll
        for (int j = 0; j < V; ++j) rows[at + j * g.HW] = x.e[j];
      }
    }
    T *out = dst + (uint64_t)n0 * g.seg_stride + (uint64_t)c1 * g.L;
    if (DCOPY_FZ_FROM_LSU_ROWS) {
      // Every thread copies 16-byte vectors of the row stage to the rows; the
      // barrier after the copy frees the stage for the next tile.
      __syncthreads();
      const uint32_t vpr = g.L * EB / 16;  // 16-byte vectors per row
      for (uint32_t u = threadIdx.x; u < valid * vpr; u += kThreads) {
        const uint32_t r = u / vpr, v = u - r * vpr;
        *reinterpret_cast<uint4 *>(reinterpret_cast<unsigned char *>(out + (uint64_t)r * g.seg_stride) +
                                   16 * v) =
            *reinterpret_cast<const uint4 *>(reinterpret_cast<const unsigned char *>(rows + r * g.P) +
                                             16 * v);
      }
      __syncthreads();
    } else {
      // Generic-proxy writes of the row stage, then bulk stores read it.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (threadIdx.x < 32) {
        for (uint32_t r = threadIdx.x; r < valid; r += 32)
          bulk::store(out + (uint64_t)r * g.seg_stride, rows + r * g.P, g.L * EB);
        bulk::commit();
      }
    }
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(&g_fz_error, 1u);
    (void)bulk::mbar_wait_bounded(&bars[k & 1], (k >> 1) & 1);
    if (next_issued) (void)bulk::mbar_wait_bounded(&bars[(k + 1) & 1], ((k + 1) >> 1) & 1);
  }
  if (threadIdx.x < 32) bulk::wait_all();
}

// FRACTAL_Z -> NCHW gathering row vectors straight from the run stage: the HW
// runs of a tile arrive as in fz_to_nchw_bulk_kernel (run pitch R chosen on the
// host to spread this kernel's bank pattern); thread u builds the 16-byte row
// vector v of weight n (u = n * L/V + v) from the V elements (c0, hw) it covers,
// each at hw*R + n*C0 + c0, and stores it to the NCHW row.
template <int EB>
__global__ void __launch_bounds__(kThreads) fz_to_nchw_gather_kernel(unsigned char *__restrict__ dst_b,
                                                                     const unsigned char *__restrict__ src_b,
                                                                     FzBGeom g, uint32_t R,
                                                                     FastDiv f_vpr, FastDiv f_hw) {
  using T = typename FzLane<EB>::T;
  constexpr int V = FzLane<EB>::V;
  union Pack {
    uint4 u;
    T e[V];
  };
  extern __shared__ __align__(128) unsigned char fzg_smem[];
  __shared__ __align__(8) uint64_t bars[2];
  T *dst = reinterpret_cast<T *>(dst_b);
  const T *src = reinterpret_cast<const T *>(src_b);
  const uint32_t run = g.NB * g.C0;
  const uint32_t run_stage = g.HW * R;
  pdl_trigger_at_entry();
  if (threadIdx.x == 0) {
    bulk::mbar_init(&bars[0], 1);
    bulk::mbar_init(&bars[1], 1);
    bulk::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  auto issue = [&](uint32_t t, int st) {
    if (threadIdx.x >= 32) return;
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    T *stage = reinterpret_cast<T *>(fzg_smem) + st * run_stage;
    if (threadIdx.x == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                       bulk::smem_u32(&bars[st])),
                   "r"(g.HW * run * EB)
                   : "memory");
    __syncwarp();
    const T *base = src + ((uint64_t)c1 * g.HW * g.N1N0 + n0) * g.C0;
    for (uint32_t hw = threadIdx.x; hw < g.HW; hw += 32)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(bulk::smem_u32(stage + hw * R)),
          "l"(base + (uint64_t)hw * g.N1N0 * g.C0), "r"(run * EB), "r"(bulk::smem_u32(&bars[st]))
          : "memory");
  };
  const uint32_t vpr = g.L / V;
  uint32_t k = 0;
  if (blockIdx.x < g.ntiles) issue(blockIdx.x, 0);
  bool ok = true, next_issued = false;
  for (uint32_t t = blockIdx.x; t < g.ntiles; t += gridDim.x, ++k) {
    const int st = (int)(k & 1);
    next_issued = t + gridDim.x < g.ntiles;
    if (next_issued) issue(t + gridDim.x, st ^ 1);
    const bool arrived = bulk::mbar_wait_bounded(&bars[st], (k >> 1) & 1);
    if (__syncthreads_or(!arrived)) {
      ok = false;
      break;
    }
    uint32_t c1, nb;
    fz_tile(g, t, &c1, &nb);
    const uint32_t n0 = nb * g.NB;
    const uint32_t valid = n0 < g.N ? min(g.NB, g.N - n0) : 0;
    const T *stage = reinterpret_cast<const T *>(fzg_smem) + st * run_stage;
    T *out = dst + (uint64_t)n0 * g.seg_stride + (uint64_t)c1 * g.L;
    for (uint32_t u = threadIdx.x; u < valid * vpr; u += kThreads) {
      const uint32_t n = f_vpr.div(u), e0 = (u - n * vpr) * V;
      uint32_t c0 = f_hw.div(e0), hw = e0 - c0 * g.HW;
      Pack x;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        x.e[j] = stage[hw * R + n * g.C0 + c0];
        if (++hw == g.HW) {
          hw = 0;
          ++c0;
        }
      }
      *reinterpret_cast<uint4 *>(out + (uint64_t)n * g.seg_stride + e0) = x.u;
    }
    __syncthreads();  // every read of this stage is done before it is refilled
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(&g_fz_error, 1u);
    (void)bulk::mbar_wait_bounded(&bars[k & 1], (k >> 1) & 1);
    if (next_issued) (void)bulk::mbar_wait_bounded(&bars[(k + 1) & 1], ((k + 1) >> 1) & 1);
  }
}

// ---- HWCN -> FRACTAL_Z with tensor-copied, double-buffered tiles ------------------
//
// For one hw and channel block c1 the HWCN weight holds C0 rows (channels) of N
// contiguous outputs; FRACTAL_Z wants the transpose, [n][c0], as one run of
// N1*16*C0 elements.  A tile is KT consecutive n of that block: one 2-D tensor
// copy (source view [H*W*C rows][N], box [C0][KT]; outputs past N arrive as
// zeros) fills one of two shared stages while the other is turned into
// FRACTAL_Z.  Each warp instruction reads one channel row for 32 consecutive n,
// so every shared load is conflict-free; lane n stores its 16-byte vector of V
// consecutive c0.  Waits are bounded as in the NCHW kernels.
struct FzHGeom {
  uint32_t HW, C0, KT, N1N0, C;  // C: channels (a multiple of C0)
  uint32_t ktiles, ntiles;
  FastDiv f_ktiles, f_hw;
};

template <int EB>
__global__ void __launch_bounds__(kThreads) fz_hwcn_tensor_kernel(unsigned char *__restrict__ dst_b,
                                                                  FzHGeom g,
                                                                  const __grid_constant__ CUtensorMap map) {
  using T = typename FzLane<EB>::T;
  constexpr int V = FzLane<EB>::V;
  union Pack {
    uint4 u;
    T e[V];
  };
  extern __shared__ __align__(128) unsigned char fzh_smem[];
  __shared__ __align__(8) uint64_t bars[2];
  T *dst = reinterpret_cast<T *>(dst_b);
  const uint32_t stage_elems = g.C0 * g.KT;
  pdl_trigger_at_entry();
  if (threadIdx.x == 0) {
    bulk::mbar_init(&bars[0], 1);
    bulk::mbar_init(&bars[1], 1);
    bulk::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  // Tile t: (c1, hw) = divmod(t / ktiles, HW), n block kt = t % ktiles.
  auto coords = [&](uint32_t t, uint32_t *c1, uint32_t *hw, uint32_t *kt) {
    const uint32_t q = g.f_ktiles.div(t);
    *kt = t - q * g.ktiles;
    *c1 = g.f_hw.div(q);
    *hw = q - *c1 * g.HW;
  };
  auto issue = [&](uint32_t t, int st) {
    if (threadIdx.x != 0) return;
    uint32_t c1, hw, kt;
    coords(t, &c1, &hw, &kt);
    T *stage = reinterpret_cast<T *>(fzh_smem) + st * stage_elems;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     bulk::smem_u32(&bars[st])),
                 "r"(stage_elems * EB)
                 : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(bulk::smem_u32(stage)),
        "l"(reinterpret_cast<uint64_t>(&map)), "r"((int32_t)(kt * g.KT)),
        "r"((int32_t)(hw * g.C + c1 * g.C0)), "r"(bulk::smem_u32(&bars[st]))
        : "memory");
  };
  uint32_t k = 0;
  if (blockIdx.x < g.ntiles) issue(blockIdx.x, 0);
  bool ok = true, next_issued = false;
  for (uint32_t t = blockIdx.x; t < g.ntiles; t += gridDim.x, ++k) {
    const int st = (int)(k & 1);
    next_issued = t + gridDim.x < g.ntiles;
    if (next_issued) issue(t + gridDim.x, st ^ 1);
    const bool arrived = bulk::mbar_wait_bounded(&bars[st], (k >> 1) & 1);
    if (__syncthreads_or(!arrived)) {
      ok = false;
      break;
    }
    uint32_t c1, hw, kt;
    coords(t, &c1, &hw, &kt);
    const uint32_t n0 = kt * g.KT, kn = min(g.KT, g.N1N0 - n0);
    const T *stage = reinterpret_cast<const T *>(fzh_smem) + st * stage_elems;
    T *out = dst + (((uint64_t)c1 * g.HW + hw) * g.N1N0 + n0) * g.C0;
    const uint32_t Q = g.C0 / V;
    for (uint32_t u = threadIdx.x; u < ((kn + 31) & ~31u) * Q; u += kThreads) {
      // Warp-uniform vector q, 32 consecutive n per warp instruction.
      const uint32_t q = (u >> 5) % Q, n = ((u >> 5) / Q << 5) + (u & 31);
      if (n >= kn) continue;
      Pack x;
#pragma unroll
      for (int j = 0; j < V; ++j) x.e[j] = stage[(q * V + j) * g.KT + n];
      *reinterpret_cast<uint4 *>(out + (uint64_t)n * g.C0 + q * V) = x.u;
    }
    __syncthreads();  // every read of this stage is done before it is refilled
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(&g_fz_error, 1u);
    (void)bulk::mbar_wait_bounded(&bars[k & 1], (k >> 1) & 1);
    if (next_issued) (void)bulk::mbar_wait_bounded(&bars[(k + 1) & 1], ((k + 1) >> 1) & 1);
  }
}

#ifndef DCOPY_FZ_HWCN_TMA
// HWCN -> FRACTAL_Z through fz_hwcn_tensor_kernel for 1-byte elements.  Measured
// on B200 as bench.py does (CUDA graph replay of two alternating weight sets, no
// L2 eviction; three interleaved rounds, GB/s against fz_vec_kernel): int8
// [2048,2048,3,3] (c0 32) 4613-4619 vs 4331-4347; fp16 3x3 5111-5132 vs
// 5457-5463, fp16 1x1 (C 8192) 4673-4675 vs 4868-4905, fp16 5x5 (C 1024)
// 5267-5282 vs 5687-5690, fp16 [4096,2048,3,3] 5230-5247 vs 5876-5885.  (With
// L2 evicted between reps the fp16 cases had read 2-14 % faster: that timing
// leaves the writes still dirty in L2 untimed.)  fp32 3x3 was 7 % slower under
// either timing.  So only 1-byte elements take this kernel.
#define DCOPY_FZ_HWCN_TMA 1
#endif

#ifndef DCOPY_FZ_NCHW_BULK
#define DCOPY_FZ_NCHW_BULK 1
#endif
#ifndef DCOPY_FZ_NCHW_BULK_FROM
// FRACTAL_Z -> NCHW through fz_to_nchw_bulk_kernel for 4-byte elements.  Measured
// on B200 ([2048,2048,3,3], three rounds, GB/s against fz_vec_kernel): fp32
// 5571-5651 vs 4956-5005; fp16 3832-3880 vs 4604-4608, int8 2748-2836 vs
// 3225-3356, fp16 5x5 3794 vs 4184-4265 -- so 1- and 2-byte elements keep the
// vector kernel.
#define DCOPY_FZ_NCHW_BULK_FROM 1
#endif
#ifndef DCOPY_FZ_FROM_GATHER
// 2-byte FRACTAL_Z -> NCHW through fz_to_nchw_gather_kernel.  Measured on B200
// (three rounds, GB/s against fz_vec_kernel): fp16 [2048,2048,3,3] 5266 vs
// 4608-4610, fp16 [2048,1024,5,5] 5063-5122 vs 4100-4267; int8 (c0 32) was
// slower (3074-3206 vs 3351-3356) and keeps the vector kernel.
#define DCOPY_FZ_FROM_GATHER 1
#endif
#ifndef DCOPY_FZ_NCHW_TMA
// 1: one 2-D tensor copy per tile of 1- or 2-byte elements when the pitch fits a
// TMA box.  Measured on B200 (NCHW -> FRACTAL_Z [2048,2048,3,3], three rounds):
// fp16 5263-5266 GB/s against 4606-4608 with one bulk copy per row; fp32 tiles
// were 7 % slower as a tensor copy (5263-5266 against 5670-5673), so 4-byte
// elements keep the row copies.
#define DCOPY_FZ_NCHW_TMA 1
#endif
#ifndef DCOPY_FZ_INT8_WORDS
// int8 NCHW -> FRACTAL_Z 3x3 / 5x5 (C0 32): the 32-bit word gather of
// fz_nchw_bulk_kernel.  Measured on B200 (dcopy_bench fz --eb 1 --c0 32 --replay
// 1, two rounds, GB/s against the byte gather): [2048,2048,3,3] 5258 vs
// 3874-3878, [4096,2048,3,3] 5575-5626 vs 4584-4589, [2048,1024,5,5] 5344-5360
// vs 4721-4769, [512,512,3,3] 1141 vs 914.
#define DCOPY_FZ_INT8_WORDS 1
#endif
#ifndef DCOPY_FZ_INT8_WORDS_FROM
// int8 FRACTAL_Z -> NCHW 3x3 / 5x5 (C0 32): the 32-bit word scatter of
// fz_to_nchw_bulk_kernel, when there are at least as many tiles as resident
// CTAs.  Measured on B200 (dcopy_bench fz --eb 1 --c0 32 --replay 1, two rounds,
// GB/s against fz_vec_kernel): [2048,2048,3,3] 4091 vs 3868-3876,
// [4096,2048,3,3] 5086-5099 vs 4334, [2048,1024,5,5] 4650-4657 vs 3578-3586;
// [512,512,3,3] (128 tiles, no second tile for any CTA) 918 vs 1146, hence the
// tile-count condition.
#define DCOPY_FZ_INT8_WORDS_FROM 1
#endif
#ifndef DCOPY_FZ_FP16_WORDS
// fp16 NCHW -> FRACTAL_Z 3x3 / 5x5 (C0 16): the word gather (one byte permute
// per FRACTAL_Z word).  Measured on B200 (dcopy_bench fz --replay 1, two rounds,
// GB/s against the element gather): [1024,2048,3,3] 5501-5534 vs 4708-4720,
// [2048,2048,3,3] 5550-5558 vs 5185, [4096,2048,3,3] 5433-5435 vs 4937-4938,
// [2048,1024,5,5] 5289-5292 vs 5053-5082, [4096,1024,5,5] 5381-5410 vs
// 5072-5079, [512,512,3,3] 3031-3035 vs 2292-2293.
#define DCOPY_FZ_FP16_WORDS 1
#endif
#ifndef DCOPY_FZ_FP16_WORDS_FROM
// fp16 FRACTAL_Z -> NCHW 3x3 / 5x5 (C0 16): the word scatter of
// fz_to_nchw_bulk_kernel instead of the row-vector gather, when there are at
// least as many tiles as resident CTAs.  Measured on B200 (dcopy_bench fz
// --replay 1, two rounds, GB/s against the gather), with the row stage copied
// out by 16-byte stores: [1024,2048,3,3] 5236-5250 vs 4573-4579,
// [2048,2048,3,3] 5300-5316 vs 5270-5283, [4096,2048,3,3] 5127-5134 vs
// 4843-4959, [2048,1024,5,5] 5550-5556 vs 5245, [4096,1024,5,5] 5942-5943 vs
// 5606-5611.  (With bulk stores out of the row stage it had lost at
// [1024,2048,3,3] and 5x5.)
#define DCOPY_FZ_FP16_WORDS_FROM 1
#endif
#ifndef DCOPY_FZ_GROUP_TILES
#define DCOPY_FZ_GROUP_TILES 1  // 0: one group (weight blocks fastest over the whole tensor)
#endif
#ifndef DCOPY_FZ_ROW_RUN
// Bytes of an NCHW row that the resident tiles of the bulk / gather kernels
// cover together (fz_tile_groups).  Measured on B200 (dcopy_bench fz --replay 1,
// fp16 3x3 [N,2048] to / from FRACTAL_Z, GB/s, against one group over the whole
// tensor): N 2048 5229-5244 / 5287-5291 vs 5187-5210 / 5113-5127, N 4096
// 4931-4938 / 4929-4931 vs 4783-4786 / 4582-4585, N 8192 4980-4992 / 4738-4742
// vs 4777-4779 / 4356-4361; fp16 5x5 [4096,1024] from 5580-5598 vs 5254-5265,
// [2048,1024] from 5242-5247 vs 5337-5343; fp32 3x3 [4096,2048] 5216-5241 /
// 5100-5104 vs 5134-5136 / 4935-5000.  16 and 32 KiB runs were in between.
#define DCOPY_FZ_ROW_RUN 65536
#endif
#ifndef DCOPY_FZ_NCHW_TMA_PROMOTION
#define DCOPY_FZ_NCHW_TMA_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif
#ifndef DCOPY_FZ_BULK_NB
#define DCOPY_FZ_BULK_NB 64  // weights per tile (a power of two)
#endif
constexpr size_t kBulkSmemMax = 96 * 1024;  // both stages

// NCHW -> FRACTAL_Z through fz_nchw_bulk_kernel when every channel block is
// whole, rows are 16-byte granules and both buffers are this GPU's memory.
int run_nchw_bulk(void *dst, const void *src, int64_t n, int64_t c, int64_t hw, int eb,
                  int64_t c0, cudaStream_t s, bool *taken) {
  *taken = false;
  if (!DCOPY_FZ_NCHW_BULK || (eb != 1 && eb != 2 && eb != 4)) return DCOPY_OK;
  const int64_t V = 16 / eb;
  if (c0 <= 0 || (c0 & (c0 - 1)) || c0 % V || c % c0 || (c * hw * eb) % 16) return DCOPY_OK;
  if (((uintptr_t)dst | (uintptr_t)src) % 16) return DCOPY_OK;
  if (!is_local_device_memory(src) || !is_local_device_memory(dst)) return DCOPY_OK;
  const int64_t Q = c0 / V;
  if (Q > 8) return DCOPY_OK;
  const int64_t NL = 8 / Q, n1n0 = ge_ceil(n, kNi) * kNi, L = c0 * hw;
  if ((uint64_t)L * eb >= (1u << 20) || n1n0 * c0 * hw > 0x7FFFFFFFll ||
      n > 0x7FFFFFFFll || c * hw > 0x7FFFFFFFll)
    return DCOPY_OK;
  int64_t words = (L * eb + 3) / 4;
  words += ((32 / NL - words % 32) % 32 + 32) % 32;
  const int64_t P = words * 4 / eb;
  int64_t nb = DCOPY_FZ_BULK_NB;
  while (nb > NL && (n1n0 % nb || (size_t)(2 * nb * P * eb) > kBulkSmemMax)) nb /= 2;
  if (n1n0 % nb || (size_t)(2 * nb * P * eb) > kBulkSmemMax || nb < NL) return DCOPY_OK;
  FzBGeom g{};
  g.N = (uint32_t)n;
  g.HW = (uint32_t)hw;
  g.C0 = (uint32_t)c0;
  g.NB = (uint32_t)nb;
  g.P = (uint32_t)P;
  g.L = (uint32_t)L;
  g.lq = log2_of((uint64_t)Q);
  g.lnl = log2_of((uint64_t)NL);
  g.lnnb = log2_of((uint64_t)(nb / NL));
  g.nblocks = (uint32_t)(n1n0 / nb);
  g.C1 = (uint32_t)(c / c0);
  const uint64_t ntiles = (uint64_t)g.C1 * g.nblocks;
  if (ntiles == 0 || ntiles > 0x7FFFFFFFull) return DCOPY_OK;
  g.ntiles = (uint32_t)ntiles;
  g.f_nblocks = FastDiv(g.nblocks);
  fz_tile_groups(g, g.nblocks);
  g.seg_stride = (uint64_t)(c * hw);
  g.N1N0 = (uint64_t)n1n0;
  const size_t smem = (size_t)(2 * nb * P * eb);
  // The tensor copy: a [N][C*HW] view, box [nb][P] (P <= 256 elements).
  CUtensorMap map{};
  bool tensor = false;
  // (Each stage must start on a 128-byte boundary for the tensor copy.)
  if (DCOPY_FZ_NCHW_TMA && eb <= 2 && P <= 256 && nb <= 256 && (nb * P * eb) % 128 == 0) {
    const uint64_t dims[2] = {(uint64_t)(c * hw), (uint64_t)n};
    const uint64_t strides[1] = {(uint64_t)(c * hw * eb)};
    const uint32_t box[2] = {(uint32_t)P, (uint32_t)nb};
    const CUtensorMapDataType dt = eb == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : eb == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                             : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    tensor = encode_tiled_map(&map, dt, 2, const_cast<void *>(src), dims, strides, box,
                              DCOPY_FZ_NCHW_TMA_PROMOTION);
  }
  using Kern = void (*)(unsigned char *, const unsigned char *, FzBGeom, const CUtensorMap);
  Kern k = tensor ? (eb == 1   ? fz_nchw_bulk_kernel<1, true>
                     : eb == 2 ? fz_nchw_bulk_kernel<2, true>
                               : fz_nchw_bulk_kernel<4, true>)
                  : (eb == 1   ? fz_nchw_bulk_kernel<1, false>
                     : eb == 2 ? fz_nchw_bulk_kernel<2, false>
                               : fz_nchw_bulk_kernel<4, false>);
  int which = (eb == 1 ? 0 : eb == 2 ? 1 : 2) + (tensor ? 3 : 0);
  // 1-byte elements with C0 = 32 (or 2-byte with C0 = 16) and 3x3 or 5x5
  // windows: the word gather (the row pitch the formula above gives is then 8
  // words modulo 32).
  const bool pitch_ok = (P * eb / 4) % 32 == 8 && (hw == 9 || hw == 25);
  if (DCOPY_FZ_INT8_WORDS && eb == 1 && c0 == 32 && !tensor && pitch_ok) {
    k = hw == 9 ? fz_nchw_bulk_kernel<1, false, 9> : fz_nchw_bulk_kernel<1, false, 25>;
    which = hw == 9 ? 6 : 7;
  } else if (DCOPY_FZ_FP16_WORDS && eb == 2 && c0 == 16 && pitch_ok) {
    k = tensor ? (hw == 9 ? fz_nchw_bulk_kernel<2, true, 9> : fz_nchw_bulk_kernel<2, true, 25>)
               : (hw == 9 ? fz_nchw_bulk_kernel<2, false, 9> : fz_nchw_bulk_kernel<2, false, 25>);
    which = 8 + (hw == 9 ? 0 : 1) + (tensor ? 2 : 0);
  }
  static std::atomic<bool> raised[12][128];
  const int dev = current_device();
  if (dev >= 0 && dev < 128 && !raised[which][dev].load()) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmemMax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fz_nchw_bulk_kernel)");
    raised[which][dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  *taken = true;
  const uint32_t grid =
      (uint32_t)std::min<uint64_t>(ntiles, (uint64_t)per_sm * (uint64_t)sm_count());
  // The resident tiles read, in every NCHW row, the segments of the channel
  // blocks they cover: group the weight blocks so that run stays near
  // DCOPY_FZ_ROW_RUN bytes (see fz_tile_groups).
  if (DCOPY_FZ_GROUP_TILES)
    fz_tile_groups(g, (uint32_t)std::max<uint64_t>(
                          1, (uint64_t)grid * g.L * (uint64_t)eb / DCOPY_FZ_ROW_RUN));
  return launch(k, std::max(1u, grid), dim3(kThreads), smem, s, "fz_nchw_bulk_kernel",
                static_cast<unsigned char *>(dst), static_cast<const unsigned char *>(src), g,
                map);
}

// Run pitch (elements) for fz_to_nchw_gather_kernel: at least NB*C0, a multiple
// of 16 bytes, with the word residue mod 32 whose simulated warp accesses (the
// first tile's row vectors) hit the fewest words per bank.
uint32_t gather_run_pitch_search(int eb, int64_t c0, int64_t hw, int64_t nb) {
  const int64_t V = 16 / eb, L = c0 * hw, vpr = L / V, run = nb * c0;
  const int64_t base_w = run * eb / 4;
  int64_t best_w = base_w, best_cost = -1;
  for (int64_t res = 0; res < 32; res += 4) {
    const int64_t rw = base_w + ((res - base_w % 32) % 32 + 32) % 32;
    int64_t cost = 0;
    for (int64_t u0 = 0; u0 < nb * vpr; u0 += 32)
      for (int64_t j = 0; j < V; ++j) {
        int64_t words[32], banks_max = 0;
        int cnt = 0;
        for (int64_t lane = 0; lane < 32 && u0 + lane < nb * vpr; ++lane) {
          const int64_t u = u0 + lane, n = u / vpr, e = (u % vpr) * V + j;
          const int64_t c = e / hw, h = e % hw;
          words[cnt++] = ((h * rw * 4) + (n * c0 + c) * eb) / 4;
        }
        for (int b = 0; b < 32; ++b) {  // distinct words in bank b
          int64_t seen[32];
          int ns = 0;
          for (int i = 0; i < cnt; ++i)
            if (words[i] % 32 == b) {
              bool dup = false;
              for (int q = 0; q < ns; ++q) dup = dup || seen[q] == words[i];
              if (!dup) seen[ns++] = words[i];
            }
          banks_max = std::max<int64_t>(banks_max, ns);
        }
        cost += banks_max;
      }
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_w = rw;
    }
  }
  return (uint32_t)(best_w * 4 / eb);
}

// The search above, done once per (eb, c0, hw, nb).
uint32_t gather_run_pitch(int eb, int64_t c0, int64_t hw, int64_t nb) {
  static std::mutex mu;
  static std::map<std::tuple<int, int64_t, int64_t, int64_t>, uint32_t> cache;
  const auto key = std::make_tuple(eb, c0, hw, nb);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const uint32_t r = gather_run_pitch_search(eb, c0, hw, nb);
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = r;
  return r;
}

int launch_from_gather(void *dst, const void *src, FzBGeom g, int eb, int64_t c0,
                       int64_t hw, int64_t nb, cudaStream_t s, bool *taken) {
  const uint32_t R = gather_run_pitch(eb, c0, hw, nb);
  const size_t smem = (size_t)2 * hw * R * eb;
  if (smem > kBulkSmemMax) return DCOPY_OK;
  using Kern = void (*)(unsigned char *, const unsigned char *, FzBGeom, uint32_t, FastDiv,
                        FastDiv);
  Kern k = fz_to_nchw_gather_kernel<2>;
  static std::atomic<bool> raised[128];
  const int dev = current_device();
  if (eb != 2) return DCOPY_OK;
  if (dev >= 0 && dev < 128 && !raised[dev].load()) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmemMax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fz_to_nchw_gather_kernel)");
    raised[dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  *taken = true;
  const uint32_t grid =
      (uint32_t)std::min<uint64_t>(g.ntiles, (uint64_t)per_sm * (uint64_t)sm_count());
  // The resident tiles write, in every NCHW row, the segments of the channel
  // blocks they cover; grouping the weight blocks keeps that run of a row near
  // DCOPY_FZ_ROW_RUN bytes however many weights there are (one group over all
  // weight blocks left it at grid / nblocks segments: 2 KiB per row for 8192
  // fp16 3x3 weights).  A run longer than the row covers whole rows.
  if (DCOPY_FZ_GROUP_TILES)
    fz_tile_groups(g, (uint32_t)std::max<uint64_t>(
                          1, (uint64_t)grid * g.L * (uint64_t)eb / DCOPY_FZ_ROW_RUN));
  const uint32_t V = 16 / (uint32_t)eb;
  return launch(k, std::max(1u, grid), dim3(kThreads), smem, s, "fz_to_nchw_gather_kernel",
                static_cast<unsigned char *>(dst), static_cast<const unsigned char *>(src), g, R,
                FastDiv(g.L / V), FastDiv(g.HW));
}

// HWCN -> FRACTAL_Z through fz_hwcn_tensor_kernel when channel blocks are whole,
// output rows (N) are 16-byte granules and both buffers are this GPU's memory.
int run_hwcn_tensor(void *dst, const void *src, int64_t n, int64_t c, int64_t hw, int eb,
                    int64_t c0, cudaStream_t s, bool *taken) {
  *taken = false;
  if (!DCOPY_FZ_HWCN_TMA || eb != 1) return DCOPY_OK;
  const int64_t V = 16 / eb;
  if (c0 <= 0 || (c0 & (c0 - 1)) || c0 % V || c0 > 256 || c % c0 || (n * eb) % 16) return DCOPY_OK;
  if (((uintptr_t)dst | (uintptr_t)src) % 16) return DCOPY_OK;
  if (!is_local_device_memory(src) || !is_local_device_memory(dst)) return DCOPY_OK;
  const int64_t n1n0 = ge_ceil(n, kNi) * kNi;
  if (n1n0 * c0 * hw * ge_ceil(c, c0) > 0x7FFFFFFFll || hw * c > 0x7FFFFFFFll || n > 0x7FFFFFFFll)
    return DCOPY_OK;
  const int64_t KT = 256;  // box width: 256 outputs (a multiple of 16 bytes for every eb)
  const size_t smem = (size_t)(2 * c0 * KT * eb);
  if (smem > kBulkSmemMax) return DCOPY_OK;
  CUtensorMap map{};
  const uint64_t dims[2] = {(uint64_t)n, (uint64_t)(hw * c)};
  const uint64_t strides[1] = {(uint64_t)(n * eb)};
  const uint32_t box[2] = {(uint32_t)KT, (uint32_t)c0};
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (!encode_tiled_map(&map, dt, 2, const_cast<void *>(src), dims, strides, box,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return DCOPY_OK;
  FzHGeom g{};
  g.HW = (uint32_t)hw;
  g.C0 = (uint32_t)c0;
  g.KT = (uint32_t)KT;
  g.N1N0 = (uint32_t)n1n0;
  g.C = (uint32_t)c;
  g.ktiles = (uint32_t)ge_ceil(n1n0, KT);
  const uint64_t ntiles = (uint64_t)(c / c0) * hw * g.ktiles;
  if (ntiles == 0 || ntiles > 0x7FFFFFFFull) return DCOPY_OK;
  g.ntiles = (uint32_t)ntiles;
  g.f_ktiles = FastDiv(g.ktiles);
  g.f_hw = FastDiv(g.HW);
  using Kern = void (*)(unsigned char *, FzHGeom, const CUtensorMap);
  Kern k = fz_hwcn_tensor_kernel<1>;
  static std::atomic<bool> raised[128];
  const int dev = current_device();
  if (dev >= 0 && dev < 128 && !raised[dev].load()) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmemMax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fz_hwcn_tensor_kernel)");
    raised[dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  *taken = true;
  const uint32_t grid =
      (uint32_t)std::min<uint64_t>(ntiles, (uint64_t)per_sm * (uint64_t)sm_count());
  return launch(k, std::max(1u, grid), dim3(kThreads), smem, s, "fz_hwcn_tensor_kernel",
                static_cast<unsigned char *>(dst), g, map);
}

// FRACTAL_Z -> NCHW through fz_to_nchw_bulk_kernel under the same conditions.
int run_nchw_bulk_from(void *dst, const void *src, int64_t n, int64_t c, int64_t hw, int eb,
                       int64_t c0, cudaStream_t s, bool *taken) {
  *taken = false;
  const bool gather = DCOPY_FZ_FROM_GATHER && eb == 2;
  const bool word_scatter =
      (hw == 9 || hw == 25) && ((DCOPY_FZ_INT8_WORDS_FROM && eb == 1 && c0 == 32) ||
                                (DCOPY_FZ_FP16_WORDS_FROM && eb == 2 && c0 == 16));
  if (!gather && !word_scatter && (!DCOPY_FZ_NCHW_BULK_FROM || eb != 4)) return DCOPY_OK;
  const int64_t V = 16 / eb;
  if (c0 <= 0 || (c0 & (c0 - 1)) || c0 % V || c % c0 || (c * hw * eb) % 16) return DCOPY_OK;
  if (((uintptr_t)dst | (uintptr_t)src) % 16) return DCOPY_OK;
  if (!is_local_device_memory(src) || !is_local_device_memory(dst)) return DCOPY_OK;
  const int64_t Q = c0 / V;
  if (Q > 8) return DCOPY_OK;
  const int64_t NL = 8 / Q, n1n0 = ge_ceil(n, kNi) * kNi, L = c0 * hw;
  if ((uint64_t)L * eb >= (1u << 20) || n1n0 * c0 * hw > 0x7FFFFFFFll ||
      n > 0x7FFFFFFFll || c * hw > 0x7FFFFFFFll || hw > 0xFFFF)
    return DCOPY_OK;
  int64_t words = (L * eb + 3) / 4;
  words += ((32 / NL - words % 32) % 32 + 32) % 32;
  const int64_t P = words * 4 / eb;
  auto smem_of = [&](int64_t nb) {
    return (size_t)((2 * hw * nb * c0 + (DCOPY_FZ_FROM_ROWS2 ? 2 : 1) * nb * P) * eb);
  };
  int64_t nb = DCOPY_FZ_BULK_NB;
  while (nb > NL && (n1n0 % nb || smem_of(nb) > kBulkSmemMax)) nb /= 2;
  if (n1n0 % nb || smem_of(nb) > kBulkSmemMax || nb < NL) return DCOPY_OK;
  if ((nb * c0 * eb) % 16) return DCOPY_OK;
  FzBGeom g{};
  g.N = (uint32_t)n;
  g.HW = (uint32_t)hw;
  g.C0 = (uint32_t)c0;
  g.NB = (uint32_t)nb;
  g.P = (uint32_t)P;
  g.L = (uint32_t)L;
  g.lq = log2_of((uint64_t)Q);
  g.lnl = log2_of((uint64_t)NL);
  g.lnnb = log2_of((uint64_t)(nb / NL));
  g.nblocks = (uint32_t)(n1n0 / nb);
  g.C1 = (uint32_t)(c / c0);
  const uint64_t ntiles = (uint64_t)g.C1 * g.nblocks;
  if (ntiles == 0 || ntiles > 0x7FFFFFFFull) return DCOPY_OK;
  g.ntiles = (uint32_t)ntiles;
  g.f_nblocks = FastDiv(g.nblocks);
  fz_tile_groups(g, g.nblocks);
  g.seg_stride = (uint64_t)(c * hw);
  g.N1N0 = (uint64_t)n1n0;
  if (gather && !word_scatter) return launch_from_gather(dst, src, g, eb, c0, hw, nb, s, taken);
  const size_t smem = smem_of(nb);
  using Kern = void (*)(unsigned char *, const unsigned char *, FzBGeom);
  Kern k = fz_to_nchw_bulk_kernel<4>;
  int which = 0;
  if (word_scatter) {
    // The word scatter needs the row pitch at 8 words modulo 32 (what the pitch
    // formula above gives for 32-byte FRACTAL_Z rows).
    if ((P * eb / 4) % 32 != 8)
      return gather ? launch_from_gather(dst, src, g, eb, c0, hw, nb, s, taken) : DCOPY_OK;
    if (eb == 1) {
      k = hw == 9 ? fz_to_nchw_bulk_kernel<1, 9> : fz_to_nchw_bulk_kernel<1, 25>;
      which = hw == 9 ? 1 : 2;
    } else {
      k = hw == 9 ? fz_to_nchw_bulk_kernel<2, 9> : fz_to_nchw_bulk_kernel<2, 25>;
      which = hw == 9 ? 3 : 4;
    }
  }
  static std::atomic<bool> raised[5][128];
  const int dev = current_device();
  if (dev >= 0 && dev < 128 && !raised[which][dev].load()) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmemMax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fz_to_nchw_bulk_kernel)");
    raised[which][dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  // The word scatter pays only when CTAs get a second tile to overlap with;
  // fewer tiles than resident CTAs stay on the vector kernel.
  if (word_scatter && ntiles < (uint64_t)per_sm * (uint64_t)sm_count())
    return gather ? launch_from_gather(dst, src, g, eb, c0, hw, nb, s, taken) : DCOPY_OK;
  *taken = true;
  const uint32_t grid =
      (uint32_t)std::min<uint64_t>(ntiles, (uint64_t)per_sm * (uint64_t)sm_count());
  if (DCOPY_FZ_GROUP_TILES)
    fz_tile_groups(g, (uint32_t)std::max<uint64_t>(
                          1, (uint64_t)grid * g.L * (uint64_t)eb / DCOPY_FZ_ROW_RUN));
  return launch(k, std::max(1u, grid), dim3(kThreads), smem, s, "fz_to_nchw_bulk_kernel",
                static_cast<unsigned char *>(dst), static_cast<const unsigned char *>(src), g);
}

}  // namespace

// ORs the bulk FRACTAL_Z kernel's give-up flag into *flag and clears it.
int fz_error_take(uint32_t *flag) {
  uint32_t v = 0, zero = 0;
  DCOPY_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fz_error, sizeof(uint32_t)));
  DCOPY_CUDA_TRY(cudaMemcpyToSymbol(g_fz_error, &zero, sizeof(uint32_t)));
  *flag |= v;
  return DCOPY_OK;
}

namespace {

// The vectorised path when its conditions hold; *taken = false otherwise.
int run_vec(int32_t fmt, void *dst, const void *src, int64_t n, int64_t c, int64_t h, int64_t w,
            int eb, int64_t c0, bool to_fz, cudaStream_t s, bool *taken) {
  *taken = false;
  if (eb != 1 && eb != 2 && eb != 4) return DCOPY_OK;
  if (c0 <= 0 || (c0 & (c0 - 1)) || (c0 * eb) % 16 || c0 > 4096) return DCOPY_OK;
  if (((uintptr_t)dst | (uintptr_t)src) % 16) return DCOPY_OK;
  const int64_t V = 16 / eb, hw = h * w, n1n0 = ge_ceil(n, kNi) * kNi, c1 = ge_ceil(c, c0);
  if (n > 0x7FFFFFFFll || c > 0x7FFFFFFFll || hw > 0x7FFFFFFFll || n1n0 * c0 > 0x7FFFFFFFll)
    return DCOPY_OK;
  FzSGeom g{};
  g.C = (uint32_t)c;
  g.C0 = (uint32_t)c0;
  g.lc0 = log2_of((uint64_t)c0);
  g.N = (uint32_t)n;
  g.N1N0 = (uint32_t)n1n0;
  g.HW = (uint32_t)hw;
  auto pitch = [&](int64_t L) {  // odd number of 4-byte words
    int64_t words = (L * eb + 3) / 4;
    if (words % 2 == 0) ++words;
    return words * 4 / eb;
  };
  uint64_t ntiles;
  size_t smem;
  if (fmt == kNchw) {
    if ((c * hw * eb) % 16) return DCOPY_OK;  // segment starts must be 16-byte aligned
    int64_t nb = DCOPY_FZ_NCHW_NB;
    while (nb > 16 && n1n0 % nb) nb /= 2;  // whole blocks: the last one may not overrun N1*16
    const int64_t L = c0 * hw, P = pitch(L);
    while (nb > 1 && (size_t)(nb * P * eb) > kVecSmemMax) nb /= 2;
    if ((size_t)(nb * P * eb) > kVecSmemMax) return DCOPY_OK;
    g.S = (uint32_t)nb;
    g.L = (uint32_t)L;
    g.P = (uint32_t)P;
    g.NB = (uint32_t)nb;
    g.nblocks = (uint32_t)(n1n0 / nb);
    g.lrv = log2_of((uint64_t)(nb * c0 / V));
    g.seg_stride = (uint64_t)(c * hw);
    ntiles = (uint64_t)c1 * g.nblocks;
    smem = (size_t)(nb * P * eb);
  } else {  // HWCN, and ND [C, N] as HWCN with H = W = 1
    if ((n * eb) % 16) return DCOPY_OK;
    int64_t kt = std::max<int64_t>(V, (DCOPY_FZ_HWCN_ELEMS / c0) / V * V);
    kt = std::min<int64_t>(kt, n1n0);
    const int64_t P = pitch(kt);
    if ((size_t)(c0 * P * eb) > kVecSmemMax) return DCOPY_OK;
    g.S = (uint32_t)c0;
    g.L = (uint32_t)kt;
    g.P = (uint32_t)P;
    g.KT = (uint32_t)kt;
    g.ktiles = (uint32_t)ge_ceil(n1n0, kt);
    g.lrv = log2_of((uint64_t)(c0 / V));
    g.seg_stride = (uint64_t)n;
    ntiles = (uint64_t)c1 * hw * g.ktiles;
    smem = (size_t)(c0 * P * eb);
  }
  g.C1 = (uint32_t)c1;
  g.c1_fast = DCOPY_FZ_C1_FAST;
  g.f_c1 = FastDiv(std::max(1u, g.C1));
  g.VPS = g.L / (uint32_t)V;
  g.f_vps = FastDiv(g.VPS);
  g.f_nblocks = FastDiv(std::max(1u, g.nblocks));
  g.f_ktiles = FastDiv(std::max(1u, g.ktiles));
  g.f_hw = FastDiv(std::max(1u, g.HW));
  *taken = true;
  if (ntiles == 0) return DCOPY_OK;
  if (ntiles > 0xFFFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "FRACTAL_Z: %llu tiles exceed 32-bit indexing",
                     (unsigned long long)ntiles);
  const bool nchw = fmt == kNchw;
  switch (eb) {
    case 1: return launch_vec<1>(nchw, to_fz, dst, src, g, (uint32_t)ntiles, smem, s);
    case 2: return launch_vec<2>(nchw, to_fz, dst, src, g, (uint32_t)ntiles, smem, s);
    default: return launch_vec<4>(nchw, to_fz, dst, src, g, (uint32_t)ntiles, smem, s);
  }
}

// The NCHW / HWCN / ND (both directions) transposing path.
int run_transpose(int32_t fmt, void *dst, const void *src, int64_t n, int64_t c, int64_t h,
                  int64_t w, int eb, int64_t c0, bool to_fz, cudaStream_t s) {
  bool taken = false;
  if (fmt == kNchw) {
    const int brc = to_fz ? run_nchw_bulk(dst, src, n, c, h * w, eb, c0, s, &taken)
                          : run_nchw_bulk_from(dst, src, n, c, h * w, eb, c0, s, &taken);
    if (taken || brc) return brc;
  }
  if (fmt == kHwcn && to_fz) {
    const int hrc = run_hwcn_tensor(dst, src, n, c, h * w, eb, c0, s, &taken);
    if (taken || hrc) return hrc;
  }
  const int vrc = run_vec(fmt, dst, src, n, c, h, w, eb, c0, to_fz, s, &taken);
  if (taken || vrc) return vrc;
  const int64_t n1n0 = ge_ceil(n, kNi) * kNi, c1 = ge_ceil(c, c0), hw = h * w;
  FzTGeom g{};
  int64_t R_ext, K_ext, B2;
  if (fmt == kNchw) {  // rows R = (n, c0), columns k = hw
    R_ext = n1n0 * c0;
    K_ext = hw;
    B2 = 1;
    g.ra_valid = (uint32_t)n;
    g.k_valid = (uint32_t)hw;
    g.s_ra = (uint64_t)(c * hw);
    g.s_rb = (uint64_t)hw;
    g.nd_c1 = (uint64_t)(c0 * hw);
    g.nd_b2 = 0;
    g.dk = (uint64_t)(n1n0 * c0);
    g.fz_c1 = (uint64_t)(hw * n1n0 * c0);
    g.fz_b2 = 0;
  } else {  // HWCN / ND: rows R = c0, columns k = n; one batch per (c1, hw)
    R_ext = c0;
    K_ext = n1n0;
    B2 = hw;
    g.ra_valid = 1;
    g.k_valid = (uint32_t)n;
    g.s_ra = 0;
    g.s_rb = (uint64_t)n;
    g.nd_c1 = (uint64_t)(c0 * n);
    g.nd_b2 = (uint64_t)(c * n);
    g.dk = (uint64_t)c0;
    g.fz_c1 = (uint64_t)(hw * n1n0 * c0);
    g.fz_b2 = (uint64_t)(n1n0 * c0);
  }
  if (R_ext > 0x7FFFFFFFll || K_ext > 0x7FFFFFFFll || n > 0x7FFFFFFFll || c > 0x7FFFFFFFll ||
      c0 > 0x7FFFFFFFll || B2 > 0x7FFFFFFFll)
    return set_error(DCOPY_ERR_UNSUPPORTED, "FRACTAL_Z: dims beyond 32-bit tile indexing");
  const int64_t budget = eb <= 4 ? 4096 : (eb == 8 ? 2048 : 1024);  // elements per tile
  const int64_t KT = std::min<int64_t>(K_ext, R_ext >= 64 ? 64 : std::max<int64_t>(1, budget / R_ext));
  const int64_t RT = std::min<int64_t>(R_ext, std::max<int64_t>(1, budget / KT));
  g.RT = (uint32_t)RT;
  g.KT = (uint32_t)KT;
  g.R_ext = (uint32_t)R_ext;
  g.K_ext = (uint32_t)K_ext;
  g.rtiles = (uint32_t)ge_ceil(R_ext, RT);
  g.ktiles = (uint32_t)ge_ceil(K_ext, KT);
  g.B2 = (uint32_t)B2;
  g.RB = (uint32_t)c0;
  g.C = (uint32_t)c;
  g.C0 = (uint32_t)c0;
  g.rw_last = (uint32_t)(R_ext - (int64_t)(g.rtiles - 1) * RT);
  g.kw_last = (uint32_t)(K_ext - (int64_t)(g.ktiles - 1) * KT);
  g.f_rb = FastDiv(g.RB);
  g.f_ktiles = FastDiv(g.ktiles);
  g.f_rtiles = FastDiv(g.rtiles);
  g.f_b2 = FastDiv(g.B2);
  g.f_kw = FastDiv(g.KT);
  g.f_kw_last = FastDiv(g.kw_last);
  g.f_rw = FastDiv(g.RT);
  g.f_rw_last = FastDiv(g.rw_last);
  const uint64_t ntiles = (uint64_t)c1 * B2 * g.rtiles * g.ktiles;
  if (ntiles == 0) return DCOPY_OK;
  if (ntiles > 0xFFFFFFFFull)
    return set_error(DCOPY_ERR_UNSUPPORTED, "FRACTAL_Z: %llu tiles exceed 32-bit indexing",
                     (unsigned long long)ntiles);
  switch (eb) {
    case 1: return launch_transpose<uint8_t>(dst, src, g, (uint32_t)ntiles, to_fz, s);
    case 2: return launch_transpose<uint16_t>(dst, src, g, (uint32_t)ntiles, to_fz, s);
    case 4: return launch_transpose<uint32_t>(dst, src, g, (uint32_t)ntiles, to_fz, s);
    case 8: return launch_transpose<uint2>(dst, src, g, (uint32_t)ntiles, to_fz, s);
    default: return launch_transpose<uint4>(dst, src, g, (uint32_t)ntiles, to_fz, s);
  }
}

// NHWC (both directions) through the tiled-format kernels: per (h, w) an
// [N x C] matrix with row pitch H*W*C, blocks of 16 rows x C0 columns.
int run_nhwc(void *dst, const void *src, int64_t n, int64_t c, int64_t h, int64_t w, int eb,
             int64_t c0, bool to_fz, dcopy_stream_t stream) {
  FracPlan p{};
  p.elem_bytes = eb;
  p.times = h * w;
  p.H = n;
  p.W = c;
  p.nd_row = h * w * c;
  p.nd_batch = c;
  p.BH = kNi;
  p.w0 = c0;
  p.H1 = ge_ceil(n, kNi);
  p.W1 = ge_ceil(c, c0);
  p.s_band = kNi * c0;
  p.fr_batch = p.H1 * kNi * c0;
  p.s_panel = h * w * p.fr_batch;
  p.batch_fast = DCOPY_FZ_NHWC_BATCH_FAST;
  return frac_launch(p, dst, src, to_fz, stream, "NHWC<->FRACTAL_Z");
}

bool width_ok(int eb) { return eb == 1 || eb == 2 || eb == 4 || eb == 8 || eb == 16; }

}  // namespace

int fz_shape(int32_t fmt, const int64_t *s, int rank, int64_t c0, int64_t groups, int64_t *out) {
  int64_t n, c, h, w;
  if (fmt == kNd) {  // TransShapeNdToFz, fractal_z_tbe.cc:32-62: every failure is FAILED
    if (!fz_dims(kNd, s, rank, &n, &c, &h, &w) || !shape_valid(s, rank))
      return set_error(DCOPY_ERR_FAILED, "ND -> FRACTAL_Z takes a valid 2-D [C, N] shape");
    if (c0 <= 0) return set_error(DCOPY_ERR_FAILED, "ND -> FRACTAL_Z: c0 %lld", (long long)c0);
    out[0] = ge_ceil(c, c0);
    out[1] = ge_ceil(n, kNi);
    out[2] = kNi;
    out[3] = c0;
    if (!shape_valid(out, 4)) return set_error(DCOPY_ERR_FAILED, "FRACTAL_Z shape is invalid");
    return DCOPY_OK;
  }
  if (fmt != kNchw && fmt != kNhwc && fmt != kHwcn)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "no FRACTAL_Z transfer from format %d", fmt);
  if (!fz_dims(fmt, s, rank, &n, &c, &h, &w) || !shape_valid(s, rank))  // CheckShapeValid(.., 4)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z source must be a valid 4-D shape");
  if (c0 < 0) return set_error(DCOPY_ERR_DATATYPE_INVALID, "c0 %lld < 0", (long long)c0);
  if (groups > 1 && fmt != kNhwc) {  // TransShapeToFzWithGroups, fractal_z.cc:64-99
    const int64_t cout = n / groups;
    if (cout == 0)
      return set_error(DCOPY_ERR_FAILED, "FRACTAL_Z groups: N %lld / groups %lld is 0",
                       (long long)n, (long long)groups);
    // The reference divides by zero here (Lcm(cin, k) / cin, Ceil(.., k) / k).
    if (c == 0 || c0 == 0)
      return set_error(DCOPY_ERR_FAILED, "FRACTAL_Z groups need C > 0 and c0 > 0");
    const GroupsLayout l = groups_layout(c, cout, c0, groups);
    out[0] = l.g_dim * l.c1_dim * h * w;
    out[1] = l.cout_opt / kNi;
  } else {  // TransShapeToFz, fractal_z.cc:41-62
    out[0] = h * w * ge_ceil(c, c0);
    out[1] = ge_ceil(n, kNi);
  }
  out[2] = kNi;
  out[3] = c0;
  if (!shape_valid(out, 4))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z shape is invalid");
  return DCOPY_OK;
}

int fz_out_elems(int32_t fmt, const int64_t *s, int rank, int64_t c0, int64_t groups,
                 int64_t *elems) {
  int64_t n, c, h, w;
  if (!fz_dims(fmt, s, rank, &n, &c, &h, &w))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z: shape of rank %d", rank);
  if (fmt == kHwcn && groups > 1) {
    const int64_t cout = n / groups;
    if (c == 0 || cout == 0 || c0 <= 0)  // GRAPH_FAILED, fractal_z.cc:283-290
      return set_error(DCOPY_ERR_FAILED, "FRACTAL_Z groups: cin %lld, cout %lld, c0 %lld",
                       (long long)c, (long long)cout, (long long)c0);
    const GroupsLayout l = groups_layout(c, cout, c0, groups);
    *elems = l.g_dim * l.c1_dim * h * w * l.cout_opt * c0;
    return DCOPY_OK;
  }
  *elems = ge_ceil(c, c0) * h * w * ge_ceil(n, kNi) * kNi * c0;
  return DCOPY_OK;
}

int to_fz(void *dst, const void *src, int32_t fmt, const int64_t *s, int rank, int eb,
          int64_t c0, int64_t groups, dcopy_stream_t stream) {
  if (!width_ok(eb))
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d not in {1,2,4,8,16}", eb);
  int64_t n, c, h, w;
  if (!fz_dims(fmt, s, rank, &n, &c, &h, &w) || !shape_valid(s, rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z: source shape of rank %d", rank);
  if (groups > 1 && fmt != kHwcn)
    return set_error(DCOPY_ERR_PARAM_INVALID, "FRACTAL_Z groups exist for HWCN sources only");
  if (c0 < 0) return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 %lld < 0", (long long)c0);
  int64_t elems = 0;
  int rc = fz_out_elems(fmt, s, rank, c0, groups, &elems);
  if (rc) return rc;
  if (elems == 0) return DCOPY_OK;
  const uint64_t out_bytes = (uint64_t)elems * eb, in_bytes = (uint64_t)(n * c * h * w) * eb;
  rc = check_device_span(src, in_bytes, "src");
  if (!rc) rc = check_device_span(dst, out_bytes, "dst");
  if (!rc) rc = check_disjoint(src, in_bytes, dst, out_bytes, "to_fractal_z");
  if (rc) return rc;
  if (((uintptr_t)src | (uintptr_t)dst) % eb)
    return set_error(DCOPY_ERR_PARAM_INVALID, "buffers must be aligned to the element size");
  cudaStream_t s_ = reinterpret_cast<cudaStream_t>(stream);
  if (fmt == kHwcn && groups > 1) {
    const int64_t cout = n / groups;
    const GroupsLayout l = groups_layout(c, cout, c0, groups);
    FzGGeom g{};
    g.total = (uint64_t)elems;
    g.k = (uint64_t)c0;
    g.cout_opt = (uint64_t)l.cout_opt;
    g.hw = (uint64_t)(h * w);
    g.c1_dim = (uint64_t)l.c1_dim;
    g.e_mult = (uint64_t)l.e_mult;
    g.groups = (uint64_t)groups;
    g.cin = (uint64_t)c;
    g.cout = (uint64_t)cout;
    g.n = (uint64_t)n;
    switch (eb) {
      case 1: return launch_groups<uint8_t>(dst, src, g, s_);
      case 2: return launch_groups<uint16_t>(dst, src, g, s_);
      case 4: return launch_groups<uint32_t>(dst, src, g, s_);
      case 8: return launch_groups<uint2>(dst, src, g, s_);
      default: return launch_groups<uint4>(dst, src, g, s_);
    }
  }
  // An NCHW weight with H = W = 1 is laid out exactly as the NHWC one ([N][C]),
  // so it takes the NHWC tiles (measured on B200, [2048,8192,1,1] fp16: 1928 GB/s
  // through the transposing tiles).
  if (fmt == kNhwc || (fmt == kNchw && h * w == 1))
    return run_nhwc(dst, src, n, c, h, w, eb, c0, true, stream);
  return run_transpose(fmt, dst, src, n, c, h, w, eb, c0, true, s_);
}

int from_fz_check(const int64_t *src_shape, int src_rank, int32_t fmt, const int64_t *dst_shape,
                  int dst_rank, int64_t c0) {
  // CheckArgsForFracZTo{Nchw,Hwcn,Nhwc} (fracz_nchw.cc:28-79 and its twins).
  int64_t n, c, h, w;
  if (fmt != kNchw && fmt != kHwcn && fmt != kNhwc)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "no transfer from FRACTAL_Z to format %d", fmt);
  if (src_rank != 4 || !shape_valid(src_shape, src_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z source must be a valid 4-D shape");
  if (!fz_dims(fmt, dst_shape, dst_rank, &n, &c, &h, &w) || !shape_valid(dst_shape, dst_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "destination must be a valid 4-D shape");
  if (c0 < 0) return set_error(DCOPY_ERR_DATATYPE_INVALID, "c0 %lld < 0", (long long)c0);
  if (src_shape[0] != h * w * ge_ceil(c, c0) || src_shape[3] != c0 || src_shape[2] != kNi ||
      src_shape[1] != ge_ceil(n, kNi))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z shape does not match the weight");
  return DCOPY_OK;
}

int from_fz(void *dst, const void *src, int32_t fmt, const int64_t *d, int rank, int eb,
            int64_t c0, dcopy_stream_t stream) {
  if (!width_ok(eb))
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "elem_bytes %d not in {1,2,4,8,16}", eb);
  int64_t n, c, h, w;
  if ((fmt != kNchw && fmt != kHwcn && fmt != kNhwc) || !fz_dims(fmt, d, rank, &n, &c, &h, &w) ||
      !shape_valid(d, rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "FRACTAL_Z: destination shape of rank %d", rank);
  const int64_t out_elems = n * c * h * w;
  if (out_elems == 0) return DCOPY_OK;
  // The reference divides by c0 (c_idx / c0 in GetDstDataAfterTransForFracZToNchw).
  if (c0 <= 0) return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 %lld must be positive", (long long)c0);
  const uint64_t in_bytes = (uint64_t)(ge_ceil(c, c0) * h * w * ge_ceil(n, kNi) * kNi * c0) * eb;
  const uint64_t out_bytes = (uint64_t)out_elems * eb;
  int rc = check_device_span(src, in_bytes, "src");
  if (!rc) rc = check_device_span(dst, out_bytes, "dst");
  if (!rc) rc = check_disjoint(src, in_bytes, dst, out_bytes, "from_fractal_z");
  if (rc) return rc;
  if (((uintptr_t)src | (uintptr_t)dst) % eb)
    return set_error(DCOPY_ERR_PARAM_INVALID, "buffers must be aligned to the element size");
  if (fmt == kNhwc || (fmt == kNchw && h * w == 1))  // same layout, see to_fz
    return run_nhwc(dst, src, n, c, h, w, eb, c0, false, stream);
  return run_transpose(fmt, dst, src, n, c, h, w, eb, c0, false,
                       reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace dcopy

using namespace dcopy;

extern "C" int dcopy_fz_shape(int32_t src_format, const int64_t *src_shape, int rank, int64_t c0,
                              int64_t groups, int64_t *fz_shape_out) {
  DCOPY_API_BEGIN
  if (!fz_shape_out || (rank && !src_shape) || rank < 0)
    return set_error(DCOPY_ERR_PARAM_INVALID, "fz_shape: invalid arguments");
  return fz_shape(src_format & 0xff, src_shape, rank, c0, groups, fz_shape_out);
  DCOPY_API_END
}

extern "C" int dcopy_to_fractal_z(void *dst, const void *src, int32_t src_format,
                                  const int64_t *src_shape, int rank, int elem_bytes, int64_t c0,
                                  int64_t groups, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return to_fz(dst, src, src_format & 0xff, src_shape, rank, elem_bytes, c0, groups, stream);
  DCOPY_API_END
}

extern "C" int dcopy_from_fractal_z(void *dst, const void *src, int32_t dst_format,
                                    const int64_t *dst_shape, int rank, int elem_bytes,
                                    int64_t c0, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  return from_fz(dst, src, dst_format & 0xff, dst_shape, rank, elem_bytes, c0, stream);
  DCOPY_API_END
}
