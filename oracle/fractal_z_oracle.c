/*
 * dcopy oracle, FRACTAL_Z family -- TEST INFRASTRUCTURE ONLY (see dcopy_oracle.h).
 *
 * Plain-C restatement of GE's FRACTAL_Z transfers (convolution weights):
 *   base/formats/format_transfers/format_transfer_fractal_z.cc      NCHW/HWCN/NHWC -> FZ
 *   base/formats/format_transfers/format_transfer_fractal_z_tbe.cc  ND [C, N] -> FZ
 *   base/formats/format_transfers/format_transfer_fracz_nchw.cc     FZ -> NCHW
 *   base/formats/format_transfers/format_transfer_fracz_hwcn.cc     FZ -> HWCN
 *   base/formats/format_transfers/format_transfer_fracz_nhwc.cc     FZ -> NHWC
 * FRACTAL_Z is [C1*H*W, N1, 16, C0]: element (c1, h, w, n, c0) holds weight
 * (n, c = c1*C0 + c0, h, w), zero where n >= N or c >= C.  Pinned by
 * tests/test_oracle_fractal_z.py against GE's unit-test vectors.
 */
#include <string.h>

#include "dcopy_oracle.h"

#define FZ_NI 16 /* kNiSize, formats_definitions.h:19 */

enum { F_NCHW = 0, F_NHWC = 1, F_ND = 2, F_HWCN = 16 };

static int64_t fz_ceil(int64_t n1, int64_t n2) { /* Ceil, formats_trans_utils.h:69-75 */
  if (n1 == 0) return 0;
  return (n2 != 0) ? (((n1 - 1) / n2) + 1) : 0;
}

static int64_t fz_gcd(int64_t x, int64_t y) { /* Measure, formats_trans_utils.h:76-88 */
  int64_t z = y;
  if (y == 0) return -1;
  while (x % y != 0) {
    z = x % y;
    x = y;
    y = z;
  }
  return z;
}

static int64_t fz_lcm(int64_t a, int64_t b) { /* Lcm, formats_trans_utils.h:90-96 */
  if (b == 0) return -1;
  return (a * b) / fz_gcd(a, b);
}

static int fz_shape_valid(const int64_t *s, int rank) { /* IsShapeValid */
  if (rank <= 0) return 0;
  int64_t num = 1;
  for (int i = 0; i < rank; ++i) {
    if (s[i] < 0) return 0;
    if (s[i] != 0 && (1099511627776LL / s[i]) < num) return 0;
    num *= s[i];
  }
  return 1;
}

/* (N, C, H, W) of a weight in `fmt`; 0 when the rank is not the format's. */
static int fz_dims(int fmt, const int64_t *s, int rank, int64_t *n, int64_t *c, int64_t *h,
                   int64_t *w) {
  switch (fmt) {
    case F_NCHW:
      if (rank != 4) return 0;
      *n = s[0], *c = s[1], *h = s[2], *w = s[3];
      return 1;
    case F_NHWC:
      if (rank != 4) return 0;
      *n = s[0], *h = s[1], *w = s[2], *c = s[3];
      return 1;
    case F_HWCN:
      if (rank != 4) return 0;
      *h = s[0], *w = s[1], *c = s[2], *n = s[3];
      return 1;
    case F_ND: /* fractal_z_tbe.cc:24-26: [C, N], H = W = 1 */
      if (rank != 2) return 0;
      *c = s[0], *n = s[1], *h = 1, *w = 1;
      return 1;
    default:
      return 0;
  }
}

/* Groups layout parameters, fractal_z.cc:77-87 and :289-298. */
static void fz_groups_params(int64_t cin, int64_t cout, int64_t k, int64_t groups,
                             int64_t *e_mult, int64_t *c1_dim, int64_t *g_dim,
                             int64_t *cout_opt) {
  int64_t a = fz_lcm(fz_lcm(cin, k) / cin, fz_lcm(cout, 16) / cout);
  *e_mult = a < groups ? a : groups;
  const int64_t cin_opt = fz_ceil(*e_mult * cin, k) * k;
  *c1_dim = cin_opt / k;
  *g_dim = fz_ceil(groups, *e_mult);
  *cout_opt = fz_ceil(cout * *e_mult, 16) * 16;
}

int oracle_fz_shape(int src_format, const int64_t *s, int rank, int64_t c0, int64_t groups,
                    int64_t *dst, int *dst_rank) {
  int64_t n, c, h, w;
  if (src_format == F_ND) { /* TransShapeNdToFz, fractal_z_tbe.cc:32-62: every failure is FAILED */
    if (!fz_dims(F_ND, s, rank, &n, &c, &h, &w) || !fz_shape_valid(s, rank)) return ORACLE_EFAILED;
    if (c0 <= 0) return ORACLE_EFAILED;
    dst[0] = h * w * fz_ceil(c, c0);
    dst[1] = fz_ceil(n, FZ_NI);
    dst[2] = FZ_NI;
    dst[3] = c0;
    *dst_rank = 4;
    return fz_shape_valid(dst, 4) ? ORACLE_OK : ORACLE_EFAILED;
  }
  if (src_format != F_NCHW && src_format != F_NHWC && src_format != F_HWCN)
    return ORACLE_EFORMAT;
  /* TransShape{Nchw,Hwcn,Nhwc}ToFz[WithGroups], fractal_z.cc:101-173 */
  if (!fz_dims(src_format, s, rank, &n, &c, &h, &w) || !fz_shape_valid(s, rank))
    return ORACLE_ESHAPE;
  if (c0 < 0) return ORACLE_EDTYPE;
  if (groups > 1 && src_format != F_NHWC) { /* TransShapeToFzWithGroups, :64-99 */
    const int64_t cout = n / groups;
    if (cout == 0) return ORACLE_EFAILED;
    /* Lcm(cin, k) / cin divides by zero in the reference when C == 0 or C0 == 0. */
    if (c == 0 || c0 == 0) return ORACLE_EFAILED;
    int64_t e_mult, c1_dim, g_dim, cout_opt;
    fz_groups_params(c, cout, c0, groups, &e_mult, &c1_dim, &g_dim, &cout_opt);
    dst[0] = g_dim * c1_dim * h * w;
    dst[1] = cout_opt / 16;
    dst[2] = 16;
    dst[3] = c0;
  } else { /* TransShapeToFz, :41-62 */
    dst[0] = h * w * fz_ceil(c, c0);
    dst[1] = fz_ceil(n, FZ_NI);
    dst[2] = FZ_NI;
    dst[3] = c0;
  }
  *dst_rank = 4;
  return fz_shape_valid(dst, 4) ? ORACLE_OK : ORACLE_ESHAPE;
}

int oracle_to_fz(void *dst_v, const void *src_v, int src_format, const int64_t *s, int rank,
                 int size, int64_t c0, int64_t groups, int64_t *out_elems) {
  int64_t n, c, h, w;
  if (!fz_dims(src_format, s, rank, &n, &c, &h, &w) || size <= 0) return ORACLE_EPARAM;
  uint8_t *dst = (uint8_t *)dst_v;
  const uint8_t *src = (const uint8_t *)src_v;
  *out_elems = 0;
  if (src_format == F_NCHW) { /* TransFormatFromNchwToFz, fractal_z.cc:175-274 */
    const int64_t c1 = fz_ceil(c, c0), hw = h * w, chw = c * hw, nchw = n * chw;
    const int64_t hwc0 = hw * c0, hf_cnt = fz_ceil(n, FZ_NI), vf_cnt = c1 * hw;
    const int64_t fractal = c0 * FZ_NI, total = hf_cnt * vf_cnt * fractal;
    *out_elems = total;
    if (total == 0 || !dst) return ORACLE_OK;
    for (int64_t vfi = 0; vfi < vf_cnt; vfi++) {
      for (int64_t hfi = 0; hfi < hf_cnt; hfi++) {
        const int64_t gfi = vfi * hf_cnt + hfi;
        const int64_t src_f = hfi * chw * FZ_NI + (vfi % hw) + (vfi / hw * hwc0);
        for (int64_t row = 0; row < c0; row++) {
          const int64_t ci = (vfi / hw * c0) + row;
          for (int64_t col = 0; col < FZ_NI; col++) {
            const int64_t ni = hfi * FZ_NI + col;
            const int64_t so = src_f + row * hw + chw * col;
            const int64_t idx = gfi * fractal + col * c0 + row;
            if (ni >= n || so >= nchw || ci >= c)
              memset(dst + idx * size, 0, (size_t)size);
            else
              memcpy(dst + idx * size, src + so * size, (size_t)size);
          }
        }
      }
    }
    return ORACLE_OK;
  }
  if (src_format == F_HWCN && groups > 1) { /* TransFormatHwcnToFzWithGroups, :276-359 */
    const int64_t cin = c, cout = n / groups;
    if (cin == 0 || cout == 0 || c0 == 0) return ORACLE_EFAILED;
    int64_t e_mult, c1_dim, g_dim, cout_opt;
    fz_groups_params(cin, cout, c0, groups, &e_mult, &c1_dim, &g_dim, &cout_opt);
    const int64_t total = g_dim * c1_dim * h * w * cout_opt * c0;
    *out_elems = total;
    if (total == 0 || !dst) return ORACLE_OK;
    memset(dst, 0, (size_t)(total * size));
    for (int64_t g = 0; g < groups; g++)
      for (int64_t ci = 0; ci < cin; ci++)
        for (int64_t hi = 0; hi < h; hi++)
          for (int64_t wi = 0; wi < w; wi++)
            for (int64_t ni = 0; ni < cout; ni++) {
              const int64_t e = g % e_mult;
              const int64_t dci = e * cin + ci, dco = e * cout + ni, sco = g * cout + ni;
              const int64_t di = (g / e_mult) * c1_dim * h * w * cout_opt * c0 +
                                 (dci / c0) * h * w * cout_opt * c0 + hi * w * cout_opt * c0 +
                                 wi * cout_opt * c0 + dco * c0 + dci % c0;
              const int64_t si = hi * w * cin * n + wi * cin * n + ci * n + sco;
              memcpy(dst + di * size, src + si * size, (size_t)size);
            }
    return ORACLE_OK;
  }
  /* HWCN (:361-448), NHWC (:450-537), ND (fractal_z_tbe.cc:64-114): dst-ordered loops */
  const int64_t n1n0 = fz_ceil(n, FZ_NI) * FZ_NI, c1 = fz_ceil(c, c0);
  const int64_t total = c1 * h * w * n1n0 * c0;
  *out_elems = total;
  if (!dst) return ORACLE_OK;
  for (int64_t c1i = 0; c1i < c1; c1i++)
    for (int64_t hi = 0; hi < h; hi++)
      for (int64_t wi = 0; wi < w; wi++)
        for (int64_t ni = 0; ni < n1n0; ni++)
          for (int64_t c0i = 0; c0i < c0; c0i++) {
            const int64_t di = (((c1i * h + hi) * w + wi) * n1n0 + ni) * c0 + c0i;
            const int64_t ci = c1i * c0 + c0i;
            if (ci >= c || ni >= n) {
              memset(dst + di * size, 0, (size_t)size);
              continue;
            }
            int64_t si;
            if (src_format == F_NHWC)
              si = ni * h * w * c + hi * w * c + wi * c + ci;
            else /* HWCN, and ND [C, N] as HWCN with H = W = 1 */
              si = hi * w * c * n + wi * c * n + ci * n + ni;
            memcpy(dst + di * size, src + si * size, (size_t)size);
          }
  return ORACLE_OK;
}

int oracle_from_fz_check(const int64_t *src_shape, int src_rank, int dst_format,
                         const int64_t *dst_shape, int dst_rank, int64_t c0) {
  /* CheckArgsForFracZTo{Nchw,Hwcn,Nhwc}, fracz_nchw.cc:28-79 (and the twins) */
  int64_t n, c, h, w;
  if (dst_format != F_NCHW && dst_format != F_HWCN && dst_format != F_NHWC) return ORACLE_EFORMAT;
  if (src_rank != 4 || !fz_shape_valid(src_shape, src_rank)) return ORACLE_ESHAPE;
  if (!fz_dims(dst_format, dst_shape, dst_rank, &n, &c, &h, &w) ||
      !fz_shape_valid(dst_shape, dst_rank))
    return ORACLE_ESHAPE;
  if (c0 < 0) return ORACLE_EDTYPE;
  const int64_t c1 = fz_ceil(c, c0), n0 = fz_ceil(n, FZ_NI);
  if (src_shape[0] != h * w * c1 || src_shape[3] != c0 || src_shape[2] != FZ_NI ||
      src_shape[1] != n0)
    return ORACLE_ESHAPE;
  return ORACLE_OK;
}

int oracle_from_fz(void *dst_v, const void *src_v, int dst_format, const int64_t *d, int rank,
                   int size, int64_t c0) {
  /* GetDstDataAfterTransForFracZTo{Nchw,Hwcn,Nhwc}: every ND element read from
   * (c1, h, w, n, c0) of the FZ source, padding dropped. */
  int64_t n, c, h, w;
  if (!fz_dims(dst_format, d, rank, &n, &c, &h, &w) || size <= 0 || c0 <= 0) return ORACLE_EPARAM;
  uint8_t *dst = (uint8_t *)dst_v;
  const uint8_t *src = (const uint8_t *)src_v;
  const int64_t nc = fz_ceil(n, FZ_NI) * FZ_NI;
  for (int64_t ni = 0; ni < n; ni++)
    for (int64_t ci = 0; ci < c; ci++)
      for (int64_t hi = 0; hi < h; hi++)
        for (int64_t wi = 0; wi < w; wi++) {
          const int64_t si = (((ci / c0 * h + hi) * w + wi) * nc + ni) * c0 + ci % c0;
          int64_t di;
          if (dst_format == F_NCHW)
            di = ((ni * c + ci) * h + hi) * w + wi;
          else if (dst_format == F_HWCN)
            di = ((hi * w + wi) * c + ci) * n + ni;
          else
            di = ((ni * h + hi) * w + wi) * c + ci;
          memcpy(dst + di * size, src + si * size, (size_t)size);
        }
  return ORACLE_OK;
}
