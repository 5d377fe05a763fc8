// GE TransData level on device buffers: the format-transfer registry
// (base/formats/formats.cc, register_format_transfer.{h,cc}), the
// FormatTransferFractalNz / FractalNzND / FractalZz / FractalZzND / FractalZ /
// FractalZTbe / FracZNchw / FracZHwcn / FracZNhwc / Transpose classes' argument
// checks, and Transpose (format_transfer_transpose.cc) on the GPU.  Every check happens on the host, in the reference's order and with its
// status class, before any launch; the data movement goes to the NZ kernels and
// to the N-D box copy.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "internal.cuh"

namespace dcopy {
namespace {

constexpr int kMaxRank = 30;

// Set while dcopy_trans_format_check runs: the transfer functions stop after
// their checks, with the result length stored, before touching memory.
thread_local bool t_check_only = false;

// GetSizeByDataType for GE's DataType enum (api/python/ge/ge/graph/types.py:15-58).
// Types without a fixed byte size (string, resource, variant, sub-byte
// floats/ints, undefined) report -1.
int32_t type_size(int32_t dt) {
  switch (dt) {
    case 0: return 4;    // DT_FLOAT
    case 1: return 2;    // DT_FLOAT16
    case 2: return 1;    // DT_INT8
    case 3: return 4;    // DT_INT32
    case 4: return 1;    // DT_UINT8
    case 6: return 2;    // DT_INT16
    case 7: return 2;    // DT_UINT16
    case 8: return 4;    // DT_UINT32
    case 9: return 8;    // DT_INT64
    case 10: return 8;   // DT_UINT64
    case 11: return 8;   // DT_DOUBLE
    case 12: return 1;   // DT_BOOL
    case 14: return 1;   // DT_DUAL_SUB_INT8
    case 15: return 1;   // DT_DUAL_SUB_UINT8
    case 16: return 8;   // DT_COMPLEX64
    case 17: return 16;  // DT_COMPLEX128
    case 18: return 1;   // DT_QINT8
    case 19: return 2;   // DT_QINT16
    case 20: return 4;   // DT_QINT32
    case 21: return 1;   // DT_QUINT8
    case 22: return 2;   // DT_QUINT16
    case 27: return 2;   // DT_BF16
    case 33: return 4;   // DT_COMPLEX32
    case 34: return 1;   // DT_HIFLOAT8
    case 35: return 1;   // DT_FLOAT8_E5M2
    case 36: return 1;   // DT_FLOAT8_E4M3FN
    case 37: return 1;   // DT_FLOAT8_E8M0
    default: return -1;
  }
}

// format_transfer_transpose.cc:26-43.
struct PermEntry {
  int32_t src, dst;
  int64_t perm[4];
};
constexpr PermEntry kPerms[] = {
    {DCOPY_FORMAT_NCHW, DCOPY_FORMAT_NHWC, {0, 2, 3, 1}},
    {DCOPY_FORMAT_NCHW, DCOPY_FORMAT_HWCN, {2, 3, 1, 0}},
    {DCOPY_FORMAT_NCHW, DCOPY_FORMAT_CHWN, {1, 2, 3, 0}},
    {DCOPY_FORMAT_NHWC, DCOPY_FORMAT_NCHW, {0, 3, 1, 2}},
    {DCOPY_FORMAT_NHWC, DCOPY_FORMAT_CHWN, {3, 1, 2, 0}},
    {DCOPY_FORMAT_NHWC, DCOPY_FORMAT_HWCN, {1, 2, 3, 0}},
    {DCOPY_FORMAT_HWCN, DCOPY_FORMAT_NCHW, {3, 2, 0, 1}},
    {DCOPY_FORMAT_HWCN, DCOPY_FORMAT_NHWC, {3, 0, 1, 2}},
    {DCOPY_FORMAT_HWCN, DCOPY_FORMAT_CHWN, {2, 0, 1, 3}},
    {DCOPY_FORMAT_CHWN, DCOPY_FORMAT_NCHW, {3, 0, 1, 2}},
    {DCOPY_FORMAT_CHWN, DCOPY_FORMAT_NHWC, {3, 1, 2, 0}},
    {DCOPY_FORMAT_CHWN, DCOPY_FORMAT_HWCN, {1, 2, 0, 3}},
};

const PermEntry *find_perm(int32_t src, int32_t dst) {
  for (const PermEntry &e : kPerms)
    if (e.src == src && e.dst == dst) return &e;
  return nullptr;
}

// The registry: which transfer class a (src, dst) primary-format pair builds
// (REGISTER_FORMAT_TRANSFER lines of both transfer files); 0 = none.
int registered_class(int32_t src, int32_t dst) {
  const bool nd_like = src == DCOPY_FORMAT_ND || src == DCOPY_FORMAT_NCHW ||
                       src == DCOPY_FORMAT_NHWC;
  const bool nd_like_dst = dst == DCOPY_FORMAT_ND || dst == DCOPY_FORMAT_NCHW ||
                           dst == DCOPY_FORMAT_NHWC;
  if (nd_like && dst == DCOPY_FORMAT_FRACTAL_NZ) return DCOPY_TRANSFER_FRACTAL_NZ;
  if (src == DCOPY_FORMAT_FRACTAL_NZ && nd_like_dst) return DCOPY_TRANSFER_FRACTAL_NZ_ND;
  if (nd_like && dst == DCOPY_FORMAT_FRACTAL_ZZ) return DCOPY_TRANSFER_FRACTAL_ZZ;
  if (src == DCOPY_FORMAT_FRACTAL_ZZ && nd_like_dst) return DCOPY_TRANSFER_FRACTAL_ZZ_ND;
  if (dst == DCOPY_FORMAT_FRACTAL_Z) {  // fractal_z.cc:606-608, fractal_z_tbe.cc:147
    if (src == DCOPY_FORMAT_NCHW || src == DCOPY_FORMAT_HWCN || src == DCOPY_FORMAT_NHWC)
      return DCOPY_TRANSFER_FRACTAL_Z;
    if (src == DCOPY_FORMAT_ND) return DCOPY_TRANSFER_FRACTAL_Z_TBE;
  }
  if (src == DCOPY_FORMAT_FRACTAL_Z) {  // fracz_{nchw,hwcn,nhwc}.cc REGISTER lines
    if (dst == DCOPY_FORMAT_NCHW) return DCOPY_TRANSFER_FRACZ_NCHW;
    if (dst == DCOPY_FORMAT_HWCN) return DCOPY_TRANSFER_FRACZ_HWCN;
    if (dst == DCOPY_FORMAT_NHWC) return DCOPY_TRANSFER_FRACZ_NHWC;
  }
  if (find_perm(src, dst)) return DCOPY_TRANSFER_TRANSPOSE;
  return 0;
}

bool same_shape(const int64_t *a, int an, const int64_t *b, int bn) {
  if (an != bn) return false;
  for (int i = 0; i < an; ++i)
    if (a[i] != b[i]) return false;
  return true;
}

int64_t item_count(const int64_t *s, int n) {  // GetItemNumByShape: empty -> 1
  int64_t v = 1;
  for (int i = 0; i < n; ++i) v *= s[i];
  return v;
}

// CheckShapeForTransShapeToFracNz (format_transfer_fractal_nz.cc:39-57); the
// FRACTAL_ZZ file's CheckShape (format_transfer_fractal_zz.cc:48-66) is the same rule.
bool check_shape_for_nz(int32_t format, const int64_t *shape, int rank) {
  switch (format) {
    case DCOPY_FORMAT_ND: return shape_valid(shape, rank);
    case DCOPY_FORMAT_NCHW:
    case DCOPY_FORMAT_NHWC: return rank == 4 && shape_valid(shape, rank);
    default: return false;
  }
}

// IsShapeArgValid (format_transfer_transpose.cc:45-77).
bool shape_arg_valid(const int64_t *shape, int rank, const int64_t *perm, int perm_rank) {
  if (rank <= 0 || !shape) return false;
  for (int i = 0; i < rank; ++i)
    if (shape[i] < 0) return false;
  if (perm_rank != rank) return false;
  int seen[kMaxRank] = {0};
  for (int i = 0; i < perm_rank; ++i) {
    if (perm[i] < 0 || perm[i] >= perm_rank || seen[perm[i]]) return false;
    seen[perm[i]] = 1;
  }
  return true;
}

int check_args(const DcopyTransArgs *a) {
  if (!a) return set_error(DCOPY_ERR_PARAM_INVALID, "TransArgs is NULL");
  if (a->src_rank < 0 || a->src_rank > kMaxRank || a->dst_rank < 0 || a->dst_rank > kMaxRank ||
      (a->src_rank && !a->src_shape) || (a->dst_rank && !a->dst_shape))
    return set_error(DCOPY_ERR_PARAM_INVALID, "TransArgs shapes: rank must be 0..%d", kMaxRank);
  return DCOPY_OK;
}

int store_length(uint64_t *len, uint64_t v) {
  if (len) *len = v;
  return DCOPY_OK;
}

// FormatTransferFractalNz::TransFormat (fractal_nz.cc:301-353).
int fractal_nz_format(const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                      dcopy_stream_t s) {
  const int32_t size = type_size(a->data_type);
  if (size <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", a->data_type);
  if (!check_shape_for_nz(a->src_format, a->src_shape, a->src_rank) ||
      !shape_valid(a->dst_shape, a->dst_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "trans format %d -> FRACTAL_NZ: invalid shapes",
                     a->src_format);
  int64_t expect[kMaxRank + 2], hw[3];
  int erank = 0;
  int rc = nz_shape(a->src_shape, a->src_rank, a->dst_c0, expect, &erank, hw);
  if (rc) return rc;
  if (a->dst_rank && !same_shape(a->dst_shape, a->dst_rank, expect, erank))  // :349-351
    return set_error(DCOPY_ERR_SHAPE_INVALID, "dst shape differs from the FRACTAL_NZ shape");
  const uint64_t bytes = (uint64_t)item_count(a->dst_shape, a->dst_rank) * size;
  if (bytes == 0) return store_length(len, 0);  // :134-137
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = nz_transfer(dst, a->data, a->src_shape, a->src_rank, size, a->dst_c0, true, s);
  return rc ? rc : store_length(len, bytes);
}

// FormatTransferFractalNzND::TransFormat (fractal_nz.cc:397-446).
int fractal_nz_nd_format(const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                         dcopy_stream_t s) {
  const int32_t size = type_size(a->data_type);
  if (size <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", a->data_type);
  if (!shape_valid(a->src_shape, a->src_rank) ||
      !check_shape_for_nz(a->dst_format, a->dst_shape, a->dst_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "trans format FRACTAL_NZ -> %d: invalid shapes",
                     a->dst_format);
  int64_t expect[kMaxRank + 2], hw[3];  // CheckShapeRelationForTransShapeToFracNz, :113-129
  int erank = 0;
  int rc = nz_shape(a->dst_shape, a->dst_rank, a->src_c0, expect, &erank, hw);
  if (rc) return rc;
  if (!same_shape(a->src_shape, a->src_rank, expect, erank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "src shape is not the FRACTAL_NZ shape of dst");
  const uint64_t bytes = (uint64_t)item_count(a->dst_shape, a->dst_rank) * size;
  if (bytes == 0) return store_length(len, 0);
  if (a->src_c0 <= 0)  // the reference divides by it (:249)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 %lld must be positive", (long long)a->src_c0);
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = nz_transfer(dst, a->data, a->dst_shape, a->dst_rank, size, a->src_c0, false, s);
  return rc ? rc : store_length(len, bytes);
}

// FormatTransferFractalZz::TransFormat (fractal_zz.cc:337-389).
int fractal_zz_format(const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                      dcopy_stream_t s) {
  const int32_t size = type_size(a->data_type);
  if (size <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", a->data_type);
  if (!check_shape_for_nz(a->src_format, a->src_shape, a->src_rank) ||
      !shape_valid(a->dst_shape, a->dst_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "trans format %d -> FRACTAL_ZZ: invalid shapes",
                     a->src_format);
  int64_t expect[kMaxRank + 2], hw[3];
  int erank = 0;
  int rc = zz_shape(a->src_shape, a->src_rank, a->dst_c0, expect, &erank, hw);
  if (rc) return rc;
  if (a->dst_rank && !same_shape(a->dst_shape, a->dst_rank, expect, erank))  // :385-387
    return set_error(DCOPY_ERR_SHAPE_INVALID, "dst shape differs from the FRACTAL_ZZ shape");
  const uint64_t bytes = (uint64_t)item_count(a->dst_shape, a->dst_rank) * size;
  if (bytes == 0) return store_length(len, 0);  // :143-146
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = frac_transfer(FracKind::kZz, dst, a->data, a->src_shape, a->src_rank, size, a->dst_c0,
                     true, s);
  return rc ? rc : store_length(len, bytes);
}

// FormatTransferFractalZzND::TransFormat (fractal_zz.cc:433-481).
int fractal_zz_nd_format(const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                         dcopy_stream_t s) {
  const int32_t size = type_size(a->data_type);
  if (size <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", a->data_type);
  if (!shape_valid(a->src_shape, a->src_rank) ||
      !check_shape_for_nz(a->dst_format, a->dst_shape, a->dst_rank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "trans format FRACTAL_ZZ -> %d: invalid shapes",
                     a->dst_format);
  int64_t expect[kMaxRank + 2], hw[3];  // CheckShapeRelation, :120-138
  int erank = 0;
  int rc = zz_shape(a->dst_shape, a->dst_rank, a->src_c0, expect, &erank, hw);
  if (rc) return rc;
  if (!same_shape(a->src_shape, a->src_rank, expect, erank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "src shape is not the FRACTAL_ZZ shape of dst");
  const uint64_t bytes = (uint64_t)item_count(a->dst_shape, a->dst_rank) * size;
  if (bytes == 0) return store_length(len, 0);
  if (a->src_c0 <= 0)  // the reference divides by it (:273)
    return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 %lld must be positive", (long long)a->src_c0);
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = frac_transfer(FracKind::kZz, dst, a->data, a->dst_shape, a->dst_rank, size, a->src_c0,
                     false, s);
  return rc ? rc : store_length(len, bytes);
}

// Transpose (transpose.cc:142-197) as a permuted copy (permute.cu): the
// destination is contiguous and the source strides are the permuted row-major
// heads.
int transpose_impl(void *dst, const void *src, const int64_t *shape, const int64_t *perm,
                   int rank, int32_t data_type, uint64_t cap, uint64_t *len, dcopy_stream_t s) {
  const int32_t size = type_size(data_type);
  if (!src) return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: the src is null");
  if (size < 0)
    return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: data type %d is not supported",
                     data_type);
  if (!shape_arg_valid(shape, rank, perm, rank))
    return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: invalid shape or perm");
  {  // the element count and its bytes must not wrap (GE would fail the allocation)
    unsigned __int128 items = 1;
    for (int i = 0; i < rank && items; ++i) {
      items *= (uint64_t)shape[i];
      if (items * (uint64_t)(size ? size : 1) >= ((unsigned __int128)1 << 62))
        return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: the tensor spans 2^62 bytes or more");
    }
  }
  int64_t heads[kMaxRank];
  for (int i = rank - 1; i >= 0; --i) heads[i] = (i == rank - 1) ? 1 : shape[i + 1] * heads[i + 1];
  uint64_t sizes[kMaxRank];
  int64_t ss[kMaxRank], ds[kMaxRank];
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) {
    sizes[i] = (uint64_t)shape[perm[i]];
    ss[i] = heads[perm[i]];
    n *= shape[perm[i]];
  }
  for (int i = rank - 1; i >= 0; --i) ds[i] = (i == rank - 1) ? 1 : (int64_t)sizes[i + 1] * ds[i + 1];
  const uint64_t bytes = (uint64_t)n * size;
  if (n == 0) return store_length(len, 0);
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  // Merge destination-adjacent dims that are also adjacent in the source, so
  // that NCHW -> NHWC style permutes become a few long runs.
  int m = 0;
  uint64_t ms[kMaxRank];
  int64_t mss[kMaxRank], mds[kMaxRank];
  for (int i = 0; i < rank; ++i) {
    if (sizes[i] == 1) continue;
    if (m > 0 && mss[m - 1] == ss[i] * (int64_t)sizes[i] && mds[m - 1] == ds[i] * (int64_t)sizes[i]) {
      ms[m - 1] *= sizes[i];
      mss[m - 1] = ss[i];
      mds[m - 1] = ds[i];
      continue;
    }
    ms[m] = sizes[i];
    mss[m] = ss[i];
    mds[m] = ds[i];
    ++m;
  }
  if (m == 0) {
    ms[0] = 1;
    mss[0] = 1;
    mds[0] = 1;
    m = 1;
  }
  if (m > 5)
    return set_error(DCOPY_ERR_UNSUPPORTED, "Transpose: %d non-trivial dims (at most 5)", m);
  int rc = check_device_span(src, bytes, "Transpose src");
  if (!rc) rc = check_device_span(dst, bytes, "Transpose dst");
  if (!rc) rc = check_disjoint(src, bytes, dst, bytes, "Transpose");
  if (!rc && ((uintptr_t)src | (uintptr_t)dst) % (uint32_t)size)
    rc = set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: buffers must be aligned to the element");
  if (!rc) rc = permute_copy(dst, src, m, ms, mss, mds, size, s);
  return rc ? rc : store_length(len, bytes);
}

// FormatTransferTranspose::TransShape (transpose.cc:253-266).
int transpose_shape(int32_t src_format, const int64_t *src_shape, int rank, int32_t dst_format,
                    int64_t *dst_shape, int32_t *dst_rank) {
  const PermEntry *e = find_perm(src_format, dst_format);
  if (!e)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "no transpose from format %d to %d", src_format,
                     dst_format);
  if (!shape_arg_valid(src_shape, rank, e->perm, 4))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "transpose: invalid src shape for the perm");
  for (int i = 0; i < 4; ++i) dst_shape[i] = src_shape[e->perm[i]];
  *dst_rank = 4;
  return DCOPY_OK;
}

// FormatTransferTranspose::TransFormat (transpose.cc:239-251).
int transpose_format(const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                     dcopy_stream_t s) {
  int64_t expect[4];
  int32_t erank = 0;
  int rc = transpose_shape(a->src_format, a->src_shape, a->src_rank, a->dst_format, expect, &erank);
  if (rc) return rc;
  if (a->dst_rank && !same_shape(a->dst_shape, a->dst_rank, expect, erank))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "transpose: dst shape differs from the permuted shape");
  const PermEntry *e = find_perm(a->src_format, a->dst_format);
  return transpose_impl(dst, a->data, a->src_shape, e->perm, a->src_rank, a->data_type, cap, len,
                        s);
}

// FormatTransferFractalZ::TransShape / FormatTransferFractalZTbe::TransShape
// (fractal_z.cc:571-604, fractal_z_tbe.cc:131-146).  `groups` is the sub format
// of the full destination format.
int fractal_z_shape(int cls, int32_t src_format, const int64_t *src_shape, int32_t src_rank,
                    int32_t data_type, int32_t dst_format, int64_t c0, int64_t groups,
                    int64_t *out) {
  if (type_size(data_type) <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", data_type);
  const bool tbe = cls == DCOPY_TRANSFER_FRACTAL_Z_TBE;
  const bool pair_ok =
      dst_format == DCOPY_FORMAT_FRACTAL_Z &&
      (tbe ? src_format == DCOPY_FORMAT_ND
           : (src_format == DCOPY_FORMAT_NCHW || src_format == DCOPY_FORMAT_HWCN ||
              src_format == DCOPY_FORMAT_NHWC));
  if (!pair_ok)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "no FRACTAL_Z transfer from %d to %d", src_format,
                     dst_format);
  return fz_shape(src_format, src_shape, src_rank, c0, groups, out);
}

// FormatTransferFractalZ::TransFormat (fractal_z.cc:540-569) and
// FormatTransferFractalZTbe::TransFormat (fractal_z_tbe.cc:117-129).
int fractal_z_format(int cls, const DcopyTransArgs *a, int64_t fmt_groups, void *dst,
                     uint64_t cap, uint64_t *len, dcopy_stream_t s) {
  int64_t expect[4];
  int rc = fractal_z_shape(cls, a->src_format, a->src_shape, a->src_rank, a->data_type,
                           a->dst_format, a->dst_c0, fmt_groups, expect);
  if (rc) return rc;
  if (a->dst_rank && !same_shape(a->dst_shape, a->dst_rank, expect, 4))
    return set_error(DCOPY_ERR_SHAPE_INVALID, "dst shape differs from the FRACTAL_Z shape");
  // The HWCN transfer takes its groups from TransArgs::dst_sub_format (:553-556);
  // NCHW and NHWC data never use groups.
  const int64_t groups = a->src_format == DCOPY_FORMAT_HWCN ? a->dst_sub_format : 0;
  if (a->dst_rank == 0 && a->src_format != DCOPY_FORMAT_NCHW && groups <= 1)
    return set_error(DCOPY_ERR_PARAM_INVALID,
                     "FRACTAL_Z from format %d sizes its result by dst_shape: pass it",
                     a->src_format);
  int64_t elems = 0;
  rc = fz_out_elems(a->src_format, a->src_shape, a->src_rank, a->dst_c0, groups, &elems);
  if (rc) return rc;
  const int32_t size = type_size(a->data_type);
  const uint64_t bytes = (uint64_t)elems * size;
  if (bytes == 0) return store_length(len, 0);
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = to_fz(dst, a->data, a->src_format, a->src_shape, a->src_rank, size, a->dst_c0, groups, s);
  return rc ? rc : store_length(len, bytes);
}

// FormatTransferFracZ{Nchw,Hwcn,Nhwc}::TransFormat (fracz_nchw.cc:154-195 and
// its twins): CheckArgsForFracZTo*, then the empty-result rule.
int fracz_to_format(int cls, const DcopyTransArgs *a, void *dst, uint64_t cap, uint64_t *len,
                    dcopy_stream_t s) {
  const int32_t want = cls == DCOPY_TRANSFER_FRACZ_NCHW   ? DCOPY_FORMAT_NCHW
                       : cls == DCOPY_TRANSFER_FRACZ_HWCN ? DCOPY_FORMAT_HWCN
                                                          : DCOPY_FORMAT_NHWC;
  if (a->src_format != DCOPY_FORMAT_FRACTAL_Z || a->dst_format != want)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "FRACTAL_Z -> %d: formats %d -> %d", want,
                     a->src_format, a->dst_format);
  const int32_t size = type_size(a->data_type);
  if (size <= 0)
    return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", a->data_type);
  int rc = from_fz_check(a->src_shape, a->src_rank, want, a->dst_shape, a->dst_rank, a->src_c0);
  if (rc) return rc;
  const uint64_t bytes = (uint64_t)item_count(a->dst_shape, a->dst_rank) * size;
  if (bytes == 0) {
    if (item_count(a->src_shape, a->src_rank) == 0) return store_length(len, 0);
    return set_error(DCOPY_ERR_SHAPE_INVALID, "empty destination from a non-empty FRACTAL_Z");
  }
  if (a->src_c0 == 0)  // the reference divides by it
    return set_error(DCOPY_ERR_SHAPE_INVALID, "c0 0 with data to move");
  if (t_check_only) return store_length(len, bytes);
  if (cap < bytes)
    return set_error(DCOPY_ERR_PARAM_INVALID, "dst holds %llu bytes, result needs %llu",
                     (unsigned long long)cap, (unsigned long long)bytes);
  rc = from_fz(dst, a->data, want, a->dst_shape, a->dst_rank, size, a->src_c0, s);
  return rc ? rc : store_length(len, bytes);
}

int class_format(int cls, const DcopyTransArgs *a, int64_t fmt_groups, void *dst, uint64_t cap,
                 uint64_t *len, dcopy_stream_t s) {
  switch (cls) {
    case DCOPY_TRANSFER_FRACTAL_Z:
    case DCOPY_TRANSFER_FRACTAL_Z_TBE: return fractal_z_format(cls, a, fmt_groups, dst, cap, len, s);
    case DCOPY_TRANSFER_FRACZ_NCHW:
    case DCOPY_TRANSFER_FRACZ_HWCN:
    case DCOPY_TRANSFER_FRACZ_NHWC: return fracz_to_format(cls, a, dst, cap, len, s);
    case DCOPY_TRANSFER_FRACTAL_NZ: return fractal_nz_format(a, dst, cap, len, s);
    case DCOPY_TRANSFER_FRACTAL_NZ_ND: return fractal_nz_nd_format(a, dst, cap, len, s);
    case DCOPY_TRANSFER_TRANSPOSE: return transpose_format(a, dst, cap, len, s);
    case DCOPY_TRANSFER_FRACTAL_ZZ: return fractal_zz_format(a, dst, cap, len, s);
    case DCOPY_TRANSFER_FRACTAL_ZZ_ND: return fractal_zz_nd_format(a, dst, cap, len, s);
    default: return set_error(DCOPY_ERR_PARAM_INVALID, "unknown transfer class %d", cls);
  }
}

int class_shape(int cls, int32_t src_format, const int64_t *src_shape, int32_t src_rank,
                int32_t data_type, int32_t dst_format, int64_t c0, int64_t fmt_groups,
                int64_t *dst_shape, int32_t *dst_rank) {
  if (!dst_shape || !dst_rank || src_rank < 0 || src_rank > kMaxRank || (src_rank && !src_shape))
    return set_error(DCOPY_ERR_PARAM_INVALID, "TransShape: invalid arguments");
  switch (cls) {
    case DCOPY_TRANSFER_FRACTAL_Z:
    case DCOPY_TRANSFER_FRACTAL_Z_TBE: {
      const int rc = fractal_z_shape(cls, src_format, src_shape, src_rank, data_type, dst_format,
                                     c0, fmt_groups, dst_shape);
      *dst_rank = rc ? 0 : 4;
      return rc;
    }
    case DCOPY_TRANSFER_FRACZ_NCHW:  // fracz_nchw.cc:197-208 and its twins
    case DCOPY_TRANSFER_FRACZ_HWCN:
    case DCOPY_TRANSFER_FRACZ_NHWC:
      return set_error(DCOPY_ERR_FORMAT_INVALID, "TransShape from FRACTAL_Z is not supported");
    case DCOPY_TRANSFER_FRACTAL_NZ: {  // fractal_nz.cc:355-395
      if (type_size(data_type) <= 0)
        return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", data_type);
      if (!check_shape_for_nz(src_format, src_shape, src_rank))
        return set_error(DCOPY_ERR_SHAPE_INVALID, "format %d shape cannot become FRACTAL_NZ",
                         src_format);
      int64_t hw[3];
      int n = 0;
      const int rc = nz_shape(src_shape, src_rank, c0, dst_shape, &n, hw);
      *dst_rank = n;
      return rc;
    }
    case DCOPY_TRANSFER_FRACTAL_NZ_ND:  // fractal_nz.cc:448-457
      return set_error(DCOPY_ERR_FORMAT_INVALID,
                       "the shape derivation from FRACTAL_NZ is not unique");
    case DCOPY_TRANSFER_TRANSPOSE:
      return transpose_shape(src_format, src_shape, src_rank, dst_format, dst_shape, dst_rank);
    case DCOPY_TRANSFER_FRACTAL_ZZ: {  // fractal_zz.cc:391-431
      if (type_size(data_type) <= 0)
        return set_error(DCOPY_ERR_DATATYPE_INVALID, "data type %d is not supported", data_type);
      if (!check_shape_for_nz(src_format, src_shape, src_rank))
        return set_error(DCOPY_ERR_SHAPE_INVALID, "format %d shape cannot become FRACTAL_ZZ",
                         src_format);
      int64_t hw[3];
      int n = 0;
      const int rc = zz_shape(src_shape, src_rank, c0, dst_shape, &n, hw);
      *dst_rank = n;
      return rc;
    }
    case DCOPY_TRANSFER_FRACTAL_ZZ_ND:  // fractal_zz.cc:483-492
      return set_error(DCOPY_ERR_FORMAT_INVALID,
                       "the shape derivation from FRACTAL_ZZ is not unique");
    default: return set_error(DCOPY_ERR_PARAM_INVALID, "unknown transfer class %d", cls);
  }
}

}  // namespace
}  // namespace dcopy

using namespace dcopy;

extern "C" int32_t dcopy_data_type_size(int32_t data_type) { return type_size(data_type); }

namespace {

int32_t primary(int32_t format) { return format & 0xff; }           // GetPrimaryFormat
int64_t sub_format(int32_t format) { return (format >> 8) & 0xffff; }  // GetSubFormat

// The arguments with primary formats; the destination format's sub format
// (FRACTAL_Z TransShape groups) goes to *fmt_groups.
DcopyTransArgs normalised(const DcopyTransArgs *a, int64_t *fmt_groups) {
  DcopyTransArgs b = *a;
  b.src_format = primary(a->src_format);
  b.dst_format = primary(a->dst_format);
  *fmt_groups = sub_format(a->dst_format);
  return b;
}

}  // namespace

extern "C" int dcopy_trans_data_format(const DcopyTransArgs *args, void *dst,
                                       uint64_t dst_capacity, uint64_t *dst_length,
                                       dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  int rc = check_args(args);
  if (rc) return rc;
  int64_t groups = 0;
  const DcopyTransArgs a = normalised(args, &groups);
  const int cls = registered_class(a.src_format, a.dst_format);  // formats.cc:31-38
  if (!cls)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "Failed to trans data from format %d to %d",
                     a.src_format, a.dst_format);
  if (!a.data && item_count(a.src_shape, a.src_rank) != 0)  // :40-49
    return set_error(DCOPY_ERR_PARAM_INVALID, "input data is null and the shape is not empty");
  return class_format(cls, &a, groups, dst, dst_capacity, dst_length, stream);
  DCOPY_API_END
}

extern "C" int dcopy_trans_format_check(int transfer_class, const DcopyTransArgs *args,
                                        uint64_t *dst_length) {
  DCOPY_API_BEGIN
  int rc = check_args(args);
  if (rc) return rc;
  int64_t groups = 0;
  const DcopyTransArgs a = normalised(args, &groups);
  int cls = transfer_class;
  if (cls == 0) {  // TransDataFormat: registry and NULL-data checks first (formats.cc:31-49)
    cls = registered_class(a.src_format, a.dst_format);
    if (!cls)
      return set_error(DCOPY_ERR_FORMAT_INVALID, "Failed to trans data from format %d to %d",
                       a.src_format, a.dst_format);
    if (!a.data && item_count(a.src_shape, a.src_rank) != 0)
      return set_error(DCOPY_ERR_PARAM_INVALID, "input data is null and the shape is not empty");
  }
  t_check_only = true;
  rc = class_format(cls, &a, groups, nullptr, 0, dst_length, nullptr);
  t_check_only = false;
  return rc;
  DCOPY_API_END
}

extern "C" int dcopy_trans_format(int transfer_class, const DcopyTransArgs *args, void *dst,
                                  uint64_t dst_capacity, uint64_t *dst_length,
                                  dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  int rc = check_args(args);
  if (rc) return rc;
  int64_t groups = 0;
  const DcopyTransArgs a = normalised(args, &groups);
  return class_format(transfer_class, &a, groups, dst, dst_capacity, dst_length, stream);
  DCOPY_API_END
}

extern "C" int dcopy_trans_shape(int transfer_class, int32_t src_format, const int64_t *src_shape,
                                 int32_t src_rank, int32_t data_type, int32_t dst_format, int64_t c0,
                                 int64_t *dst_shape, int32_t *dst_rank) {
  DCOPY_API_BEGIN
  return class_shape(transfer_class, primary(src_format), src_shape, src_rank, data_type,
                     primary(dst_format), c0, sub_format(dst_format), dst_shape, dst_rank);
  DCOPY_API_END
}

extern "C" int dcopy_trans_tensor_shape(int32_t src_format, const int64_t *src_shape,
                                        int32_t src_rank, int32_t data_type, int32_t dst_format,
                                        int64_t c0, int64_t *dst_shape, int32_t *dst_rank) {
  DCOPY_API_BEGIN
  const int cls = registered_class(primary(src_format), primary(dst_format));
  if (!cls)
    return set_error(DCOPY_ERR_FORMAT_INVALID, "Failed to trans shape from format %d to %d",
                     primary(src_format), primary(dst_format));
  return class_shape(cls, primary(src_format), src_shape, src_rank, data_type,
                     primary(dst_format), c0, sub_format(dst_format), dst_shape, dst_rank);
  DCOPY_API_END
}

extern "C" int dcopy_transpose(void *dst, const void *src, const int64_t *src_shape,
                               const int64_t *perm, int32_t rank, int32_t data_type,
                               dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (rank < 0 || rank > kMaxRank || !perm)
    return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: rank %d", rank);
  return transpose_impl(dst, src, src_shape, perm, rank, data_type, UINT64_MAX, nullptr, stream);
  DCOPY_API_END
}

extern "C" int dcopy_transpose_with_shape_check(void *dst, const void *src,
                                                const int64_t *src_shape, const int64_t *dst_shape,
                                                const int64_t *perm, int32_t rank,
                                                int32_t data_type, dcopy_stream_t stream) {
  DCOPY_API_BEGIN
  if (rank < 0 || rank > kMaxRank || !perm)
    return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: rank %d", rank);
  // transpose.cc:203-205: the argument check comes first.
  const int32_t size = type_size(data_type);
  if (!src || size < 0 || !shape_arg_valid(src_shape, rank, perm, rank))
    return set_error(DCOPY_ERR_PARAM_INVALID, "Transpose: invalid arguments");
  bool mismatch = !dst_shape;
  for (int i = 0; !mismatch && i < rank; ++i) mismatch = dst_shape[i] != src_shape[perm[i]];
  const int rc =
      transpose_impl(dst, src, src_shape, perm, rank, data_type, UINT64_MAX, nullptr, stream);
  // transpose.cc:207-212 logs a dst_shape mismatch and carries on.
  if (!rc && mismatch) set_error(DCOPY_OK, "Failed to trans axis: invalid dst shape");
  return rc;
  DCOPY_API_END
}
