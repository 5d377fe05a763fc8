// GE-compatible TransData host API on the B200 kernels (header-only C++17).
//
// Mirrors the interface GE's callers use (ge/base/formats/formats.h/.cc,
// register_format_transfer.h:25-48, format_transfer_fractal_nz.h:21-38,
// format_transfer_fractal_zz.h, format_transfer_transpose.h): TransArgs in, TransResult out, host buffers on
// both sides, GE status codes.  The data movement runs on the GPU through the C
// ABI: the source is copied to the device, converted by the library's kernels
// and copied back into a new host buffer owned by the TransResult, as GE's own
// TransResult owns its buffer.  TransdataKernel::Compute
// (compiler/host_kernels/transformation_ops/transdata_kernel.cc:51-140) and
// TransVarOnHost (runtime/v1/graph/manager/trans_var_data_utils.cc:169-205) can
// call these in place of ge::formats::TransDataFormat.
//
// Differences, all on purpose:
//   * formats are the PRIMARY GE formats; C0 comes from TransArgs'
//     src_c0_format / dst_c0_format fields (GE decodes it from the full format);
//   * the registry holds {ND, NCHW, NHWC} <-> FRACTAL_NZ / FRACTAL_ZZ, {NCHW, HWCN,
//     NHWC, ND} -> FRACTAL_Z, FRACTAL_Z -> {NCHW, HWCN, NHWC} and the 12
//     transposes among NCHW/NHWC/HWCN/CHWN; other pairs are
//     ACL_ERROR_GE_FORMAT_INVALID;
//   * device work runs on an internal stream and the call returns after the
//     result is on the host (GE's transfers are synchronous too).
#ifndef DCOPY_GE_FORMATS_HPP_
#define DCOPY_GE_FORMATS_HPP_

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include "dcopy/dcopy.h"

namespace dcopy {
namespace ge {

using Status = uint32_t;
constexpr Status SUCCESS = 0;
constexpr Status ACL_ERROR_GE_PARAM_INVALID = 145000U;
constexpr Status ACL_ERROR_GE_FORMAT_INVALID = 145020U;
constexpr Status ACL_ERROR_GE_SHAPE_INVALID = 145021U;
constexpr Status ACL_ERROR_GE_DATATYPE_INVALID = 145022U;
constexpr Status ACL_ERROR_GE_MEMORY_ALLOCATION = 245000U;
constexpr Status ACL_ERROR_GE_MEMORY_OPERATE_FAILED = 245001U;
constexpr Status FAILED = 0xFFFFFFFFU;  // GE's generic failure (and GRAPH_FAILED)

// GE enum values (metadef graph/types.h; api/python/ge/ge/graph/types.py).
enum Format : int32_t {
  FORMAT_NCHW = 0, FORMAT_NHWC = 1, FORMAT_ND = 2, FORMAT_NC1HWC0 = 3, FORMAT_FRACTAL_Z = 4,
  FORMAT_C1HWNC0 = 9, FORMAT_CHWN = 14, FORMAT_HWCN = 16, FORMAT_FRACTAL_ZZ = 28,
  FORMAT_FRACTAL_NZ = 29, FORMAT_RESERVED = 40
};
enum DataType : int32_t {
  DT_FLOAT = 0, DT_FLOAT16 = 1, DT_INT8 = 2, DT_INT32 = 3, DT_UINT8 = 4, DT_INT16 = 6,
  DT_UINT16 = 7, DT_UINT32 = 8, DT_INT64 = 9, DT_UINT64 = 10, DT_DOUBLE = 11, DT_BOOL = 12,
  DT_STRING = 13, DT_COMPLEX64 = 16, DT_COMPLEX128 = 17, DT_BF16 = 27, DT_UNDEFINED = 28
};

namespace formats {

// register_format_transfer.h:25-42, field for field (aggregate-initialised the
// way GE's callers and unit tests do).
struct TransArgs {
  const uint8_t *data;
  Format src_format;
  Format dst_format;
  Format src_primary_format;
  Format dst_primary_format;
  Format src_sub_format;
  Format dst_sub_format;
  int64_t src_c0_format;
  int64_t dst_c0_format;
  std::vector<int64_t> src_shape;
  std::vector<int64_t> dst_shape;
  DataType src_data_type;
};

// register_format_transfer.h:44-48: a host buffer and its length in bytes.
struct TransResult {
  std::shared_ptr<uint8_t> data;
  size_t length;
};

inline int32_t GetSizeByDataType(DataType dt) { return dcopy_data_type_size(dt); }

namespace detail {

inline DcopyTransArgs c_args(const TransArgs &a, const void *data) {
  DcopyTransArgs c{};
  c.data = data;
  // Primary formats from their own fields, sub formats (FRACTAL_Z groups) from
  // the full formats, as GE's transfers read them.
  c.src_format = (a.src_format & 0xffff00) | (a.src_primary_format & 0xff);
  c.dst_format = (a.dst_format & 0xffff00) | (a.dst_primary_format & 0xff);
  c.src_sub_format = a.src_sub_format;
  c.dst_sub_format = a.dst_sub_format;
  c.src_c0 = a.src_c0_format;
  c.dst_c0 = a.dst_c0_format;
  c.src_shape = a.src_shape.data();
  c.src_rank = static_cast<int32_t>(a.src_shape.size());
  c.dst_shape = a.dst_shape.data();
  c.dst_rank = static_cast<int32_t>(a.dst_shape.size());
  c.data_type = a.src_data_type;
  return c;
}

// Runs one TransFormat (transfer_class 0 = the registry) on the GPU with host
// buffers on both sides.
inline Status run(int transfer_class, const TransArgs &args, TransResult &result) {
  DcopyTransArgs c = c_args(args, args.data);
  uint64_t out_bytes = 0;
  int rc = dcopy_trans_format_check(transfer_class, &c, &out_bytes);
  if (rc != DCOPY_OK) return dcopy_status_to_ge(rc);
  if (out_bytes == 0) {
    result.data.reset();
    result.length = 0;
    return SUCCESS;
  }
  int64_t in_items = 1;
  for (int64_t d : args.src_shape) in_items *= d;
  const uint64_t in_bytes = static_cast<uint64_t>(in_items) *
                            static_cast<uint64_t>(GetSizeByDataType(args.src_data_type));
  std::shared_ptr<uint8_t> host(new (std::nothrow) uint8_t[out_bytes],
                                std::default_delete<uint8_t[]>());
  if (!host) return ACL_ERROR_GE_MEMORY_ALLOCATION;
  cudaStream_t s = nullptr;
  void *d_in = nullptr, *d_out = nullptr;
  Status status = SUCCESS;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMallocAsync(&d_in, in_bytes ? in_bytes : 1, s) != cudaSuccess ||
      cudaMallocAsync(&d_out, out_bytes, s) != cudaSuccess) {
    status = ACL_ERROR_GE_MEMORY_ALLOCATION;
  } else if (cudaMemcpyAsync(d_in, args.data, in_bytes, cudaMemcpyHostToDevice, s) !=
             cudaSuccess) {
    status = ACL_ERROR_GE_MEMORY_OPERATE_FAILED;
  } else {
    c = c_args(args, d_in);
    uint64_t written = 0;
    const auto ds = reinterpret_cast<dcopy_stream_t>(s);
    rc = transfer_class == 0 ? dcopy_trans_data_format(&c, d_out, out_bytes, &written, ds)
                             : dcopy_trans_format(transfer_class, &c, d_out, out_bytes, &written,
                                                  ds);
    if (rc != DCOPY_OK)
      status = dcopy_status_to_ge(rc);
    else if (cudaMemcpyAsync(host.get(), d_out, out_bytes, cudaMemcpyDeviceToHost, s) !=
                 cudaSuccess ||
             cudaStreamSynchronize(s) != cudaSuccess)
      status = ACL_ERROR_GE_MEMORY_OPERATE_FAILED;
  }
  if (s) {
    if (d_in) cudaFreeAsync(d_in, s);
    if (d_out) cudaFreeAsync(d_out, s);
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
  }
  if (status == SUCCESS) {
    result.data = host;
    result.length = static_cast<size_t>(out_bytes);
  }
  return status;
}

}  // namespace detail

// formats.cc:30-52.
inline Status TransDataFormat(const TransArgs &args, TransResult &result) {
  return detail::run(0, args, result);
}

// formats.cc:73-75: is the (src, dst) primary-format pair registered?  The
// registry check of TransDataFormat is the only one that answers FORMAT_INVALID.
inline bool IsTransFormatSupport(const TransArgs &args) {
  DcopyTransArgs c{};
  c.data = &c;  // any non-NULL address: only the registry is consulted
  c.src_format = args.src_primary_format;
  c.dst_format = args.dst_primary_format;
  uint64_t len = 0;
  return dcopy_trans_format_check(0, &c, &len) != DCOPY_ERR_FORMAT_INVALID;
}

// formats.cc:54-71 with the destination format's C0 made explicit.
inline Status TransTensorShape(Format src_format, const std::vector<int64_t> &src_shape,
                               DataType data_type, Format dst_format,
                               std::vector<int64_t> &dst_shape, int64_t dst_c0 = 16) {
  std::vector<int64_t> out(src_shape.size() + 4);
  int32_t rank = 0;
  const int rc = dcopy_trans_tensor_shape(src_format, src_shape.data(),
                                          static_cast<int32_t>(src_shape.size()), data_type,
                                          dst_format, dst_c0, out.data(), &rank);
  if (rc != DCOPY_OK) return dcopy_status_to_ge(rc);
  dst_shape.assign(out.begin(), out.begin() + rank);
  return SUCCESS;
}

// The FormatTransfer classes (format_transfer_fractal_nz.h:21-38,
// format_transfer_fractal_zz.h, format_transfer_fractal_z.h, format_transfer_fractal_z_tbe.h,
// format_transfer_fracz_{nchw,hwcn,nhwc}.h, format_transfer_transpose.h): TransFormat
// runs that class's own checks.
template <int kClass>
class FormatTransferClass {
 public:
  Status TransFormat(const TransArgs &args, TransResult &result) {
    return detail::run(kClass, args, result);
  }
  Status TransShape(Format src_format, const std::vector<int64_t> &src_shape, DataType data_type,
                    Format dst_format, std::vector<int64_t> &dst_shape, int64_t c0 = 16) {
    std::vector<int64_t> out(src_shape.size() + 4);
    int32_t rank = 0;
    const int rc = dcopy_trans_shape(kClass, src_format, src_shape.data(),
                                     static_cast<int32_t>(src_shape.size()), data_type,
                                     dst_format, c0, out.data(), &rank);
    if (rc != DCOPY_OK) return dcopy_status_to_ge(rc);
    dst_shape.assign(out.begin(), out.begin() + rank);
    return SUCCESS;
  }
};
using FormatTransferFractalNz = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_NZ>;
using FormatTransferFractalNzND = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_NZ_ND>;
using FormatTransferTranspose = FormatTransferClass<DCOPY_TRANSFER_TRANSPOSE>;
using FormatTransferFractalZz = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_ZZ>;
using FormatTransferFractalZzND = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_ZZ_ND>;
using FormatTransferFractalZ = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_Z>;
using FormatTransferFractalZTbe = FormatTransferClass<DCOPY_TRANSFER_FRACTAL_Z_TBE>;
using FormatTransferFracZNchw = FormatTransferClass<DCOPY_TRANSFER_FRACZ_NCHW>;
using FormatTransferFracZHwcn = FormatTransferClass<DCOPY_TRANSFER_FRACZ_HWCN>;
using FormatTransferFracZNhwc = FormatTransferClass<DCOPY_TRANSFER_FRACZ_NHWC>;

// format_transfer_transpose.cc:142-215 with host buffers.
inline Status TransposeWithShapeCheck(const uint8_t *src, const std::vector<int64_t> &src_shape,
                                      const std::vector<int64_t> &dst_shape,
                                      DataType src_data_type, const std::vector<int64_t> &perm_arg,
                                      TransResult &result) {
  const int32_t size = GetSizeByDataType(src_data_type);
  if (!src || size < 0 || src_shape.empty() || perm_arg.size() != src_shape.size())
    return ACL_ERROR_GE_PARAM_INVALID;
  int64_t n = 1;
  for (int64_t d : src_shape) {
    if (d < 0) return ACL_ERROR_GE_PARAM_INVALID;
    n *= d;
  }
  const uint64_t bytes = static_cast<uint64_t>(n) * static_cast<uint64_t>(size);
  if (bytes == 0) {
    result.data.reset();
    result.length = 0;
    return SUCCESS;
  }
  std::shared_ptr<uint8_t> host(new (std::nothrow) uint8_t[bytes],
                                std::default_delete<uint8_t[]>());
  if (!host) return ACL_ERROR_GE_MEMORY_ALLOCATION;
  void *d_in = nullptr, *d_out = nullptr;
  if (cudaMalloc(&d_in, bytes) != cudaSuccess || cudaMalloc(&d_out, bytes) != cudaSuccess) {
    cudaFree(d_in);
    return ACL_ERROR_GE_MEMORY_ALLOCATION;
  }
  Status status = SUCCESS;
  if (cudaMemcpy(d_in, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
    status = ACL_ERROR_GE_MEMORY_OPERATE_FAILED;
  } else {
    const std::vector<int64_t> &dst = dst_shape.size() == src_shape.size() ? dst_shape : src_shape;
    const int rc = dcopy_transpose_with_shape_check(d_out, d_in, src_shape.data(), dst.data(),
                                                    perm_arg.data(),
                                                    static_cast<int32_t>(src_shape.size()),
                                                    src_data_type, nullptr);
    if (rc != DCOPY_OK)
      status = dcopy_status_to_ge(rc);
    else if (cudaMemcpy(host.get(), d_out, bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
      status = ACL_ERROR_GE_MEMORY_OPERATE_FAILED;
  }
  cudaFree(d_in);
  cudaFree(d_out);
  if (status == SUCCESS) {
    result.data = host;
    result.length = static_cast<size_t>(bytes);
  }
  return status;
}

inline Status Transpose(const uint8_t *src, const std::vector<int64_t> &src_shape,
                        DataType src_data_type, const std::vector<int64_t> &perm_arg,
                        TransResult &result) {
  std::vector<int64_t> dst(src_shape.size());
  for (size_t i = 0; i < perm_arg.size() && i < dst.size(); ++i)
    dst[i] = (perm_arg[i] >= 0 && static_cast<size_t>(perm_arg[i]) < src_shape.size())
                 ? src_shape[static_cast<size_t>(perm_arg[i])]
                 : 0;
  return TransposeWithShapeCheck(src, src_shape, dst, src_data_type, perm_arg, result);
}

}  // namespace formats
}  // namespace ge
}  // namespace dcopy

#endif  // DCOPY_GE_FORMATS_HPP_
