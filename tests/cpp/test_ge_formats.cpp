// GE-style use of dcopy/ge_formats.hpp, checked against the oracle.
//
// The calls are written the way GE's own format-transfer unit tests and its
// TransData callers write them (TransArgs aggregate-initialised field by field,
// TransDataFormat / FormatTransfer*::TransFormat / TransShape returning GE
// status codes), with host buffers in and out.  Built and run by
// tests/test_ge_formats_cpp.py; prints one line per failure and exits non-zero
// if any check fails.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "dcopy/ge_formats.hpp"
#include "dcopy_oracle.h"

using namespace dcopy::ge;
using namespace dcopy::ge::formats;

static int g_failures = 0;
static int g_checks = 0;
#define EXPECT(cond)                                                    \
  do {                                                                  \
    ++g_checks;                                                         \
    if (!(cond)) {                                                      \
      ++g_failures;                                                     \
      std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);       \
    }                                                                   \
  } while (0)

template <typename T>
static std::vector<T> random_vec(size_t n, unsigned seed) {
  std::mt19937_64 rng(seed);
  std::vector<T> v(n);
  for (auto &x : v) x = static_cast<T>(rng());
  return v;
}

static void nd_nz_round_trip(Format src_fmt, const std::vector<int64_t> &nd, DataType dt,
                             int elem, unsigned seed) {
  int64_t nz[40], hw[3];
  int nz_rank = 0;
  EXPECT(oracle_nz_shape(nd.data(), (int)nd.size(), 16, nz, &nz_rank, hw) == 0);
  std::vector<int64_t> nz_shape(nz, nz + nz_rank);
  size_t n = 1, m = 1;
  for (auto d : nd) n *= d;
  for (auto d : nz_shape) m *= d;
  auto data = random_vec<uint8_t>(n * elem, seed);
  std::vector<uint8_t> expect(m * elem);
  EXPECT(oracle_nd_to_nz(expect.data(), data.data(), nd.data(), (int)nd.size(), elem, 16) == 0);

  TransArgs args{data.data(), src_fmt, FORMAT_FRACTAL_NZ, src_fmt, FORMAT_FRACTAL_NZ,
                 FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, nd, nz_shape, dt};
  TransResult result;
  EXPECT(TransDataFormat(args, result) == SUCCESS);
  EXPECT(result.length == expect.size());
  EXPECT(result.data && std::memcmp(result.data.get(), expect.data(), expect.size()) == 0);
  FormatTransferFractalNz transfer;
  std::vector<int64_t> shape_out;
  EXPECT(transfer.TransShape(src_fmt, nd, dt, FORMAT_FRACTAL_NZ, shape_out) == SUCCESS);
  EXPECT(shape_out == nz_shape);

  TransArgs args2{expect.data(), FORMAT_FRACTAL_NZ, src_fmt, FORMAT_FRACTAL_NZ, src_fmt,
                  FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, nz_shape, nd, dt};
  TransResult result2;
  EXPECT(TransDataFormat(args2, result2) == SUCCESS);
  EXPECT(result2.length == data.size());
  EXPECT(result2.data && std::memcmp(result2.data.get(), data.data(), data.size()) == 0);
  FormatTransferFractalNzND transfer2;
  EXPECT(transfer2.TransShape(FORMAT_FRACTAL_NZ, nz_shape, dt, src_fmt, shape_out) ==
         ACL_ERROR_GE_FORMAT_INVALID);
}

static void nd_zz_round_trip(Format src_fmt, const std::vector<int64_t> &nd, DataType dt,
                             int elem, int64_t c0, unsigned seed) {
  int64_t zz[40], hw[3];
  int zz_rank = 0;
  EXPECT(oracle_zz_shape(nd.data(), (int)nd.size(), c0, zz, &zz_rank, hw) == 0);
  std::vector<int64_t> zz_shape(zz, zz + zz_rank);
  size_t n = 1, m = 1;
  for (auto d : nd) n *= d;
  for (auto d : zz_shape) m *= d;
  auto data = random_vec<uint8_t>(n * elem, seed);
  std::vector<uint8_t> expect(m * elem);
  EXPECT(oracle_nd_to_zz(expect.data(), data.data(), nd.data(), (int)nd.size(), elem, c0) == 0);

  TransArgs args{data.data(), src_fmt, FORMAT_FRACTAL_ZZ, src_fmt, FORMAT_FRACTAL_ZZ,
                 FORMAT_RESERVED, FORMAT_RESERVED, c0, c0, nd, zz_shape, dt};
  TransResult result;
  EXPECT(FormatTransferFractalZz().TransFormat(args, result) == SUCCESS);
  EXPECT(result.length == expect.size());
  EXPECT(result.data && std::memcmp(result.data.get(), expect.data(), expect.size()) == 0);
  std::vector<int64_t> shape_out;
  EXPECT(FormatTransferFractalZz().TransShape(src_fmt, nd, dt, FORMAT_FRACTAL_ZZ, shape_out,
                                              c0) == SUCCESS);
  EXPECT(shape_out == zz_shape);

  TransArgs args2{expect.data(), FORMAT_FRACTAL_ZZ, src_fmt, FORMAT_FRACTAL_ZZ, src_fmt,
                  FORMAT_RESERVED, FORMAT_RESERVED, c0, c0, zz_shape, nd, dt};
  TransResult result2;
  EXPECT(TransDataFormat(args2, result2) == SUCCESS);
  EXPECT(result2.length == data.size());
  EXPECT(result2.data && std::memcmp(result2.data.get(), data.data(), data.size()) == 0);
  EXPECT(FormatTransferFractalZzND().TransShape(FORMAT_FRACTAL_ZZ, zz_shape, dt, src_fmt,
                                                shape_out) == ACL_ERROR_GE_FORMAT_INVALID);
}

static void fractal_z_round_trip() {
  // NCHW fp16 [31, 17, 4, 4] -> FRACTAL_Z [32, 2, 16, 16] (GE's fp16_2c_2n_pad shape) and back.
  const std::vector<int64_t> nchw = {31, 17, 4, 4}, fz = {32, 2, 16, 16};
  auto data = random_vec<uint16_t>(31 * 17 * 16, 21);
  std::vector<uint16_t> expect(32 * 2 * 16 * 16);
  int64_t written = 0;
  EXPECT(oracle_to_fz(expect.data(), data.data(), FORMAT_NCHW, nchw.data(), 4, 2, 16, 0,
                      &written) == 0 && written == (int64_t)expect.size());
  TransArgs args{reinterpret_cast<uint8_t *>(data.data()), FORMAT_NCHW, FORMAT_FRACTAL_Z,
                 FORMAT_NCHW, FORMAT_FRACTAL_Z, FORMAT_RESERVED, FORMAT_NCHW, 16, 16, nchw, fz,
                 DT_FLOAT16};
  TransResult result;
  EXPECT(FormatTransferFractalZ().TransFormat(args, result) == SUCCESS);
  EXPECT(result.length == expect.size() * 2 &&
         std::memcmp(result.data.get(), expect.data(), result.length) == 0);
  std::vector<int64_t> shape_out;
  EXPECT(FormatTransferFractalZ().TransShape(FORMAT_NCHW, nchw, DT_FLOAT16, FORMAT_FRACTAL_Z,
                                             shape_out) == SUCCESS && shape_out == fz);
  TransArgs back{reinterpret_cast<uint8_t *>(expect.data()), FORMAT_FRACTAL_Z, FORMAT_NCHW,
                 FORMAT_FRACTAL_Z, FORMAT_NCHW, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, fz, nchw,
                 DT_FLOAT16};
  TransResult result2;
  EXPECT(TransDataFormat(back, result2) == SUCCESS);
  EXPECT(result2.length == data.size() * 2 &&
         std::memcmp(result2.data.get(), data.data(), result2.length) == 0);
  // NCHW with the group count 40 in the destination format: N / groups = 0 -> FAILED.
  TransArgs bad{reinterpret_cast<uint8_t *>(data.data()),
                static_cast<Format>(FORMAT_NCHW), static_cast<Format>(FORMAT_FRACTAL_Z | (40 << 8)),
                FORMAT_NCHW, FORMAT_FRACTAL_Z, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16,
                {1, 1, 1, 1}, {1, 1, 16, 16}, DT_FLOAT16};
  EXPECT(FormatTransferFractalZ().TransFormat(bad, result) == FAILED);
}

static void transposes() {
  const struct {
    Format src, dst;
    std::vector<int64_t> perm;
  } pairs[] = {{FORMAT_NCHW, FORMAT_NHWC, {0, 2, 3, 1}}, {FORMAT_NCHW, FORMAT_HWCN, {2, 3, 1, 0}},
               {FORMAT_NHWC, FORMAT_NCHW, {0, 3, 1, 2}}, {FORMAT_HWCN, FORMAT_CHWN, {2, 0, 1, 3}},
               {FORMAT_CHWN, FORMAT_NHWC, {3, 1, 2, 0}}, {FORMAT_CHWN, FORMAT_HWCN, {1, 2, 0, 3}}};
  const std::vector<int64_t> shape = {2, 3, 4, 5};
  auto data = random_vec<uint16_t>(120, 7);
  for (const auto &p : pairs) {
    std::vector<int64_t> dst(4);
    for (int i = 0; i < 4; ++i) dst[i] = shape[p.perm[i]];
    std::vector<uint16_t> expect(120);
    EXPECT(oracle_transpose(expect.data(), data.data(), shape.data(), p.perm.data(), 4, 2) == 0);
    TransArgs args{reinterpret_cast<uint8_t *>(data.data()), p.src, p.dst, p.src, p.dst,
                   FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, shape, dst, DT_FLOAT16};
    TransResult result;
    EXPECT(TransDataFormat(args, result) == SUCCESS);
    EXPECT(result.length == 240 && std::memcmp(result.data.get(), expect.data(), 240) == 0);
    FormatTransferTranspose transfer;
    std::vector<int64_t> shape_out;
    EXPECT(transfer.TransShape(p.src, shape, DT_FLOAT16, p.dst, shape_out) == SUCCESS);
    EXPECT(shape_out == dst);
  }
  // TransposeWithShapeCheck, 2-D (format_transfer_transpose_unittest.cc transpose_with_shape_check_2d shape)
  uint8_t d2[4] = {1, 2, 3, 4};
  TransResult r2;
  EXPECT(TransposeWithShapeCheck(d2, {2, 2}, {2, 2}, DT_UINT8, {1, 0}, r2) == SUCCESS);
  EXPECT(r2.length == 4 && r2.data.get()[1] == 3 && r2.data.get()[2] == 2);
}

static void failures() {
  uint16_t data[16] = {0};
  TransResult result;
  {  // NHWC needs 4-D
    TransArgs a{reinterpret_cast<uint8_t *>(data), FORMAT_NHWC, FORMAT_FRACTAL_NZ, FORMAT_NHWC,
                FORMAT_FRACTAL_NZ, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, {1, 4, 4},
                {1, 1, 1, 16, 16}, DT_FLOAT16};
    EXPECT(FormatTransferFractalNz().TransFormat(a, result) == ACL_ERROR_GE_SHAPE_INVALID);
  }
  {  // undefined data type
    TransArgs a{reinterpret_cast<uint8_t *>(data), FORMAT_ND, FORMAT_FRACTAL_NZ, FORMAT_ND,
                FORMAT_FRACTAL_NZ, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, {4, 4},
                {1, 1, 16, 16}, DT_UNDEFINED};
    EXPECT(TransDataFormat(a, result) == ACL_ERROR_GE_DATATYPE_INVALID);
  }
  {  // unregistered pair
    TransArgs a{reinterpret_cast<uint8_t *>(data), FORMAT_FRACTAL_NZ, FORMAT_HWCN,
                FORMAT_FRACTAL_NZ, FORMAT_HWCN, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16,
                {1, 1, 1, 1, 16, 16}, {1, 1, 4, 4}, DT_FLOAT16};
    EXPECT(TransDataFormat(a, result) == ACL_ERROR_GE_FORMAT_INVALID);
    EXPECT(!IsTransFormatSupport(a));
  }
  {  // NULL data with a non-empty shape
    TransArgs a{nullptr, FORMAT_ND, FORMAT_FRACTAL_NZ, FORMAT_ND, FORMAT_FRACTAL_NZ,
                FORMAT_RESERVED, FORMAT_RESERVED, 16, 16, {4, 4}, {1, 1, 16, 16}, DT_FLOAT16};
    EXPECT(TransDataFormat(a, result) == ACL_ERROR_GE_PARAM_INVALID);
    EXPECT(IsTransFormatSupport(a));
  }
  {  // src / dst shape relation (ZZ -> ND)
    TransArgs a{reinterpret_cast<uint8_t *>(data), FORMAT_FRACTAL_ZZ, FORMAT_NHWC,
                FORMAT_FRACTAL_ZZ, FORMAT_NHWC, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16,
                {1, 1, 2, 1, 16, 16}, {1, 1, 15, 17}, DT_FLOAT16};
    EXPECT(FormatTransferFractalZzND().TransFormat(a, result) == ACL_ERROR_GE_SHAPE_INVALID);
    EXPECT(IsTransFormatSupport(a));
  }
  {  // src / dst shape relation (NZ -> ND)
    TransArgs a{reinterpret_cast<uint8_t *>(data), FORMAT_FRACTAL_NZ, FORMAT_NHWC,
                FORMAT_FRACTAL_NZ, FORMAT_NHWC, FORMAT_RESERVED, FORMAT_RESERVED, 16, 16,
                {1, 1, 2, 1, 16, 16}, {1, 1, 17, 15}, DT_FLOAT16};
    EXPECT(FormatTransferFractalNzND().TransFormat(a, result) == ACL_ERROR_GE_SHAPE_INVALID);
  }
}

int main(int argc, char **argv) {
  const bool with_gpu = !(argc > 1 && std::strcmp(argv[1], "--host-only") == 0);
  failures();
  if (with_gpu) {
    nd_nz_round_trip(FORMAT_ND, {2, 2, 17, 4}, DT_FLOAT16, 2, 1);
    nd_nz_round_trip(FORMAT_ND, {2, 2, 2, 17, 4}, DT_FLOAT16, 2, 2);
    nd_nz_round_trip(FORMAT_NCHW, {2, 2, 17, 4}, DT_FLOAT, 4, 3);
    nd_nz_round_trip(FORMAT_NHWC, {2, 2, 4, 17}, DT_FLOAT, 4, 4);
    nd_nz_round_trip(FORMAT_ND, {3, 100, 256}, DT_BF16, 2, 5);
    fractal_z_round_trip();
    nd_zz_round_trip(FORMAT_ND, {2, 3, 4, 33}, DT_UINT8, 1, 32, 6);
    nd_zz_round_trip(FORMAT_NHWC, {2, 2, 17, 4}, DT_FLOAT, 4, 16, 7);
    nd_zz_round_trip(FORMAT_ND, {3, 100, 256}, DT_BF16, 2, 16, 8);
    transposes();
  }
  std::printf("%s: %d checks, %d failures\n", g_failures ? "FAIL" : "PASS", g_checks, g_failures);
  return g_failures ? 1 : 0;
}
