/*
 * dcopy oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-address-space restatement of the reference's algorithms for
 * the data-movement hot path.  It exists to CHECK the CUDA library: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load it.
 * The product (libdcopy.so) never links, calls or falls back to it.
 *
 * Parity pins (checked by tests/test_oracle_*.py):
 *   - tiling planner and RunTiles address model: fixtures generated from the
 *     reference's own Python twin (standalone_datacopy/profile.py:88-99,
 *     test_address_model.py:13-34) by tests/golden/make_golden.py;
 *   - ND<->FRACTAL_NZ, ND<->FRACTAL_ZZ, FRACTAL_Z and N-D transpose: GE's golden
 *     vectors (tests/ge/ut/ge/common/format_transfer_fractal_nz_unittest.cc,
 *      format_transfer_fractal_zz_unittest.cc, format_transfer_*fractalz_unittest.cc,
 *      format_transfer_fracz_*_unittest.cc, format_transfer_fractal_z_tbe_unittest.cc,
 *      format_transfer_transpose_unittest.cc), parsed at test time.
 *   - DataCopyExt gap addressing: test_address_model.py:24 (pinned through the
 *     RunTiles model, which is a DataCopyExt gather with blockLen=4).
 * Normal-mode UB padding and LoopModeParams have no reference vectors: unpinned.
 */
#ifndef DCOPY_ORACLE_H_
#define DCOPY_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#include "../include/dcopy/tiling_datacopy.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Status classes, numerically equal to the library's DCOPY_ERR_* codes. */
enum {
  ORACLE_OK = 0,
  ORACLE_EPARAM = -1,   /* ACL_ERROR_GE_PARAM_INVALID / std::runtime_error in the demo host */
  ORACLE_ESHAPE = -2,   /* ACL_ERROR_GE_SHAPE_INVALID */
  ORACLE_EDTYPE = -3,   /* ACL_ERROR_GE_DATATYPE_INVALID */
  ORACLE_EFORMAT = -4,  /* ACL_ERROR_GE_FORMAT_INVALID */
  ORACLE_EFAILED = -8,  /* GE's generic FAILED / GRAPH_FAILED */
};

/* ---- standalone_datacopy ------------------------------------------------ */

/* Tile planner: datacopy_data_collection.asc:115-123 and profile.py:88-99. */
int oracle_plan_tiling(uint32_t rows, uint32_t cols, uint32_t tile_kib, uint32_t store,
                       DataCopyTiling *out);

/* Validates a caller-filled tiling against what RunTiles can execute
 * (a tiling that would loop forever or overflow its UB buffer is rejected). */
int oracle_check_tiling(const DataCopyTiling *t);

/* RunTiles<phase> (datacopy_data_collection.asc:16-62), byte for byte, through
 * a UB buffer of t->ub_bytes bytes.  phase 0 = small/large, 1 = pretranspose,
 * 2 = contiguous.  `output` is only written when phase == 1 or t->store. */
int oracle_run_tiles(int phase, const void *input, void *output, const DataCopyTiling *t);

/* The demo host's input pattern input[i] = int32(i*17+3) (asc:124-125). */
void oracle_fill_pattern(int32_t *dst, uint64_t n);

/* ---- DataCopyExtParams (gap semantics) ----------------------------------- */

/* Block i: src + i*(block_len+src_gap) -> dst + i*(block_len+dst_gap), block_len
 * bytes.  test_address_model.py:24; ascendc/api/datacopy.h:14-40.
 * Regions must not overlap. */
void oracle_copy_ext(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                     uint64_t src_gap, uint64_t dst_gap);
/* The gap copy inside LoopModeParams' two outer loops, as GE's codegen writes
 * the loop nest (v35/codegen/reg_api_call/reg_api_call_utils.h:17-25):
 *   for i < loop2_size, j < loop1_size: copy_ext(dst + i*loop2_dst + j*loop1_dst,
 *                                                src + i*loop2_src + j*loop1_src)
 * loop strides in bytes (reg_api_call_utils.cpp:64-73 multiplies by the
 * element size). */
void oracle_copy_ext_loop(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                          uint64_t src_gap, uint64_t dst_gap, uint64_t loop1_size,
                          uint64_t loop2_size, uint64_t loop1_src, uint64_t loop1_dst,
                          uint64_t loop2_src, uint64_t loop2_dst);
/* Same, blockCount range split over `nthreads` pthreads (CPU baseline). */
int oracle_copy_ext_mt(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                       uint64_t src_gap, uint64_t dst_gap, int nthreads);

/* ---- DataCopyPad with the UB-side conventions ------------------------------ */

/* The destination (GM -> UB) or source (UB -> GM) is laid out as the Unified
 * Buffer holds it: its stride is a gap in 32-byte blocks (ascendc/api/
 * datacopy.h:20-21 GM->UB dstStride = dst_stride / align_num, :36-37 UB->GM
 * srcStride = src_stride / align_num, align_num = 32 / sizeof(T)).
 *   mode 0 (PaddingMode::Normal): each UB block starts on a 32-byte boundary and
 *     occupies round_up(left*eb + block_len + right*eb, 32) bytes;
 *   mode 1 (PaddingMode::Compact, v35/ascendc/api_regbase/datacopy.h:14-25 and
 *     standalone_datacopy/README.md: Compact packs UB without per-block 32-byte
 *     padding): each UB block occupies left*eb + block_len + right*eb bytes,
 *     and only the end of the whole transfer is rounded up to 32 bytes.
 * GM -> UB (DataCopyPad(LocalTensor, GlobalTensor, DataCopyExtParams,
 * DataCopyPadExtParams{is_pad, left, right, value})): block i of block_len
 * bytes from gm + i*(block_len + src_gap) goes to ub + i*(slot + dst_blocks*32)
 * + left*eb; when is_pad, the padding bytes (left, right and the round-up) hold
 * `value` (the low eb bytes, element by element); otherwise they are untouched
 * (the reference leaves their contents unspecified).
 * UB -> GM (DataCopyPad(GlobalTensor, LocalTensor, DataCopyExtParams)): block i
 * of block_len bytes from ub + i*(slot + src_blocks*32) (slot without padding
 * elements) to gm + i*(block_len + dst_gap).
 * Hardware results for the padding bytes are unpinned: the reference holds no
 * vectors for them.  Returns ORACLE_EPARAM for eb not 1/2/4/8, block_len not a
 * multiple of eb, or left/right padding above 32 bytes. */
int oracle_copy_pad_gm_to_ub(void *ub, const void *gm, uint64_t block_count, uint64_t block_len,
                             uint64_t src_gap, uint64_t dst_blocks, int mode, int is_pad,
                             uint32_t left, uint32_t right, uint64_t value, uint32_t eb);
int oracle_copy_pad_ub_to_gm(void *gm, const void *ub, uint64_t block_count, uint64_t block_len,
                             uint64_t src_blocks, uint64_t dst_gap, int mode);
/* Bytes a GM -> UB transfer spans in UB (first byte to the end of its last slot). */
uint64_t oracle_pad_ub_span(uint64_t block_count, uint64_t block_len, uint64_t ub_blocks, int mode,
                            uint32_t left, uint32_t right, uint32_t eb);

/* DataCopyNddma (v35/ascendc/api_regbase/datacopy_nddma.h:15-29): an N-D box
 * copy.  sizes/strides are outermost-first, strides in elements. */
int oracle_copy_nd(void *dst, const void *src, int ndim, const uint64_t *sizes,
                   const int64_t *src_strides, const int64_t *dst_strides, uint32_t elem_bytes);

/* ---- ND <-> FRACTAL_NZ ---------------------------------------------------- */

/* TransShapeToFracNz (format_transfer_fractal_nz.cc:65-111).  dst_shape needs
 * room for rank+2 entries; hw_shape receives {times, H, W}. */
int oracle_nz_shape(const int64_t *nd_shape, int rank, int64_t w0, int64_t *dst_shape,
                    int *dst_rank, int64_t *hw_shape);
/* TransFormatFromNdToFracNz (:131-213).  dst is zero-filled first (:139). */
int oracle_nd_to_nz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t w0);
/* TransFormatFromFracNzToNd (:215-298).  Padding is dropped. */
int oracle_nz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t w0);
/* Multi-threaded versions (times x H split over pthreads) for the CPU baseline. */
int oracle_nd_to_nz_mt(void *dst, const void *src, const int64_t *nd_shape, int rank,
                       int elem_bytes, int64_t w0, int nthreads);
int oracle_nz_to_nd_mt(void *dst, const void *src, const int64_t *nd_shape, int rank,
                       int elem_bytes, int64_t w0, int nthreads);

/* ---- ND <-> FRACTAL_ZZ ---------------------------------------------------- */

/* TransShapeToFracZz (format_transfer_fractal_zz.cc:74-118): [..., H, W] ->
 * [..., ceil(H/c0), ceil(W/c0), c0, c0]; rank 1 [N] -> [1, ceil(N/c0), c0, c0]. */
int oracle_zz_shape(const int64_t *nd_shape, int rank, int64_t c0, int64_t *dst_shape,
                    int *dst_rank, int64_t *hw_shape);
/* TransFormatFromNdToFracZz (:140-236), zero-filled padding (:148). */
int oracle_nd_to_zz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t c0);
/* TransFormatFromFracZzToNd (:238-334). */
int oracle_zz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t c0);

/* ---- FRACTAL_Z (convolution weights; fractal_z_oracle.c) ------------------- */

/* TransShape of FormatTransferFractalZ (fractal_z.cc:41-173, src_format NCHW 0,
 * NHWC 1, HWCN 16; groups = the destination format's sub format, used when > 1
 * for NCHW/HWCN) and of FormatTransferFractalZTbe (fractal_z_tbe.cc:32-62,
 * src_format ND 2 = [C, N]).  dst_shape receives [C1*H*W, N1, 16, C0]. */
int oracle_fz_shape(int src_format, const int64_t *src_shape, int rank, int64_t c0,
                    int64_t groups, int64_t *dst_shape, int *dst_rank);
/* The data movement of FormatTransferFractalZ::TransFormat / FractalZTbe
 * (groups = TransArgs::dst_sub_format, used for HWCN when > 1).  *out_elems
 * receives the element count the reference writes. */
int oracle_to_fz(void *dst, const void *src, int src_format, const int64_t *src_shape, int rank,
                 int elem_bytes, int64_t c0, int64_t groups, int64_t *out_elems);
/* CheckArgsForFracZTo{Nchw,Hwcn,Nhwc} (fracz_nchw.cc:28-79 and twins). */
int oracle_from_fz_check(const int64_t *src_shape, int src_rank, int dst_format,
                         const int64_t *dst_shape, int dst_rank, int64_t c0);
/* GetDstDataAfterTransForFracZTo{Nchw,Hwcn,Nhwc}: FZ -> NCHW / HWCN / NHWC. */
int oracle_from_fz(void *dst, const void *src, int dst_format, const int64_t *dst_shape,
                   int rank, int elem_bytes, int64_t c0);

/* ---- N-D transpose -------------------------------------------------------- */

/* Transpose (format_transfer_transpose.cc:94-197): dst[i] = src[sum idx_k *
 * src_heads[perm_k]] over the dst odometer. */
int oracle_transpose(void *dst, const void *src, const int64_t *src_shape, const int64_t *perm,
                     int rank, int elem_bytes);

#ifdef __cplusplus
}
#endif

#endif  /* DCOPY_ORACLE_H_ */
