/*
 * dcopy -- B200 (sm_100a) data-movement library: C ABI.
 *
 * Drop-in boundary for the data-movement hot path of the reference:
 *   - the standalone_datacopy kernels and their DataCopyTiling contract
 *     (standalone_datacopy/datacopy_data_collection.asc, tiling_datacopy.h);
 *   - the DataCopyExtParams strided copy that GE's DataCopyPadExtend wrappers
 *     drive (compiler/graph/optimize/autofuse/ascendc/api/datacopy.h) and the
 *     N-D DataCopyNddma box copy (v35/ascendc/api_regbase/datacopy_nddma.h);
 *   - the ND <-> FRACTAL_NZ TransData layout conversion
 *     (base/formats/format_transfers/format_transfer_fractal_nz.cc).
 *
 * Conventions
 *   - Every function returns an int status: DCOPY_OK (0) or a negative
 *     DCOPY_ERR_* code.  Nothing throws across this ABI.  After a failure,
 *     dcopy_last_error_message() (thread-local) describes it.
 *   - The caller owns every buffer.  Buffers passed to kernels must be device
 *     memory of the current CUDA device (or memory mapped into it); each one is
 *     checked against its allocation before any launch, so a wrong pointer or a
 *     size that runs past the allocation is refused on the host instead of
 *     faulting on the GPU.
 *   - Launches are asynchronous on `stream` (NULL = the legacy default stream);
 *     no function synchronises unless its comment says so.
 *   - All copies move bits: any element type, NaN payloads included, comes out
 *     byte-identical.
 */
#ifndef DCOPY_DCOPY_H_
#define DCOPY_DCOPY_H_

#include <stddef.h>
#include <stdint.h>

#include "tiling_datacopy.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream, without requiring the CUDA headers. */
typedef struct CUstream_st *dcopy_stream_t;

/* ---- status codes ---------------------------------------------------------
 * The first four mirror the GE status classes the reference returns
 * (inc/external/ge/ge_error_codes.h:34,51-53); the demo host's validation
 * failures (asc:115-123, a std::runtime_error there) map to PARAM_INVALID. */
#define DCOPY_OK 0
#define DCOPY_ERR_PARAM_INVALID (-1)    /* ACL_ERROR_GE_PARAM_INVALID    145000 */
#define DCOPY_ERR_SHAPE_INVALID (-2)    /* ACL_ERROR_GE_SHAPE_INVALID    145021 */
#define DCOPY_ERR_DATATYPE_INVALID (-3) /* ACL_ERROR_GE_DATATYPE_INVALID 145022 */
#define DCOPY_ERR_FORMAT_INVALID (-4)   /* ACL_ERROR_GE_FORMAT_INVALID   145020 */
#define DCOPY_ERR_CUDA (-5)             /* a CUDA runtime/driver call failed */
#define DCOPY_ERR_TIMEOUT (-6)          /* a bounded device-side wait gave up */
#define DCOPY_ERR_UNSUPPORTED (-7)      /* valid request outside this build's limits */
#define DCOPY_ERR_FAILED (-8)           /* GE's generic FAILED / GRAPH_FAILED 0xFFFFFFFF */

/* Thread-local description of the last failure on this thread ("" if none). */
const char *dcopy_last_error_message(void);
/* The GE status code (ACL_ERROR_GE_*) for a DCOPY_ERR_* code; 0 for DCOPY_OK. */
uint32_t dcopy_status_to_ge(int status);
/* Library version, major*10000 + minor*100 + patch. */
int dcopy_version(void);

/* ---- standalone_datacopy ---------------------------------------------------- */

/* Tile planner.  Replaces the host planning in datacopy_data_collection.asc:108-123
 * (and its Python twin profile.py:88-99 tile_plan): validates rows (8..4088,
 * multiple of 8), cols (1..65535), tile_kib (1..240), store (0/1) and the 64 MiB
 * input limit, then fills tile_cols = min(cols, tile_kib*1024/(rows*4)) and
 * ub_bytes = tile_cols*rows*4.  Returns DCOPY_ERR_PARAM_INVALID on any rule the
 * reference rejects. */
int dcopy_plan_tiling(uint32_t rows, uint32_t cols, uint32_t tile_kib, uint32_t store,
                      DataCopyTiling *out);

/* The four kernels of datacopy_data_collection.asc:64-71, launched by the
 * reference as kernel<<<1, nullptr, stream>>>(x, y, tiling) (asc:141-147).
 * `tiling` may point to host or device memory; a device pointer costs one
 * synchronising 20-byte read on `stream`, a host pointer none.  The library
 * chooses the grid.
 *   small / large   : y[c*rows + r] = x[r*cols + c] if tiling->store, else
 *                     x is read and y is left untouched (load-only timing mode);
 *   pretranspose    : b[c*rows + r] = x[r*cols + c] always (store ignored);
 *   contiguous      : y = b (rows*cols int32) if tiling->store, else load only.
 * x, y, b are int32 buffers of rows*cols elements. */
int dcopy_datacopy_small(const void *x, void *y, const DataCopyTiling *tiling,
                         dcopy_stream_t stream);
int dcopy_datacopy_large(const void *x, void *y, const DataCopyTiling *tiling,
                         dcopy_stream_t stream);
int dcopy_datacopy_pretranspose(const void *x, void *b, const DataCopyTiling *tiling,
                                dcopy_stream_t stream);
int dcopy_datacopy_contiguous(const void *b, void *y, const DataCopyTiling *tiling,
                              dcopy_stream_t stream);

/* RunTiles<phase> (0 small/large, 1 pretranspose, 2 contiguous) over the
 * reference's tiles [tile_begin, tile_begin + tile_count) only: tile k covers
 * columns [k*tile_cols, min((k+1)*tile_cols, cols)) of x (asc:36) and writes
 * out[c*rows + r] for those columns, a contiguous range of out.  In, out and
 * tiling are those of the whole problem.  This is one Ascend core's share of
 * the tiles, and how the transpose shards across GPUs (dcopy_shard_range over
 * the tile count; each GPU writes a disjoint slice of y).  Tiles past the end
 * are PARAM_INVALID; an empty range is a no-op. */
int dcopy_datacopy_tiles(int32_t phase, const void *in, void *out, const DataCopyTiling *tiling,
                         uint32_t tile_begin, uint32_t tile_count, dcopy_stream_t stream);

/* The whole pretranspose workflow (x -> B -> y, as datacopy_pretranspose
 * followed by datacopy_contiguous) for callers that cannot allocate device
 * memory for B: a runtime that owns the whole device-memory budget, or a
 * latency-critical path where cudaMalloc/cudaFree would synchronise the device.
 * No counterpart in the reference (its host allocates B, asc:131).
 *   - Allocates nothing: B is a 16 MiB array in the library's own device memory,
 *     held by every GPU that loads this part of the library until exit.
 *     rows*cols*4 above 16 MiB is refused with DCOPY_ERR_PARAM_INVALID.
 *   - The first call on a device looks up the array's device address (with that
 *     device current) and caches it for the device's current context; a call
 *     after the context was replaced (cudaDeviceReset) looks it up again.  Make
 *     the first call on a device before any stream capture on it.
 *   - Every call on a device shares the one array: calls whose work overlaps on
 *     the GPU (other streams, other threads) race on it.  B needs no clearing:
 *     each call overwrites all of the part it reads.
 *   - y is written only when tiling->store is 1, as for datacopy_contiguous. */
int dcopy_datacopy_pretranspose_noalloc(const void *x, void *y, const DataCopyTiling *tiling,
                                        dcopy_stream_t stream);

/* ---- DataCopyExtParams strided copy ---------------------------------------- */

/* AscendC::DataCopyExtParams as filled by DataCopyPadExtend (ascendc/api/
 * datacopy.h:14-40) and by RunTiles (asc:32-40), widened so every BASELINE
 * configuration fits: blockLen in bytes, strides are GAPS in bytes between the
 * end of one block and the start of the next (test_address_model.py:24):
 *   src block i = src + i*(blockLen + srcStride)
 *   dst block i = dst + i*(blockLen + dstStride)                            */
typedef struct DcopyExtParams {
  uint32_t blockCount;
  uint32_t blockLen;   /* bytes */
  uint64_t srcStride;  /* gap bytes */
  uint64_t dstStride;  /* gap bytes */
} DcopyExtParams;

/* GM->GM copy of blockCount bursts.  Any byte alignment is accepted; 16-byte
 * aligned bursts take the vectorised path.  Source and destination ranges must
 * not overlap (DCOPY_ERR_PARAM_INVALID). */
int dcopy_copy_ext(void *dst, const void *src, const DcopyExtParams *params,
                   dcopy_stream_t stream);

/* DataCopyExt whose source and destination are host memory, through a device
 * staging buffer the caller provides (`staging`, `staging_bytes`, memory of the
 * current device; no allocation inside).  The copy engine gathers the bursts
 * host -> device chunk by chunk on `stream` (a 2-D copy reads only the bursts);
 * each staged chunk is written to dst, with its gaps, on the library's
 * per-device return stream while the next chunk is gathered, so both PCIe
 * directions are busy at once.  The return write is the copy kernel (dst must
 * be pinned host memory) unless flags has DCOPY_STAGED_COPY_ENGINE_RETURN (any
 * host memory).  `stream` waits for the last write: the call is ordered on it.
 * Staging must hold at least two bursts; the whole transfer (six chunks) keeps
 * the pipeline full.  Calls on one device share the return stream (they serialise there);
 * capturing one in a CUDA graph while another thread issues staged copies on
 * the same device is not supported.  No counterpart in the reference. */
#define DCOPY_STAGED_COPY_ENGINE_RETURN 1
int dcopy_copy_ext_staged(void *dst, const void *src, const DcopyExtParams *params, void *staging,
                          uint64_t staging_bytes, int32_t flags, dcopy_stream_t stream);

/* LoopModeParams of the v35 DataCopyPadExtend (v35/ascendc/api_regbase/datacopy.h:29-45,
 * 60-72), field order as GE's codegen emits it (v35/codegen/reg_api_call/
 * reg_api_call_utils.cpp:64-73); strides in bytes, absolute (not gaps). */
typedef struct DcopyLoopModeParams {
  uint32_t loop1Size;
  uint32_t loop2Size;
  uint64_t loop1SrcStride;
  uint64_t loop1DstStride;
  uint64_t loop2SrcStride;
  uint64_t loop2DstStride;
} DcopyLoopModeParams;

/* The DataCopyExt copy inside two outer loops (reg_api_call_utils.h:17-25):
 *   for i < loop2Size, j < loop1Size:
 *     dcopy_copy_ext(dst + i*loop2DstStride + j*loop1DstStride,
 *                    src + i*loop2SrcStride + j*loop1SrcStride, params)
 * run as one N-D box.  Destinations of different (i, j) must not overlap
 * (a zero destination stride with a loop size above 1 is PARAM_INVALID). */
int dcopy_copy_ext_loop(void *dst, const void *src, const DcopyExtParams *params,
                        const DcopyLoopModeParams *loop, dcopy_stream_t stream);

/* One copy of a batch: dcopy_copy_ext(dst, src, &params) as a record. */
typedef struct DcopyExtCopy {
  void *dst;
  const void *src;
  DcopyExtParams params;
} DcopyExtCopy;

/* `count` independent dcopy_copy_ext copies in as few launches as possible (one
 * per 256 copies; copies above 2^30 elements launch on their own).  An Ascend C
 * kernel issues many DataCopy calls per launch (the standalone kernel moves
 * each tile with one, datacopy_data_collection.asc:16-62); this is that shape
 * for a host ABI.  Every copy is validated as dcopy_copy_ext validates it, and
 * because the copies run concurrently no destination may overlap another
 * copy's destination or source (DCOPY_ERR_PARAM_INVALID, nothing launched).
 * No counterpart in the reference's host API. */
int dcopy_copy_ext_batch(const DcopyExtCopy *copies, uint32_t count, dcopy_stream_t stream);

/* Same copy with blockLen and both gaps in 32-byte units (AscendC DataCopyParams
 * units; BASELINE expresses configs 1, 2, 3 and 5 this way). */
int dcopy_copy_ext_32b(void *dst, const void *src, uint32_t blockCount, uint32_t blockLen32,
                       uint32_t srcStride32, uint32_t dstStride32, dcopy_stream_t stream);

/* ---- DataCopyPad with the Unified-Buffer side conventions ------------------ */

/* AscendC::DataCopyPadExtParams<T> {isPad, leftPadding, rightPadding,
 * paddingValue} (the GM->UB padding of DataCopyPad, ascendc/api/datacopy.h:24),
 * with T given by its size: paddingValue holds T's bits in its low elemBytes
 * bytes; leftPadding / rightPadding count elements (at most 32 bytes each). */
typedef struct DcopyPadParams {
  uint8_t isPad;
  uint8_t leftPadding;
  uint8_t rightPadding;
  uint8_t reserved;
  uint32_t elemBytes;    /* sizeof(T): 1, 2, 4 or 8 */
  uint64_t paddingValue;
} DcopyPadParams;

/* AscendC::PaddingMode (v35/ascendc/api_regbase/datacopy.h:13). */
#define DCOPY_PAD_NORMAL 0  /* every UB block starts on a 32-byte boundary */
#define DCOPY_PAD_COMPACT 1 /* UB blocks packed; the transfer's end rounded up to 32 bytes */

/* DataCopyPad GM -> UB as DataCopyPadExtend drives it (ascendc/api/datacopy.h:
 * 14-25; v35/ascendc/api_regbase/datacopy.h:14-25).  `ub` is a device buffer
 * laid out as the Unified Buffer would hold the tile.  params->blockLen is in
 * bytes, params->srcStride a GM gap in bytes, params->dstStride a UB gap in
 * 32-BYTE BLOCKS.  Block i (blockLen bytes from gm + i*(blockLen + srcStride))
 * fills UB slot i at ub + i*(slot + 32*dstStride), after leftPadding elements;
 * slot = left*eb + blockLen + right*eb, rounded up to 32 bytes in Normal mode.
 * With pad->isPad, every padding byte of a slot (and, in Compact mode, the bytes
 * that round the transfer's end up to 32) holds paddingValue element by element;
 * without it they are left untouched (their contents are unspecified on Ascend).
 * blockLen must be a whole number of elements.  The padding bytes' exact
 * hardware contents are unpinned (the reference holds no vectors for them). */
int dcopy_copy_pad_gm_to_ub(void *ub, const void *gm, const DcopyExtParams *params,
                            const DcopyPadParams *pad, int32_t mode, dcopy_stream_t stream);

/* DataCopyPad UB -> GM (ascendc/api/datacopy.h:28-40): params->srcStride is a
 * UB gap in 32-BYTE BLOCKS, params->dstStride a GM gap in bytes.  Block i of
 * blockLen bytes goes from UB slot i at ub + i*(slot + 32*srcStride), slot =
 * blockLen rounded up to 32 in Normal mode (blockLen in Compact mode), to
 * gm + i*(blockLen + dstStride). */
int dcopy_copy_pad_ub_to_gm(void *gm, const void *ub, const DcopyExtParams *params, int32_t mode,
                            dcopy_stream_t stream);

/* DataCopyPadExtend itself, arguments in elements of T exactly as GE's codegen
 * emits them (e.g. `DataCopyPadExtend(local_1[0 + 0], local_0, 1, 1, 16 - 1, 0)`,
 * tests/autofuse/ut/codegen/api_call/test_codegen_store_api_call.cpp:131):
 *   load  (GM -> UB, datacopy.h:14-25): blockLen = block_len*eb, srcStride =
 *         src_stride*eb bytes, dstStride = dst_stride / (32/eb) blocks (rounded
 *         down), padding {true, 0, 0, 0};
 *   store (UB -> GM, datacopy.h:28-40): blockLen = block_len*eb, srcStride =
 *         src_stride / (32/eb) blocks, dstStride = dst_stride*eb bytes.
 * block_len*eb must fit 32 bits (the reference truncates; here PARAM_INVALID). */
int dcopy_datacopy_pad_extend_load(void *ub, const void *gm, uint32_t elem_bytes,
                                   uint32_t block_count, uint32_t block_len, uint32_t src_stride,
                                   uint32_t dst_stride, int32_t mode, dcopy_stream_t stream);
int dcopy_datacopy_pad_extend_store(void *gm, const void *ub, uint32_t elem_bytes,
                                    uint32_t block_count, uint32_t block_len, uint32_t src_stride,
                                    uint32_t dst_stride, int32_t mode, dcopy_stream_t stream);

/* DataCopyNddma<T, dim> (v35/ascendc/api_regbase/datacopy_nddma.h:15-29): an
 * N-D box copy, 1 <= ndim <= 5.  sizes, src_strides and dst_strides are
 * outermost-first (like its output_dims argument) and strides count elements
 * of elem_bytes (1, 2, 4, 8 or 16) bytes.  Negative strides are refused.
 * Boxes whose innermost axis is contiguous on both sides run as rows in the
 * widest unit (<= 16 bytes) dividing the row, both bases and every stride;
 * other boxes run element by element.  With the TMA path selected
 * (dcopy_set_nd_tma), 3- to 5-D boxes whose rows are whole 16-byte granules,
 * with 16-byte aligned bases and 16-byte multiple strides, run as TMA tensor
 * copies (cp.async.bulk.tensor through two tensor maps) instead. */
int dcopy_copy_nd(void *dst, const void *src, int ndim, const uint64_t *sizes,
                  const int64_t *src_strides, const int64_t *dst_strides, uint32_t elem_bytes,
                  dcopy_stream_t stream);

/* Selects (enable = 1) or deselects (0) the TMA tensor-copy path of
 * dcopy_copy_nd for the whole process; *previous (may be NULL) receives the
 * former setting.  The initial setting is DCOPY_ND_TMA from the environment
 * (unset: 0).  Off by default: on B200 the row kernel measured as fast or faster
 * on every box tried.  No counterpart in the reference. */
int dcopy_set_nd_tma(int enable, int *previous);

/* Reads and clears the current device's TMA error words: 1 when a launch that
 * moved data with the copy engine inside a kernel -- the tensor-copy box path,
 * the bulk-copy burst path (both with dcopy_set_nd_tma(1)), the tensor copy that
 * dcopy_copy_ext uses by default for bursts of at most 32 bytes with source gaps
 * of at least 4x the burst, or the bulk-copied FRACTAL_Z tiles -- gave up waiting
 * on one of its own loads (that copy is then incomplete), else 0.  Synchronises
 * the device.  No counterpart in the reference. */
int dcopy_tma_error(uint32_t *flag);

/* ---- ND <-> FRACTAL_NZ ------------------------------------------------------ */

/* TransShapeToFracNz (format_transfer_fractal_nz.cc:65-111): ND [..., H, W] ->
 * NZ [..., ceil(W/w0), ceil(H/16), 16, w0]; rank 1 [N] -> [ceil(N/w0), 1, 16, w0].
 * nz_shape needs room for rank+2 (rank 1: 4) entries; hw_shape (3 entries,
 * may be NULL) receives {times, H, W}.  Also a host-only query. */
int dcopy_nz_shape(const int64_t *nd_shape, int rank, int64_t w0, int64_t *nz_shape,
                   int *nz_rank, int64_t *hw_shape);

/* TransFormatFromNdToFracNz (:131-213) on the GPU.  dst holds prod(nz_shape)
 * elements of elem_bytes bytes; its H and W padding is written as zeros (the
 * reference zero-initialises its output, :139).  w0 is the C0 of the NZ format
 * (16 for fp16/fp32 in the reference tests, 32 for 1-byte types). */
int dcopy_nd_to_nz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                   int elem_bytes, int64_t w0, dcopy_stream_t stream);

/* TransFormatFromFracNzToNd (:215-298) on the GPU: the exact inverse; padding
 * is dropped.  nd_shape is the DESTINATION (ND) shape. */
int dcopy_nz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                   int elem_bytes, int64_t w0, dcopy_stream_t stream);

/* ---- ND <-> FRACTAL_ZZ ------------------------------------------------------ */

/* TransShapeToFracZz (format_transfer_fractal_zz.cc:74-118): ND [..., H, W] ->
 * ZZ [..., ceil(H/c0), ceil(W/c0), c0, c0]; rank 1 [N] -> [1, ceil(N/c0), c0, c0].
 * Same buffer contract as dcopy_nz_shape. */
int dcopy_zz_shape(const int64_t *nd_shape, int rank, int64_t c0, int64_t *zz_shape,
                   int *zz_rank, int64_t *hw_shape);

/* TransFormatFromNdToFracZz (fractal_zz.cc:140-236) on the GPU: c0 x c0 blocks,
 * row bands outermost; H and W padding written as zeros (:148). */
int dcopy_nd_to_zz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                   int elem_bytes, int64_t c0, dcopy_stream_t stream);

/* TransFormatFromFracZzToNd (fractal_zz.cc:238-334) on the GPU: the exact
 * inverse; nd_shape is the DESTINATION (ND) shape. */
int dcopy_zz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                   int elem_bytes, int64_t c0, dcopy_stream_t stream);

/* ---- FRACTAL_Z (convolution weights) ---------------------------------------- */

/* FRACTAL_Z is [C1*H*W, N1, 16, C0]: element (c1, h, w, n, c0) holds weight
 * (n, c = c1*C0 + c0, h, w), zero where n >= N or c >= C.  Weight formats:
 * NCHW (0), NHWC (1), HWCN (16), and ND (2) = a 2-D [C, N] weight.
 *
 * TransShape of FormatTransferFractalZ (format_transfer_fractal_z.cc:41-173,
 * 571-604) and FormatTransferFractalZTbe (format_transfer_fractal_z_tbe.cc:
 * 32-62, 131-146): fz_shape receives the 4 dims.  `groups` > 1 selects the
 * group-convolution layout for NCHW and HWCN (GE takes it from the destination
 * format's sub format).  Status as the reference: SHAPE_INVALID for a source
 * that is not a valid 4-D shape, DATATYPE_INVALID for c0 < 0, FAILED when N /
 * groups is 0 (and, where the reference divides by zero, for C == 0 or c0 == 0
 * with groups) and for every ND failure. */
int dcopy_fz_shape(int32_t src_format, const int64_t *src_shape, int rank, int64_t c0,
                   int64_t groups, int64_t *fz_shape);

/* NCHW / NHWC / HWCN / ND -> FRACTAL_Z on the GPU (the data movement of
 * fractal_z.cc:175-537 and fractal_z_tbe.cc:64-114).  dst holds the whole
 * FRACTAL_Z tensor, padding written as zeros.  groups > 1 is the HWCN group
 * layout (fractal_z.cc:276-359) and is refused for the other formats. */
int dcopy_to_fractal_z(void *dst, const void *src, int32_t src_format, const int64_t *src_shape,
                       int rank, int elem_bytes, int64_t c0, int64_t groups,
                       dcopy_stream_t stream);

/* FRACTAL_Z -> NCHW / HWCN / NHWC on the GPU (format_transfer_fracz_nchw.cc,
 * fracz_hwcn.cc, fracz_nhwc.cc): dst_shape is the weight's shape; padding is
 * dropped. */
int dcopy_from_fractal_z(void *dst, const void *src, int32_t dst_format,
                         const int64_t *dst_shape, int rank, int elem_bytes, int64_t c0,
                         dcopy_stream_t stream);

/* ---- GE TransData level ------------------------------------------------------
 * The format-transfer registry of GE (base/formats/formats.cc:30-71,
 * register_format_transfer.h:25-95) on device buffers.  Formats and data types
 * use GE's enum values (metadef graph/types.h, mirrored in
 * api/python/ge/ge/graph/types.py); only PRIMARY formats are passed, with the
 * C0 of each side given explicitly (TransArgs::src_c0_format/dst_c0_format).
 * Registered pairs: {ND, NCHW, NHWC} <-> FRACTAL_NZ
 * (format_transfer_fractal_nz.cc:459-464), {ND, NCHW, NHWC} <-> FRACTAL_ZZ
 * (format_transfer_fractal_zz.cc:494-499), {NCHW, HWCN, NHWC, ND} ->
 * FRACTAL_Z and FRACTAL_Z -> {NCHW, HWCN, NHWC} (fractal_z.cc:606-608,
 * fractal_z_tbe.cc:147, fracz_{nchw,hwcn,nhwc}.cc) and the 12 transposes among NCHW, NHWC,
 * HWCN, CHWN (format_transfer_transpose.cc:268-279).
 * A format argument is a GE Format value: the primary format in bits 0-7, the
 * sub format (GetSubFormat; FRACTAL_Z's group count) in bits 8-23.  Higher bits
 * (GE's C0 field) are ignored: C0 is passed explicitly. */
#define DCOPY_FORMAT_NCHW 0
#define DCOPY_FORMAT_NHWC 1
#define DCOPY_FORMAT_ND 2
#define DCOPY_FORMAT_FRACTAL_Z 4
#define DCOPY_FORMAT_CHWN 14
#define DCOPY_FORMAT_HWCN 16
#define DCOPY_FORMAT_FRACTAL_ZZ 28
#define DCOPY_FORMAT_FRACTAL_NZ 29

/* Transfer classes (the reference's FormatTransfer subclasses). */
#define DCOPY_TRANSFER_FRACTAL_NZ 1    /* FormatTransferFractalNz   (ND/NCHW/NHWC -> NZ) */
#define DCOPY_TRANSFER_FRACTAL_NZ_ND 2 /* FormatTransferFractalNzND (NZ -> ND/NCHW/NHWC) */
#define DCOPY_TRANSFER_TRANSPOSE 3     /* FormatTransferTranspose   (4-D permutes)       */
#define DCOPY_TRANSFER_FRACTAL_ZZ 4    /* FormatTransferFractalZz   (ND/NCHW/NHWC -> ZZ) */
#define DCOPY_TRANSFER_FRACTAL_ZZ_ND 5 /* FormatTransferFractalZzND (ZZ -> ND/NCHW/NHWC) */
#define DCOPY_TRANSFER_FRACTAL_Z 6     /* FormatTransferFractalZ    (NCHW/HWCN/NHWC -> FZ) */
#define DCOPY_TRANSFER_FRACTAL_Z_TBE 7 /* FormatTransferFractalZTbe (ND [C, N] -> FZ)     */
#define DCOPY_TRANSFER_FRACZ_NCHW 8    /* FormatTransferFracZNchw   (FZ -> NCHW)          */
#define DCOPY_TRANSFER_FRACZ_HWCN 9    /* FormatTransferFracZHwcn   (FZ -> HWCN)          */
#define DCOPY_TRANSFER_FRACZ_NHWC 10   /* FormatTransferFracZNhwc   (FZ -> NHWC)          */

/* TransArgs (register_format_transfer.h:25-42) with device data. */
typedef struct DcopyTransArgs {
  const void *data;         /* source, device memory */
  int32_t src_format;       /* GE Format of the source (primary + sub bits) */
  int32_t dst_format;       /* GE Format of the destination (primary + sub bits) */
  int64_t src_c0;           /* C0 of the source format (used by NZ/ZZ -> ND) */
  int64_t dst_c0;           /* C0 of the destination format (used by ND -> NZ/ZZ) */
  const int64_t *src_shape;
  int32_t src_rank;
  const int64_t *dst_shape; /* required by the transfers, as in the reference */
  int32_t dst_rank;
  int32_t data_type;        /* GE DataType */
  int32_t src_sub_format;   /* TransArgs::src_sub_format (unused by these transfers) */
  int32_t dst_sub_format;   /* TransArgs::dst_sub_format: HWCN -> FRACTAL_Z groups */
} DcopyTransArgs;

/* GetSizeByDataType: bytes of one element, or -1 for types without a fixed
 * byte size (string, resource, sub-byte types, undefined). */
int32_t dcopy_data_type_size(int32_t data_type);

/* TransDataFormat (formats.cc:30-52): FORMAT_INVALID for an unregistered pair,
 * PARAM_INVALID for a NULL source with a non-empty shape, then the registered
 * transfer's TransFormat.  The result (prod(dst_shape) elements) is written to
 * `dst` (device, dst_capacity bytes; too small -> PARAM_INVALID) and its byte
 * length stored in *dst_length. */
int dcopy_trans_data_format(const DcopyTransArgs *args, void *dst, uint64_t dst_capacity,
                            uint64_t *dst_length, dcopy_stream_t stream);

/* Every check of dcopy_trans_data_format (transfer_class 0) or of one transfer
 * class's TransFormat, with the same status, but no data movement: *dst_length
 * receives the result length in bytes.  args->data is only tested for NULL
 * (it may be host memory), so callers can size their buffers first. */
int dcopy_trans_format_check(int transfer_class, const DcopyTransArgs *args,
                             uint64_t *dst_length);

/* FormatTransfer::TransFormat of one transfer class, with that class's own
 * checks and status codes (format_transfer_fractal_nz.cc:301-353, 397-446;
 * format_transfer_fractal_zz.cc:337-389, 433-481;
 * format_transfer_transpose.cc:239-251). */
int dcopy_trans_format(int transfer_class, const DcopyTransArgs *args, void *dst,
                       uint64_t dst_capacity, uint64_t *dst_length, dcopy_stream_t stream);

/* FormatTransfer::TransShape of one transfer class (fractal_nz.cc:355-395,
 * 448-457; fractal_zz.cc:391-431, 483-492; transpose.cc:253-266).  `c0` is the
 * C0 of dst_format.  dst_shape needs room for src_rank + 2 entries. */
int dcopy_trans_shape(int transfer_class, int32_t src_format, const int64_t *src_shape,
                      int32_t src_rank, int32_t data_type, int32_t dst_format, int64_t c0,
                      int64_t *dst_shape, int32_t *dst_rank);

/* TransTensorShape (formats.cc:54-71): registry dispatch of TransShape. */
int dcopy_trans_tensor_shape(int32_t src_format, const int64_t *src_shape, int32_t src_rank,
                             int32_t data_type, int32_t dst_format, int64_t c0,
                             int64_t *dst_shape, int32_t *dst_rank);

/* Transpose (format_transfer_transpose.cc:142-197) on the GPU:
 * dst[i] = src[sum_k idx_k * src_heads[perm_k]] over the destination odometer,
 * rank 1..5.  Every argument failure is PARAM_INVALID, as in the reference. */
int dcopy_transpose(void *dst, const void *src, const int64_t *src_shape, const int64_t *perm,
                    int32_t rank, int32_t data_type, dcopy_stream_t stream);

/* TransposeWithShapeCheck (transpose.cc:200-215): like the reference, a
 * dst_shape that differs from the permuted source shape is reported in
 * dcopy_last_error_message() but does not fail the call. */
int dcopy_transpose_with_shape_check(void *dst, const void *src, const int64_t *src_shape,
                                     const int64_t *dst_shape, const int64_t *perm,
                                     int32_t rank, int32_t data_type, dcopy_stream_t stream);

/* ---- runtime memcpy task --------------------------------------------------------
 * The D2D memcpy task of GE's runtime (runtime/v1/graph/load/model_manager/
 * task_info/rts/memcpy_async_task_info.cc:88-111 -> rtMemcpyAsyncWithCfg,
 * runtime/v1/common/runtime_api_wrapper.h:42-49).  Kinds take rtMemcpyKind_t's
 * values (compiler/engines/rts_engine/ops_kernel_store/op/acl_rt_memcpy_kind.h). */
#define DCOPY_MEMCPY_HOST_TO_HOST 0
#define DCOPY_MEMCPY_HOST_TO_DEVICE 1
#define DCOPY_MEMCPY_DEVICE_TO_HOST 2
#define DCOPY_MEMCPY_DEVICE_TO_DEVICE 3  /* one device or peer-to-peer */
#define DCOPY_MEMCPY_MANAGED 4
#define DCOPY_MEMCPY_HOST_TO_DEVICE_EX 6
#define DCOPY_MEMCPY_DEVICE_TO_HOST_EX 7
#define DCOPY_MEMCPY_DEFAULT 8           /* infer the direction from the pointers */

typedef struct DcopyMemcpyInfo {  /* MemcpyAsyncMemInfo */
  void *dst;
  uint64_t destMax;               /* capacity of dst in bytes */
  const void *src;
  uint64_t cnt;                   /* bytes to copy */
} DcopyMemcpyInfo;

/* cnt > destMax is PARAM_INVALID (nothing copied).  Device-to-device copies
 * (DEVICE_TO_DEVICE, or DEFAULT between two device buffers) run the library's
 * copy kernel on `stream`, peer memory included; host-side kinds go to
 * cudaMemcpyAsync.  RT_MEMCPY_ADDR_DEVICE_TO_DEVICE (5) is UNSUPPORTED. */
int dcopy_memcpy_async(const DcopyMemcpyInfo *info, int32_t kind, dcopy_stream_t stream);

/* `count` memcpy tasks of one kind, each checked as dcopy_memcpy_async checks
 * it (nothing runs if one fails).  Tasks whose buffers are device or pinned
 * host memory, below 8 MiB when a host side is involved, run together on the
 * batched copy kernel (one launch per 256 tasks; host buffers are read and
 * written over PCIe); pageable host memory, larger host-side transfers and
 * HOST_TO_HOST take cudaMemcpyAsync, one per task.  The result is that of the
 * tasks issued one by one in order: the tasks of one kernel launch run
 * concurrently, so a launch is issued before each copy-engine task and before
 * any task that reads or writes what a task already in the launch writes (or
 * writes what one reads).  A task whose own source and destination overlap is
 * PARAM_INVALID.  No counterpart in the reference (its tasks are issued one by
 * one). */
int dcopy_memcpy_async_batch(const DcopyMemcpyInfo *infos, uint32_t count, int32_t kind,
                             dcopy_stream_t stream);

/* ---- multi-GPU ----------------------------------------------------------------
 * No counterpart in the reference (its kernels run on one device).
 * Copies shard by splitting the blockCount range over devices with no
 * exchange; the separate ring shift moves each device's shard to the next
 * device with in-kernel stores over NVLink.  No TMA multicast is used. */

/* Contiguous block range [*begin, *begin + *count) of `block_count` blocks that
 * `rank` of `world` owns: the first block_count % world ranks get one more. */
int dcopy_shard_range(uint64_t block_count, int32_t rank, int32_t world, uint64_t *begin,
                      uint64_t *count);

/* One strided copy per device, launched from one host thread (each on its own
 * device and stream).  The current device is restored on return. */
typedef struct DcopyDevCopy {
  int32_t device;
  void *dst;
  const void *src;
  DcopyExtParams params;
  dcopy_stream_t stream;
} DcopyDevCopy;
int dcopy_copy_ext_multi(const DcopyDevCopy *copies, int32_t n);

/* Lets `device` address `peer`'s memory (cudaDeviceEnablePeerAccess); OK when
 * already enabled, PARAM_INVALID when the pair cannot be peers.  Process-wide
 * and released with the process; it changes no setting of the GPU itself. */
int dcopy_enable_peer_access(int32_t device, int32_t peer);

/* bytes from `src` to `dst`, either of which may be another GPU's memory mapped
 * into this process (peer access or IPC), on `stream`.  Engine (see
 * dcopy_set_p2p_engine), automatic choice: a push (src this GPU's memory, dst
 * not) runs on the copy engine, which measured faster than every SM write path
 * at every size from 64 KiB to 1 GiB; every other case (pulls, local copies)
 * runs the 128-bit load/store kernel.  With the SM engine forced, a push of
 * 16-byte granular buffers runs an SM bulk-copy (TMA, no multicast) pipeline --
 * local loads into shared memory, bulk stores over NVLink.  No counterpart in
 * the reference (its multi-device transfers go through HCCL). */
int dcopy_p2p_copy(void *dst, const void *src, uint64_t bytes, dcopy_stream_t stream);

/* Engine selection of dcopy_p2p_copy for the whole process; *previous (may be
 * NULL) receives the former setting.  AUTO as above; SM: the kernels only;
 * COPY: the copy engine for every transfer.  The initial setting is
 * DCOPY_P2P_ENGINE from the environment (auto, sm or copy; unset: auto). */
#define DCOPY_P2P_ENGINE_AUTO 0
#define DCOPY_P2P_ENGINE_SM 1
#define DCOPY_P2P_ENGINE_COPY 2
int dcopy_set_p2p_engine(int32_t engine, int32_t *previous);

/* The route dcopy_p2p_copy(dst, src, bytes, ...) takes under the current engine
 * setting and the current device, without copying anything or checking the
 * buffers: the copy engine, the SM bulk-copy push, or the SM load/store kernel. */
#define DCOPY_P2P_ROUTE_COPY_ENGINE 0
#define DCOPY_P2P_ROUTE_SM_BULK_PUSH 1
#define DCOPY_P2P_ROUTE_SM_LOAD_STORE 2
int dcopy_p2p_route(const void *dst, const void *src, uint64_t bytes, int32_t *route);

/* Reads and clears the current device's P2P error word: 1 when a bulk-copy
 * push gave up waiting on one of its own copies (the copy is then incomplete),
 * else 0.  Synchronises the device. */
int dcopy_p2p_error(uint32_t *flag);

/* Ring shift inside one process: device devices[i] copies src[i] (its own
 * memory) into dst[(i + 1) % n] (memory of the next device), on streams[i]
 * (NULL entries = that device's legacy default stream).  Peer access between
 * ring neighbours is enabled as needed. */
int dcopy_p2p_ring_shift(const int32_t *devices, void *const *src, void *const *dst,
                         const dcopy_stream_t *streams, int32_t n, uint64_t bytes);

/* CUDA IPC (multi-process): the 64-byte handle of the allocation holding
 * dev_ptr and dev_ptr's byte offset inside it; another process of the same node
 * opens the handle (peer access enabled lazily) and adds the offset.  Close the
 * BASE pointer that dcopy_ipc_open_handle returned.  The library records every
 * mapping opened here until it is closed: the driver reports an IPC mapping as
 * memory of the opening GPU, and the record is what makes dcopy_p2p_copy treat
 * a copy into it as a push to another GPU. */
#define DCOPY_IPC_HANDLE_BYTES 64
int dcopy_ipc_get_handle(const void *dev_ptr, void *handle, uint64_t *offset);
int dcopy_ipc_open_handle(const void *handle, void **base_ptr);
int dcopy_ipc_close_handle(void *base_ptr);

/* Completion flags.  dcopy_signal stores `value` to *flag with release
 * semantics at system scope after all earlier work on `stream` (the flag may
 * live on another GPU).  Flag values are sequence numbers that only grow.
 * dcopy_wait_signal launches a one-thread kernel that waits, with acquire
 * loads, until *flag has reached or passed value ((int32_t)(*flag - value) >= 0,
 * so a signaller already a step ahead counts), at most timeout_ns nanoseconds
 * (and a fixed iteration bound), then writes 0 (seen) or 1 (timed out) to
 * *status (device memory) and returns; later work on `stream` runs after it
 * either way.  The wait must not run on the same GPU as the kernel
 * that sets the flag, unless that kernel is already complete. */
int dcopy_signal(uint32_t *flag, uint32_t value, dcopy_stream_t stream);
int dcopy_wait_signal(const uint32_t *flag, uint32_t value, uint64_t timeout_ns,
                      uint32_t *status, dcopy_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
static_assert(sizeof(DcopyExtParams) == 24, "DcopyExtParams layout");
static_assert(sizeof(DcopyExtCopy) == 40, "DcopyExtCopy layout");
static_assert(sizeof(DcopyLoopModeParams) == 40, "DcopyLoopModeParams layout");
#endif

#endif /* DCOPY_DCOPY_H_ */
