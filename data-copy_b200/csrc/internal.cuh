// Host-side helpers shared between translation units of libdcopy.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dcopy/dcopy.h"

namespace dcopy {

// The unique id of the calling thread's current CUDA context (driver API, looked
// up through the runtime, so the library needs no link against libcuda); false
// when there is none or the driver lacks the call.  Caches of per-context
// objects (addresses, events) compare it to notice a device reset.
bool current_context_id(unsigned long long *id);

// IsShapeValid (formats_trans_utils.cc:88-107): non-empty, no negative dim,
// item count below 2^40.
bool shape_valid(const int64_t *shape, int rank);
// TransShapeToFracNz (format_transfer_fractal_nz.cc:65-111).  Sets the error
// slot (SHAPE_INVALID) when the result is not a valid shape.
int nz_shape(const int64_t *nd, int rank, int64_t w0, int64_t *nz, int *nz_rank, int64_t *hw);
// TransShapeToFracZz (format_transfer_fractal_zz.cc:74-118), same contract.
int zz_shape(const int64_t *nd, int rank, int64_t c0, int64_t *zz, int *zz_rank, int64_t *hw);

// One tiled-format transfer: `times` ND matrices of H x W elements (row pitch
// nd_row, batch pitch nd_batch) <-> blocks of BH rows x w0 columns, zero-padded
// to H1 x W1 blocks, where block (band, panel) of batch t starts at
// t*fr_batch + band*s_band + panel*s_panel and is stored row-major.  All
// pitches and strides in elements of elem_bytes bytes.
struct FracPlan {
  int64_t times, H, W, nd_row, nd_batch;
  int64_t BH, w0, H1, W1, s_band, s_panel, fr_batch;
  int elem_bytes;
  bool batch_fast;  // order tiles batch-first (neighbouring batches are adjacent in memory)
};
// Launches the shared tiled-format kernels for a plan whose buffers the caller
// has already checked.
int frac_launch(const FracPlan &plan, void *dst, const void *src, bool to_frac,
                dcopy_stream_t stream, const char *name);

enum class FracKind { kNz, kZz };
// ND <-> FRACTAL_NZ / FRACTAL_ZZ with all argument checks of the public entries
// (dcopy_nd_to_nz, dcopy_nz_to_nd, dcopy_nd_to_zz, dcopy_zz_to_nd).
int frac_transfer(FracKind kind, void *dst, const void *src, const int64_t *nd_shape, int rank,
                  int elem_bytes, int64_t w0, bool to_frac, dcopy_stream_t stream);
int nz_transfer(void *dst, const void *src, const int64_t *nd_shape, int rank, int elem_bytes,
                int64_t w0, bool to_nz, dcopy_stream_t stream);

// FRACTAL_Z (fz.cu).  Formats are primary GE formats (NCHW 0, NHWC 1, ND 2,
// HWCN 16).  fz_shape: TransShape with the reference's statuses (out: 4 dims).
int fz_shape(int32_t fmt, const int64_t *shape, int rank, int64_t c0, int64_t groups,
             int64_t *out);
// Elements the reference writes for a (fmt, shape, c0, groups) -> FRACTAL_Z transfer.
int fz_out_elems(int32_t fmt, const int64_t *shape, int rank, int64_t c0, int64_t groups,
                 int64_t *elems);
int to_fz(void *dst, const void *src, int32_t fmt, const int64_t *shape, int rank, int eb,
          int64_t c0, int64_t groups, dcopy_stream_t stream);
// CheckArgsForFracZTo{Nchw,Hwcn,Nhwc}.
int from_fz_check(const int64_t *src_shape, int src_rank, int32_t fmt, const int64_t *dst_shape,
                  int dst_rank, int64_t c0);
int from_fz(void *dst, const void *src, int32_t fmt, const int64_t *dst_shape, int rank, int eb,
            int64_t c0, dcopy_stream_t stream);

// dst (contiguous) = the m-D (m <= 5) strided view of src: sizes and strides in
// elements of eb bytes, dst strides the row-major heads of `size`.  Buffers are
// checked by the caller.
int permute_copy(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
                 const int64_t *ds, int eb, dcopy_stream_t stream);

// A 3- to 5-D box copy through TMA tensor maps when both views allow it
// (*taken = true); otherwise nothing is launched and *taken = false.  Sizes and
// strides outermost first, in elements.  Buffers are checked by the caller.
// Rows of size[m-1] elements, m <= 5, whose length, bases or strides are not
// 16-byte multiples: aligned 16-byte destination vectors assembled with funnel
// shifts (rows.cu).  ds == NULL: contiguous destination.
int rows_shift(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
               const int64_t *ds, int eb, cudaStream_t s);
// Whether rows of row_bytes whose widest common unit is `unit` bytes move faster
// through rows_shift than in units (measured on B200).  N-D rows (the row kernel
// with an odometer per unit): 1-, 2- and 4-byte units (112-byte rows in 4-byte
// units: 2358 -> 4978 GB/s).  2-D bursts (the strided kernel, one division per
// unit): 1- and 2-byte units, and 4-byte units from 256-byte bursts on (36-byte
// bursts stay faster in units: 4608 against 3880 GB/s).  8-byte units never.
inline bool shift_rows_pay(uint32_t unit, uint64_t row_bytes, bool nd_rows) {
  if (row_bytes < 16 || unit >= 8) return false;
  return unit <= 2 || nd_rows || row_bytes >= 256;
}

// Rows of a <=5-D box whose innermost axis is contiguous on both sides
// (permute.cu); *taken = false when the row kernel does not apply.
int rows_copy(void *dst, const void *src, int m, const uint64_t *size, const int64_t *ss,
              const int64_t *ds, int eb, dcopy_stream_t stream, bool *taken);

int nd_copy_tma(void *dst, const void *src, int ndim, const uint64_t *sizes,
                const int64_t *src_strides, const int64_t *dst_strides, uint32_t eb,
                dcopy_stream_t stream, bool *taken);

// With the TMA paths selected: a 2-D strided copy through shared memory with
// the bulk-copy engine (bulk.cu) when its bursts are 16-byte granules of at
// least DCOPY_BULK_MIN_BURST bytes in this GPU's memory (*taken = true);
// otherwise nothing is launched.
int bulk_bursts(void *dst, const void *src, uint64_t rows, uint64_t row_bytes,
                uint64_t src_pitch, uint64_t dst_pitch, cudaStream_t s, bool *taken);
// A tiled TMA tensor map (cuTensorMapEncodeTiled through the runtime's driver
// entry point, no swizzle, no interleave, zero fill): dims innermost first,
// strides[i] = bytes between steps of dim i+1 (rank - 1 entries).  False when
// the driver refuses it or lacks the call.
bool encode_tiled_map(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                      const uint64_t *dims, const uint64_t *strides, const uint32_t *box,
                      CUtensorMapL2promotion promotion);
// Whether the TMA paths are selected (dcopy_set_nd_tma / DCOPY_ND_TMA): the
// tensor-copy box kernel and the bulk-copy and tensor-copy 2-D burst kernels.
bool tma_paths_selected();
// With the TMA paths selected: gapped 2-D bursts of whole 16-byte granules
// shorter than 128 bytes as 2-D tensor copies (nd_tma.cu; *taken = true), else
// nothing is launched.
int tma_short_bursts(void *dst, const void *src, uint64_t rows, uint64_t row_bytes,
                     uint64_t src_pitch, uint64_t dst_pitch, cudaStream_t s, bool *taken);
// ORs the bulk-copy kernel's give-up flag into *flag and clears it.
int bulk_error_take(uint32_t *flag);
// The same for the bulk-copied NCHW -> FRACTAL_Z kernel (fz.cu).
int fz_error_take(uint32_t *flag);

// The reference's pretranspose workflow (asc:144-146): x -> B with RunTiles<1>,
// then B -> y with RunTiles<2>, through a B buffer of scratch_bytes bytes that
// the caller of this function guarantees is device memory (it is not checked).
int run_pretranspose_workflow(const void *x, void *scratch, uint64_t scratch_bytes, void *y,
                              const DataCopyTiling *tiling, dcopy_stream_t stream);

}  // namespace dcopy
