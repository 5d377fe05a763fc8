// Host-side helpers shared between translation units of libdcopy.
#pragma once

#include <stdint.h>

#include "dcopy/dcopy.h"

namespace dcopy {

// IsShapeValid (formats_trans_utils.cc:88-107): non-empty, no negative dim,
// item count below 2^40.
bool shape_valid(const int64_t *shape, int rank);
// TransShapeToFracNz (format_transfer_fractal_nz.cc:65-111).  Sets the error
// slot (SHAPE_INVALID) when the result is not a valid shape.
int nz_shape(const int64_t *nd, int rank, int64_t w0, int64_t *nz, int *nz_rank, int64_t *hw);
// TransShapeToFracZz (format_transfer_fractal_zz.cc:74-118), same contract.
int zz_shape(const int64_t *nd, int rank, int64_t c0, int64_t *zz, int *zz_rank, int64_t *hw);

enum class FracKind { kNz, kZz };
// ND <-> FRACTAL_NZ / FRACTAL_ZZ with all argument checks of the public entries
// (dcopy_nd_to_nz, dcopy_nz_to_nd, dcopy_nd_to_zz, dcopy_zz_to_nd).
int frac_transfer(FracKind kind, void *dst, const void *src, const int64_t *nd_shape, int rank,
                  int elem_bytes, int64_t w0, bool to_frac, dcopy_stream_t stream);
int nz_transfer(void *dst, const void *src, const int64_t *nd_shape, int rank, int elem_bytes,
                int64_t w0, bool to_nz, dcopy_stream_t stream);

// The reference's pretranspose workflow (asc:144-146): x -> B with RunTiles<1>,
// then B -> y with RunTiles<2>, through a B buffer of scratch_bytes bytes that
// the caller of this function guarantees is device memory (it is not checked).
int run_pretranspose_workflow(const void *x, void *scratch, uint64_t scratch_bytes, void *y,
                              const DataCopyTiling *tiling, dcopy_stream_t stream);

}  // namespace dcopy
