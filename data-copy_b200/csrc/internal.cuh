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
// ND <-> FRACTAL_NZ with all argument checks of dcopy_nd_to_nz / dcopy_nz_to_nd.
int nz_transfer(void *dst, const void *src, const int64_t *nd_shape, int rank, int elem_bytes,
                int64_t w0, bool to_nz, dcopy_stream_t stream);

// The reference's pretranspose workflow (asc:144-146): x -> B with RunTiles<1>,
// then B -> y with RunTiles<2>, through a B buffer of scratch_bytes bytes that
// the caller of this function guarantees is device memory (it is not checked).
int run_pretranspose_workflow(const void *x, void *scratch, uint64_t scratch_bytes, void *y,
                              const DataCopyTiling *tiling, dcopy_stream_t stream);

}  // namespace dcopy
