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

}  // namespace dcopy
