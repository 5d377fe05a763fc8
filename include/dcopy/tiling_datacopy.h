/*
 * DataCopyTiling: the tiling contract of the standalone datacopy kernels.
 *
 * Byte-identical to the reference struct (standalone_datacopy/tiling_datacopy.h:7-13):
 * five little-endian uint32 fields, 20 bytes, no padding.  A caller that fills
 * these fields the way the reference host does (datacopy_data_collection.asc:108-121)
 * gets the same output bytes from this library.
 *
 *   A[rows, cols] int32 -> B[cols, rows]; tiles cover the whole rows axis.
 *   rows % 8 == 0 keeps every output row 32-byte aligned.
 */
#ifndef DCOPY_TILING_DATACOPY_H_
#define DCOPY_TILING_DATACOPY_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct DataCopyTiling {
  uint32_t rows;       /* A rows (M); 8..4088, multiple of 8 */
  uint32_t cols;       /* A cols (N); 1..65535 */
  uint32_t tile_cols;  /* columns of A per tile; 1..cols */
  uint32_t ub_bytes;   /* tile_cols * rows * 4 (the reference's UB buffer size) */
  uint32_t store;      /* 1: write the tile to the output; 0: load only */
} DataCopyTiling;

#ifdef __cplusplus
}  /* extern "C" */
static_assert(sizeof(DataCopyTiling) == 20, "DataCopyTiling must stay 20 bytes");
#else
_Static_assert(sizeof(DataCopyTiling) == 20, "DataCopyTiling must stay 20 bytes");
#endif

#endif  /* DCOPY_TILING_DATACOPY_H_ */
