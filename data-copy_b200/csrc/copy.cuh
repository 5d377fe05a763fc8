// Copy primitives shared by the entry points (copy.cu implements them).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcopy {

// dst[0, bytes) = src[0, bytes); any alignment.
int copy_linear(void *dst, const void *src, uint64_t bytes, cudaStream_t s);
// Reads src[0, bytes) and discards it (load-only timing modes).
int load_linear(const void *src, uint64_t bytes, cudaStream_t s);
// rows bursts of row_bytes: src + r*src_pitch -> dst + r*dst_pitch.
int copy2d(void *dst, const void *src, uint64_t rows, uint64_t row_bytes, uint64_t src_pitch,
           uint64_t dst_pitch, cudaStream_t s);

}  // namespace dcopy
