// Shared host/device helpers for libdcopy: status reporting, buffer checks,
// invariant-divisor division and the sm_100a global-memory access helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dcopy/dcopy.h"

namespace dcopy {

// ---- status -----------------------------------------------------------------

// Records `code` and a printf-style message in the calling thread's error slot
// and returns `code`.
int set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// Clears the calling thread's error slot; every entry point starts with it.
void clear_error();
// Turns a failed CUDA runtime call into DCOPY_ERR_CUDA with its name and text.
int cuda_fail(cudaError_t err, const char *what);
// Checks the launch that was just issued (cudaGetLastError).
int check_launch(const char *kernel);

// ---- buffers ----------------------------------------------------------------

// Refuses `ptr` unless [ptr, ptr+bytes) lies inside one device allocation that
// the current device can address (device memory, managed memory or a peer /
// IPC mapping).  bytes == 0 only checks nothing.  Disabled when the environment
// sets DCOPY_CHECK_POINTERS=0.
int check_device_span(const void *ptr, uint64_t bytes, const char *name);
// True when ptr is device memory of the current device (not a peer's, not an
// IPC mapping opened through dcopy_ipc_open_handle, not host memory).  Kernels
// L2-prefetch only such sources: a prefetch of another GPU's memory stalls the
// copy (measured 100x).
bool is_local_device_memory(const void *ptr);
// Records (opened) or forgets (!opened) the IPC mapping that starts at base;
// in_ipc_mapping tells whether ptr lies in a recorded one.
void note_ipc_mapping(const void *base, bool opened);
bool in_ipc_mapping(const void *ptr);
// Start address of the allocation holding ptr (0 when it cannot be determined).
uint64_t allocation_base(const void *ptr);
// 0 when the byte ranges [a, a+an) and [b, b+bn) are disjoint, else PARAM_INVALID.
int check_disjoint(const void *a, uint64_t an, const void *b, uint64_t bn, const char *what);
// Bytes spanned by `count` (>= 1) blocks of `len` bytes, `pitch` bytes apart:
// (count - 1) * pitch + len, computed without wrapping.  0 (OK) with *span set,
// or PARAM_INVALID (`what` in the message) when the span reaches 2^62 bytes.
int block_span(uint64_t count, uint64_t pitch, uint64_t len, uint64_t *span, const char *what);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();
// Ordinal of the current device.
int current_device();

// ---- invariant division ---------------------------------------------------------
// Unsigned 32-bit division by a run-time invariant divisor with one multiply-high,
// following Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication" (PLDI 1994), Figure 4.1: for 1 <= d < 2^32,
//   l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
//   q = (t + ((n - t) >> min(l,1))) >> max(l-1, 0),  t = mulhi(m, n).
struct FastDiv {
  uint32_t d = 1, m = 0, s1 = 0, s2 = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) : d(divisor) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < divisor) ++l;
    m = (uint32_t)((((1ull << l) - divisor) << 32) / divisor + 1);
    s1 = l < 1 ? l : 1;
    s2 = l > 1 ? l - 1 : 0;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    const uint32_t t = __umulhi(m, n);
    return (t + ((n - t) >> s1)) >> s2;
  }
};

// ---- global memory access (sm_100a) -------------------------------------------
// Source reads go through the non-coherent path without allocating in L1: every
// byte is read once.  Writes use the default write-back policy.

template <typename T>
__device__ __forceinline__ T ld_stream(const T *p);

template <>
__device__ __forceinline__ uint4 ld_stream<uint4>(const uint4 *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint2 ld_stream<uint2>(const uint2 *p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint32_t ld_stream<uint32_t>(const uint32_t *p) {
  uint32_t v;
  asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint16_t ld_stream<uint16_t>(const uint16_t *p) {
  uint16_t v;
  asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint8_t ld_stream<uint8_t>(const uint8_t *p) {
  uint16_t v;
  asm("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (uint8_t)v;
}

// The same streaming loads with the `.L2::64B` size qualifier: the L2 fills the
// 64-byte half line the load touches instead of the whole 128-byte line.  For
// bursts that end inside a line with a gap behind them this halves the DRAM read
// (measured on B200: 32 B bursts with a 128 B gap 2648 -> 3542 GB/s, 64 B bursts
// with a 64 B gap 4443 -> 5242 GB/s); bursts of whole lines are unchanged.
template <typename T>
__device__ __forceinline__ T ld_stream_half_line(const T *p);

template <>
__device__ __forceinline__ uint4 ld_stream_half_line<uint4>(const uint4 *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::64B.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint2 ld_stream_half_line<uint2>(const uint2 *p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.L2::64B.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint32_t ld_stream_half_line<uint32_t>(const uint32_t *p) {
  uint32_t v;
  asm("ld.global.nc.L1::no_allocate.L2::64B.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint16_t ld_stream_half_line<uint16_t>(const uint16_t *p) {
  uint16_t v;
  asm("ld.global.nc.L1::no_allocate.L2::64B.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint8_t ld_stream_half_line<uint8_t>(const uint8_t *p) {
  uint16_t v;
  asm("ld.global.nc.L1::no_allocate.L2::64B.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (uint8_t)v;
}

// L2 prefetch hint for the line holding p.  Kernels issue these for their source
// before waiting on the previous kernel of the stream (programmatic dependent
// launch): a prefetch returns no data to the SM and has no effect on memory
// ordering, so it is safe even when that kernel writes the same addresses.
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// A read that the compiler must keep even though its value is unused: the
// load-only (store == 0) modes of the standalone kernels time reads alone.
__device__ __forceinline__ uint32_t ld_keep_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_keep_u8(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_keep_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace dcopy

// Entry-point boilerplate: clear the error slot, run `body`, never throw.
#define DCOPY_API_BEGIN \
  dcopy::clear_error(); \
  try {
#define DCOPY_API_END                                                          \
  }                                                                            \
  catch (...) {                                                                \
    return dcopy::set_error(DCOPY_ERR_UNSUPPORTED, "internal exception");      \
  }

#define DCOPY_CUDA_TRY(call)                                   \
  do {                                                         \
    cudaError_t _e = (call);                                   \
    if (_e != cudaSuccess) return dcopy::cuda_fail(_e, #call); \
  } while (0)
