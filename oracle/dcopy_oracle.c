/*
 * dcopy oracle -- TEST INFRASTRUCTURE ONLY (see dcopy_oracle.h).
 *
 * Plain C restatement of the reference algorithms; every function cites the
 * reference file:line it follows.  Nothing here is optimised beyond splitting
 * independent work over pthreads for the timed CPU baseline.
 */
#include "dcopy_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* standalone_datacopy                                                        */
/* ------------------------------------------------------------------------ */

/* datacopy_data_collection.asc:115-123 (host validation + plan), with the
 * same limits as profile.py:88-99 (rows 8..4088 %8, cols 1..65535,
 * tile 1..240 KiB, input <= 64 MiB, tile_cols > 0). */
int oracle_plan_tiling(uint32_t rows, uint32_t cols, uint32_t tile_kib, uint32_t store,
                       DataCopyTiling *out) {
  if (!out) return ORACLE_EPARAM;
  if (!rows || rows > 4095 || rows % 8 || !cols || cols > 65535 || !tile_kib || tile_kib > 240 ||
      store > 1)
    return ORACLE_EPARAM;
  uint32_t tile_cols = tile_kib * 1024u / (rows * 4u);
  if (tile_cols > cols) tile_cols = cols;
  if (!tile_cols) return ORACLE_EPARAM;
  const uint64_t bytes = (uint64_t)rows * cols * 4u;
  if (bytes > 64ull * 1024 * 1024) return ORACLE_EPARAM;
  out->rows = rows;
  out->cols = cols;
  out->tile_cols = tile_cols;
  out->ub_bytes = tile_cols * rows * 4u;
  out->store = store;
  return ORACLE_OK;
}

int oracle_check_tiling(const DataCopyTiling *t) {
  if (!t) return ORACLE_EPARAM;
  if (!t->rows || t->rows > 4095 || t->rows % 8 || !t->cols || t->cols > 65535 || t->store > 1)
    return ORACLE_EPARAM;
  if (!t->tile_cols || t->tile_cols > t->cols) return ORACLE_EPARAM; /* c0 += 0 never ends */
  if ((uint64_t)t->tile_cols * t->rows * 4u > t->ub_bytes) return ORACLE_EPARAM; /* UB overflow */
  if (t->ub_bytes > 240u * 1024u) return ORACLE_EPARAM;                          /* UB budget */
  if ((uint64_t)t->rows * t->cols * 4u > 64ull * 1024 * 1024) return ORACLE_EPARAM;
  return ORACLE_OK;
}

/* RunTiles<phase>, datacopy_data_collection.asc:16-62.
 *  - phase 0/1: per column c of the tile, DataCopyPad<Compact> with
 *    {blockCount=rows, blockLen=4, srcStride=(cols-1)*4} from gm[c0+c] into
 *    ub[c*rows] (:32-35, :45-48); the byte address of block `b` is
 *    (c0+c)*4 + b*(4 + (cols-1)*4)  (test_address_model.py:24).
 *  - phase 2: one linear burst of count*rows*4 bytes from gm[c0*rows] (:41-43).
 *  - store when phase == 1 or t->store: ub -> out[c0*rows], linear (:52-59). */
int oracle_run_tiles(int phase, const void *input, void *output, const DataCopyTiling *t) {
  int rc = oracle_check_tiling(t);
  if (rc) return rc;
  if (phase < 0 || phase > 2 || !input) return ORACLE_EPARAM;
  if ((phase == 1 || t->store) && !output) return ORACLE_EPARAM;
  const uint64_t rows = t->rows, cols = t->cols, tile_cols = t->tile_cols;
  uint8_t *ub = (uint8_t *)malloc(t->ub_bytes);
  if (!ub) return ORACLE_EPARAM;
  const uint8_t *gm = (const uint8_t *)input;
  uint8_t *out = (uint8_t *)output;
  for (uint64_t c0 = 0; c0 < cols; c0 += tile_cols) {
    const uint64_t count = (cols - c0 < tile_cols) ? cols - c0 : tile_cols;
    const uint64_t linear_len = count * rows * 4u;
    if (phase == 2) {
      memcpy(ub, gm + c0 * rows * 4u, linear_len);
    } else {
      for (uint64_t c = 0; c < count; ++c) {
        const uint64_t base = (c0 + c) * 4u;
        for (uint64_t block = 0; block < rows; ++block) {
          const uint64_t source_byte = base + block * (4u + (cols - 1u) * 4u);
          memcpy(ub + (c * rows + block) * 4u, gm + source_byte, 4u);
        }
      }
    }
    if (phase == 1 || t->store) memcpy(out + c0 * rows * 4u, ub, linear_len);
  }
  free(ub);
  return ORACLE_OK;
}

void oracle_fill_pattern(int32_t *dst, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) dst[i] = (int32_t)(uint32_t)(i * 17u + 3u);
}

/* ------------------------------------------------------------------------ */
/* DataCopyExt gap copy                                                       */
/* ------------------------------------------------------------------------ */

void oracle_copy_ext(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                     uint64_t src_gap, uint64_t dst_gap) {
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  const uint64_t sp = block_len + src_gap, dp = block_len + dst_gap;
  for (uint64_t i = 0; i < block_count; ++i) memcpy(d + i * dp, s + i * sp, block_len);
}

void oracle_copy_ext_loop(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                          uint64_t src_gap, uint64_t dst_gap, uint64_t loop1_size,
                          uint64_t loop2_size, uint64_t loop1_src, uint64_t loop1_dst,
                          uint64_t loop2_src, uint64_t loop2_dst) {
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  for (uint64_t i = 0; i < loop2_size; ++i)
    for (uint64_t j = 0; j < loop1_size; ++j)
      oracle_copy_ext(d + i * loop2_dst + j * loop1_dst, s + i * loop2_src + j * loop1_src,
                      block_count, block_len, src_gap, dst_gap);
}

/* ------------------------------------------------------------------------ */
/* DataCopyPad with the UB-side conventions (ascendc/api/datacopy.h:14-40;    */
/* v35/ascendc/api_regbase/datacopy.h:14-72)                                  */
/* ------------------------------------------------------------------------ */

static uint64_t round_up32(uint64_t x) { return (x + 31) / 32 * 32; }

/* Bytes block i's UB slot occupies before the stride gap. */
static uint64_t pad_slot(uint64_t block_len, int mode, uint32_t left, uint32_t right,
                         uint32_t eb) {
  const uint64_t used = (uint64_t)left * eb + block_len + (uint64_t)right * eb;
  return mode == 0 ? round_up32(used) : used;
}

uint64_t oracle_pad_ub_span(uint64_t block_count, uint64_t block_len, uint64_t ub_blocks, int mode,
                            uint32_t left, uint32_t right, uint32_t eb) {
  if (!block_count) return 0;
  const uint64_t slot = pad_slot(block_len, mode, left, right, eb);
  const uint64_t end = (block_count - 1) * (slot + ub_blocks * 32) + slot;
  return mode == 0 ? end : round_up32(end);
}

int oracle_copy_pad_gm_to_ub(void *ub, const void *gm, uint64_t block_count, uint64_t block_len,
                             uint64_t src_gap, uint64_t dst_blocks, int mode, int is_pad,
                             uint32_t left, uint32_t right, uint64_t value, uint32_t eb) {
  if ((eb != 1 && eb != 2 && eb != 4 && eb != 8) || block_len % eb || (uint64_t)left * eb > 32 ||
      (uint64_t)right * eb > 32 || (mode != 0 && mode != 1))
    return ORACLE_EPARAM;
  const uint8_t *s = (const uint8_t *)gm;
  uint8_t *d = (uint8_t *)ub;
  const uint64_t slot = pad_slot(block_len, mode, left, right, eb);
  const uint64_t ub_pitch = slot + dst_blocks * 32, lead = (uint64_t)left * eb;
  for (uint64_t i = 0; i < block_count; ++i) {
    uint8_t *b = d + i * ub_pitch;
    memcpy(b + lead, s + i * (block_len + src_gap), block_len);
    if (is_pad) /* the element-aligned padding positions of the slot hold `value` */
      for (uint64_t o = 0; o < slot; ++o)
        if (o < lead || o >= lead + block_len) b[o] = (uint8_t)(value >> (8 * (o % eb)));
  }
  if (mode == 1 && is_pad && block_count) { /* Compact: round the whole transfer up to 32 B */
    const uint64_t end = (block_count - 1) * ub_pitch + slot;
    for (uint64_t o = end; o < round_up32(end); ++o) d[o] = (uint8_t)(value >> (8 * (o % eb)));
  }
  return ORACLE_OK;
}

int oracle_copy_pad_ub_to_gm(void *gm, const void *ub, uint64_t block_count, uint64_t block_len,
                             uint64_t src_blocks, uint64_t dst_gap, int mode) {
  if (mode != 0 && mode != 1) return ORACLE_EPARAM;
  const uint8_t *s = (const uint8_t *)ub;
  uint8_t *d = (uint8_t *)gm;
  const uint64_t ub_pitch = pad_slot(block_len, mode, 0, 0, 1) + src_blocks * 32;
  for (uint64_t i = 0; i < block_count; ++i)
    memcpy(d + i * (block_len + dst_gap), s + i * ub_pitch, block_len);
  return ORACLE_OK;
}

typedef struct {
  uint8_t *dst;
  const uint8_t *src;
  uint64_t b0, b1, block_len, sp, dp;
} ext_job;

static void *ext_worker(void *arg) {
  ext_job *j = (ext_job *)arg;
  for (uint64_t i = j->b0; i < j->b1; ++i)
    memcpy(j->dst + i * j->dp, j->src + i * j->sp, j->block_len);
  return NULL;
}

int oracle_copy_ext_mt(void *dst, const void *src, uint64_t block_count, uint64_t block_len,
                       uint64_t src_gap, uint64_t dst_gap, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  ext_job jobs[256];
  const uint64_t per = (block_count + nthreads - 1) / nthreads;
  int started = 0;
  for (int k = 0; k < nthreads; ++k) {
    uint64_t b0 = (uint64_t)k * per, b1 = b0 + per;
    if (b0 >= block_count) break;
    if (b1 > block_count) b1 = block_count;
    jobs[k] = (ext_job){(uint8_t *)dst, (const uint8_t *)src, b0, b1, block_len,
                        block_len + src_gap, block_len + dst_gap};
    if (pthread_create(&th[k], NULL, ext_worker, &jobs[k]) != 0) {
      ext_worker(&jobs[k]);
      th[k] = 0;
    }
    started = k + 1;
  }
  for (int k = 0; k < started; ++k)
    if (th[k]) pthread_join(th[k], NULL);
  return ORACLE_OK;
}

/* DataCopyNddma: loop sizes and per-dimension src/dst strides
 * (datacopy_nddma.h:18-23 fills loopSize/loopSrcStride/loopDstStride from
 * output_dims/input_stride/output_stride, innermost first).  The arrays here
 * are outermost-first like output_dims.  Elements are moved bit-exactly. */
int oracle_copy_nd(void *dst, const void *src, int ndim, const uint64_t *sizes,
                   const int64_t *src_strides, const int64_t *dst_strides, uint32_t elem_bytes) {
  if (ndim < 1 || ndim > 8 || !elem_bytes || !sizes || !src_strides || !dst_strides)
    return ORACLE_EPARAM;
  uint64_t total = 1;
  for (int k = 0; k < ndim; ++k) total *= sizes[k];
  if (!total) return ORACLE_OK;
  if (!dst || !src) return ORACLE_EPARAM;
  uint64_t idx[8] = {0};
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  for (uint64_t n = 0; n < total; ++n) {
    int64_t so = 0, dof = 0;
    for (int k = 0; k < ndim; ++k) {
      so += (int64_t)idx[k] * src_strides[k];
      dof += (int64_t)idx[k] * dst_strides[k];
    }
    memcpy(d + dof * (int64_t)elem_bytes, s + so * (int64_t)elem_bytes, elem_bytes);
    for (int k = ndim - 1; k >= 0; --k) {
      if (++idx[k] < sizes[k]) break;
      idx[k] = 0;
    }
  }
  return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* ND <-> FRACTAL_NZ                                                          */
/* ------------------------------------------------------------------------ */

#define KCUBE 16               /* kCubeSize, formats_definitions.h:18 */
#define KSHAPE_MAX 1099511627776LL /* kShapeItemNumMAX, formats_definitions.h:20 */

/* Ceil, formats_trans_utils.h:69-74. */
static int64_t ge_ceil(int64_t n1, int64_t n2) {
  if (n1 == 0) return 0;
  return (n2 != 0) ? (((n1 - 1) / n2) + 1) : 0;
}

/* IsShapeValid, formats_trans_utils.cc:88-107. */
static int shape_valid(const int64_t *shape, int rank) {
  if (rank <= 0) return 0;
  int64_t num = 1;
  for (int i = 0; i < rank; ++i) {
    const int64_t dim = shape[i];
    if (dim < 0) return 0;
    if (dim != 0 && (KSHAPE_MAX / dim) < num) return 0;
    num *= dim;
  }
  return 1;
}

/* TransShapeToFracNz, format_transfer_fractal_nz.cc:65-111. */
int oracle_nz_shape(const int64_t *src, int rank, int64_t w0, int64_t *dst, int *dst_rank,
                    int64_t *hw) {
  if (!src || !dst || !dst_rank || !hw || rank <= 0) return ORACLE_ESHAPE;
  int n = 0;
  if (rank == 1) {
    dst[n++] = ge_ceil(src[0], w0);
    dst[n++] = 1;
    dst[n++] = KCUBE;
    dst[n++] = w0;
    hw[0] = 1;
    hw[1] = 1;
    hw[2] = src[0];
  } else {
    int64_t times = 1;
    for (int i = 0; i < rank - 2; ++i) {
      dst[n++] = src[i];
      times *= src[i];
    }
    dst[n++] = ge_ceil(src[rank - 1], w0);
    dst[n++] = ge_ceil(src[rank - 2], KCUBE);
    dst[n++] = KCUBE;
    dst[n++] = w0;
    hw[0] = times;
    hw[1] = src[rank - 2];
    hw[2] = src[rank - 1];
  }
  *dst_rank = n;
  return shape_valid(dst, n) ? ORACLE_OK : ORACLE_ESHAPE;
}

/* TransShapeToFracZz, format_transfer_fractal_zz.cc:74-118. */
int oracle_zz_shape(const int64_t *src, int rank, int64_t c0, int64_t *dst, int *dst_rank,
                    int64_t *hw) {
  if (!src || !dst || !dst_rank || !hw || rank <= 0) return ORACLE_ESHAPE;
  int n = 0;
  if (rank == 1) {
    dst[n++] = 1;
    dst[n++] = ge_ceil(src[0], c0);
    dst[n++] = c0;
    dst[n++] = c0;
    hw[0] = 1;
    hw[1] = 1;
    hw[2] = src[0];
  } else {
    int64_t times = 1;
    for (int i = 0; i < rank - 2; ++i) {
      dst[n++] = src[i];
      times *= src[i];
    }
    dst[n++] = ge_ceil(src[rank - 2], c0);
    dst[n++] = ge_ceil(src[rank - 1], c0);
    dst[n++] = c0;
    dst[n++] = c0;
    hw[0] = times;
    hw[1] = src[rank - 2];
    hw[2] = src[rank - 1];
  }
  *dst_rank = n;
  return shape_valid(dst, n) ? ORACLE_OK : ORACLE_ESHAPE;
}

/* One job of the FRACTAL_NZ / FRACTAL_ZZ copy loops over ND rows [r0, r1) of
 * times*H.  ND row hi of batch t starts, in the tiled buffer, at
 *   t*batch + (hi / band_rows)*band_stride + (hi % band_rows)*w0
 * and its column block w1 sits `panel` elements further per block:
 *   NZ: band_rows >= H (no bands; rows of a panel are adjacent), panel = H1*16*w0;
 *   ZZ: band_rows = h0, band_stride = W1*h0*w0, panel = h0*w0. */
typedef struct {
  uint8_t *dst;
  const uint8_t *src;
  int64_t r0, r1;
  int64_t h, w, size, w0, panel, batch, band_rows, band_stride, num_w1;
  int to_frac;
} frac_job;

/* The hot loops of TransFormatFromNdToFracNz (fractal_nz.cc:168-209),
 * TransFormatFromFracNzToNd (:251-294), TransFormatFromNdToFracZz
 * (fractal_zz.cc:176-230) and TransFormatFromFracZzToNd (:275-328):
 * whole W0-element runs for the full column blocks, then the W tail
 * element by element. */
static void *frac_worker(void *arg) {
  const frac_job *j = (const frac_job *)arg;
  const int64_t size = j->size, w0 = j->w0;
  for (int64_t r = j->r0; r < j->r1; ++r) {
    const int64_t t = r / j->h, hi = r % j->h;
    const int64_t fr_h_head =
        t * j->batch + (hi / j->band_rows) * j->band_stride + (hi % j->band_rows) * w0;
    const int64_t nd_h_head = t * j->h * j->w + hi * j->w;
    for (int64_t w1i = 0; w1i < j->num_w1; ++w1i) {
      const int64_t fr_off = (fr_h_head + w1i * j->panel) * size;
      const int64_t nd_off = (nd_h_head + w1i * w0) * size;
      if (j->to_frac)
        memcpy(j->dst + fr_off, j->src + nd_off, (size_t)(size * w0));
      else
        memcpy(j->dst + nd_off, j->src + fr_off, (size_t)(size * w0));
    }
    const int64_t w1_head = j->num_w1 * w0;
    for (int64_t w0i = 0; w1_head + w0i < j->w; ++w0i) {
      const int64_t fr_off = (fr_h_head + j->num_w1 * j->panel + w0i) * size;
      const int64_t nd_off = (nd_h_head + w1_head + w0i) * size;
      if (j->to_frac)
        memcpy(j->dst + fr_off, j->src + nd_off, (size_t)size);
      else
        memcpy(j->dst + nd_off, j->src + fr_off, (size_t)size);
    }
  }
  return NULL;
}

typedef struct {
  uint8_t *p;
  size_t n;
} zero_job;

static void *zero_worker(void *arg) {
  zero_job *z = (zero_job *)arg;
  memset(z->p, 0, z->n);
  return NULL;
}

static int frac_run(int zz, void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t w0, int to_nz, int nthreads) {
  /* IsDataTypeSupportForTransShapeToFracNz (fractal_nz.cc:36),
   * CheckDataTypeSupportForFractalZz (fractal_zz.cc:45). */
  if (elem_bytes <= 0) return ORACLE_EDTYPE;
  if (!shape_valid(nd_shape, rank)) return ORACLE_ESHAPE;
  /* The tiled -> ND loops divide by w0 (fractal_nz.cc:249, fractal_zz.cc:273);
   * a C0 of 0 never comes out of a format's C0 bits. */
  if (!to_nz && w0 <= 0) return ORACLE_ESHAPE;
  int64_t nz[16], hw[3];
  int nz_rank = 0;
  if (rank > 14) return ORACLE_ESHAPE;
  int rc = zz ? oracle_zz_shape(nd_shape, rank, w0, nz, &nz_rank, hw)
              : oracle_nz_shape(nd_shape, rank, w0, nz, &nz_rank, hw);
  if (rc) return rc;
  int64_t nz_items = 1, nd_items = 1;
  for (int i = 0; i < nz_rank; ++i) nz_items *= nz[i];
  for (int i = 0; i < rank; ++i) nd_items *= nd_shape[i];
  const int64_t dst_size = (to_nz ? nz_items : nd_items) * elem_bytes;
  if (dst_size == 0) return ORACLE_OK;
  if (!dst || !src) return ORACLE_EPARAM;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  if (to_nz) { /* new uint8_t[dst_size]() zero-initialises the padding (fractal_nz.cc:139,
                 fractal_zz.cc:148) */
    zero_job zj[256];
    const size_t per = ((size_t)dst_size + nthreads - 1) / nthreads;
    int started = 0;
    for (int k = 0; k < nthreads; ++k) {
      size_t b0 = (size_t)k * per;
      if (b0 >= (size_t)dst_size) break;
      size_t n = per;
      if (b0 + n > (size_t)dst_size) n = (size_t)dst_size - b0;
      zj[k] = (zero_job){(uint8_t *)dst + b0, n};
      if (nthreads == 1 || pthread_create(&th[k], NULL, zero_worker, &zj[k]) != 0) {
        zero_worker(&zj[k]);
        th[k] = 0;
      }
      started = k + 1;
    }
    for (int k = 0; k < started; ++k)
      if (th[k]) pthread_join(th[k], NULL);
  }
  const int64_t h0 = nz[nz_rank - 2];
  const int64_t w1 = zz ? nz[nz_rank - 3] : nz[nz_rank - 4];
  const int64_t h1 = zz ? nz[nz_rank - 4] : nz[nz_rank - 3];
  const int64_t block = h0 * w0;
  const int64_t rows = hw[0] * hw[1];
  if (rows == 0) return ORACLE_OK;
  frac_job base = {(uint8_t *)dst, (const uint8_t *)src, 0, 0, hw[1], hw[2], elem_bytes, w0,
                   zz ? block : h1 * block,          /* panel */
                   h1 * w1 * block,                   /* batch */
                   zz ? h0 : h1 * h0,                 /* band_rows */
                   zz ? w1 * block : 0,               /* band_stride */
                   hw[2] / w0, to_nz};
  frac_job jobs[256];
  const int64_t per = (rows + nthreads - 1) / nthreads;
  int started = 0;
  for (int k = 0; k < nthreads; ++k) {
    int64_t r0 = (int64_t)k * per, r1 = r0 + per;
    if (r0 >= rows) break;
    if (r1 > rows) r1 = rows;
    jobs[k] = base;
    jobs[k].r0 = r0;
    jobs[k].r1 = r1;
    if (nthreads == 1 || pthread_create(&th[k], NULL, frac_worker, &jobs[k]) != 0) {
      frac_worker(&jobs[k]);
      th[k] = 0;
    }
    started = k + 1;
  }
  for (int k = 0; k < started; ++k)
    if (th[k]) pthread_join(th[k], NULL);
  return ORACLE_OK;
}

int oracle_nd_to_nz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t w0) {
  return frac_run(0, dst, src, nd_shape, rank, elem_bytes, w0, 1, 1);
}

int oracle_nz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t w0) {
  return frac_run(0, dst, src, nd_shape, rank, elem_bytes, w0, 0, 1);
}

int oracle_nd_to_nz_mt(void *dst, const void *src, const int64_t *nd_shape, int rank,
                       int elem_bytes, int64_t w0, int nthreads) {
  return frac_run(0, dst, src, nd_shape, rank, elem_bytes, w0, 1, nthreads);
}

int oracle_nz_to_nd_mt(void *dst, const void *src, const int64_t *nd_shape, int rank,
                       int elem_bytes, int64_t w0, int nthreads) {
  return frac_run(0, dst, src, nd_shape, rank, elem_bytes, w0, 0, nthreads);
}

int oracle_nd_to_zz(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t c0) {
  return frac_run(1, dst, src, nd_shape, rank, elem_bytes, c0, 1, 1);
}

int oracle_zz_to_nd(void *dst, const void *src, const int64_t *nd_shape, int rank,
                    int elem_bytes, int64_t c0) {
  return frac_run(1, dst, src, nd_shape, rank, elem_bytes, c0, 0, 1);
}

/* ------------------------------------------------------------------------ */
/* N-D transpose                                                              */
/* ------------------------------------------------------------------------ */

/* Transpose, format_transfer_transpose.cc:142-197, with the argument checks of
 * IsTransposeArgValid / IsShapeArgValid (:45-92): every failure there makes
 * Transpose return ACL_ERROR_GE_PARAM_INVALID (:144-145). */
int oracle_transpose(void *dst, const void *src, const int64_t *src_shape, const int64_t *perm,
                     int rank, int elem_bytes) {
  if (!src || elem_bytes < 0 || rank <= 0 || rank > 16 || !src_shape || !perm)
    return ORACLE_EPARAM;
  int seen[16] = {0};
  for (int i = 0; i < rank; ++i) {
    if (src_shape[i] < 0) return ORACLE_EPARAM;
    if (perm[i] < 0 || perm[i] >= rank || seen[perm[i]]) return ORACLE_EPARAM;
    seen[perm[i]] = 1;
  }
  int64_t heads[16], dst_shape[16], src_heads[16], idx[16] = {0};
  for (int i = rank - 1; i >= 0; --i) /* GenHeads, :94-108 */
    heads[i] = (i == rank - 1) ? 1 : src_shape[i + 1] * heads[i + 1];
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) { /* TransShapeByPerm, :133-139 */
    dst_shape[i] = src_shape[perm[i]];
    src_heads[i] = heads[perm[i]];
    n *= dst_shape[i];
  }
  if (n == 0) return ORACLE_OK;
  if (!dst) return ORACLE_EPARAM;
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  for (int64_t di = 0; di < n; ++di) {
    int64_t off = 0; /* GenOffset, :110-116 */
    for (int k = 0; k < rank; ++k) off += src_heads[k] * idx[k];
    memcpy(d + di * elem_bytes, s + off * elem_bytes, (size_t)elem_bytes);
    int k = rank - 1; /* AddOne, :118-131 */
    idx[k] += 1;
    while (k > 0 && idx[k] >= dst_shape[k]) {
      idx[k] = 0;
      idx[--k] += 1;
    }
  }
  return ORACLE_OK;
}
