"""ctypes binding of the C oracle (dcopy_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
use this module, as the checker or as the timed CPU restatement of the
reference.  The product library never imports it.

Arrays are numpy arrays (C-contiguous); the functions work on raw bytes, so any
dtype moves bit-exactly.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

OK, EPARAM, ESHAPE, EDTYPE, EFORMAT, EFAILED = 0, -1, -2, -3, -4, -8


class Tiling(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32),
                ("tile_cols", ctypes.c_uint32), ("ub_bytes", ctypes.c_uint32),
                ("store", ctypes.c_uint32)]


_lib = None
_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)
_u64p = ctypes.POINTER(ctypes.c_uint64)


def build() -> str:
    """Compile liboracle.so with make (a no-op when it is up to date)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        h = ctypes.CDLL(LIB_PATH)
        sig = {
            "oracle_plan_tiling": [ctypes.c_uint32] * 4 + [ctypes.POINTER(Tiling)],
            "oracle_check_tiling": [ctypes.POINTER(Tiling)],
            "oracle_run_tiles": [ctypes.c_int, _vp, _vp, ctypes.POINTER(Tiling)],
            "oracle_fill_pattern": [_vp, ctypes.c_uint64],
            "oracle_copy_ext": [_vp, _vp] + [ctypes.c_uint64] * 4,
            "oracle_copy_ext_loop": [_vp, _vp] + [ctypes.c_uint64] * 10,
            "oracle_copy_ext_mt": [_vp, _vp] + [ctypes.c_uint64] * 4 + [ctypes.c_int],
            "oracle_copy_nd": [_vp, _vp, ctypes.c_int, _u64p, _i64p, _i64p, ctypes.c_uint32],
            "oracle_copy_pad_gm_to_ub": [_vp, _vp] + [ctypes.c_uint64] * 4 +
                                        [ctypes.c_int, ctypes.c_int, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32],
            "oracle_copy_pad_ub_to_gm": [_vp, _vp] + [ctypes.c_uint64] * 4 + [ctypes.c_int],
            "oracle_pad_ub_span": [ctypes.c_uint64] * 3 + [ctypes.c_int] + [ctypes.c_uint32] * 3,
            "oracle_nz_shape": [_i64p, ctypes.c_int, ctypes.c_int64, _i64p,
                                ctypes.POINTER(ctypes.c_int), _i64p],
            "oracle_nd_to_nz": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64],
            "oracle_fz_shape": [ctypes.c_int, _i64p, ctypes.c_int, ctypes.c_int64,
                                ctypes.c_int64, _i64p, ctypes.POINTER(ctypes.c_int)],
            "oracle_to_fz": [_vp, _vp, ctypes.c_int, _i64p, ctypes.c_int, ctypes.c_int,
                             ctypes.c_int64, ctypes.c_int64, _i64p],
            "oracle_from_fz_check": [_i64p, ctypes.c_int, ctypes.c_int, _i64p, ctypes.c_int,
                                     ctypes.c_int64],
            "oracle_from_fz": [_vp, _vp, ctypes.c_int, _i64p, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int64],
            "oracle_zz_shape": [_i64p, ctypes.c_int, ctypes.c_int64, _i64p,
                                ctypes.POINTER(ctypes.c_int), _i64p],
            "oracle_nd_to_zz": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64],
            "oracle_zz_to_nd": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64],
            "oracle_nz_to_nd": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64],
            "oracle_nd_to_nz_mt": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                   ctypes.c_int],
            "oracle_nz_to_nd_mt": [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                   ctypes.c_int],
            "oracle_transpose": [_vp, _vp, _i64p, _i64p, ctypes.c_int, ctypes.c_int],
        }
        for name, args in sig.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = (None if name in ("oracle_fill_pattern", "oracle_copy_ext",
                                           "oracle_copy_ext_loop") else
                          ctypes.c_uint64 if name == "oracle_pad_ub_span" else ctypes.c_int)
        _lib = h
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _i64(vals: Sequence[int]):
    return (ctypes.c_int64 * max(len(vals), 1))(*vals)


def plan_tiling(rows, cols, kib, store=1):
    t = Tiling()
    rc = lib().oracle_plan_tiling(rows, cols, kib, store, ctypes.byref(t))
    return rc, t


def check_tiling(t: Tiling) -> int:
    return lib().oracle_check_tiling(ctypes.byref(t))


def run_tiles(phase: int, inp: np.ndarray, out, t: Tiling) -> int:
    return lib().oracle_run_tiles(phase, _p(inp), _p(out), ctypes.byref(t))


def fill_pattern(n: int) -> np.ndarray:
    a = np.empty(n, dtype=np.int32)
    lib().oracle_fill_pattern(_p(a), n)
    return a


def copy_ext(dst: np.ndarray, src: np.ndarray, count, blen, sgap=0, dgap=0, threads=1) -> None:
    if threads > 1:
        lib().oracle_copy_ext_mt(_p(dst), _p(src), count, blen, sgap, dgap, threads)
    else:
        lib().oracle_copy_ext(_p(dst), _p(src), count, blen, sgap, dgap)


def copy_ext_loop(dst: np.ndarray, src: np.ndarray, count, blen, sgap, dgap, loop1,
                  loop2=(1, 0, 0)) -> None:
    """LoopModeParams around the gap copy; loop1/loop2 = (size, src stride, dst stride) bytes."""
    lib().oracle_copy_ext_loop(_p(dst), _p(src), count, blen, sgap, dgap, loop1[0], loop2[0],
                               loop1[1], loop1[2], loop2[1], loop2[2])


def copy_pad_gm_to_ub(ub: np.ndarray, gm: np.ndarray, count, blen, src_gap, dst_blocks, mode=0,
                      pad=(True, 0, 0, 0), eb=1) -> int:
    """DataCopyPad GM -> UB; pad = DataCopyPadExtParams (is_pad, left, right, value)."""
    return lib().oracle_copy_pad_gm_to_ub(_p(ub), _p(gm), count, blen, src_gap, dst_blocks, mode,
                                          int(bool(pad[0])), pad[1], pad[2], pad[3], eb)


def copy_pad_ub_to_gm(gm: np.ndarray, ub: np.ndarray, count, blen, src_blocks, dst_gap,
                      mode=0) -> int:
    return lib().oracle_copy_pad_ub_to_gm(_p(gm), _p(ub), count, blen, src_blocks, dst_gap, mode)


def pad_ub_span(count, blen, ub_blocks, mode=0, left=0, right=0, eb=1) -> int:
    return lib().oracle_pad_ub_span(count, blen, ub_blocks, mode, left, right, eb)


def copy_nd(dst, src, sizes, src_strides, dst_strides, elem_bytes) -> int:
    n = len(sizes)
    return lib().oracle_copy_nd(_p(dst), _p(src), n, (ctypes.c_uint64 * n)(*sizes),
                                _i64(src_strides), _i64(dst_strides), elem_bytes)


def nz_shape(nd_shape: Sequence[int], w0: int):
    out = (ctypes.c_int64 * (len(nd_shape) + 4))()
    rank = ctypes.c_int(0)
    hw = (ctypes.c_int64 * 3)()
    rc = lib().oracle_nz_shape(_i64(nd_shape), len(nd_shape), w0, out, ctypes.byref(rank), hw)
    return rc, [out[i] for i in range(rank.value)], tuple(hw)


def nd_to_nz(dst, src, nd_shape, elem_bytes, w0, threads=1) -> int:
    if threads > 1:
        return lib().oracle_nd_to_nz_mt(_p(dst), _p(src), _i64(nd_shape), len(nd_shape),
                                        elem_bytes, w0, threads)
    return lib().oracle_nd_to_nz(_p(dst), _p(src), _i64(nd_shape), len(nd_shape), elem_bytes, w0)


def nz_to_nd(dst, src, nd_shape, elem_bytes, w0, threads=1) -> int:
    if threads > 1:
        return lib().oracle_nz_to_nd_mt(_p(dst), _p(src), _i64(nd_shape), len(nd_shape),
                                        elem_bytes, w0, threads)
    return lib().oracle_nz_to_nd(_p(dst), _p(src), _i64(nd_shape), len(nd_shape), elem_bytes, w0)


def zz_shape(nd_shape: Sequence[int], c0: int):
    out = (ctypes.c_int64 * (len(nd_shape) + 4))()
    rank = ctypes.c_int(0)
    hw = (ctypes.c_int64 * 3)()
    rc = lib().oracle_zz_shape(_i64(nd_shape), len(nd_shape), c0, out, ctypes.byref(rank), hw)
    return rc, [out[i] for i in range(rank.value)], tuple(hw)


def nd_to_zz(dst, src, nd_shape, elem_bytes, c0) -> int:
    return lib().oracle_nd_to_zz(_p(dst), _p(src), _i64(nd_shape), len(nd_shape), elem_bytes, c0)


def zz_to_nd(dst, src, nd_shape, elem_bytes, c0) -> int:
    return lib().oracle_zz_to_nd(_p(dst), _p(src), _i64(nd_shape), len(nd_shape), elem_bytes, c0)


# GE format enum values used by the FRACTAL_Z family.
NCHW, NHWC, ND, HWCN, FRACTAL_Z = 0, 1, 2, 16, 4


def fz_shape(src_format: int, shape: Sequence[int], c0: int, groups: int = 0):
    out = (ctypes.c_int64 * 4)()
    rank = ctypes.c_int(0)
    rc = lib().oracle_fz_shape(src_format, _i64(shape), len(shape), c0, groups, out,
                               ctypes.byref(rank))
    return rc, [out[i] for i in range(rank.value)]


def to_fz(src: np.ndarray, src_format: int, c0: int, groups: int = 0) -> np.ndarray:
    """FormatTransferFractalZ / FractalZTbe data movement (groups = the
    TransArgs dst_sub_format); returns the written elements, flat."""
    n = ctypes.c_int64(0)
    src = np.ascontiguousarray(src)
    args = (src_format, _i64(src.shape), src.ndim, src.dtype.itemsize, c0, groups,
            ctypes.byref(n))
    rc = lib().oracle_to_fz(None, _p(src), *args)  # sizing call: nothing written
    if rc:
        raise ValueError(f"to_fz rc={rc}")
    out = np.empty(max(n.value, 1), dtype=src.dtype)
    rc = lib().oracle_to_fz(_p(out), _p(src), *args)
    if rc:
        raise ValueError(f"to_fz rc={rc}")
    return out[:n.value]


def from_fz_check(src_shape, dst_format, dst_shape, c0) -> int:
    return lib().oracle_from_fz_check(_i64(src_shape), len(src_shape), dst_format,
                                      _i64(dst_shape), len(dst_shape), c0)


def from_fz(src: np.ndarray, dst_format: int, dst_shape, c0: int) -> np.ndarray:
    out = np.empty(dst_shape, dtype=src.dtype)
    rc = lib().oracle_from_fz(_p(out), _p(np.ascontiguousarray(src)), dst_format,
                              _i64(dst_shape), len(dst_shape), src.dtype.itemsize, c0)
    if rc:
        raise ValueError(f"from_fz rc={rc}")
    return out


def transpose(dst, src, src_shape, perm, elem_bytes) -> int:
    if len(perm) != len(src_shape):
        raise ValueError("perm and src_shape must have the same rank")
    return lib().oracle_transpose(_p(dst), _p(src), _i64(src_shape), _i64(perm), len(src_shape),
                                  elem_bytes)


# ---- convenience wrappers returning new arrays -------------------------------------

def nd_to_nz_array(src: np.ndarray, w0: int, threads: int = 1) -> np.ndarray:
    rc, nz, _ = nz_shape(src.shape, w0)
    if rc:
        raise ValueError(f"nz_shape rc={rc}")
    out = np.empty(nz, dtype=src.dtype)
    rc = nd_to_nz(out, np.ascontiguousarray(src), src.shape, src.dtype.itemsize, w0, threads)
    if rc:
        raise ValueError(f"nd_to_nz rc={rc}")
    return out


def nz_to_nd_array(src: np.ndarray, nd_shape, w0: int, threads: int = 1) -> np.ndarray:
    out = np.empty(nd_shape, dtype=src.dtype)
    rc = nz_to_nd(out, np.ascontiguousarray(src), nd_shape, src.dtype.itemsize, w0, threads)
    if rc:
        raise ValueError(f"nz_to_nd rc={rc}")
    return out


def nd_to_zz_array(src: np.ndarray, c0: int) -> np.ndarray:
    rc, zz, _ = zz_shape(src.shape, c0)
    if rc:
        raise ValueError(f"zz_shape rc={rc}")
    out = np.empty(zz, dtype=src.dtype)
    rc = nd_to_zz(out, np.ascontiguousarray(src), src.shape, src.dtype.itemsize, c0)
    if rc:
        raise ValueError(f"nd_to_zz rc={rc}")
    return out


def zz_to_nd_array(src: np.ndarray, nd_shape, c0: int) -> np.ndarray:
    out = np.empty(nd_shape, dtype=src.dtype)
    rc = zz_to_nd(out, np.ascontiguousarray(src), nd_shape, src.dtype.itemsize, c0)
    if rc:
        raise ValueError(f"zz_to_nd rc={rc}")
    return out


def transpose_rows_cols(a: np.ndarray) -> np.ndarray:
    """RunTiles small/large output for A[rows, cols] int32 with store=1, via the tile model."""
    rows, cols = a.shape
    rc, t = plan_tiling(rows, cols, 240, 1)
    if rc:
        raise ValueError(f"plan_tiling rc={rc}")
    out = np.empty((cols, rows), dtype=np.int32)
    rc = run_tiles(0, np.ascontiguousarray(a), out, t)
    if rc:
        raise ValueError(f"run_tiles rc={rc}")
    return out
