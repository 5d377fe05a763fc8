"""dcopy: Python binding of the B200 data-movement library (libdcopy.so).

A thin ctypes layer over the C ABI declared in include/dcopy/dcopy.h.  Every
call goes to the CUDA kernels in libdcopy.so; there is no CPU implementation
behind this module, and it raises ``DcopyUnavailable`` when the library has not
been built.

Buffers may be given as CUDA ``torch.Tensor`` objects (their ``data_ptr()`` is
used) or as raw integer device addresses.  ``stream`` defaults to torch's
current CUDA stream when torch is loaded, else the legacy default stream.

Names follow the reference's host interface:
  * ``plan_tiling`` / ``datacopy_small|large|pretranspose|contiguous``
    -- standalone_datacopy/datacopy_data_collection.asc:64-123;
  * ``copy_ext`` -- AscendC::DataCopyExtParams via DataCopyPadExtend
    (compiler/graph/optimize/autofuse/ascendc/api/datacopy.h:14-40);
  * ``copy_nd`` -- DataCopyNddma (v35/ascendc/api_regbase/datacopy_nddma.h);
  * ``nz_shape`` / ``nd_to_nz`` / ``nz_to_nd`` -- TransShapeToFracNz and the
    FRACTAL_NZ transfers (base/formats/format_transfers/format_transfer_fractal_nz.cc);
  * ``zz_shape`` / ``nd_to_zz`` / ``zz_to_nd`` -- the same for FRACTAL_ZZ
    (base/formats/format_transfers/format_transfer_fractal_zz.cc).
"""
from __future__ import annotations

import ctypes
import os
import sys
from typing import Optional, Sequence

__all__ = [
    "DataCopyTiling", "DcopyExtParams", "DcopyError", "DcopyUnavailable", "lib", "lib_path",
    "plan_tiling", "datacopy_small", "datacopy_large", "datacopy_pretranspose",
    "datacopy_contiguous", "datacopy_pretranspose_noalloc", "copy_ext", "copy_ext_32b", "copy_nd", "nz_shape", "nd_to_nz",
    "DcopyPadParams", "PAD_NORMAL", "PAD_COMPACT", "copy_pad_gm_to_ub", "copy_pad_ub_to_gm",
    "datacopy_pad_extend",
    "nz_to_nd", "zz_shape", "nd_to_zz", "zz_to_nd", "TRANSFER_FRACTAL_ZZ", "TRANSFER_FRACTAL_ZZ_ND", "status_to_ge", "DcopyTransArgs", "data_type_size", "trans_data_format",
    "trans_format", "trans_format_check", "trans_shape", "trans_tensor_shape", "transpose",
    "transpose_with_shape_check", "FORMAT", "DATA_TYPE", "TRANSFER_FRACTAL_NZ",
    "TRANSFER_FRACTAL_NZ_ND", "TRANSFER_TRANSPOSE", "shard_range", "enable_peer_access",
    "p2p_copy", "set_p2p_engine", "P2P_ENGINE_AUTO", "P2P_ENGINE_SM", "P2P_ENGINE_COPY",
    "p2p_route", "P2P_ROUTE_COPY_ENGINE", "P2P_ROUTE_SM_BULK_PUSH", "P2P_ROUTE_SM_LOAD_STORE",
    "p2p_ring_shift", "ipc_get_handle", "ipc_open_handle", "ipc_close_handle",
    "signal", "wait_signal", "p2p_error", "tma_error", "DcopyDevCopy", "copy_ext_multi", "DcopyMemcpyInfo", "memcpy_async",
    "MEMCPY_KIND",
    "OK", "ERR_PARAM_INVALID", "ERR_SHAPE_INVALID", "ERR_DATATYPE_INVALID",
    "ERR_FORMAT_INVALID", "ERR_CUDA", "ERR_TIMEOUT", "ERR_UNSUPPORTED", "ERR_FAILED",
    "fz_shape", "to_fractal_z", "from_fractal_z", "TRANSFER_FRACTAL_Z", "TRANSFER_FRACTAL_Z_TBE",
    "TRANSFER_FRACZ_NCHW", "TRANSFER_FRACZ_HWCN", "TRANSFER_FRACZ_NHWC", "format_with_sub",
]

OK = 0
ERR_PARAM_INVALID = -1
ERR_SHAPE_INVALID = -2
ERR_DATATYPE_INVALID = -3
ERR_FORMAT_INVALID = -4
ERR_CUDA = -5
ERR_TIMEOUT = -6
ERR_UNSUPPORTED = -7
ERR_FAILED = -8

_HERE = os.path.dirname(os.path.abspath(__file__))
# DCOPY_LIBRARY selects an alternative build of the same library (e.g. one built
# with different compile-time options); the default is the in-tree libdcopy.so.
lib_path = os.environ.get("DCOPY_LIBRARY") or os.path.join(_HERE, "libdcopy.so")


class DcopyUnavailable(RuntimeError):
    """libdcopy.so is missing or cannot be loaded (build it with __graft_entry__.build())."""


class DcopyError(RuntimeError):
    """A libdcopy call returned a non-zero status."""

    def __init__(self, code: int, message: str, func: str):
        super().__init__(f"{func}: status {code}: {message}")
        self.code = code
        self.message = message


class DataCopyTiling(ctypes.Structure):
    """Byte-identical to the reference's DataCopyTiling (tiling_datacopy.h:7-13)."""
    _fields_ = [("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32),
                ("tile_cols", ctypes.c_uint32), ("ub_bytes", ctypes.c_uint32),
                ("store", ctypes.c_uint32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class DcopyExtParams(ctypes.Structure):
    """blockCount bursts of blockLen bytes; srcStride/dstStride are gaps in bytes."""
    _fields_ = [("blockCount", ctypes.c_uint32), ("blockLen", ctypes.c_uint32),
                ("srcStride", ctypes.c_uint64), ("dstStride", ctypes.c_uint64)]


class DcopyPadParams(ctypes.Structure):
    """AscendC::DataCopyPadExtParams<T> with T given by its size (include/dcopy/dcopy.h)."""
    _fields_ = [("isPad", ctypes.c_uint8), ("leftPadding", ctypes.c_uint8),
                ("rightPadding", ctypes.c_uint8), ("reserved", ctypes.c_uint8),
                ("elemBytes", ctypes.c_uint32), ("paddingValue", ctypes.c_uint64)]


P2P_ENGINE_AUTO = 0  # pushes on the copy engine, pulls and local copies on the SM kernel
P2P_ENGINE_SM = 1    # SM kernels only
P2P_ENGINE_COPY = 2  # the copy engine for every p2p_copy
P2P_ROUTE_COPY_ENGINE = 0
P2P_ROUTE_SM_BULK_PUSH = 1
P2P_ROUTE_SM_LOAD_STORE = 2

PAD_NORMAL = 0   # AscendC::PaddingMode::Normal
PAD_COMPACT = 1  # AscendC::PaddingMode::Compact


class DcopyTransArgs(ctypes.Structure):
    """TransArgs (register_format_transfer.h:25-42) with device data; formats carry the
    primary format in bits 0-7 and the sub format in bits 8-23."""
    _fields_ = [("data", ctypes.c_void_p), ("src_format", ctypes.c_int32),
                ("dst_format", ctypes.c_int32), ("src_c0", ctypes.c_int64),
                ("dst_c0", ctypes.c_int64), ("src_shape", ctypes.POINTER(ctypes.c_int64)),
                ("src_rank", ctypes.c_int32), ("dst_shape", ctypes.POINTER(ctypes.c_int64)),
                ("dst_rank", ctypes.c_int32), ("data_type", ctypes.c_int32),
                ("src_sub_format", ctypes.c_int32), ("dst_sub_format", ctypes.c_int32)]


# GE enum values (metadef graph/types.h; api/python/ge/ge/graph/types.py).
FORMAT = {"NCHW": 0, "NHWC": 1, "ND": 2, "NC1HWC0": 3, "FRACTAL_Z": 4, "C1HWNC0": 9,
          "CHWN": 14, "HWCN": 16, "FRACTAL_ZZ": 28, "FRACTAL_NZ": 29, "RESERVED": 40}
DATA_TYPE = {"FLOAT": 0, "FLOAT16": 1, "INT8": 2, "INT32": 3, "UINT8": 4, "INT16": 6,
             "UINT16": 7, "UINT32": 8, "INT64": 9, "UINT64": 10, "DOUBLE": 11, "BOOL": 12,
             "STRING": 13, "COMPLEX64": 16, "COMPLEX128": 17, "BF16": 27, "UNDEFINED": 28}
TRANSFER_FRACTAL_NZ, TRANSFER_FRACTAL_NZ_ND, TRANSFER_TRANSPOSE = 1, 2, 3
TRANSFER_FRACTAL_ZZ, TRANSFER_FRACTAL_ZZ_ND = 4, 5
TRANSFER_FRACTAL_Z, TRANSFER_FRACTAL_Z_TBE = 6, 7
TRANSFER_FRACZ_NCHW, TRANSFER_FRACZ_HWCN, TRANSFER_FRACZ_NHWC = 8, 9, 10


def format_with_sub(primary: int, sub: int) -> int:
    """A GE Format value with a sub format (GetFormatFromSub): FRACTAL_Z groups."""
    return (primary & 0xff) | ((sub & 0xffff) << 8)


class DcopyMemcpyInfo(ctypes.Structure):
    """MemcpyAsyncMemInfo (runtime/v1/common/runtime_api_wrapper.h:42-47)."""
    _fields_ = [("dst", ctypes.c_void_p), ("destMax", ctypes.c_uint64), ("src", ctypes.c_void_p),
                ("cnt", ctypes.c_uint64)]


# rtMemcpyKind_t values (acl_rt_memcpy_kind.h:16-27).
MEMCPY_KIND = {"HOST_TO_HOST": 0, "HOST_TO_DEVICE": 1, "DEVICE_TO_HOST": 2,
               "DEVICE_TO_DEVICE": 3, "MANAGED": 4, "ADDR_DEVICE_TO_DEVICE": 5,
               "HOST_TO_DEVICE_EX": 6, "DEVICE_TO_HOST_EX": 7, "DEFAULT": 8}


class DcopyDevCopy(ctypes.Structure):
    """One device's strided copy for dcopy_copy_ext_multi."""
    _fields_ = [("device", ctypes.c_int32), ("dst", ctypes.c_void_p), ("src", ctypes.c_void_p),
                ("params", DcopyExtParams), ("stream", ctypes.c_void_p)]

assert ctypes.sizeof(DataCopyTiling) == 20
assert ctypes.sizeof(DcopyExtParams) == 24

_lib = None

_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_SIGNATURES = {
    "dcopy_last_error_message": (ctypes.c_char_p, []),
    "dcopy_status_to_ge": (ctypes.c_uint32, [ctypes.c_int]),
    "dcopy_version": (ctypes.c_int, []),
    "dcopy_plan_tiling": (ctypes.c_int, [ctypes.c_uint32] * 4 + [ctypes.POINTER(DataCopyTiling)]),
    "dcopy_datacopy_small": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DataCopyTiling), _vp]),
    "dcopy_datacopy_large": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DataCopyTiling), _vp]),
    "dcopy_datacopy_pretranspose": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DataCopyTiling), _vp]),
    "dcopy_datacopy_contiguous": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DataCopyTiling), _vp]),
    "dcopy_datacopy_tiles": (ctypes.c_int, [ctypes.c_int32, _vp, _vp, ctypes.POINTER(DataCopyTiling),
                                            ctypes.c_uint32, ctypes.c_uint32, _vp]),
    "dcopy_datacopy_pretranspose_noalloc": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DataCopyTiling),
                                                           _vp]),
    "dcopy_copy_ext": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DcopyExtParams), _vp]),
    "dcopy_copy_ext_32b": (ctypes.c_int, [_vp, _vp] + [ctypes.c_uint32] * 4 + [_vp]),
    "dcopy_copy_pad_gm_to_ub": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DcopyExtParams),
                                               ctypes.POINTER(DcopyPadParams), ctypes.c_int32,
                                               _vp]),
    "dcopy_copy_pad_ub_to_gm": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(DcopyExtParams),
                                               ctypes.c_int32, _vp]),
    "dcopy_datacopy_pad_extend_load": (ctypes.c_int, [_vp, _vp] + [ctypes.c_uint32] * 5 +
                                       [ctypes.c_int32, _vp]),
    "dcopy_datacopy_pad_extend_store": (ctypes.c_int, [_vp, _vp] + [ctypes.c_uint32] * 5 +
                                        [ctypes.c_int32, _vp]),
    "dcopy_copy_nd": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _u64p, _i64p, _i64p,
                                     ctypes.c_uint32, _vp]),
    "dcopy_nz_shape": (ctypes.c_int, [_i64p, ctypes.c_int, ctypes.c_int64, _i64p,
                                      ctypes.POINTER(ctypes.c_int), _i64p]),
    "dcopy_nd_to_nz": (ctypes.c_int, [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int64, _vp]),
    "dcopy_nz_to_nd": (ctypes.c_int, [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int64, _vp]),
    "dcopy_fz_shape": (ctypes.c_int, [ctypes.c_int32, _i64p, ctypes.c_int, ctypes.c_int64,
                                      ctypes.c_int64, _i64p]),
    "dcopy_to_fractal_z": (ctypes.c_int, [_vp, _vp, ctypes.c_int32, _i64p, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _vp]),
    "dcopy_from_fractal_z": (ctypes.c_int, [_vp, _vp, ctypes.c_int32, _i64p, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int64, _vp]),
    "dcopy_zz_shape": (ctypes.c_int, [_i64p, ctypes.c_int, ctypes.c_int64, _i64p,
                                      ctypes.POINTER(ctypes.c_int), _i64p]),
    "dcopy_nd_to_zz": (ctypes.c_int, [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int64, _vp]),
    "dcopy_zz_to_nd": (ctypes.c_int, [_vp, _vp, _i64p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int64, _vp]),
    "dcopy_data_type_size": (ctypes.c_int32, [ctypes.c_int32]),
    "dcopy_trans_data_format": (ctypes.c_int, [ctypes.POINTER(DcopyTransArgs), _vp,
                                               ctypes.c_uint64, _u64p, _vp]),
    "dcopy_trans_format_check": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(DcopyTransArgs),
                                                ctypes.POINTER(ctypes.c_uint64)]),
    "dcopy_trans_format": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(DcopyTransArgs), _vp,
                                          ctypes.c_uint64, _u64p, _vp]),
    "dcopy_trans_shape": (ctypes.c_int, [ctypes.c_int, ctypes.c_int32, _i64p, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, _i64p,
                                         ctypes.POINTER(ctypes.c_int32)]),
    "dcopy_trans_tensor_shape": (ctypes.c_int, [ctypes.c_int32, _i64p, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                                _i64p, ctypes.POINTER(ctypes.c_int32)]),
    "dcopy_transpose": (ctypes.c_int, [_vp, _vp, _i64p, _i64p, ctypes.c_int32, ctypes.c_int32,
                                       _vp]),
    "dcopy_transpose_with_shape_check": (ctypes.c_int, [_vp, _vp, _i64p, _i64p, _i64p,
                                                        ctypes.c_int32, ctypes.c_int32, _vp]),
    "dcopy_memcpy_async": (ctypes.c_int, [ctypes.POINTER(DcopyMemcpyInfo), ctypes.c_int32, _vp]),
    "dcopy_shard_range": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32, _u64p,
                                         _u64p]),
    "dcopy_copy_ext_multi": (ctypes.c_int, [ctypes.POINTER(DcopyDevCopy), ctypes.c_int32]),
    "dcopy_enable_peer_access": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32]),
    "dcopy_p2p_copy": (ctypes.c_int, [_vp, _vp, ctypes.c_uint64, _vp]),
    "dcopy_p2p_ring_shift": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32),
                                            ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
                                            ctypes.c_uint64]),
    "dcopy_ipc_get_handle": (ctypes.c_int, [_vp, ctypes.c_char_p, _u64p]),
    "dcopy_ipc_open_handle": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "dcopy_ipc_close_handle": (ctypes.c_int, [_vp]),
    "dcopy_p2p_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "dcopy_set_p2p_engine": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]),
    "dcopy_p2p_route": (ctypes.c_int, [_vp, _vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_int32)]),
    "dcopy_signal": (ctypes.c_int, [_vp, ctypes.c_uint32, _vp]),
    "dcopy_wait_signal": (ctypes.c_int, [_vp, ctypes.c_uint32, ctypes.c_uint64, _vp, _vp]),
    "dcopy_tma_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "dcopy_set_nd_tma": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "dcopy_copy_ext_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
    "dcopy_copy_ext_loop": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_void_p]),
    "dcopy_copy_ext_staged": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32,
                                             ctypes.c_void_p]),
    "dcopy_memcpy_async_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int32,
                                                ctypes.c_void_p]),
}


def lib() -> ctypes.CDLL:
    """Load libdcopy.so once and bind the declared signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(lib_path):
            raise DcopyUnavailable(f"{lib_path} is not built; run __graft_entry__.build()")
        try:
            handle = ctypes.CDLL(lib_path)
        except OSError as exc:  # pragma: no cover - depends on the machine
            raise DcopyUnavailable(f"cannot load {lib_path}: {exc}") from exc
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if getattr(x, "is_cuda", True) is False and not x.is_pinned():
            # Pinned host memory is GPU-addressable (the kernels read and write it over
            # PCIe); pageable host memory is not.
            raise ValueError("dcopy kernels need CUDA or pinned host tensors (got a pageable "
                             "CPU tensor)")
        return x.data_ptr()
    raise TypeError(f"expected a CUDA tensor or a device address, got {type(x).__name__}")


def _stream(stream) -> Optional[int]:
    if stream is None:
        torch = sys.modules.get("torch")
        if torch is not None and torch.cuda.is_available() and torch.cuda.is_initialized():
            return torch.cuda.current_stream().cuda_stream or None
        return None
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


def _check(rc: int, func: str) -> None:
    if rc != OK:
        msg = lib().dcopy_last_error_message() or b""
        raise DcopyError(rc, msg.decode(errors="replace"), func)


def status_to_ge(status: int) -> int:
    return lib().dcopy_status_to_ge(status)


def plan_tiling(rows: int, cols: int, tile_kib: int, store: int = 1) -> DataCopyTiling:
    """asc:115-123: validate and plan; raises DcopyError(ERR_PARAM_INVALID) like the reference."""
    for v in (rows, cols, tile_kib, store):
        if not 0 <= v <= 0xFFFFFFFF:
            raise DcopyError(ERR_PARAM_INVALID, "Integer overflow", "dcopy_plan_tiling")
    t = DataCopyTiling()
    _check(lib().dcopy_plan_tiling(rows, cols, tile_kib, store, ctypes.byref(t)),
           "dcopy_plan_tiling")
    return t


def _datacopy(name: str, src, dst, tiling: DataCopyTiling, stream=None) -> None:
    fn = getattr(lib(), name)
    _check(fn(_ptr(src), _ptr(dst), ctypes.byref(tiling), _stream(stream)), name)


def datacopy_small(x, y, tiling: DataCopyTiling, stream=None) -> None:
    _datacopy("dcopy_datacopy_small", x, y, tiling, stream)


def datacopy_large(x, y, tiling: DataCopyTiling, stream=None) -> None:
    _datacopy("dcopy_datacopy_large", x, y, tiling, stream)


def datacopy_pretranspose(x, b, tiling: DataCopyTiling, stream=None) -> None:
    _datacopy("dcopy_datacopy_pretranspose", x, b, tiling, stream)


def datacopy_contiguous(b, y, tiling: DataCopyTiling, stream=None) -> None:
    _datacopy("dcopy_datacopy_contiguous", b, y, tiling, stream)


def datacopy_tiles(phase: int, inp, out, tiling: DataCopyTiling, tile_begin: int,
                   tile_count: int, stream=None) -> None:
    """RunTiles<phase> over the tiles [tile_begin, tile_begin + tile_count) only (one core's
    or one GPU's share); in, out and tiling are those of the whole problem."""
    _check(lib().dcopy_datacopy_tiles(phase, _ptr(inp), _ptr(out), ctypes.byref(tiling),
                                      tile_begin, tile_count, _stream(stream)),
           "dcopy_datacopy_tiles")


def datacopy_pretranspose_noalloc(x, y, tiling: DataCopyTiling, stream=None) -> None:
    """x -> B -> y without any allocation (B lives in the library's 16 MiB device array)."""
    _datacopy("dcopy_datacopy_pretranspose_noalloc", x, y, tiling, stream)


class DcopyLoopModeParams(ctypes.Structure):
    """LoopModeParams: two outer loops around a DataCopyExt copy; strides in bytes."""
    _fields_ = [("loop1Size", ctypes.c_uint32), ("loop2Size", ctypes.c_uint32),
                ("loop1SrcStride", ctypes.c_uint64), ("loop1DstStride", ctypes.c_uint64),
                ("loop2SrcStride", ctypes.c_uint64), ("loop2DstStride", ctypes.c_uint64)]


STAGED_COPY_ENGINE_RETURN = 1


def copy_ext_staged(dst, src, block_count: int, block_len: int, src_gap: int, dst_gap: int,
                    staging, staging_bytes: int = None, flags: int = 0, stream=None) -> None:
    """DataCopyExt between host buffers through a device staging buffer (copy-engine
    gather host -> device, return write overlapped on a second stream)."""
    if staging_bytes is None:
        staging_bytes = staging.numel() * staging.element_size()
    p = DcopyExtParams(block_count, block_len, src_gap, dst_gap)
    _check(lib().dcopy_copy_ext_staged(_host_or_dev(dst), _host_or_dev(src), ctypes.byref(p),
                                       _ptr(staging), staging_bytes, flags, _stream(stream)),
           "dcopy_copy_ext_staged")


def _host_or_dev(x):
    """Address of a tensor in any memory (pageable host included), a numpy array or an int."""
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    return x


def copy_ext_loop(dst, src, block_count: int, block_len: int, src_gap: int, dst_gap: int,
                  loop1, loop2=(1, 0, 0), stream=None) -> None:
    """DataCopyPadExtend with LoopModeParams: loop1/loop2 = (size, src stride, dst stride),
    strides in bytes; the inner copy is copy_ext(block_count, block_len, gaps)."""
    p = DcopyExtParams(block_count, block_len, src_gap, dst_gap)
    lp = DcopyLoopModeParams(loop1[0], loop2[0], loop1[1], loop1[2], loop2[1], loop2[2])
    _check(lib().dcopy_copy_ext_loop(_ptr(dst), _ptr(src), ctypes.byref(p), ctypes.byref(lp),
                                     _stream(stream)), "dcopy_copy_ext_loop")


class DcopyExtCopy(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("src", ctypes.c_void_p), ("params", DcopyExtParams)]


def copy_ext_batch(copies, stream=None) -> None:
    """Independent copies (dst, src, block_count, block_len, src_stride, dst_stride) in one
    batch: one launch per 256 copies; destinations may not overlap other copies' spans."""
    arr = (DcopyExtCopy * max(len(copies), 1))()
    for i, (dst, src, count, blen, sgap, dgap) in enumerate(copies):
        arr[i].dst = _ptr(dst)
        arr[i].src = _ptr(src)
        arr[i].params = DcopyExtParams(count, blen, sgap, dgap)
    _check(lib().dcopy_copy_ext_batch(arr if copies else None, len(copies), _stream(stream)),
           "dcopy_copy_ext_batch")


def copy_ext(dst, src, block_count: int, block_len: int, src_stride: int = 0,
             dst_stride: int = 0, stream=None) -> None:
    """blockCount bursts of blockLen bytes; strides are gap bytes (test_address_model.py:24)."""
    p = DcopyExtParams(block_count, block_len, src_stride, dst_stride)
    _check(lib().dcopy_copy_ext(_ptr(dst), _ptr(src), ctypes.byref(p), _stream(stream)),
           "dcopy_copy_ext")


def copy_ext_32b(dst, src, block_count: int, block_len32: int, src_stride32: int = 0,
                 dst_stride32: int = 0, stream=None) -> None:
    _check(lib().dcopy_copy_ext_32b(_ptr(dst), _ptr(src), block_count, block_len32,
                                    src_stride32, dst_stride32, _stream(stream)),
           "dcopy_copy_ext_32b")


def copy_pad_gm_to_ub(ub, gm, block_count: int, block_len: int, src_gap: int, dst_blocks: int,
                      mode: int = PAD_NORMAL, pad=(True, 0, 0, 0), elem_bytes: int = 1,
                      stream=None) -> None:
    """DataCopyPad GM -> UB: blockLen and the GM gap in bytes, the UB gap in 32-byte
    blocks; pad = DataCopyPadExtParams (isPad, leftPadding, rightPadding, paddingValue)
    with paddingValue given as the element's bits."""
    p = DcopyExtParams(block_count, block_len, src_gap, dst_blocks)
    pp = DcopyPadParams(int(bool(pad[0])), pad[1], pad[2], 0, elem_bytes, pad[3])
    _check(lib().dcopy_copy_pad_gm_to_ub(_ptr(ub), _ptr(gm), ctypes.byref(p), ctypes.byref(pp),
                                         mode, _stream(stream)), "dcopy_copy_pad_gm_to_ub")


def copy_pad_ub_to_gm(gm, ub, block_count: int, block_len: int, src_blocks: int, dst_gap: int,
                      mode: int = PAD_NORMAL, stream=None) -> None:
    """DataCopyPad UB -> GM: the UB gap in 32-byte blocks, the GM gap in bytes."""
    p = DcopyExtParams(block_count, block_len, src_blocks, dst_gap)
    _check(lib().dcopy_copy_pad_ub_to_gm(_ptr(gm), _ptr(ub), ctypes.byref(p), mode,
                                         _stream(stream)), "dcopy_copy_pad_ub_to_gm")


def datacopy_pad_extend(dst, src, elem_bytes: int, block_count: int, block_len: int,
                        src_stride: int, dst_stride: int, to_ub: bool, mode: int = PAD_NORMAL,
                        stream=None) -> None:
    """DataCopyPadExtend (ascendc/api/datacopy.h:14-40) in elements of T: to_ub=True is
    the GM -> UB overload (dst is the UB image), False the UB -> GM one."""
    fn = lib().dcopy_datacopy_pad_extend_load if to_ub else lib().dcopy_datacopy_pad_extend_store
    _check(fn(_ptr(dst), _ptr(src), elem_bytes, block_count, block_len, src_stride, dst_stride,
              mode, _stream(stream)), "dcopy_datacopy_pad_extend")


def copy_nd(dst, src, sizes: Sequence[int], src_strides: Sequence[int],
            dst_strides: Sequence[int], elem_bytes: int, stream=None) -> None:
    n = len(sizes)
    s = (ctypes.c_uint64 * n)(*sizes)
    ss = (ctypes.c_int64 * n)(*src_strides)
    ds = (ctypes.c_int64 * n)(*dst_strides)
    _check(lib().dcopy_copy_nd(_ptr(dst), _ptr(src), n, s, ss, ds, elem_bytes, _stream(stream)),
           "dcopy_copy_nd")


def nz_shape(nd_shape: Sequence[int], w0: int):
    """TransShapeToFracNz: returns (nz_shape, (times, H, W))."""
    n = len(nd_shape)
    src = (ctypes.c_int64 * max(n, 1))(*nd_shape)
    out = (ctypes.c_int64 * (n + 4))()
    rank = ctypes.c_int(0)
    hw = (ctypes.c_int64 * 3)()
    _check(lib().dcopy_nz_shape(src, n, w0, out, ctypes.byref(rank), hw), "dcopy_nz_shape")
    return [out[i] for i in range(rank.value)], tuple(hw)


def _shape_arg(shape: Sequence[int]):
    return (ctypes.c_int64 * max(len(shape), 1))(*shape), len(shape)


def nd_to_nz(dst, src, nd_shape: Sequence[int], elem_bytes: int, w0: int, stream=None) -> None:
    arr, n = _shape_arg(nd_shape)
    _check(lib().dcopy_nd_to_nz(_ptr(dst), _ptr(src), arr, n, elem_bytes, w0, _stream(stream)),
           "dcopy_nd_to_nz")


def nz_to_nd(dst, src, nd_shape: Sequence[int], elem_bytes: int, w0: int, stream=None) -> None:
    arr, n = _shape_arg(nd_shape)
    _check(lib().dcopy_nz_to_nd(_ptr(dst), _ptr(src), arr, n, elem_bytes, w0, _stream(stream)),
           "dcopy_nz_to_nd")


def zz_shape(nd_shape: Sequence[int], c0: int):
    """TransShapeToFracZz: returns (zz_shape, (times, H, W))."""
    n = len(nd_shape)
    src = (ctypes.c_int64 * max(n, 1))(*nd_shape)
    out = (ctypes.c_int64 * (n + 4))()
    rank = ctypes.c_int(0)
    hw = (ctypes.c_int64 * 3)()
    _check(lib().dcopy_zz_shape(src, n, c0, out, ctypes.byref(rank), hw), "dcopy_zz_shape")
    return [out[i] for i in range(rank.value)], tuple(hw)


def nd_to_zz(dst, src, nd_shape: Sequence[int], elem_bytes: int, c0: int, stream=None) -> None:
    arr, n = _shape_arg(nd_shape)
    _check(lib().dcopy_nd_to_zz(_ptr(dst), _ptr(src), arr, n, elem_bytes, c0, _stream(stream)),
           "dcopy_nd_to_zz")


def zz_to_nd(dst, src, nd_shape: Sequence[int], elem_bytes: int, c0: int, stream=None) -> None:
    arr, n = _shape_arg(nd_shape)
    _check(lib().dcopy_zz_to_nd(_ptr(dst), _ptr(src), arr, n, elem_bytes, c0, _stream(stream)),
           "dcopy_zz_to_nd")


def fz_shape(src_format: int, src_shape: Sequence[int], c0: int, groups: int = 0):
    """FRACTAL_Z TransShape: [C1*H*W, N1, 16, C0] of a NCHW/NHWC/HWCN/ND weight."""
    arr, n = _shape_arg(src_shape)
    out = (ctypes.c_int64 * 4)()
    _check(lib().dcopy_fz_shape(src_format, arr, n, c0, groups, out), "dcopy_fz_shape")
    return list(out)


def to_fractal_z(dst, src, src_format: int, src_shape: Sequence[int], elem_bytes: int, c0: int,
                 groups: int = 0, stream=None) -> None:
    arr, n = _shape_arg(src_shape)
    _check(lib().dcopy_to_fractal_z(_ptr(dst), _ptr(src), src_format, arr, n, elem_bytes, c0,
                                    groups, _stream(stream)), "dcopy_to_fractal_z")


def from_fractal_z(dst, src, dst_format: int, dst_shape: Sequence[int], elem_bytes: int,
                   c0: int, stream=None) -> None:
    arr, n = _shape_arg(dst_shape)
    _check(lib().dcopy_from_fractal_z(_ptr(dst), _ptr(src), dst_format, arr, n, elem_bytes, c0,
                                      _stream(stream)), "dcopy_from_fractal_z")


# ---- GE TransData level -------------------------------------------------------------

def data_type_size(data_type: int) -> int:
    """GetSizeByDataType: bytes per element, -1 for types without a fixed size."""
    return lib().dcopy_data_type_size(data_type)


def _trans_args(data, src_format, dst_format, src_shape, dst_shape, data_type, src_c0=16,
                dst_c0=16, src_sub=0, dst_sub=0):
    src = (ctypes.c_int64 * max(len(src_shape), 1))(*src_shape)
    dst = (ctypes.c_int64 * max(len(dst_shape), 1))(*dst_shape)
    a = DcopyTransArgs(_ptr(data), src_format, dst_format, src_c0, dst_c0, src, len(src_shape),
                       dst, len(dst_shape), data_type, src_sub, dst_sub)
    a._keep = (src, dst)
    return a


def trans_data_format(dst, data, src_format, dst_format, src_shape, dst_shape, data_type,
                      dst_capacity, src_c0=16, dst_c0=16, stream=None, src_sub=0,
                      dst_sub=0) -> int:
    """TransDataFormat (formats.cc:30-52) into `dst`; returns the result length in bytes."""
    a = _trans_args(data, src_format, dst_format, src_shape, dst_shape, data_type, src_c0, dst_c0,
                    src_sub, dst_sub)
    n = ctypes.c_uint64(0)
    _check(lib().dcopy_trans_data_format(ctypes.byref(a), _ptr(dst), dst_capacity,
                                         ctypes.byref(n), _stream(stream)),
           "dcopy_trans_data_format")
    return n.value


def trans_format(transfer_class, dst, data, src_format, dst_format, src_shape, dst_shape,
                 data_type, dst_capacity, src_c0=16, dst_c0=16, stream=None, src_sub=0,
                 dst_sub=0) -> int:
    """FormatTransfer<class>::TransFormat; returns the result length in bytes."""
    a = _trans_args(data, src_format, dst_format, src_shape, dst_shape, data_type, src_c0, dst_c0,
                    src_sub, dst_sub)
    n = ctypes.c_uint64(0)
    _check(lib().dcopy_trans_format(transfer_class, ctypes.byref(a), _ptr(dst), dst_capacity,
                                    ctypes.byref(n), _stream(stream)), "dcopy_trans_format")
    return n.value


def trans_format_check(transfer_class, data, src_format, dst_format, src_shape, dst_shape,
                       data_type, src_c0=16, dst_c0=16, src_sub=0, dst_sub=0) -> int:
    """Every check of TransDataFormat (class 0) or of one class's TransFormat, no data
    movement; returns the result length in bytes."""
    a = _trans_args(data, src_format, dst_format, src_shape, dst_shape, data_type, src_c0, dst_c0,
                    src_sub, dst_sub)
    n = ctypes.c_uint64(0)
    _check(lib().dcopy_trans_format_check(transfer_class, ctypes.byref(a), ctypes.byref(n)),
           "dcopy_trans_format_check")
    return n.value


def _shape_call(fn, name, *head, src_shape, rest):
    src = (ctypes.c_int64 * max(len(src_shape), 1))(*src_shape)
    out = (ctypes.c_int64 * (len(src_shape) + 4))()
    rank = ctypes.c_int32(0)
    _check(fn(*head, src, len(src_shape), *rest, out, ctypes.byref(rank)), name)
    return [out[i] for i in range(rank.value)]


def trans_shape(transfer_class, src_format, src_shape, data_type, dst_format, c0=16):
    """FormatTransfer<class>::TransShape."""
    return _shape_call(lib().dcopy_trans_shape, "dcopy_trans_shape", transfer_class, src_format,
                       src_shape=src_shape, rest=(data_type, dst_format, c0))


def trans_tensor_shape(src_format, src_shape, data_type, dst_format, c0=16):
    """TransTensorShape (formats.cc:54-71)."""
    return _shape_call(lib().dcopy_trans_tensor_shape, "dcopy_trans_tensor_shape", src_format,
                       src_shape=src_shape, rest=(data_type, dst_format, c0))


def transpose(dst, src, src_shape, perm, data_type, stream=None) -> None:
    """Transpose (format_transfer_transpose.cc:142-197) on the GPU."""
    n = len(src_shape)
    s = (ctypes.c_int64 * max(n, 1))(*src_shape)
    p = (ctypes.c_int64 * max(len(perm), 1))(*perm)
    if len(perm) != n:
        raise DcopyError(ERR_PARAM_INVALID, "perm and shape ranks differ", "dcopy_transpose")
    _check(lib().dcopy_transpose(_ptr(dst), _ptr(src), s, p, n, data_type, _stream(stream)),
           "dcopy_transpose")


def transpose_with_shape_check(dst, src, src_shape, dst_shape, perm, data_type,
                               stream=None) -> None:
    n = len(src_shape)
    if len(perm) != n or len(dst_shape) != n:
        raise DcopyError(ERR_PARAM_INVALID, "perm/shape ranks differ",
                         "dcopy_transpose_with_shape_check")
    s = (ctypes.c_int64 * max(n, 1))(*src_shape)
    d = (ctypes.c_int64 * max(n, 1))(*dst_shape)
    p = (ctypes.c_int64 * max(n, 1))(*perm)
    _check(lib().dcopy_transpose_with_shape_check(_ptr(dst), _ptr(src), s, d, p, n, data_type,
                                                  _stream(stream)),
           "dcopy_transpose_with_shape_check")


# ---- multi-GPU ------------------------------------------------------------------------

def shard_range(block_count: int, rank: int, world: int):
    """(begin, count) of the blocks `rank` of `world` owns (contiguous split)."""
    b, c = ctypes.c_uint64(0), ctypes.c_uint64(0)
    _check(lib().dcopy_shard_range(block_count, rank, world, ctypes.byref(b), ctypes.byref(c)),
           "dcopy_shard_range")
    return b.value, c.value


def copy_ext_multi(copies) -> None:
    """copies: iterable of (device, dst, src, (count, blen, sgap, dgap), stream)."""
    items = list(copies)
    arr = (DcopyDevCopy * max(len(items), 1))()
    for i, (dev, dst, src, prm, stream) in enumerate(items):
        arr[i] = DcopyDevCopy(dev, _ptr(dst), _ptr(src), DcopyExtParams(*prm),
                              _stream(stream) if stream is not None else None)
    _check(lib().dcopy_copy_ext_multi(arr, len(items)), "dcopy_copy_ext_multi")


def enable_peer_access(device: int, peer: int) -> None:
    _check(lib().dcopy_enable_peer_access(device, peer), "dcopy_enable_peer_access")


def p2p_copy(dst, src, nbytes: int, stream=None) -> None:
    """nbytes from src to dst (this GPU's or a peer's memory): pushes on the copy engine,
    pulls on the SM load/store kernel (see set_p2p_engine)."""
    _check(lib().dcopy_p2p_copy(_ptr(dst), _ptr(src), nbytes, _stream(stream)), "dcopy_p2p_copy")


def set_p2p_engine(engine: int) -> int:
    """Selects p2p_copy's engine (P2P_ENGINE_AUTO / _SM / _COPY, process-wide);
    returns the former setting."""
    prev = ctypes.c_int32(0)
    _check(lib().dcopy_set_p2p_engine(int(engine), ctypes.byref(prev)), "dcopy_set_p2p_engine")
    return prev.value


def p2p_route(dst, src, nbytes: int) -> int:
    """The route p2p_copy would take (P2P_ROUTE_*), on the current device."""
    r = ctypes.c_int32(-1)
    _check(lib().dcopy_p2p_route(_ptr(dst), _ptr(src), nbytes, ctypes.byref(r)), "dcopy_p2p_route")
    return r.value


def p2p_ring_shift(devices, srcs, dsts, nbytes: int, streams=None) -> None:
    """One process: device i copies srcs[i] into dsts[(i+1) % n]."""
    n = len(devices)
    devs = (ctypes.c_int32 * n)(*devices)
    s = (ctypes.c_void_p * n)(*[_ptr(x) for x in srcs])
    d = (ctypes.c_void_p * n)(*[_ptr(x) for x in dsts])
    st = None
    if streams is not None:
        st = (ctypes.c_void_p * n)(*[_stream(x) for x in streams])
    _check(lib().dcopy_p2p_ring_shift(devs, s, d, st, n, nbytes), "dcopy_p2p_ring_shift")


def set_nd_tma(enable: bool) -> bool:
    """Selects the TMA tensor-copy path of copy_nd (process-wide); returns the former setting."""
    prev = ctypes.c_int(0)
    _check(lib().dcopy_set_nd_tma(1 if enable else 0, ctypes.byref(prev)), "dcopy_set_nd_tma")
    return bool(prev.value)


def tma_error() -> int:
    """Reads and clears the device's TMA box-copy error word (1 = a copy gave up)."""
    v = ctypes.c_uint32(0)
    _check(lib().dcopy_tma_error(ctypes.byref(v)), "dcopy_tma_error")
    return v.value


def p2p_error() -> int:
    """Reads and clears this device's P2P error word (1 = a bulk push gave up)."""
    v = ctypes.c_uint32(0)
    _check(lib().dcopy_p2p_error(ctypes.byref(v)), "dcopy_p2p_error")
    return v.value


def ipc_get_handle(ptr):
    """(64-byte handle, offset) of the allocation holding a device pointer/tensor."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64(0)
    _check(lib().dcopy_ipc_get_handle(_ptr(ptr), buf, ctypes.byref(off)), "dcopy_ipc_get_handle")
    return buf.raw, off.value


def ipc_open_handle(handle: bytes) -> int:
    """Maps another process's allocation; returns its base address here."""
    out = ctypes.c_void_p()
    _check(lib().dcopy_ipc_open_handle(handle, ctypes.byref(out)), "dcopy_ipc_open_handle")
    return out.value


def ipc_close_handle(base: int) -> None:
    _check(lib().dcopy_ipc_close_handle(base), "dcopy_ipc_close_handle")


def signal(flag, value: int, stream=None) -> None:
    """Release-store `value` into a (possibly peer) 4-byte flag after earlier stream work."""
    _check(lib().dcopy_signal(_ptr(flag), value, _stream(stream)), "dcopy_signal")


def wait_signal(flag, value: int, timeout_ns: int, status, stream=None) -> None:
    """Bounded device-side wait for *flag == value; writes 0 (seen) / 1 (timeout) to status."""
    _check(lib().dcopy_wait_signal(_ptr(flag), value, timeout_ns, _ptr(status), _stream(stream)),
           "dcopy_wait_signal")


def memcpy_async_batch(tasks, kind, stream=None) -> None:
    """Many memcpy tasks (dst, dst_max, src, count) of one kind; small tasks between
    device or pinned host buffers run as one batched launch."""
    if isinstance(kind, str):
        kind = MEMCPY_KIND[kind]

    def addr(x):
        if hasattr(x, "data_ptr"):
            return x.data_ptr()
        if hasattr(x, "ctypes"):
            return x.ctypes.data
        return x
    arr = (DcopyMemcpyInfo * max(len(tasks), 1))()
    for i, (dst, dst_max, src, count) in enumerate(tasks):
        arr[i] = DcopyMemcpyInfo(addr(dst), dst_max, addr(src), count)
    _check(lib().dcopy_memcpy_async_batch(arr if tasks else None, len(tasks), kind,
                                          _stream(stream)), "dcopy_memcpy_async_batch")


def memcpy_async(dst, dst_max: int, src, count: int, kind, stream=None) -> None:
    """rtMemcpyAsyncWithCfg(MemcpyAsyncMemInfo{dst, destMax, src, cnt}, kind, stream)."""
    if isinstance(kind, str):
        kind = MEMCPY_KIND[kind]

    def addr(x):
        if hasattr(x, "data_ptr"):
            return x.data_ptr()
        if hasattr(x, "ctypes"):
            return x.ctypes.data
        return x
    info = DcopyMemcpyInfo(addr(dst), dst_max, addr(src), count)
    _check(lib().dcopy_memcpy_async(ctypes.byref(info), kind, _stream(stream)),
           "dcopy_memcpy_async")
