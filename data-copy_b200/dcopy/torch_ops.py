"""PyTorch operators over libdcopy, registered with torch.library.

The reference exposes its Ascend C kernels to PyTorch as custom operators
(ge/examples/custom_op/ascendc_add_custom registers add_custom with
TORCH_LIBRARY_FRAGMENT).  These are the data-movement kernels of this library
as operators in the ``dcopy`` namespace, on CUDA tensors:

  torch.ops.dcopy.nd_to_nz(x, c0)                     ND -> FRACTAL_NZ
  torch.ops.dcopy.nz_to_nd(x_nz, nd_shape, c0)        FRACTAL_NZ -> ND
  torch.ops.dcopy.transpose(x, perm)                  GE Transpose (contiguous result)
  torch.ops.dcopy.datacopy_transpose(x)               standalone datacopy: int32 [r, c] -> [c, r]
  torch.ops.dcopy.strided_gather(x, count, block_len, src_gap)
                                                      DataCopyExt gather into a packed tensor
  torch.ops.dcopy.copy_ext_(dst, src, count, block_len, src_gap, dst_gap)
                                                      DataCopyExt in place (mutates dst)
  torch.ops.dcopy.box(x, sizes, strides, offset)      DataCopyNddma: the strided box of x
                                                      (element strides/offset) packed
  torch.ops.dcopy.nd_to_zz(x, c0) / zz_to_nd(x_zz, nd_shape, c0)
                                                      ND <-> FRACTAL_ZZ
  torch.ops.dcopy.to_fractal_z(w, src_format, c0)     NCHW / NHWC / HWCN / ND weight -> FRACTAL_Z
  torch.ops.dcopy.from_fractal_z(w_fz, dst_format, dst_shape, c0)
                                                      FRACTAL_Z -> NCHW / NHWC / HWCN

Lengths and gaps of the DataCopyExt operators count ELEMENTS of the tensors'
dtype (as DataCopyPadExtend's arguments do, datacopy.h:14-40).  Each operator
has a fake implementation, so shapes propagate under FakeTensor / torch.compile
tracing without a GPU.  Every call runs on torch's current CUDA stream.
"""
from __future__ import annotations

from typing import List

import torch
from torch.library import custom_op

import dcopy

# A GE data type of each element width, for the dtype-agnostic Transpose.
_GE_TYPE_OF_WIDTH = {1: dcopy.DATA_TYPE["UINT8"], 2: dcopy.DATA_TYPE["FLOAT16"],
                     4: dcopy.DATA_TYPE["FLOAT"], 8: dcopy.DATA_TYPE["INT64"],
                     16: dcopy.DATA_TYPE["COMPLEX128"]}


def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("dcopy operators take CUDA tensors")


@custom_op("dcopy::nd_to_nz", mutates_args=(), device_types="cuda")
def nd_to_nz(x: torch.Tensor, c0: int = 16) -> torch.Tensor:
    _require_cuda(x)
    x = x.contiguous()
    nz, _ = dcopy.nz_shape(list(x.shape), c0)
    out = torch.empty(nz, dtype=x.dtype, device=x.device)
    dcopy.nd_to_nz(out, x, list(x.shape), x.element_size(), c0)
    return out


@nd_to_nz.register_fake
def _nd_to_nz_fake(x, c0=16):
    nz, _ = dcopy.nz_shape(list(x.shape), c0)
    return x.new_empty(nz)


@custom_op("dcopy::nz_to_nd", mutates_args=(), device_types="cuda")
def nz_to_nd(x: torch.Tensor, nd_shape: List[int], c0: int = 16) -> torch.Tensor:
    _require_cuda(x)
    nz, _ = dcopy.nz_shape(list(nd_shape), c0)
    if list(x.shape) != nz:
        raise ValueError(f"NZ tensor shape {list(x.shape)} is not the NZ shape {nz} of {nd_shape}")
    x = x.contiguous()
    out = torch.empty(list(nd_shape), dtype=x.dtype, device=x.device)
    dcopy.nz_to_nd(out, x, list(nd_shape), x.element_size(), c0)
    return out


@nz_to_nd.register_fake
def _nz_to_nd_fake(x, nd_shape, c0=16):
    return x.new_empty(list(nd_shape))


@custom_op("dcopy::transpose", mutates_args=(), device_types="cuda")
def transpose(x: torch.Tensor, perm: List[int]) -> torch.Tensor:
    _require_cuda(x)
    x = x.contiguous()
    out = torch.empty([x.shape[p] for p in perm], dtype=x.dtype, device=x.device)
    dcopy.transpose(out, x, list(x.shape), list(perm), _GE_TYPE_OF_WIDTH[x.element_size()])
    return out


@transpose.register_fake
def _transpose_fake(x, perm):
    return x.new_empty([x.shape[p] for p in perm])


@custom_op("dcopy::datacopy_transpose", mutates_args=(), device_types="cuda")
def datacopy_transpose(x: torch.Tensor) -> torch.Tensor:
    _require_cuda(x)
    if x.dtype != torch.int32 or x.dim() != 2:
        raise ValueError("datacopy_transpose takes a 2-D int32 tensor")
    rows, cols = x.shape
    t = dcopy.plan_tiling(rows, cols, 240, 1)
    out = torch.empty(cols, rows, dtype=x.dtype, device=x.device)
    dcopy.datacopy_large(x.contiguous(), out, t)
    return out


@datacopy_transpose.register_fake
def _datacopy_transpose_fake(x):
    return x.new_empty(x.shape[1], x.shape[0])


@custom_op("dcopy::strided_gather", mutates_args=(), device_types="cuda")
def strided_gather(x: torch.Tensor, count: int, block_len: int, src_gap: int) -> torch.Tensor:
    _require_cuda(x)
    x = x.contiguous()
    e = x.element_size()
    out = torch.empty(count * block_len, dtype=x.dtype, device=x.device)
    dcopy.copy_ext(out, x, count, block_len * e, src_gap * e, 0)
    return out


@strided_gather.register_fake
def _strided_gather_fake(x, count, block_len, src_gap):
    return x.new_empty(count * block_len)


@custom_op("dcopy::copy_ext_", mutates_args=("dst",), device_types="cuda")
def copy_ext_(dst: torch.Tensor, src: torch.Tensor, count: int, block_len: int, src_gap: int,
              dst_gap: int) -> None:
    _require_cuda(dst, src)
    if dst.dtype != src.dtype or not dst.is_contiguous():
        raise ValueError("copy_ext_ needs a contiguous dst of src's dtype")
    e = src.element_size()
    dcopy.copy_ext(dst, src.contiguous(), count, block_len * e, src_gap * e, dst_gap * e)


@copy_ext_.register_fake
def _copy_ext_fake(dst, src, count, block_len, src_gap, dst_gap):
    return None


@custom_op("dcopy::box", mutates_args=(), device_types="cuda")
def box(x: torch.Tensor, sizes: List[int], strides: List[int], offset: int = 0) -> torch.Tensor:
    """torch.as_strided(x, sizes, strides, offset).contiguous(), moved by dcopy_copy_nd."""
    _require_cuda(x)
    if len(sizes) != len(strides) or not 1 <= len(sizes) <= 5:
        raise ValueError("box: sizes and strides must have the same rank, 1..5")
    x = x.contiguous()
    last = offset + sum((n - 1) * st for n, st in zip(sizes, strides) if n > 0)
    if offset < 0 or min(strides) < 0 or (all(n > 0 for n in sizes) and last >= x.numel()):
        raise ValueError("box: the box runs outside x")
    out = torch.empty(list(sizes), dtype=x.dtype, device=x.device)
    if out.numel():
        dense = [1] * len(sizes)
        for k in range(len(sizes) - 2, -1, -1):
            dense[k] = dense[k + 1] * sizes[k + 1]
        dcopy.copy_nd(out, x.data_ptr() + offset * x.element_size(), list(sizes), list(strides),
                      dense, x.element_size())
    return out


@box.register_fake
def _box_fake(x, sizes, strides, offset=0):
    return x.new_empty(list(sizes))


@custom_op("dcopy::nd_to_zz", mutates_args=(), device_types="cuda")
def nd_to_zz(x: torch.Tensor, c0: int = 16) -> torch.Tensor:
    _require_cuda(x)
    x = x.contiguous()
    zz, _ = dcopy.zz_shape(list(x.shape), c0)
    out = torch.empty(zz, dtype=x.dtype, device=x.device)
    dcopy.nd_to_zz(out, x, list(x.shape), x.element_size(), c0)
    return out


@nd_to_zz.register_fake
def _nd_to_zz_fake(x, c0=16):
    zz, _ = dcopy.zz_shape(list(x.shape), c0)
    return x.new_empty(zz)


@custom_op("dcopy::zz_to_nd", mutates_args=(), device_types="cuda")
def zz_to_nd(x: torch.Tensor, nd_shape: List[int], c0: int = 16) -> torch.Tensor:
    _require_cuda(x)
    zz, _ = dcopy.zz_shape(list(nd_shape), c0)
    if list(x.shape) != zz:
        raise ValueError(f"ZZ tensor shape {list(x.shape)} is not the ZZ shape {zz} of {nd_shape}")
    x = x.contiguous()
    out = torch.empty(list(nd_shape), dtype=x.dtype, device=x.device)
    dcopy.zz_to_nd(out, x, list(nd_shape), x.element_size(), c0)
    return out


@zz_to_nd.register_fake
def _zz_to_nd_fake(x, nd_shape, c0=16):
    return x.new_empty(list(nd_shape))


def _weight_format(name: str) -> int:
    if name not in ("NCHW", "NHWC", "HWCN", "ND"):
        raise ValueError(f"FRACTAL_Z weights are NCHW, NHWC, HWCN or ND, not {name}")
    return dcopy.FORMAT[name]


@custom_op("dcopy::to_fractal_z", mutates_args=(), device_types="cuda")
def to_fractal_z(w: torch.Tensor, src_format: str, c0: int = 16) -> torch.Tensor:
    _require_cuda(w)
    fmt = _weight_format(src_format)
    w = w.contiguous()
    out = torch.empty(dcopy.fz_shape(fmt, list(w.shape), c0), dtype=w.dtype, device=w.device)
    dcopy.to_fractal_z(out, w, fmt, list(w.shape), w.element_size(), c0)
    return out


@to_fractal_z.register_fake
def _to_fractal_z_fake(w, src_format, c0=16):
    return w.new_empty(dcopy.fz_shape(_weight_format(src_format), list(w.shape), c0))


@custom_op("dcopy::from_fractal_z", mutates_args=(), device_types="cuda")
def from_fractal_z(w: torch.Tensor, dst_format: str, dst_shape: List[int],
                   c0: int = 16) -> torch.Tensor:
    _require_cuda(w)
    fmt = _weight_format(dst_format)
    w = w.contiguous()
    out = torch.empty(list(dst_shape), dtype=w.dtype, device=w.device)
    dcopy.from_fractal_z(out, w, fmt, list(dst_shape), w.element_size(), c0)
    return out


@from_fractal_z.register_fake
def _from_fractal_z_fake(w, dst_format, dst_shape, c0=16):
    return w.new_empty(list(dst_shape))
