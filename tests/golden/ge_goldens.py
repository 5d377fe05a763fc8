"""Parse GE's format-transfer unit tests into golden cases (read at test time).

The reference's golden vectors for the layout conversions live in gtest sources
that cannot be built here (they need securec, gtest and the metadef headers):
  tests/ge/ut/ge/common/format_transfer_fractal_nz_unittest.cc
  tests/ge/ut/ge/common/format_transfer_fractal_zz_unittest.cc
  tests/ge/ut/ge/common/format_transfer_transpose_unittest.cc
This module reads them as text: for every TEST_F it extracts the literal
`data` / `ret` arrays, each `TransArgs{...}` (primary formats, shapes, data
type) or `TransposeWithShapeCheck(...)` call, and the status each EXPECT_EQ
asserts.  Nothing is copied into this repository; the tests that use it skip
when the reference checkout is absent.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np

NZ_TEST = "ge-develop/tests/ge/ut/ge/common/format_transfer_fractal_nz_unittest.cc"
ZZ_TEST = "ge-develop/tests/ge/ut/ge/common/format_transfer_fractal_zz_unittest.cc"
TRANSPOSE_TEST = "ge-develop/tests/ge/ut/ge/common/format_transfer_transpose_unittest.cc"

_CTYPES = {"uint8_t": np.uint8, "uint16_t": np.uint16, "float": np.float32,
           "int32_t": np.int32, "int64_t": np.int64, "double": np.float64}

# GE DataType enum values and sizes (api/python/ge/ge/graph/types.py:15-58 mirrors
# metadef/inc/external/graph/types.h).
DT = {"DT_FLOAT": 0, "DT_FLOAT16": 1, "DT_INT8": 2, "DT_INT32": 3, "DT_UINT8": 4,
      "DT_INT16": 6, "DT_UINT16": 7, "DT_UINT32": 8, "DT_INT64": 9, "DT_UINT64": 10,
      "DT_DOUBLE": 11, "DT_BOOL": 12, "DT_STRING": 13, "DT_BF16": 27, "DT_UNDEFINED": 28}
FMT = {"FORMAT_NCHW": 0, "FORMAT_NHWC": 1, "FORMAT_ND": 2, "FORMAT_NC1HWC0": 3,
       "FORMAT_FRACTAL_Z": 4, "FORMAT_C1HWNC0": 9, "FORMAT_CHWN": 14, "FORMAT_HWCN": 16,
       "FORMAT_FRACTAL_ZZ": 28, "FORMAT_FRACTAL_NZ": 29, "FORMAT_RESERVED": 40}
STATUS = {"SUCCESS": 0, "ACL_ERROR_GE_PARAM_INVALID": 145000,
          "ACL_ERROR_GE_FORMAT_INVALID": 145020, "ACL_ERROR_GE_SHAPE_INVALID": 145021,
          "ACL_ERROR_GE_DATATYPE_INVALID": 145022}


@dataclass
class Args:
    name: str                 # variable name (args, args2, ...)
    data_var: Optional[str]   # array passed as data (None for nullptr)
    src_format: str
    dst_format: str
    src_shape: List[int]
    dst_shape: List[int]
    dtype: str
    c0: List[int] = field(default_factory=list)


@dataclass
class Expect:
    call: str                 # TransDataFormat | TransFormat | TransShape | TransposeWithShapeCheck
    args: Optional[str]       # TransArgs variable the call uses
    status: int
    transfer_class: Optional[str] = None
    shape_call: Optional[dict] = None   # literal TransShape(...) / TransposeWithShapeCheck(...) args


@dataclass
class Case:
    name: str
    arrays: Dict[str, np.ndarray]
    args: Dict[str, Args]
    expects: List[Expect]


def _nums(text: str):
    return [int(x) for x in re.findall(r"-?\d+", text)]


def _array_values(body: str, ctype: str) -> np.ndarray:
    body = re.sub(r"//[^\n]*", "", body)
    toks = [t for t in re.split(r"[,\s]+", body) if t]
    if _CTYPES[ctype] in (np.float32, np.float64):
        # A C++ double literal converted to float: parse as double, then round.
        return np.array([float(t) for t in toks], dtype=np.float64).astype(_CTYPES[ctype])
    return np.array([int(t) for t in toks], dtype=np.int64).astype(_CTYPES[ctype])


def _split_tests(text: str):
    heads = list(re.finditer(r"TEST_F\(\s*\w+\s*,\s*(\w+)\s*\)\s*\{", text))
    for i, m in enumerate(heads):
        end = heads[i + 1].start() if i + 1 < len(heads) else len(text)
        yield m.group(1), text[m.end():end]


def _parse_args(var: str, body: str) -> Args:
    body = body.replace("std::vector<int64_t>(", "(")
    data = re.match(r"\s*(?:reinterpret_cast<uint8_t\s*\*>\(\s*(\w+)\s*\)|(\w+))", body)
    data_var = (data.group(1) or data.group(2)) if data else None
    fmts = re.findall(r"\bFORMAT_\w+", body)
    shapes = re.findall(r"\{([-\d,\s]*)\}", body)
    dtype = re.findall(r"\bDT_\w+", body)[-1]
    # c0 values sit between the 4 formats and the shapes: "..., FORMAT_RESERVED, 16, 16, {".
    c0 = _nums(re.search(r"FORMAT_RESERVED\s*,\s*FORMAT_RESERVED\s*,([^{]*)\{", body).group(1))
    return Args(var, data_var, fmts[0], fmts[1], _nums(shapes[0]), _nums(shapes[1]), dtype, c0)


def _vector(text: str):
    return _nums(text)


def parse(path: Path) -> List[Case]:
    text = path.read_text(encoding="utf-8", errors="replace")
    cases = []
    for name, body in _split_tests(text):
        arrays = {}
        for m in re.finditer(r"\b(uint8_t|uint16_t|float|int32_t|int64_t|double)\s+(\w+)\s*"
                             r"\[([^\]]*)\]\s*=\s*\{(.*?)\};", body, re.S):
            values = _array_values(m.group(4), m.group(1))
            # A shorter initializer list leaves the remaining elements zero (C++
            # aggregate initialisation): pad to the declared extent when it is
            # a product of integer literals.
            dims = m.group(3).split("*")
            if all(d.strip().isdigit() for d in dims):
                n = int(np.prod([int(d) for d in dims]))
                if n > values.size:
                    values = np.concatenate([values, np.zeros(n - values.size, values.dtype)])
            arrays[m.group(2)] = values
        args = {}
        for m in re.finditer(r"TransArgs\s+(\w+)\s*\{(.*?)\};", body, re.S):
            args[m.group(1)] = _parse_args(m.group(1), m.group(2))
        var_class = {v: k for k, v in re.findall(r"\b(FormatTransfer\w+)\s+(\w+)\s*;", body)}
        expects = []
        for m in re.finditer(r"EXPECT_EQ\(\s*((?:(?!EXPECT_EQ).)*?)\s*,\s*(SUCCESS|ACL_ERROR_GE_\w+)"
                             r"\s*\)\s*;", body, re.S):
            call, status = m.group(1), STATUS[m.group(2)]
            if call.startswith("TransDataFormat("):
                a = re.match(r"TransDataFormat\(\s*(\w+)", call).group(1)
                expects.append(Expect("TransDataFormat", a, status))
            elif ".TransFormat(" in call:
                obj, a = re.match(r"(\w+)\.TransFormat\(\s*(\w+)", call).groups()
                expects.append(Expect("TransFormat", a, status, var_class.get(obj)))
            elif ".TransShape(" in call:
                obj = re.match(r"(\w+)\.TransShape\(", call).group(1)
                am = re.search(r"TransShape\(\s*(\w+)\.src_format", call)
                if am:
                    expects.append(Expect("TransShape", am.group(1), status, var_class.get(obj)))
                else:
                    fm = re.findall(r"FORMAT_\w+", call)
                    vec = re.search(r"std::vector<int64_t>\(\{([-\d,\s]*)\}\)", call)
                    shape = _vector(vec.group(1)) if vec else []
                    dt = re.search(r"DT_\w+", call).group(0)
                    expects.append(Expect("TransShape", None, status, var_class.get(obj),
                                          {"src_format": fm[0], "dst_format": fm[1],
                                           "src_shape": shape, "dtype": dt}))
            elif call.startswith("TransposeWithShapeCheck("):
                vecs = re.findall(r"std::vector<int64_t>\(\{([-\d,\s]*)\}\)", call)
                dm = re.match(r"TransposeWithShapeCheck\(\s*(?:reinterpret_cast<uint8_t\s*\*>\()?"
                              r"\s*(\w+)", call)
                dt = re.search(r"DT_\w+", call).group(0)
                expects.append(Expect("TransposeWithShapeCheck", None, status, None,
                                      {"data": dm.group(1), "src_shape": _vector(vecs[0]),
                                       "dst_shape": _vector(vecs[1]), "perm": _vector(vecs[2]),
                                       "dtype": dt}))
        cases.append(Case(name, arrays, args, expects))
    return cases


def load(reference_root: Path, which: str) -> List[Case]:
    rel = {"nz": NZ_TEST, "zz": ZZ_TEST, "transpose": TRANSPOSE_TEST}[which]
    return parse(Path(reference_root) / rel)
