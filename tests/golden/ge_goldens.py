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
FZ_TESTS = {
    "hwcn_fz": "ge-develop/tests/ge/ut/ge/common/format_transfer_hwcn_fractalz_unittest.cc",
    "nchw_fz": "ge-develop/tests/ge/ut/ge/common/format_transfer_nchw_fractalz_unittest.cc",
    "nhwc_fz": "ge-develop/tests/ge/ut/ge/common/format_transfer_nhwc_fractalz_unittest.cc",
    "nd_fz": "ge-develop/tests/ge/ut/ge/common/format_transfer_fractal_z_tbe_unittest.cc",
    "fz_nchw": "ge-develop/tests/ge/ut/ge/common/format_transfer_fracz_nchw_unittest.cc",
    "fz_hwcn": "ge-develop/tests/ge/ut/ge/common/format_transfer_fracz_hwcn_unittest.cc",
    "fz_nhwc": "ge-develop/tests/ge/ut/ge/common/format_transfer_fracz_nhwc_unittest.cc",
}
TRANSPOSE_TEST = "ge-develop/tests/ge/ut/ge/common/format_transfer_transpose_unittest.cc"

_CTYPES = {"uint8_t": np.uint8, "int8_t": np.int8, "uint16_t": np.uint16, "float": np.float32,
           "int32_t": np.int32, "int64_t": np.int64, "double": np.float64}

# GE DataType enum values and sizes (api/python/ge/ge/graph/types.py:15-58 mirrors
# metadef/inc/external/graph/types.h).
DT = {"DT_FLOAT": 0, "DT_FLOAT16": 1, "DT_INT8": 2, "DT_INT32": 3, "DT_UINT8": 4,
      "DT_INT16": 6, "DT_UINT16": 7, "DT_UINT32": 8, "DT_INT64": 9, "DT_UINT64": 10,
      "DT_DOUBLE": 11, "DT_BOOL": 12, "DT_STRING": 13, "DT_BF16": 27, "DT_UNDEFINED": 28}
FMT = {"FORMAT_NCHW": 0, "FORMAT_NHWC": 1, "FORMAT_ND": 2, "FORMAT_NC1HWC0": 3,
       "FORMAT_FRACTAL_Z": 4, "FORMAT_C1HWNC0": 9, "FORMAT_CHWN": 14, "FORMAT_HWCN": 16,
       "FORMAT_FRACTAL_ZZ": 28, "FORMAT_FRACTAL_NZ": 29, "FORMAT_RESERVED": 40}
_FMT_NAME = {v: k for k, v in FMT.items()}
# GE's generic FAILED and GRAPH_FAILED (external metadef headers): 0xFFFFFFFF.
STATUS = {"SUCCESS": 0, "FAILED": 0xFFFFFFFF, "GRAPH_FAILED": 0xFFFFFFFF,
          "ACL_ERROR_GE_PARAM_INVALID": 145000,
          "ACL_ERROR_GE_FORMAT_INVALID": 145020, "ACL_ERROR_GE_SHAPE_INVALID": 145021,
          "ACL_ERROR_GE_DATATYPE_INVALID": 145022}


@dataclass
class Args:
    name: str                 # variable name (args, args2, ...)
    data_var: Optional[str]   # array passed as data (None for nullptr)
    src_format: str           # primary formats (TransArgs::src/dst_primary_format)
    dst_format: str
    src_shape: List[int]
    dst_shape: List[int]
    dtype: str
    c0: List[int] = field(default_factory=list)
    src_sub: int = 0          # TransArgs::src_sub_format / dst_sub_format
    dst_sub: int = 0
    src_format_sub: int = 0   # sub format carried by the full src_format / dst_format
    dst_format_sub: int = 0


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
    # TransArgs variable -> name of the array its result is compared with
    outputs: Dict[str, str] = field(default_factory=dict)


def _nums(text: str):
    return [int(x) for x in re.findall(r"-?\d+", text)]


def _array_values(body: str, ctype: str) -> np.ndarray:
    body = re.sub(r"//[^\n]*", "", body)
    toks = [t for t in re.split(r"[,\s]+", body) if t]
    if _CTYPES[ctype] in (np.float32, np.float64):
        # A C++ double literal converted to float: parse as double, then round.
        return np.array([float(t) for t in toks], dtype=np.float64).astype(_CTYPES[ctype])
    return np.array([int(t, 0) for t in toks], dtype=np.int64).astype(_CTYPES[ctype])


def _split_tests(text: str):
    heads = list(re.finditer(r"TEST_F\(\s*\w+\s*,\s*(\w+)\s*\)\s*\{", text))
    for i, m in enumerate(heads):
        end = heads[i + 1].start() if i + 1 < len(heads) else len(text)
        yield m.group(1), text[m.end():end]


def _split_top(text: str) -> List[str]:
    """Splits at commas outside (), {} and <>."""
    out, depth, cur = [], 0, []
    for ch in text:
        if ch in "({<":
            depth += 1
        elif ch in ")}>":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur).strip())
    return out


def _symbols(body: str):
    """Integer and Format variables of one test body, and the (primary, sub)
    of every full format built with GetFormatFromSub / GetFormatFromSubAndC0."""
    sym, full = {}, {}

    def val(tok):
        tok = tok.strip()
        if tok in FMT:
            return FMT[tok]
        if re.fullmatch(r"-?\d+", tok):
            return int(tok)
        return sym.get(tok)

    for line in body.split(";"):
        line = " ".join(line.split())
        m = re.search(r"\b(?:int32_t|int64_t|int)\s+(\w+)\s*=\s*(-?\d+)$", line)
        if m:
            sym[m.group(1)] = int(m.group(2))
            continue
        m = re.search(r"Format\s+(\w+)\s*=\s*(FORMAT_\w+)$", line)
        if m:
            sym[m.group(1)] = FMT.get(m.group(2))
            continue
        m = re.search(r"(\w+)\s*=.*GetFormatFromSubAndC0\(\s*(\w+)\s*,\s*(\w+)\s*,\s*(\d+)\s*\)", line)
        if m:
            full[m.group(1)] = (val(m.group(2)), val(m.group(3)))
            continue
        m = re.search(r"(\w+)\s*=.*GetFormatFromSub\(\s*(\w+)\s*,\s*(\w+)\s*\)", line)
        if m:
            full[m.group(1)] = (val(m.group(2)), val(m.group(3)))
            continue
        m = re.search(r"(\w+)\s*=.*Get(Sub|Primary)Format\(\s*(?:static_cast<int32_t>\()?\s*(\w+)", line)
        if m and m.group(3) in full:
            sym[m.group(1)] = full[m.group(3)][1 if m.group(2) == "Sub" else 0]
    return sym, full, val


def _parse_args_positional(var: str, body: str, test_body: str) -> Optional[Args]:
    """TransArgs{data, src_format, dst_format, src_primary, dst_primary, src_sub,
    dst_sub, src_c0, dst_c0, src_shape, dst_shape, data_type} by position."""
    f = _split_top(body)
    if len(f) != 12:
        return None
    sym, full, val = _symbols(test_body)
    data = re.match(r"\s*(?:reinterpret_cast<uint8_t\s*\*>\(\s*(\w+)\s*\)|(\w+))", f[0])
    data_var = (data.group(1) or data.group(2)) if data else None
    prim = [val(f[3]), val(f[4])]
    if None in prim:
        return None
    shapes = [_nums(re.search(r"\{([-\d,\s]*)\}", x).group(1)) for x in (f[9], f[10])]
    subs = [val(f[5]) or 0, val(f[6]) or 0]
    fsub = [full.get(f[1].strip(), (None, 0))[1] or 0, full.get(f[2].strip(), (None, 0))[1] or 0]
    return Args(var, data_var, _FMT_NAME[prim[0]], _FMT_NAME[prim[1]], shapes[0], shapes[1],
                f[11].strip(), [int(f[7]), int(f[8])], subs[0], subs[1], fsub[0], fsub[1])


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
        for m in re.finditer(r"\b(uint8_t|int8_t|uint16_t|float|int32_t|int64_t|double)\s+(\w+)\s*"
                             r"\[([^\]]*)\]\s*=?\s*\{(.*?)\};", body, re.S):
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
            a = _parse_args_positional(m.group(1), m.group(2), body)
            args[m.group(1)] = a if a is not None else _parse_args(m.group(1), m.group(2))
        var_class = {v: k for k, v in re.findall(r"\b(FormatTransfer\w+)\s+(\w+)\s*;", body)}
        expects = []
        for m in re.finditer(r"EXPECT_EQ\(\s*((?:(?!EXPECT_EQ).)*?)\s*,\s*(SUCCESS|FAILED|GRAPH_FAILED|ACL_ERROR_GE_\w+)"
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
        result_of = {}
        for m in re.finditer(r"(?:\.TransFormat|TransDataFormat)\(\s*(\w+)\s*,\s*(\w+)\s*\)", body):
            result_of[m.group(2)] = m.group(1)
        outputs = {}
        for m in re.finditer(r"(\w+)\.data\.get\(\)\)\)\[i\]\s*,\s*(\w+)\[i\]", body):
            if m.group(1) in result_of and m.group(2) in arrays:
                outputs[result_of[m.group(1)]] = m.group(2)
        cases.append(Case(name, arrays, args, expects, outputs))
    return cases


def load(reference_root: Path, which: str) -> List[Case]:
    rel = {"nz": NZ_TEST, "zz": ZZ_TEST, "transpose": TRANSPOSE_TEST, **FZ_TESTS}[which]
    return parse(Path(reference_root) / rel)
