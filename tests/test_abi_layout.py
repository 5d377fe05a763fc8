"""The ctypes records of the Python binding have the C ABI's layout: a small C
program compiled here against include/dcopy/dcopy.h prints sizeof and every
field's offset, and each must match the binding's ctypes.Structure."""
import ctypes
import json
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

STRUCTS = {
    "DataCopyTiling": ["rows", "cols", "tile_cols", "ub_bytes", "store"],
    "DcopyExtParams": ["blockCount", "blockLen", "srcStride", "dstStride"],
    "DcopyExtCopy": ["dst", "src", "params"],
    "DcopyLoopModeParams": ["loop1Size", "loop2Size", "loop1SrcStride", "loop1DstStride",
                            "loop2SrcStride", "loop2DstStride"],
    "DcopyMemcpyInfo": ["dst", "destMax", "src", "cnt"],
    "DcopyPadParams": ["isPad", "leftPadding", "rightPadding", "reserved", "elemBytes",
                       "paddingValue"],
    "DcopyDevCopy": ["device", "dst", "src", "params", "stream"],
    "DcopyTransArgs": ["data", "src_format", "dst_format", "src_c0", "dst_c0", "src_shape",
                       "src_rank", "dst_shape", "dst_rank", "data_type", "src_sub_format",
                       "dst_sub_format"],
}


def _c_layout(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "dcopy/dcopy.h"',
             'int main(void) {', '  printf("{");']
    first = True
    for name, fields in STRUCTS.items():
        sep = "" if first else ","
        first = False
        offs = ", ".join(f'\\"{f}\\": %zu' for f in fields)
        args = ", ".join(f"offsetof({name}, {f})" for f in fields)
        lines.append(f'  printf("{sep}\\"{name}\\": {{\\"size\\": %zu, {offs}}}", sizeof({name}), {args});')
    lines += ['  printf("}\\n");', '  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    return json.loads(subprocess.run([str(exe)], check=True, capture_output=True,
                                     text=True).stdout)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_records_match_the_c_abi(dcopy, tmp_path):
    c = _c_layout(tmp_path)
    for name, fields in STRUCTS.items():
        py = getattr(dcopy, name)
        assert ctypes.sizeof(py) == c[name]["size"], name
        for f in fields:
            assert getattr(py, f).offset == c[name][f], (name, f)
