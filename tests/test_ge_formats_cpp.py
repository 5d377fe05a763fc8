"""Builds and runs tests/cpp/test_ge_formats.cpp: GE-style C++ use of
include/dcopy/ge_formats.hpp (host buffers, GE status codes) against the oracle."""
import subprocess

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def test_binary(dcopy, oracle, tmp_path_factory):
    out = tmp_path_factory.mktemp("ge_cpp") / "test_ge_formats"
    lib = ROOT / "data-copy_b200" / "dcopy"
    orc = ROOT / "oracle" / "_build"
    cmd = ["nvcc", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", str(ROOT / "oracle"),
           str(ROOT / "tests" / "cpp" / "test_ge_formats.cpp"), "-o", str(out),
           "-L", str(lib), "-ldcopy", "-L", str(orc), "-loracle",
           "-Xlinker", f"-rpath,{lib}", "-Xlinker", f"-rpath,{orc}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return out


def test_host_side_statuses(test_binary):
    r = subprocess.run([str(test_binary), "--host-only"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("PASS")


@pytest.mark.gpu
def test_round_trips_on_gpu(test_binary, torch_cuda):
    r = subprocess.run([str(test_binary)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("PASS")
