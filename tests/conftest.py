"""Shared pytest setup: import paths, the `gpu` marker and session fixtures."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "data-copy_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

# Reference checkout, only present where the golden vectors can be re-read: the
# directory DCOPY_REFERENCE names, else a checkout called `reference` beside this
# repository.  Tests that need it skip when neither exists.
REFERENCE = Path(os.environ.get("DCOPY_REFERENCE") or (ROOT.parent / "reference"))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def reference_root():
    if not (REFERENCE / "ge-develop").is_dir():
        pytest.skip("reference checkout not present")
    return REFERENCE


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    O.lib()
    return O


@pytest.fixture(scope="session")
def dcopy():
    import dcopy as D
    D.lib()
    return D


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch


@pytest.fixture(scope="session")
def cuda_malloc(torch_cuda):
    """Context manager giving a raw cudaMalloc'd device address (exact-size allocation)."""
    import contextlib
    import ctypes

    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
    rt.cudaFree.argtypes = [ctypes.c_void_p]

    @contextlib.contextmanager
    def alloc(nbytes):
        p = ctypes.c_void_p()
        assert rt.cudaMalloc(ctypes.byref(p), nbytes) == 0
        try:
            yield p.value
        finally:
            torch_cuda.cuda.synchronize()
            rt.cudaFree(p)

    return alloc
