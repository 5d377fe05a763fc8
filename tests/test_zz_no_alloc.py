"""The allocation-free pretranspose entry point, checked against the entry points
that take a caller-allocated B buffer.

dcopy_datacopy_pretranspose_noalloc serves callers that cannot allocate device
memory (a runtime that owns the whole device-memory budget, or a latency-critical
path where cudaMalloc would synchronise the device): it keeps B in the library's
own 16 MiB device array.  Its first call on a device looks the array up, so this
file also runs alone in a fresh process; pytest collects it last, so a run that
stops at the first failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(dcopy):
    fn = dcopy.lib().dcopy_datacopy_pretranspose_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(dcopy.DataCopyTiling),
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _reference_output(torch, dcopy, x, t):
    """The same workflow through the existing entry points, B allocated here."""
    b = torch.empty_like(x)
    y = torch.full_like(x, -1)
    dcopy.datacopy_pretranspose(x, b, t)
    dcopy.datacopy_contiguous(b, y, t)
    return y


@pytest.mark.parametrize("calls", [[(256, 768, 240, 1), (256, 768, 240, 2), (128, 513, 4, 3)]])
def test_noalloc_matches_caller_buffer_entry_points(torch_cuda, dcopy, calls):
    torch = torch_cuda
    fn = _noalloc(dcopy)
    stream = torch.cuda.current_stream().cuda_stream or None
    for rows, cols, kib, seed in calls:  # two calls in a row on one shape, then another shape
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = torch.randint(-2**31, 2**31 - 1, (rows * cols,), dtype=torch.int32, device="cuda",
                          generator=g)
        t = dcopy.plan_tiling(rows, cols, kib, 1)
        expect = _reference_output(torch, dcopy, x, t)
        y = torch.full_like(x, -1)
        rc = fn(x.data_ptr(), y.data_ptr(), ctypes.byref(t), stream)
        assert rc == 0, dcopy.lib().dcopy_last_error_message()
        torch.cuda.synchronize()
        assert torch.equal(y, expect)  # bit-exact, the tolerance of every copy test here
        assert torch.equal(y.view(cols, rows), x.view(rows, cols).t())


def test_noalloc_refuses_shapes_beyond_its_array(torch_cuda, dcopy):
    torch = torch_cuda
    fn = _noalloc(dcopy)
    t = dcopy.plan_tiling(4088, 1100, 240, 1)  # 17.2 MB > 16 MiB
    x = torch.zeros(4088 * 1100, dtype=torch.int32, device="cuda")
    y = torch.zeros_like(x)
    assert fn(x.data_ptr(), y.data_ptr(), ctypes.byref(t), None) == dcopy.ERR_PARAM_INVALID
    assert b"16777216-byte static B buffer" in dcopy.lib().dcopy_last_error_message()


def test_noalloc_store0_leaves_y_untouched(torch_cuda, dcopy):
    """With store = 0 the workflow writes only the library's array, never y (as
    dcopy_datacopy_contiguous with store = 0); two calls in a row."""
    torch = torch_cuda
    fn = _noalloc(dcopy)
    rows, cols = 256, 768
    x = torch.arange(rows * cols, dtype=torch.int32, device="cuda")
    t = dcopy.plan_tiling(rows, cols, 240, 0)
    y = torch.full_like(x, -0x5A5A5A5B)
    for _ in range(2):
        assert fn(x.data_ptr(), y.data_ptr(), ctypes.byref(t), None) == 0
        torch.cuda.synchronize()
        assert bool((y == -0x5A5A5A5B).all())
    # A store = 1 call right after still gives the transpose.
    t1 = dcopy.plan_tiling(rows, cols, 240, 1)
    assert fn(x.data_ptr(), y.data_ptr(), ctypes.byref(t1), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(y.view(cols, rows), x.view(rows, cols).t())


def test_noalloc_on_a_second_device(torch_cuda, dcopy):
    """Each device has its own copy of the array, looked up with that device current."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    fn = _noalloc(dcopy)
    rows, cols = 128, 513
    t = dcopy.plan_tiling(rows, cols, 4, 1)
    outs = []
    for dev in (1, 0, 1):
        with torch.cuda.device(dev):
            x = torch.arange(rows * cols, dtype=torch.int32, device=f"cuda:{dev}") * 7 + dev
            y = torch.full_like(x, -1)
            stream = torch.cuda.current_stream(dev).cuda_stream or None
            assert fn(x.data_ptr(), y.data_ptr(), ctypes.byref(t), stream) == 0, \
                dcopy.lib().dcopy_last_error_message()
            torch.cuda.synchronize(dev)
            assert torch.equal(y.view(cols, rows), x.view(rows, cols).t())
            outs.append(y.cpu())
    assert torch.equal(outs[0], outs[2])
