"""GPU parity: the standalone_datacopy kernels (C ABI) vs the oracle's RunTiles, bit-exact.

Covers every shape of the reference's address-model tests plus ragged tails,
rows = 4088 and the 64 MiB maximum, store = 0 (output untouched), tilings read
from device memory, and the reference's validation failures.
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

CANARY = 0xA5


def _dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)).cuda()


def _canary(torch, nbytes):
    return torch.full((nbytes,), CANARY, dtype=torch.uint8, device="cuda")


def _host(t):
    return t.cpu().numpy()


SHAPES = [(256, 768, 8, 240), (8, 37, 1, 2), (128, 513, 4, 128), (4088, 19, 16, 240),
          (8, 1, 1, 240), (24, 100, 1, 7), (16, 255, 3, 5), (64, 1000, 1, 3), (72, 33, 2, 9)]


@pytest.mark.parametrize("rows,cols,small,large", SHAPES)
def test_small_large_pretranspose_bit_exact(torch_cuda, dcopy, oracle, rows, cols, small, large):
    torch = torch_cuda
    a = oracle.fill_pattern(rows * cols)  # asc:124-125 input[i] = i*17+3
    x = _dev(torch, a)
    for mode, kib in (("small", small), ("large", large)):
        t = dcopy.plan_tiling(rows, cols, kib, 1)
        ot = oracle.Tiling(*[getattr(t, f) for f in ("rows", "cols", "tile_cols", "ub_bytes",
                                                      "store")])
        expect = np.full(rows * cols, -0x5A5A5A5B, dtype=np.int32)
        assert oracle.run_tiles(0, a, expect, ot) == 0
        y = _canary(torch, a.nbytes)
        getattr(dcopy, f"datacopy_{mode}")(x, y, t)
        torch.cuda.synchronize()
        assert _host(y).tobytes() == expect.tobytes(), mode
    t = dcopy.plan_tiling(rows, cols, large, 1)
    b = _canary(torch, a.nbytes)
    y = _canary(torch, a.nbytes)
    dcopy.datacopy_pretranspose(x, b, t)
    dcopy.datacopy_contiguous(b, y, t)
    torch.cuda.synchronize()
    expect_b = a.reshape(rows, cols).T.copy()
    assert _host(b).tobytes() == expect_b.tobytes()
    assert _host(y).tobytes() == expect_b.tobytes()


def test_address_model_digests(torch_cuda, dcopy):
    """The GPU output hashes to the reference's own model() digest (input a[i] = i)."""
    import hashlib
    torch = torch_cuda
    for case in json.loads((GOLDEN / "address_model.json").read_text())["cases"]:
        rows, cols, kib = case["rows"], case["cols"], case["kib"]
        x = _dev(torch, np.arange(rows * cols, dtype=np.int32))
        t = dcopy.plan_tiling(rows, cols, kib, 1)
        y = _canary(torch, rows * cols * 4)
        if case["pretranspose"]:
            b = _canary(torch, rows * cols * 4)
            dcopy.datacopy_pretranspose(x, b, t)
            dcopy.datacopy_contiguous(b, y, t)
        else:
            dcopy.datacopy_small(x, y, t)
        torch.cuda.synchronize()
        assert hashlib.sha256(_host(y).tobytes()).hexdigest() == case["sha256"], case


def test_store0_leaves_y_untouched(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    rows, cols = 128, 513
    x = _dev(torch, oracle.fill_pattern(rows * cols))
    t = dcopy.plan_tiling(rows, cols, 4, 0)
    y = _canary(torch, rows * cols * 4)
    dcopy.datacopy_small(x, y, t)
    dcopy.datacopy_large(x, y, t)
    dcopy.datacopy_contiguous(x, y, t)
    torch.cuda.synchronize()
    assert (_host(y) == CANARY).all()
    # pretranspose always stores (asc:52).
    b = _canary(torch, rows * cols * 4)
    dcopy.datacopy_pretranspose(x, b, t)
    torch.cuda.synchronize()
    assert not (_host(b) == CANARY).all()


def test_max_input_64mib(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    rows, cols = 4088, 4104  # 67,108,608 bytes <= 64 MiB
    a = oracle.fill_pattern(rows * cols)
    t = dcopy.plan_tiling(rows, cols, 240, 1)
    x = _dev(torch, a)
    y = _canary(torch, a.nbytes)
    dcopy.datacopy_large(x, y, t)
    torch.cuda.synchronize()
    assert (_host(y).view(np.int32).reshape(cols, rows) == a.reshape(rows, cols).T).all()
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.plan_tiling(4088, 4105, 240, 1)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


def test_tiling_in_device_memory(torch_cuda, dcopy, oracle):
    import ctypes
    torch = torch_cuda
    rows, cols = 64, 300
    a = oracle.fill_pattern(rows * cols)
    t = dcopy.plan_tiling(rows, cols, 8, 1)
    td = torch.from_numpy(np.frombuffer(bytes(t), dtype=np.uint8).copy()).cuda()
    x = _dev(torch, a)
    y = _canary(torch, a.nbytes)
    rc = dcopy.lib().dcopy_datacopy_small(x.data_ptr(), y.data_ptr(),
                                          ctypes.cast(td.data_ptr(),
                                                      ctypes.POINTER(dcopy.DataCopyTiling)),
                                          None)
    assert rc == 0
    torch.cuda.synchronize()
    assert (_host(y).view(np.int32).reshape(cols, rows) == a.reshape(rows, cols).T).all()


def test_invalid_tilings_refused(torch_cuda, dcopy):
    torch = torch_cuda
    x = torch.zeros(64 * 100, dtype=torch.int32, device="cuda")
    y = torch.zeros_like(x)
    good = dcopy.plan_tiling(64, 100, 8, 1)
    for field, value in [("tile_cols", 0), ("tile_cols", 101), ("ub_bytes", good.ub_bytes - 4),
                         ("rows", 60), ("store", 2), ("cols", 0), ("rows", 4096)]:
        bad = dcopy.DataCopyTiling(good.rows, good.cols, good.tile_cols, good.ub_bytes, good.store)
        setattr(bad, field, value)
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.datacopy_small(x, y, bad)
        assert e.value.code == dcopy.ERR_PARAM_INVALID, field


def test_buffer_extent_checked(torch_cuda, dcopy, cuda_malloc):
    torch = torch_cuda
    t = dcopy.plan_tiling(64, 100, 8, 1)
    x = torch.zeros(64 * 100, dtype=torch.int32, device="cuda")
    with cuda_malloc(1 << 16) as small:
        # rows*cols*4 = 25600 bytes starting 64 bytes before the end of a 64 KiB
        # allocation would run past it: refused on the host, nothing launched.
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.datacopy_small(x, small + (1 << 16) - 64, t)
        assert e.value.code == dcopy.ERR_PARAM_INVALID
    host = np.zeros(64 * 100, dtype=np.int32)
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.datacopy_small(x, host.ctypes.data, t)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


@pytest.mark.parametrize("rows,cols,kib,parts", [(256, 768, 8, 3), (128, 513, 4, 5), (72, 33, 2, 2),
                                                  (4088, 19, 240, 1), (16, 255, 3, 7)])
def test_tile_ranges_compose(torch_cuda, dcopy, oracle, rows, cols, kib, parts):
    """The tiles split over `parts` shards (dcopy_shard_range, as GPUs or cores would take
    them), each run on its own: together they write exactly the whole result, for every
    phase; store = 0 shards write nothing."""
    torch = torch_cuda
    a = oracle.fill_pattern(rows * cols)
    x = _dev(torch, a)
    t = dcopy.plan_tiling(rows, cols, kib, 1)
    ntiles = -(-cols // t.tile_cols)
    expect = a.reshape(rows, cols).T.copy()
    y, b, y2 = _canary(torch, a.nbytes), _canary(torch, a.nbytes), _canary(torch, a.nbytes)
    for r in range(parts):
        begin, count = dcopy.shard_range(ntiles, r, parts)
        dcopy.datacopy_tiles(0, x, y, t, begin, count)
        dcopy.datacopy_tiles(1, x, b, t, begin, count)
    torch.cuda.synchronize()
    for r in reversed(range(parts)):
        begin, count = dcopy.shard_range(ntiles, r, parts)
        dcopy.datacopy_tiles(2, b, y2, t, begin, count)
    torch.cuda.synchronize()
    assert _host(y).tobytes() == expect.tobytes()
    assert _host(b).tobytes() == expect.tobytes()
    assert _host(y2).tobytes() == expect.tobytes()
    # One shard alone writes exactly its own columns.
    begin, count = dcopy.shard_range(ntiles, parts - 1, parts)
    y3 = _canary(torch, a.nbytes)
    dcopy.datacopy_tiles(0, x, y3, t, begin, count)
    torch.cuda.synchronize()
    c_lo = min(cols, begin * t.tile_cols)
    c_hi = min(cols, (begin + count) * t.tile_cols)
    got = _host(y3).view(np.int32).reshape(cols, rows)
    assert got[c_lo:c_hi].tobytes() == expect[c_lo:c_hi].tobytes()
    untouched = _host(_canary(torch, a.nbytes)).view(np.int32).reshape(cols, rows)
    assert got[:c_lo].tobytes() == untouched[:c_lo].tobytes()
    assert got[c_hi:].tobytes() == untouched[c_hi:].tobytes()
    t0 = dcopy.plan_tiling(rows, cols, kib, 0)
    y4 = _canary(torch, a.nbytes)
    dcopy.datacopy_tiles(0, x, y4, t0, 0, ntiles)
    torch.cuda.synchronize()
    assert _host(y4).tobytes() == untouched.tobytes()
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.datacopy_tiles(0, x, y, t, ntiles, 1)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
