"""Pins the oracle's ND<->FRACTAL_NZ and transpose restatements to GE's golden vectors.

The vectors are read at test time from the reference's gtest sources
(format_transfer_fractal_nz_unittest.cc, format_transfer_transpose_unittest.cc)
by tests/golden/ge_goldens.py; the tests skip without the reference checkout.
Shape rules and size-independent properties are checked without it.
"""
import numpy as np
import pytest

import ge_goldens

# format_transfer_transpose.cc:26-43 (the perm table a transpose pair uses).
PERMS = {
    ("FORMAT_NCHW", "FORMAT_NHWC"): [0, 2, 3, 1], ("FORMAT_NCHW", "FORMAT_HWCN"): [2, 3, 1, 0],
    ("FORMAT_NCHW", "FORMAT_CHWN"): [1, 2, 3, 0], ("FORMAT_NHWC", "FORMAT_NCHW"): [0, 3, 1, 2],
    ("FORMAT_NHWC", "FORMAT_CHWN"): [3, 1, 2, 0], ("FORMAT_NHWC", "FORMAT_HWCN"): [1, 2, 3, 0],
    ("FORMAT_HWCN", "FORMAT_NCHW"): [3, 2, 0, 1], ("FORMAT_HWCN", "FORMAT_NHWC"): [3, 0, 1, 2],
    ("FORMAT_HWCN", "FORMAT_CHWN"): [2, 0, 1, 3], ("FORMAT_CHWN", "FORMAT_NCHW"): [3, 0, 1, 2],
    ("FORMAT_CHWN", "FORMAT_NHWC"): [3, 1, 2, 0], ("FORMAT_CHWN", "FORMAT_HWCN"): [1, 2, 0, 3],
}


@pytest.fixture(scope="module")
def nz_cases(reference_root):
    return ge_goldens.load(reference_root, "nz")


@pytest.fixture(scope="module")
def transpose_cases(reference_root):
    return ge_goldens.load(reference_root, "transpose")


def test_nz_golden_vectors(oracle, nz_cases):
    checked = 0
    for case in nz_cases:
        if "data" not in case.arrays or "ret" not in case.arrays:
            continue
        fwd = case.args["args"]
        data, ret = case.arrays["data"], case.arrays["ret"]
        w0 = fwd.dst_shape[-1]
        rc, nz, _ = oracle.nz_shape(fwd.src_shape, w0)
        assert rc == 0 and nz == fwd.dst_shape, case.name
        out = oracle.nd_to_nz_array(data.reshape(fwd.src_shape), w0)
        assert out.tobytes() == ret.tobytes(), case.name
        back = oracle.nz_to_nd_array(ret.reshape(fwd.dst_shape), fwd.src_shape, w0)
        assert back.tobytes() == data.tobytes(), case.name
        checked += 1
    assert checked == 5  # nd_shape4_fp16, nd_shape5_fp16, nd_shape4_fp32, nchw/nhwc fp32


def test_nz_golden_padding_is_zero(oracle, nz_cases):
    case = next(c for c in nz_cases if c.name == "nd_shape4_fp16")
    ret = case.arrays["ret"].reshape(2, 2, 1, 2, 16, 16)
    assert (ret[..., 17:, :] == 0).all() and (ret[..., 4:] == 0).all()


def test_transpose_golden_vectors(oracle, transpose_cases):
    checked = 0
    for case in transpose_cases:
        for e in case.expects:
            if e.call == "TransposeWithShapeCheck" and e.status == 0:
                sc = e.shape_call
                data, ret = case.arrays[sc["data"]], case.arrays["ret"]
                out = np.empty_like(ret)
                assert oracle.transpose(out, data, sc["src_shape"], sc["perm"],
                                        data.dtype.itemsize) == 0
                assert out.tobytes() == ret.tobytes(), case.name
                checked += 1
            elif e.call == "TransFormat" and e.status == 0:
                a = case.args[e.args]
                data, ret = case.arrays[a.data_var], case.arrays["ret"]
                perm = PERMS[(a.src_format, a.dst_format)]
                assert [a.src_shape[p] for p in perm] == a.dst_shape
                out = np.empty_like(ret)
                assert oracle.transpose(out, data, a.src_shape, perm, data.dtype.itemsize) == 0
                assert out.tobytes() == ret.tobytes(), case.name
                checked += 1
    assert checked >= 25


def test_transpose_2d_equals_run_tiles(oracle):
    # The standalone kernels' B[c, r] = A[r, c] is Transpose with perm {1, 0}.
    rows, cols = 64, 77
    a = oracle.fill_pattern(rows * cols)
    t_out = np.empty_like(a)
    assert oracle.transpose(t_out, a, [rows, cols], [1, 0], 4) == 0
    assert (oracle.transpose_rows_cols(a.reshape(rows, cols)).ravel() == t_out).all()


def test_transpose_invalid_args(oracle):
    a = np.zeros(8, dtype=np.uint8)
    out = np.zeros(8, dtype=np.uint8)
    assert oracle.transpose(out, a, [2, 4], [0, 0], 1) == oracle.EPARAM
    assert oracle.transpose(out, a, [2, 4], [0, 2], 1) == oracle.EPARAM
    assert oracle.transpose(out, a, [2, -4], [1, 0], 1) == oracle.EPARAM
    with pytest.raises(ValueError):
        oracle.transpose(out, a, [2, 4, 1], [1, 0], 1)  # perm and shape ranks differ


@pytest.mark.parametrize("shape,w0,expect", [
    ([2, 2, 17, 4], 16, [2, 2, 1, 2, 16, 16]),
    ([100], 16, [7, 1, 16, 16]),
    ([0], 16, [0, 1, 16, 16]),
    ([5, 33], 32, [2, 1, 16, 32]),
    ([3, 0, 7], 16, [3, 1, 0, 16, 16]),
    ([16, 4096, 4096], 16, [16, 256, 256, 16, 16]),
])
def test_nz_shape_rules(oracle, shape, w0, expect):
    rc, nz, hw = oracle.nz_shape(shape, w0)
    assert rc == 0 and nz == expect


def test_nz_shape_invalid(oracle):
    assert oracle.nz_shape([4, 4], -1)[0] == oracle.ESHAPE  # no C0 in the format -> -1
    assert oracle.nz_shape([1 << 21, 1 << 21], 16)[0] == oracle.ESHAPE  # > 2^40 items


@pytest.mark.parametrize("dtype", [np.uint8, np.uint16, np.uint32, np.uint64])
@pytest.mark.parametrize("shape", [[1], [15], [17, 3], [16, 16], [2, 33, 47], [3, 2, 5, 16],
                                   [40, 1], [1, 40]])
def test_nz_round_trip(oracle, dtype, shape):
    rng = np.random.default_rng(11)
    a = rng.integers(0, np.iinfo(dtype).max, size=shape, dtype=dtype, endpoint=True)
    w0 = 32 if np.dtype(dtype).itemsize == 1 else 16
    nz = oracle.nd_to_nz_array(a, w0)
    back = oracle.nz_to_nd_array(nz, shape, w0)
    assert back.tobytes() == a.tobytes()
    # Only padding positions are zero-filled: the NZ holds every ND element once.
    assert np.sort(nz.ravel())[-a.size:].tobytes() == np.sort(a.ravel()).tobytes()


def test_nz_threads_agree(oracle):
    rng = np.random.default_rng(12)
    a = rng.integers(0, 65535, size=(3, 100, 70), dtype=np.uint16)
    assert oracle.nd_to_nz_array(a, 16).tobytes() == oracle.nd_to_nz_array(a, 16, 5).tobytes()
    nz = oracle.nd_to_nz_array(a, 16)
    assert (oracle.nz_to_nd_array(nz, a.shape, 16, 6) == a).all()


# ---- ND <-> FRACTAL_ZZ --------------------------------------------------------------

@pytest.fixture(scope="module")
def zz_cases(reference_root):
    return ge_goldens.load(reference_root, "zz")


def _zz_numpy(a: np.ndarray, c0: int) -> np.ndarray:
    """FRACTAL_ZZ by array reshaping, independent of the C oracle: pad [.., H, W]
    to whole c0 x c0 blocks, split into [.., H1, c0, W1, c0], swap to
    [.., H1, W1, c0, c0]."""
    if a.ndim == 1:
        a = a.reshape(1, -1)
    *batch, h, w = a.shape
    h1, w1 = -(-h // c0), -(-w // c0)
    p = np.zeros((*batch, h1 * c0, w1 * c0), dtype=a.dtype)
    p[..., :h, :w] = a
    p = p.reshape(*batch, h1, c0, w1, c0)
    return np.ascontiguousarray(np.swapaxes(p, -3, -2))


def test_zz_golden_vectors(oracle, zz_cases):
    checked = 0
    for case in zz_cases:
        if "data" not in case.arrays or "ret" not in case.arrays:
            continue
        fwd = case.args["args"]
        data, ret = case.arrays["data"], case.arrays["ret"]
        c0 = fwd.c0[1]
        rc, zz, _ = oracle.zz_shape(fwd.src_shape, c0)
        assert rc == 0 and zz == fwd.dst_shape, case.name
        out = oracle.nd_to_zz_array(data.reshape(fwd.src_shape), c0)
        assert out.tobytes() == ret.tobytes(), case.name
        back = oracle.zz_to_nd_array(ret.reshape(fwd.dst_shape), fwd.src_shape, c0)
        assert back.tobytes() == data.tobytes(), case.name
        # The reshaping restatement agrees with GE's vectors too.
        assert _zz_numpy(data.reshape(fwd.src_shape), c0).tobytes() == ret.tobytes(), case.name
        checked += 1
    assert checked == 18  # every data-moving case of the ZZ unit test (uint8, fp16, fp32)


@pytest.mark.parametrize("shape,c0,expect", [
    ([1], 32, [1, 1, 32, 32]),
    ([100], 16, [1, 7, 16, 16]),
    ([0], 16, [1, 0, 16, 16]),
    ([30, 33], 32, [1, 2, 32, 32]),
    ([2, 3, 4, 33], 32, [2, 3, 1, 2, 32, 32]),
    ([3, 0, 7], 16, [3, 0, 1, 16, 16]),
    ([8, 4096, 4096], 16, [8, 256, 256, 16, 16]),
])
def test_zz_shape_rules(oracle, shape, c0, expect):
    rc, zz, hw = oracle.zz_shape(shape, c0)
    assert rc == 0 and zz == expect


def test_zz_shape_invalid(oracle):
    assert oracle.zz_shape([4, 4], -1)[0] == oracle.ESHAPE
    assert oracle.zz_shape([1 << 21, 1 << 21], 16)[0] == oracle.ESHAPE


@pytest.mark.parametrize("dtype", [np.uint8, np.uint16, np.uint32, np.uint64])
@pytest.mark.parametrize("shape", [[1], [15], [17, 3], [16, 16], [2, 33, 47], [3, 2, 5, 16],
                                   [40, 1], [1, 40]])
@pytest.mark.parametrize("c0", [4, 16, 32])
def test_zz_round_trip(oracle, dtype, shape, c0):
    rng = np.random.default_rng(13)
    a = rng.integers(0, np.iinfo(dtype).max, size=shape, dtype=dtype, endpoint=True)
    zz = oracle.nd_to_zz_array(a, c0)
    assert zz.tobytes() == _zz_numpy(a, c0).tobytes()
    assert oracle.zz_to_nd_array(zz, shape, c0).tobytes() == a.tobytes()
