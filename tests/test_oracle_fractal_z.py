"""Pins the oracle's FRACTAL_Z restatement to GE's golden vectors.

Every data-moving case of GE's seven FRACTAL_Z unit tests (HWCN / NCHW / NHWC /
ND -> FRACTAL_Z including the groups layout, FRACTAL_Z -> NCHW / HWCN / NHWC)
is replayed through the oracle: the shape derivation must give the test's
destination shape and the bytes must equal the test's expected array.  The
vectors are read at test time from the reference's gtest sources by
tests/golden/ge_goldens.py; the tests skip without the reference checkout.
"""
import numpy as np
import pytest

import ge_goldens

FORWARD = {"hwcn_fz": 16, "nchw_fz": 0, "nhwc_fz": 1, "nd_fz": 2}
REVERSE = {"fz_nchw": 0, "fz_hwcn": 16, "fz_nhwc": 1}


def _data_cases(reference_root, which):
    for case in ge_goldens.load(reference_root, which):
        for var, out_name in case.outputs.items():
            yield case, case.args[var], case.arrays[case.args[var].data_var], case.arrays[out_name]


@pytest.mark.parametrize("which", sorted(FORWARD))
def test_to_fractal_z_golden_vectors(oracle, reference_root, which):
    fmt = FORWARD[which]
    checked = 0
    for case, a, data, expect in _data_cases(reference_root, which):
        c0 = a.c0[1]
        # TransShape reads the groups from the full destination format.
        rc, shape = oracle.fz_shape(fmt, a.src_shape, c0, a.dst_format_sub)
        assert rc == 0 and shape == a.dst_shape, (case.name, rc, shape)
        src = data[:int(np.prod(a.src_shape))].reshape(a.src_shape)
        # The transfer reads them from TransArgs::dst_sub_format.
        out = oracle.to_fz(src, fmt, c0, a.dst_sub)
        assert out.tobytes() == expect.tobytes(), case.name
        checked += 1
    assert checked == {"hwcn_fz": 8, "nchw_fz": 9, "nhwc_fz": 5, "nd_fz": 1}[which]


@pytest.mark.parametrize("which", sorted(REVERSE))
def test_from_fractal_z_golden_vectors(oracle, reference_root, which):
    fmt = REVERSE[which]
    checked = 0
    for case, a, data, expect in _data_cases(reference_root, which):
        c0 = a.c0[0]
        assert oracle.from_fz_check(a.src_shape, fmt, a.dst_shape, c0) == 0, case.name
        src = data[:int(np.prod(a.src_shape))].reshape(a.src_shape)
        out = oracle.from_fz(src, fmt, a.dst_shape, c0)
        assert out.tobytes() == expect[:out.size].tobytes(), case.name
        checked += 1
    assert checked == {"fz_nchw": 11, "fz_hwcn": 8, "fz_nhwc": 5}[which]


def _numpy_fz(w: np.ndarray, fmt: int, c0: int) -> np.ndarray:
    """FRACTAL_Z by array reshaping, independent of the C oracle."""
    n, c, h, ww = {0: lambda s: (s[0], s[1], s[2], s[3]), 1: lambda s: (s[0], s[3], s[1], s[2]),
                   16: lambda s: (s[3], s[2], s[0], s[1]),
                   2: lambda s: (s[1], s[0], 1, 1)}[fmt](w.shape)
    nchw = {0: lambda a: a, 1: lambda a: a.transpose(0, 3, 1, 2),
            16: lambda a: a.transpose(3, 2, 0, 1),
            2: lambda a: a.T.reshape(n, c, 1, 1)}[fmt](w)
    c1, n1 = -(-c // c0), -(-n // 16)
    p = np.zeros((n1 * 16, c1 * c0, h, ww), dtype=w.dtype)
    p[:n, :c] = nchw
    # [n1n0, c1, c0, h, w] -> [c1, h, w, n1n0, c0]
    return np.ascontiguousarray(p.reshape(n1 * 16, c1, c0, h, ww).transpose(1, 3, 4, 0, 2))


@pytest.mark.parametrize("fmt", [0, 1, 16, 2])
@pytest.mark.parametrize("shape", [[1, 1, 1, 1], [17, 5, 3, 3], [33, 64, 1, 1], [16, 16, 2, 2],
                                   [5, 40, 4, 7]])
@pytest.mark.parametrize("dtype,c0", [(np.uint16, 16), (np.uint8, 32), (np.float32, 16),
                                      (np.float32, 8)])
def test_fractal_z_round_trip(oracle, fmt, shape, dtype, c0):
    if fmt == 2:
        shape = [shape[1] * shape[2], shape[0]]  # ND [C, N]
    elif fmt == 1:
        shape = [shape[0], shape[2], shape[3], shape[1]]
    elif fmt == 16:
        shape = [shape[2], shape[3], shape[1], shape[0]]
    rng = np.random.default_rng(sum(shape) + c0)
    w = rng.integers(0, 250, size=shape).astype(dtype)
    fz = oracle.to_fz(w, fmt, c0)
    assert fz.tobytes() == _numpy_fz(w, fmt, c0).tobytes()
    if fmt != 2:  # FRACTAL_Z -> ND is not registered
        rc, fz_shape = oracle.fz_shape(fmt, shape, c0)
        back = oracle.from_fz(fz.reshape(fz_shape), fmt, shape, c0)
        assert back.tobytes() == w.tobytes()


def test_fractal_z_shape_rules(oracle):
    assert oracle.fz_shape(0, [1, 1, 1, 1], 16, 40)[0] == oracle.EFAILED  # cout = 1 / 40 = 0
    assert oracle.fz_shape(0, [4, 3, 2, 2], 16, 2) == (0, [4, 1, 16, 16])
    assert oracle.fz_shape(16, [3, 3, 4, 8], 16, 2) == (0, [9, 1, 16, 16])
    assert oracle.fz_shape(1, [1, 4, 4], 16)[0] == oracle.ESHAPE
    assert oracle.fz_shape(0, [1, 1, 1, 1], -1)[0] == oracle.EDTYPE
    assert oracle.fz_shape(2, [1, 4, 4], 16)[0] == oracle.EFAILED  # TBE: 2-D only
    assert oracle.fz_shape(2, [4, 4], 0)[0] == oracle.EFAILED
    assert oracle.fz_shape(14, [1, 1, 4, 4], 16)[0] == oracle.EFORMAT
