"""Randomised GPU parity: seeded random shapes, strides, element widths and base
offsets for every entry point, each result compared byte for byte with the
oracle (canary-filled destinations: bytes the reference does not write must
keep their canary).  Shapes stay small so the oracle finishes in milliseconds;
the seeds make every case reproducible.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5
DT = {1: 4, 2: 1, 4: 0, 8: 9, 16: 17}  # element bytes -> a GE data type of that size


def _bytes(n, rng):
    return rng.integers(0, 256, size=n, dtype=np.uint8)


@pytest.mark.parametrize("seed", range(80))
def test_transpose_random(torch_cuda, dcopy, oracle, seed):
    torch = torch_cuda
    rng = np.random.default_rng(5000 + seed)
    rank = int(rng.integers(2, 6))
    eb = int(rng.choice([1, 2, 4, 8, 16]))
    shape = [int(rng.integers(1, 24)) for _ in range(rank)]
    while int(np.prod(shape)) * eb > (1 << 20):
        shape[int(np.argmax(shape))] //= 2
    perm = [int(p) for p in rng.permutation(rank)]
    off_s, off_d = int(rng.integers(0, 16 // eb + 1)) * eb, int(rng.integers(0, 16 // eb + 1)) * eb
    n = int(np.prod(shape)) * eb
    src_np = _bytes(n + off_s, rng)
    expect = np.empty(n, dtype=np.uint8)
    assert oracle.transpose(expect, src_np[off_s:], shape, perm, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((n + off_d + 32,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.transpose(dst.data_ptr() + off_d, src.data_ptr() + off_s, shape, perm, DT[eb])
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[off_d:off_d + n].tobytes() == expect.tobytes(), (shape, perm, eb)
    assert (out[:off_d] == CANARY).all() and (out[off_d + n:] == CANARY).all()


@pytest.mark.parametrize("seed", range(80))
def test_copy_ext_random(torch_cuda, dcopy, oracle, seed):
    torch = torch_cuda
    rng = np.random.default_rng(6000 + seed)
    count = int(rng.integers(1, 600))
    blen = int(rng.choice([int(rng.integers(1, 300)), 16 * int(rng.integers(1, 64))]))
    sgap, dgap = int(rng.integers(0, 200)), int(rng.integers(0, 50))
    soff, doff = int(rng.integers(0, 32)), int(rng.integers(0, 32))
    src_span = (count - 1) * (blen + sgap) + blen
    dst_span = (count - 1) * (blen + dgap) + blen
    src_np = _bytes(src_span + soff, rng)
    expect = np.full(dst_span + doff + 32, CANARY, dtype=np.uint8)
    oracle.copy_ext(expect[doff:], src_np[soff:], count, blen, sgap, dgap)
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_ext(dst.data_ptr() + doff, src.data_ptr() + soff, count, blen, sgap, dgap)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes(), (count, blen, sgap, dgap, soff, doff)


@pytest.mark.parametrize("seed", range(80))
def test_copy_nd_random(torch_cuda, dcopy, oracle, seed):
    """Random boxes: destination strides are a padded dense layout in a random axis
    order (no two elements share a destination), source strides are arbitrary
    (broadcast axes and overlapping reads included)."""
    torch = torch_cuda
    rng = np.random.default_rng(7000 + seed)
    ndim = int(rng.integers(1, 6))
    eb = int(rng.choice([1, 2, 4, 8, 16]))
    sizes = [int(rng.integers(1, 12)) for _ in range(ndim)]
    sizes[-1] = int(rng.integers(1, 80))
    order = [int(k) for k in rng.permutation(ndim)]  # innermost first in the destination
    if rng.random() < 0.6:  # mostly keep the innermost axis innermost (the row paths)
        order = [ndim - 1] + [k for k in order if k != ndim - 1]
    ds = [0] * ndim
    step = 1
    for k in order:
        ds[k] = step
        step *= sizes[k] + int(rng.integers(0, 3))
    ss = [int(rng.integers(0, 3)) if rng.random() < 0.1 else 0 for _ in range(ndim)]
    step = 1
    for k in reversed(range(ndim)):
        if ss[k] == 0 and rng.random() < 0.1 and k != ndim - 1:
            continue  # a broadcast source axis
        ss[k] = step if k == ndim - 1 and rng.random() < 0.8 else step + int(rng.integers(0, 3))
        step = ss[k] * sizes[k] + int(rng.integers(0, 5))
    soff, doff = int(rng.integers(0, 16 // eb + 1)) * eb, int(rng.integers(0, 16 // eb + 1)) * eb
    src_elems = sum((s - 1) * st for s, st in zip(sizes, ss)) + 1
    dst_elems = sum((s - 1) * st for s, st in zip(sizes, ds)) + 1
    src_np = _bytes(src_elems * eb + soff, rng)
    expect = np.full(dst_elems * eb + doff + 32, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(expect[doff:], src_np[soff:], sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_nd(dst.data_ptr() + doff, src.data_ptr() + soff, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes(), (sizes, ss, ds, eb)


NZ_KINDS = [(2, 16), (1, 32), (4, 16), (4, 8), (8, 16), (2, 8)]  # (element bytes, W0 / C0)


@pytest.mark.parametrize("seed", range(40))
def test_nz_zz_random(torch_cuda, dcopy, oracle, seed):
    torch = torch_cuda
    rng = np.random.default_rng(8000 + seed)
    eb, w0 = NZ_KINDS[seed % len(NZ_KINDS)]
    rank = int(rng.integers(1, 5))
    shape = [int(rng.integers(1, 5)) for _ in range(rank - 2)] + \
            [int(rng.integers(1, 70)) for _ in range(min(rank, 2))]
    src_np = _bytes(int(np.prod(shape)) * eb, rng)
    src = torch.from_numpy(src_np).cuda()
    for kind in ("nz", "zz"):
        if kind == "nz":
            rc, fr, _ = oracle.nz_shape(shape, w0)
            to_o, to_g, back_g = oracle.nd_to_nz, dcopy.nd_to_nz, dcopy.nz_to_nd
        else:
            if eb * w0 > 64:
                continue
            rc, fr, _ = oracle.zz_shape(shape, w0)
            to_o, to_g, back_g = oracle.nd_to_zz, dcopy.nd_to_zz, dcopy.zz_to_nd
        assert rc == 0
        nbytes = int(np.prod(fr)) * eb
        expect = np.empty(nbytes, dtype=np.uint8)
        assert to_o(expect, src_np, shape, eb, w0) == 0
        dst = torch.full((nbytes,), CANARY, dtype=torch.uint8, device="cuda")
        to_g(dst, src, shape, eb, w0)
        back = torch.full((src_np.size,), CANARY, dtype=torch.uint8, device="cuda")
        back_g(back, dst, shape, eb, w0)
        torch.cuda.synchronize()
        assert dst.cpu().numpy().tobytes() == expect.tobytes(), (kind, shape, eb, w0)
        assert back.cpu().numpy().tobytes() == src_np.tobytes(), (kind, shape, eb, w0)


NCHW, NHWC, HWCN = 0, 1, 16
FZ_KINDS = [(2, 16), (1, 32), (4, 16), (4, 8)]


@pytest.mark.parametrize("seed", range(40))
def test_fractal_z_random(torch_cuda, dcopy, oracle, seed):
    torch = torch_cuda
    rng = np.random.default_rng(9000 + seed)
    eb, c0 = FZ_KINDS[seed % len(FZ_KINDS)]
    fmt = [NCHW, NHWC, HWCN][(seed // len(FZ_KINDS)) % 3]
    n, c = int(rng.integers(1, 40)), int(rng.integers(1, 70))
    h, w = int(rng.integers(1, 6)), int(rng.integers(1, 6))
    shape = {NCHW: [n, c, h, w], NHWC: [n, h, w, c], HWCN: [h, w, c, n]}[fmt]
    dtype = {1: np.uint8, 2: np.uint16, 4: np.uint32}[eb]
    src_np = _bytes(n * c * h * w * eb, rng)
    expect = oracle.to_fz(src_np.view(dtype).reshape(shape), fmt, c0)
    fz = torch.full((expect.nbytes,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(fz, torch.from_numpy(src_np).cuda(), fmt, shape, eb, c0)
    back = torch.full((src_np.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.from_fractal_z(back, fz, fmt, shape, eb, c0)
    torch.cuda.synchronize()
    assert fz.cpu().numpy().tobytes() == expect.tobytes(), (fmt, shape, eb, c0)
    assert back.cpu().numpy().tobytes() == src_np.tobytes(), (fmt, shape, eb, c0)
