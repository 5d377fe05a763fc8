"""GPU parity for the GE TransData-level entry points (C ABI) vs the oracle, bit-exact.

Shapes follow GE's format-transfer tests (the oracle is pinned to their golden
vectors on the CPU side); data is random so every byte position is checked.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = {"NCHW": 0, "NHWC": 1, "ND": 2, "CHWN": 14, "HWCN": 16, "FRACTAL_NZ": 29}
DT = {1: ("FLOAT16", 2), 0: ("FLOAT", 4), 9: ("INT64", 8), 2: ("INT8", 1)}
PERMS = {  # format_transfer_transpose.cc:26-43
    ("NCHW", "NHWC"): [0, 2, 3, 1], ("NCHW", "HWCN"): [2, 3, 1, 0], ("NCHW", "CHWN"): [1, 2, 3, 0],
    ("NHWC", "NCHW"): [0, 3, 1, 2], ("NHWC", "CHWN"): [3, 1, 2, 0], ("NHWC", "HWCN"): [1, 2, 3, 0],
    ("HWCN", "NCHW"): [3, 2, 0, 1], ("HWCN", "NHWC"): [3, 0, 1, 2], ("HWCN", "CHWN"): [2, 0, 1, 3],
    ("CHWN", "NCHW"): [3, 0, 1, 2], ("CHWN", "NHWC"): [3, 1, 2, 0], ("CHWN", "HWCN"): [1, 2, 0, 3],
}


def _rand(nbytes, seed):
    return np.random.default_rng(seed).integers(0, 256, size=nbytes, dtype=np.uint8)


@pytest.mark.parametrize("src_fmt,shape,dt", [
    ("ND", [2, 2, 17, 4], 1), ("ND", [2, 2, 2, 17, 4], 1), ("ND", [2, 2, 17, 4], 0),
    ("NCHW", [2, 2, 17, 4], 0), ("NHWC", [2, 2, 4, 17], 0), ("ND", [100], 1),
    ("ND", [3, 64, 96], 2), ("ND", [5, 33, 70], 9)])
def test_trans_data_format_nz_round_trip(torch_cuda, dcopy, oracle, src_fmt, shape, dt):
    torch = torch_cuda
    eb = DT[dt][1]
    c0 = 32 if eb == 1 else 16
    rc, nz, _ = oracle.nz_shape(shape, c0)
    nd_np = _rand(int(np.prod(shape)) * eb, sum(shape))
    expect = np.empty(int(np.prod(nz)) * eb, dtype=np.uint8)
    assert oracle.nd_to_nz(expect, nd_np, shape, eb, c0) == 0
    src = torch.from_numpy(nd_np).cuda()
    dst = torch.full((expect.size,), 0xA5, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_data_format(dst, src, F[src_fmt], F["FRACTAL_NZ"], shape, nz, dt, dst.numel(),
                                dst_c0=c0)
    torch.cuda.synchronize()
    assert n == expect.size and dst.cpu().numpy().tobytes() == expect.tobytes()
    back = torch.full((nd_np.size,), 0xA5, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_data_format(back, dst, F["FRACTAL_NZ"], F[src_fmt], nz, shape, dt,
                                back.numel(), src_c0=c0)
    torch.cuda.synchronize()
    assert n == nd_np.size and back.cpu().numpy().tobytes() == nd_np.tobytes()


@pytest.mark.parametrize("pair", sorted(PERMS), ids=lambda p: f"{p[0]}->{p[1]}")
@pytest.mark.parametrize("shape", [[1, 2, 3, 4], [2, 3, 4, 5], [8, 3, 16, 16], [3, 1, 7, 9]])
def test_trans_data_format_transpose(torch_cuda, dcopy, oracle, pair, shape):
    torch = torch_cuda
    perm = PERMS[pair]
    src_np = np.random.default_rng(sum(shape)).integers(0, 65535, size=shape, dtype=np.uint16)
    dst_shape = [shape[p] for p in perm]
    expect = np.empty(dst_shape, dtype=np.uint16)
    assert oracle.transpose(expect, src_np, shape, perm, 2) == 0
    src = torch.from_numpy(src_np.view(np.int16)).cuda()
    dst = torch.full(dst_shape, -1, dtype=torch.int16, device="cuda")
    n = dcopy.trans_data_format(dst, src, F[pair[0]], F[pair[1]], shape, dst_shape, 1,
                                dst.numel() * 2)
    torch.cuda.synchronize()
    assert n == expect.nbytes and dst.cpu().numpy().tobytes() == expect.tobytes()


@pytest.mark.parametrize("shape,perm,eb", [
    ([1, 1, 1, 1], [3, 2, 1, 0], 1), ([1, 1, 1, 5], [2, 1, 0, 3], 1), ([2, 2], [1, 0], 1),
    ([1, 3, 4, 4], [2, 3, 1, 0], 2), ([8, 3, 16, 16], [2, 3, 1, 0], 2),
    ([8, 8, 1, 1], [3, 2, 0, 1], 2), ([4, 4, 3, 16], [3, 2, 0, 1], 2),
    ([1, 3, 16, 16], [0, 2, 3, 1], 2), ([8, 1, 24, 24], [0, 2, 3, 1], 4),
    ([1, 24, 24, 3], [0, 3, 1, 2], 4), ([3, 5, 7, 2, 4], [4, 0, 3, 1, 2], 8),
    ([33, 65], [1, 0], 16)])
def test_transpose_with_shape_check(torch_cuda, dcopy, oracle, shape, perm, eb):
    torch = torch_cuda
    dt = {1: 4, 2: 1, 4: 0, 8: 9, 16: 17}[eb]
    src_np = _rand(int(np.prod(shape)) * eb, len(shape) * 7 + eb)
    dst_shape = [shape[p] for p in perm]
    expect = np.empty(src_np.size, dtype=np.uint8)
    assert oracle.transpose(expect, src_np, shape, perm, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((src_np.size,), 0xA5, dtype=torch.uint8, device="cuda")
    dcopy.transpose_with_shape_check(dst, src, shape, dst_shape, perm, dt)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


def test_large_nchw_to_nhwc(torch_cuda, dcopy):
    torch = torch_cuda
    x = torch.randn(8, 64, 128, 128, device="cuda", dtype=torch.float16)
    y = torch.empty(8, 128, 128, 64, device="cuda", dtype=torch.float16)
    dcopy.trans_data_format(y, x, F["NCHW"], F["NHWC"], list(x.shape), list(y.shape), 1,
                            y.numel() * 2)
    torch.cuda.synchronize()
    assert torch.equal(y, x.permute(0, 2, 3, 1))
