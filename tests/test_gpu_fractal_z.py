"""GPU parity: FRACTAL_Z (convolution weight) transfers through the C ABI vs the
oracle, bit-exact.

The oracle's FRACTAL_Z restatement is pinned to every data-moving golden vector
of GE's seven FRACTAL_Z unit tests on the CPU side; here the GPU is checked
against it with random bytes: NCHW / NHWC / HWCN / ND sources and the three
FRACTAL_Z -> weight directions, every element width, ragged N and C (padding),
1x1 and 3x3 kernels, the HWCN group layout, unaligned base addresses, and the
GE-level transfer classes.  Destinations are canary-filled around the written
range.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5
NCHW, NHWC, ND, HWCN = 0, 1, 2, 16

WEIGHTS = [  # (N, C, H, W)
    (1, 1, 1, 1), (16, 16, 1, 1), (17, 5, 3, 3), (64, 64, 3, 3), (33, 70, 1, 1),
    (5, 40, 4, 7), (128, 3, 7, 7), (31, 17, 4, 4), (2, 300, 2, 2), (40, 33, 5, 5),
    (20, 32, 11, 11), (20, 16, 15, 15), (48, 64, 1, 1),
]


def _shape(fmt, n, c, h, w):
    return {NCHW: [n, c, h, w], NHWC: [n, h, w, c], HWCN: [h, w, c, n], ND: [c * h * w, n]}[fmt]


def _rand(nbytes, seed):
    return np.random.default_rng(seed).integers(0, 256, size=nbytes, dtype=np.uint8)


def _as(arr, eb):
    return arr.view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[eb])


@pytest.mark.parametrize("fmt", [NCHW, NHWC, HWCN, ND], ids=["NCHW", "NHWC", "HWCN", "ND"])
@pytest.mark.parametrize("eb,c0", [(2, 16), (1, 32), (4, 16), (4, 8), (8, 4)])
@pytest.mark.parametrize("weight", WEIGHTS, ids=lambda w: "x".join(map(str, w)))
def test_to_fractal_z_and_back(torch_cuda, dcopy, oracle, fmt, eb, c0, weight):
    torch = torch_cuda
    shape = _shape(fmt, *weight)
    src_np = _rand(int(np.prod(shape)) * eb, sum(shape) * 7 + eb + fmt)
    expect = oracle.to_fz(_as(src_np, eb).reshape(shape), fmt, c0)
    fz_shape = dcopy.fz_shape(fmt, shape, c0)
    assert int(np.prod(fz_shape)) == expect.size
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((expect.nbytes + 64,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(dst, src, fmt, shape, eb, c0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[:expect.nbytes].tobytes() == expect.tobytes()
    assert (out[expect.nbytes:] == CANARY).all()
    if fmt == ND:
        return  # FRACTAL_Z -> ND is not a registered transfer
    back = torch.full((src_np.size + 64,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.from_fractal_z(back, dst, fmt, shape, eb, c0)
    torch.cuda.synchronize()
    b = back.cpu().numpy()
    assert b[:src_np.size].tobytes() == src_np.tobytes() and (b[src_np.size:] == CANARY).all()


@pytest.mark.parametrize("fmt", [NCHW, NHWC, HWCN], ids=["NCHW", "NHWC", "HWCN"])
def test_from_fractal_z_ignores_padding(torch_cuda, dcopy, oracle, fmt):
    """A FRACTAL_Z buffer with garbage in its padding converts like the oracle does."""
    torch = torch_cuda
    n, c, h, w, eb, c0 = 23, 21, 3, 3, 2, 16
    shape = _shape(fmt, n, c, h, w)
    fz_shape = dcopy.fz_shape(fmt, shape, c0)
    fz_np = _rand(int(np.prod(fz_shape)) * eb, 99)
    expect = oracle.from_fz(_as(fz_np, eb).reshape(fz_shape), fmt, shape, c0)
    out = torch.full((expect.nbytes,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.from_fractal_z(out, torch.from_numpy(fz_np).cuda(), fmt, shape, eb, c0)
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == expect.tobytes()


@pytest.mark.parametrize("weight,groups", [((2, 1, 1, 1), 2), ((8, 4, 3, 3), 2), ((12, 5, 1, 1), 3),
                                           ((64, 16, 3, 3), 4), ((30, 7, 2, 2), 6),
                                           ((32, 32, 3, 3), 32)])
@pytest.mark.parametrize("eb", [2, 4])
def test_hwcn_groups(torch_cuda, dcopy, oracle, weight, groups, eb):
    torch = torch_cuda
    n, c, h, w = weight
    shape = [h, w, c, n]
    src_np = _rand(int(np.prod(shape)) * eb, n * c + groups)
    expect = oracle.to_fz(_as(src_np, eb).reshape(shape), HWCN, 16, groups)
    assert int(np.prod(dcopy.fz_shape(HWCN, shape, 16, groups))) == expect.size
    dst = torch.full((expect.nbytes + 32,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(dst, torch.from_numpy(src_np).cuda(), HWCN, shape, eb, 16, groups)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[:expect.nbytes].tobytes() == expect.tobytes() and (out[expect.nbytes:] == CANARY).all()


def test_unaligned_base_addresses(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    shape, eb, c0 = [20, 24, 3, 3], 2, 16
    src_np = _rand(int(np.prod(shape)) * eb, 5)
    expect = oracle.to_fz(_as(src_np, eb).reshape(shape), NCHW, c0)
    src = torch.from_numpy(np.concatenate([np.zeros(2, np.uint8), src_np])).cuda()
    dst = torch.full((expect.nbytes + 6,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(dst.data_ptr() + 6, src.data_ptr() + 2, NCHW, shape, eb, c0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[6:].tobytes() == expect.tobytes() and (out[:6] == CANARY).all()


@pytest.mark.parametrize("fmt", [NCHW, NHWC, HWCN], ids=["NCHW", "NHWC", "HWCN"])
def test_large_weight_against_torch(torch_cuda, dcopy, fmt):
    """fp16 [1024, 1024, 3, 3] (18 MiB) against a reshape/permute restatement in torch."""
    torch = torch_cuda
    n, c, h, w = 1024, 1024, 3, 3
    g = torch.Generator(device="cuda").manual_seed(fmt + 1)
    wt = torch.randint(-32768, 32767, (n, c, h, w), generator=g, device="cuda",
                       dtype=torch.int16)
    src = {NCHW: wt, NHWC: wt.permute(0, 2, 3, 1), HWCN: wt.permute(2, 3, 1, 0)}[fmt].contiguous()
    fz = torch.empty(c // 16 * h * w, n // 16, 16, 16, dtype=torch.int16, device="cuda")
    dcopy.to_fractal_z(fz, src, fmt, list(src.shape), 2, 16)
    expect = wt.view(n, c // 16, 16, h, w).permute(1, 3, 4, 0, 2).reshape(fz.shape)
    back = torch.empty_like(src)
    dcopy.from_fractal_z(back, fz, fmt, list(src.shape), 2, 16)
    torch.cuda.synchronize()
    assert torch.equal(fz, expect) and torch.equal(back, src)


def test_ge_level_classes(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    f, d = dcopy.FORMAT, dcopy.DATA_TYPE
    shape = [3, 3, 30, 20]  # HWCN uint8, c0 32 (GE's uint8_1c_2n_pad_cn shape)
    src_np = _rand(int(np.prod(shape)), 11)
    expect = oracle.to_fz(src_np.reshape(shape), HWCN, 32)
    dst = torch.full((expect.nbytes,), CANARY, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_data_format(dst, torch.from_numpy(src_np).cuda(), f["HWCN"], f["FRACTAL_Z"],
                                shape, [9, 2, 16, 32], d["UINT8"], dst.numel(), src_c0=32,
                                dst_c0=32)
    torch.cuda.synchronize()
    assert n == expect.nbytes and dst.cpu().numpy().tobytes() == expect.tobytes()
    back = torch.full((src_np.size,), CANARY, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_format(dcopy.TRANSFER_FRACZ_HWCN, back, dst, f["FRACTAL_Z"], f["HWCN"],
                           [9, 2, 16, 32], shape, d["UINT8"], back.numel(), src_c0=32)
    torch.cuda.synchronize()
    assert n == src_np.size and back.cpu().numpy().tobytes() == src_np.tobytes()
    # ND [C, N] through the TBE class.
    nd_np = _rand(17 * 4 * 2, 12)
    expect = oracle.to_fz(nd_np.view(np.uint16).reshape(17, 4), ND, 16)
    out = torch.full((expect.nbytes,), CANARY, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_data_format(out, torch.from_numpy(nd_np).cuda(), f["ND"], f["FRACTAL_Z"],
                                [17, 4], [2, 1, 16, 16], d["FLOAT16"], out.numel())
    torch.cuda.synchronize()
    assert n == expect.nbytes and out.cpu().numpy().tobytes() == expect.tobytes()


def test_invalid_arguments(torch_cuda, dcopy, cuda_malloc):
    with cuda_malloc(1 << 16) as buf, cuda_malloc(1 << 16) as out:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.to_fractal_z(out, buf, NCHW, [4, 4, 1, 1], 3, 16)
        assert e.value.code == dcopy.ERR_DATATYPE_INVALID
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.to_fractal_z(out, buf, NCHW, [4, 4, 1], 2, 16)
        assert e.value.code == dcopy.ERR_SHAPE_INVALID
        with pytest.raises(dcopy.DcopyError) as e:  # groups exist for HWCN only
            dcopy.to_fractal_z(out, buf, NCHW, [4, 4, 1, 1], 2, 16, 2)
        assert e.value.code == dcopy.ERR_PARAM_INVALID
        with pytest.raises(dcopy.DcopyError) as e:  # [256, 256, 3, 3] fp16 -> 1.1 MiB > 64 KiB
            dcopy.to_fractal_z(out, buf, NCHW, [256, 256, 3, 3], 2, 16)
        assert e.value.code == dcopy.ERR_PARAM_INVALID
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.from_fractal_z(out, buf, NHWC, [4, 4, 4, 4], 2, 0)
        assert e.value.code == dcopy.ERR_SHAPE_INVALID
        dcopy.to_fractal_z(out, buf, HWCN, [3, 3, 0, 16], 2, 16)  # empty: nothing written


@pytest.mark.parametrize("weight,eb,c0", [
    ((2048, 1024, 3, 3), 2, 16),   # 2048 tiles: every CTA cycles both stages several times
    ((200, 64, 5, 5), 2, 16),      # padding weights 200..207 in the last tile
    ((96, 64, 3, 3), 1, 32),
    ((2048, 1024, 3, 3), 1, 32),   # int8 3x3 / 5x5 with C0 32: the 32-bit word gather
    ((200, 128, 5, 5), 1, 32),     # padding weights in the last tile of the word gather
    ((80, 32, 2, 2), 4, 16),       # even H*W
    ((33, 16, 1, 1), 4, 8),
    ((1000, 256, 7, 7), 2, 16),
], ids=lambda v: "x".join(map(str, v)) if isinstance(v, tuple) else str(v))
def test_nchw_to_fractal_z_bulk_tiles(torch_cuda, dcopy, oracle, weight, eb, c0):
    """NCHW -> FRACTAL_Z with whole channel blocks: the bulk-copied, double-buffered tile
    kernel, against the oracle byte for byte, with no give-up of its bounded waits."""
    torch = torch_cuda
    shape = list(weight)
    src_np = _rand(int(np.prod(shape)) * eb, sum(shape) + eb)
    expect = oracle.to_fz(_as(src_np, eb).reshape(shape), NCHW, c0)
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((expect.nbytes + 64,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(dst, src, NCHW, shape, eb, c0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[:expect.nbytes].tobytes() == expect.tobytes()
    assert (out[expect.nbytes:] == CANARY).all()
    assert dcopy.tma_error() == 0


@pytest.mark.parametrize("shape,eb,c0", [
    ((3, 3, 1024, 2048), 2, 16),
    ((5, 5, 64, 200), 2, 16),
    ((3, 3, 1024, 2048), 1, 32),   # 2304 tiles: every CTA cycles both stages several times
    ((5, 5, 64, 208), 1, 32),      # N = 208: the last tile is partial, its padding zero-filled
    ((3, 3, 64, 96), 1, 32),
    ((2, 2, 32, 80), 4, 16),
    ((1, 1, 256, 1000), 2, 16),
], ids=lambda v: "x".join(map(str, v)) if isinstance(v, tuple) else str(v))
def test_hwcn_to_fractal_z_tensor_tiles(torch_cuda, dcopy, oracle, shape, eb, c0):
    """HWCN -> FRACTAL_Z with whole channel blocks and 16-byte output rows (the
    tensor-copied, double-buffered tile kernel for 1-byte elements, the vector kernel
    for wider ones), against the oracle byte for byte."""
    torch = torch_cuda
    shape = list(shape)
    src_np = _rand(int(np.prod(shape)) * eb, sum(shape) * 3 + eb)
    expect = oracle.to_fz(_as(src_np, eb).reshape(shape), HWCN, c0)
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((expect.nbytes + 64,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.to_fractal_z(dst, src, HWCN, shape, eb, c0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[:expect.nbytes].tobytes() == expect.tobytes()
    assert (out[expect.nbytes:] == CANARY).all()
    assert dcopy.tma_error() == 0


@pytest.mark.parametrize("weight,eb,c0", [
    ((2048, 1024, 3, 3), 1, 32),   # int8 3x3 / 5x5 with C0 32: the 32-bit word scatter
    ((2040, 1024, 3, 3), 1, 32),   # word scatter, padding rows 2040..2047 not stored
    ((1000, 1024, 5, 5), 1, 32),   # word scatter at 5x5, 2016 tiles, padding rows
    ((200, 128, 5, 5), 1, 32),     # fewer tiles than CTAs: the vector kernel
    ((96, 64, 3, 3), 1, 32),
    ((2048, 1024, 3, 3), 2, 16),   # the fp16 row-vector gather
    ((80, 32, 2, 2), 4, 16),       # the fp32 bulk kernel
], ids=lambda v: "x".join(map(str, v)) if isinstance(v, tuple) else str(v))
def test_fractal_z_to_nchw_bulk_tiles(torch_cuda, dcopy, oracle, weight, eb, c0):
    """FRACTAL_Z (made by the oracle) -> NCHW through the bulk-copied tile kernels: the
    result is the original weight byte for byte, nothing written past it, no give-up."""
    torch = torch_cuda
    shape = list(weight)
    src_np = _rand(int(np.prod(shape)) * eb, sum(shape) * 5 + eb)
    fz = oracle.to_fz(_as(src_np, eb).reshape(shape), NCHW, c0)
    z = torch.from_numpy(np.ascontiguousarray(fz).view(np.uint8).reshape(-1)).cuda()
    back = torch.full((src_np.size + 64,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.from_fractal_z(back, z, NCHW, shape, eb, c0)
    torch.cuda.synchronize()
    out = back.cpu().numpy()
    assert out[:src_np.size].tobytes() == src_np.tobytes()
    assert (out[src_np.size:] == CANARY).all()
    assert dcopy.tma_error() == 0
