"""GPU parity: ND <-> FRACTAL_ZZ kernels (C ABI) vs the oracle, bit-exact.

The oracle's ZZ restatement is pinned to every data-moving golden vector of GE's
format_transfer_fractal_zz_unittest.cc on the CPU side; here the GPU is checked
against it with random bytes on the golden shapes, on every element width, on
C0 values that take the shared-memory path (16-byte units, power-of-two blocks)
and the direct path (small or very large blocks, odd widths), on unaligned base
addresses, and at 512 MiB against a reshape/permute restatement in torch.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5

SHAPES = [
    # GE's golden shapes: (nd shape, element bytes, c0)
    ([1], 1, 32), ([32], 1, 32), ([32, 32], 1, 32), ([30, 33], 1, 32), ([2, 30, 32], 1, 32),
    ([2, 3, 4, 32], 1, 32), ([2, 3, 4, 33], 1, 32), ([1], 2, 16), ([15], 2, 16),
    ([1, 16], 2, 16), ([15, 17], 2, 16), ([2, 4, 17], 2, 16), ([1, 1, 17, 4], 2, 16),
    ([2, 2, 17, 4], 2, 16), ([2, 3, 2, 3, 17], 2, 16), ([2, 2, 4, 17], 4, 16),
    # ragged, wide and deep shapes, every element width, shared-memory and direct paths
    ([3, 100, 256], 2, 16), ([5, 31, 200], 1, 32), ([2, 48, 40], 8, 16), ([7, 129, 33], 4, 16),
    ([1, 16, 4096], 2, 16), ([4, 20, 24], 2, 8), ([2, 3, 3, 9], 16, 16), ([3, 70, 130], 4, 4),
    ([2, 200, 300], 2, 64), ([2, 130, 260], 4, 128), ([1, 33, 1000], 2, 8), ([4, 64, 64], 4, 16),
    ([2, 17, 19], 1, 3), ([3, 5], 8, 2), ([40, 1], 4, 16), ([1, 40], 4, 16),
]


def _rand(shape, eb, seed):
    n = int(np.prod(shape)) * eb
    return np.random.default_rng(seed).integers(0, 256, size=n, dtype=np.uint8)


@pytest.mark.parametrize("shape,eb,c0", SHAPES, ids=lambda v: str(v))
def test_nd_to_zz_and_back(torch_cuda, dcopy, oracle, shape, eb, c0):
    torch = torch_cuda
    rc, zz, _ = oracle.zz_shape(shape, c0)
    assert rc == 0
    assert dcopy.zz_shape(shape, c0)[0] == zz
    src_np = _rand(shape, eb, seed=sum(shape) + eb + c0)
    zz_bytes = int(np.prod(zz)) * eb
    expect = np.empty(zz_bytes, dtype=np.uint8)
    assert oracle.nd_to_zz(expect, src_np, shape, eb, c0) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((zz_bytes,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.nd_to_zz(dst, src, shape, eb, c0)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()
    back = torch.full((src_np.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.zz_to_nd(back, dst, shape, eb, c0)
    torch.cuda.synchronize()
    assert back.cpu().numpy().tobytes() == src_np.tobytes()


def test_unaligned_base_addresses(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    shape, eb, c0 = [3, 40, 64], 2, 16
    src_np = _rand(shape, eb, 19)
    rc, zz, _ = oracle.zz_shape(shape, c0)
    expect = np.empty(int(np.prod(zz)) * eb, dtype=np.uint8)
    oracle.nd_to_zz(expect, src_np, shape, eb, c0)
    src = torch.from_numpy(np.concatenate([np.zeros(2, np.uint8), src_np])).cuda()
    dst = torch.full((expect.size + 6,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.nd_to_zz(dst.data_ptr() + 6, src.data_ptr() + 2, shape, eb, c0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[6:].tobytes() == expect.tobytes() and (out[:6] == CANARY).all()


def test_full_size_against_torch_permute(torch_cuda, dcopy, oracle):
    """fp16 [8, 4096, 4096] (256 MiB each way) -> [8, 256, 256, 16, 16] and back."""
    torch = torch_cuda
    shape = [8, 4096, 4096]
    g = torch.Generator(device="cuda").manual_seed(5)
    nd = torch.randint(-32768, 32767, shape, generator=g, device="cuda", dtype=torch.int16)
    zz = torch.empty(8, 256, 256, 16, 16, dtype=torch.int16, device="cuda")
    dcopy.nd_to_zz(zz, nd, shape, 2, 16)
    back = torch.empty_like(nd)
    dcopy.zz_to_nd(back, zz, shape, 2, 16)
    torch.cuda.synchronize()
    assert torch.equal(back, nd)
    expect = nd.view(8, 256, 16, 256, 16).permute(0, 1, 3, 2, 4)
    assert torch.equal(zz, expect)
    one = nd[5].cpu().numpy().view(np.uint8)
    ref = np.empty(4096 * 4096 * 2, dtype=np.uint8)
    assert oracle.nd_to_zz(ref, one, [4096, 4096], 2, 16) == 0
    assert zz[5].cpu().numpy().view(np.uint8).tobytes() == ref.tobytes()


@pytest.mark.parametrize("src_fmt,shape,dt,eb", [
    ("ND", [2, 2, 17, 4], 1, 2), ("ND", [2, 3, 2, 3, 17], 1, 2), ("ND", [2, 2, 4, 17], 0, 4),
    ("NCHW", [1, 2, 4, 17], 0, 4), ("NHWC", [2, 2, 17, 4], 0, 4), ("ND", [2, 3, 4, 33], 4, 1),
    ("ND", [100], 1, 2), ("ND", [5, 33, 70], 9, 8)])
def test_trans_data_format_zz_round_trip(torch_cuda, dcopy, oracle, src_fmt, shape, dt, eb):
    torch = torch_cuda
    f = dcopy.FORMAT
    c0 = 32 if eb == 1 else 16
    rc, zz, _ = oracle.zz_shape(shape, c0)
    nd_np = _rand(shape, eb, sum(shape) + 3)
    expect = np.empty(int(np.prod(zz)) * eb, dtype=np.uint8)
    assert oracle.nd_to_zz(expect, nd_np, shape, eb, c0) == 0
    src = torch.from_numpy(nd_np).cuda()
    dst = torch.full((expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_data_format(dst, src, f[src_fmt], f["FRACTAL_ZZ"], shape, zz, dt,
                                dst.numel(), dst_c0=c0)
    torch.cuda.synchronize()
    assert n == expect.size and dst.cpu().numpy().tobytes() == expect.tobytes()
    back = torch.full((nd_np.size,), CANARY, dtype=torch.uint8, device="cuda")
    n = dcopy.trans_format(dcopy.TRANSFER_FRACTAL_ZZ_ND, back, dst, f["FRACTAL_ZZ"], f[src_fmt],
                           zz, shape, dt, back.numel(), src_c0=c0)
    torch.cuda.synchronize()
    assert n == nd_np.size and back.cpu().numpy().tobytes() == nd_np.tobytes()


def test_invalid_arguments(torch_cuda, dcopy, cuda_malloc):
    with cuda_malloc(1 << 16) as buf, cuda_malloc(1 << 16) as out:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.nd_to_zz(out, buf, [4, 4], 3, 16)
        assert e.value.code == dcopy.ERR_DATATYPE_INVALID
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.zz_to_nd(out, buf, [4, 4], 2, -16)
        assert e.value.code == dcopy.ERR_SHAPE_INVALID
        with pytest.raises(dcopy.DcopyError) as e:  # ZZ of [300, 300] fp16 needs 180 KiB > 64 KiB
            dcopy.nd_to_zz(out, buf, [300, 300], 2, 16)
        assert e.value.code == dcopy.ERR_PARAM_INVALID
        dcopy.nd_to_zz(out, buf, [0, 16], 2, 16)  # empty: success, nothing written
