"""GPU parity: ND <-> FRACTAL_NZ kernels (C ABI) vs the oracle, bit-exact.

The oracle is pinned to GE's golden vectors on the CPU side; here the GPU is
checked against it on the golden shapes with random data, on ragged and
unaligned shapes that take the element-granular path, on every element width,
and on BASELINE config 4 ([16, 4096, 4096] fp16) at full size: byte-exact
against the oracle and as a round trip.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5

SHAPES = [
    ([2, 2, 17, 4], 2, 16), ([2, 2, 2, 17, 4], 2, 16), ([2, 2, 17, 4], 4, 16),
    ([2, 2, 4, 17], 4, 16), ([1], 2, 16), ([100], 2, 16), ([17, 3], 1, 32), ([16, 16], 2, 16),
    ([2, 33, 47], 2, 16), ([3, 2, 5, 16], 8, 16), ([40, 1], 4, 16), ([1, 40], 4, 16),
    ([64, 128], 2, 16), ([3, 100, 256], 2, 16), ([5, 31, 200], 1, 32), ([2, 48, 40], 8, 16),
    ([7, 129, 33], 4, 16), ([1, 16, 4096], 2, 16), ([4, 20, 24], 2, 8), ([2, 3, 3, 9], 16, 16),
]


def _rand(shape, eb, seed):
    n = int(np.prod(shape)) * eb
    return np.random.default_rng(seed).integers(0, 256, size=n, dtype=np.uint8)


@pytest.mark.parametrize("shape,eb,w0", SHAPES, ids=lambda v: str(v))
def test_nd_to_nz_and_back(torch_cuda, dcopy, oracle, shape, eb, w0):
    torch = torch_cuda
    rc, nz, _ = oracle.nz_shape(shape, w0)
    assert rc == 0
    assert dcopy.nz_shape(shape, w0)[0] == nz
    src_np = _rand(shape, eb, seed=sum(shape) + eb)
    nz_bytes = int(np.prod(nz)) * eb
    expect = np.empty(nz_bytes, dtype=np.uint8)
    assert oracle.nd_to_nz(expect, src_np, shape, eb, w0) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((nz_bytes,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.nd_to_nz(dst, src, shape, eb, w0)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()
    back = torch.full((src_np.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.nz_to_nd(back, dst, shape, eb, w0)
    torch.cuda.synchronize()
    assert back.cpu().numpy().tobytes() == src_np.tobytes()


def test_unaligned_base_addresses(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    shape, eb, w0 = [3, 40, 64], 2, 16
    src_np = _rand(shape, eb, 9)
    rc, nz, _ = oracle.nz_shape(shape, w0)
    expect = np.empty(int(np.prod(nz)) * eb, dtype=np.uint8)
    oracle.nd_to_nz(expect, src_np, shape, eb, w0)
    src = torch.from_numpy(np.concatenate([np.zeros(2, np.uint8), src_np])).cuda()
    dst = torch.full((expect.size + 6,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.nd_to_nz(dst.data_ptr() + 6, src.data_ptr() + 2, shape, eb, w0)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[6:].tobytes() == expect.tobytes() and (out[:6] == CANARY).all()


def test_config4_full_size(torch_cuda, dcopy, oracle):
    """fp16 [16, 4096, 4096] normal(0,1) seed 2 -> [16, 256, 256, 16, 16]."""
    torch = torch_cuda
    shape = [16, 4096, 4096]
    g = torch.Generator(device="cuda").manual_seed(2)
    nd = torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).half()
    nz = torch.empty(16, 256, 256, 16, 16, dtype=torch.float16, device="cuda")
    dcopy.nd_to_nz(nz, nd, shape, 2, 16)
    back = torch.empty_like(nd)
    dcopy.nz_to_nd(back, nz, shape, 2, 16)
    torch.cuda.synchronize()
    assert torch.equal(back.view(torch.int16), nd.view(torch.int16))
    # The NZ bytes equal the reference layout: panel w1 holds columns w1*16..w1*16+15.
    expect = nd.view(16, 4096, 256, 16).permute(0, 2, 1, 3).contiguous()
    assert torch.equal(nz.view(torch.int16).view(16, 256, 4096, 16), expect.view(torch.int16))
    # And byte for byte against the oracle on one batch.
    one = nd[3].cpu().numpy().view(np.uint8)
    ref = np.empty(4096 * 4096 * 2, dtype=np.uint8)
    assert oracle.nd_to_nz(ref, one, [4096, 4096], 2, 16, threads=8) == 0
    assert nz[3].cpu().numpy().view(np.uint8).tobytes() == ref.tobytes()


def test_invalid_arguments(torch_cuda, dcopy, cuda_malloc):
    with cuda_malloc(1 << 16) as buf, cuda_malloc(1 << 16) as out:
        _invalid_arguments(dcopy, buf, out)


def _invalid_arguments(dcopy, buf, out):
    for eb, code in [(0, dcopy.ERR_DATATYPE_INVALID), (-2, dcopy.ERR_DATATYPE_INVALID),
                     (3, dcopy.ERR_DATATYPE_INVALID)]:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.nd_to_nz(out, buf, [4, 4], eb, 16)
        assert e.value.code == code
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_nz(out, buf, [4, -4], 2, 16)
    assert e.value.code == dcopy.ERR_SHAPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nz_to_nd(out, buf, [4, 4], 2, 0)
    assert e.value.code == dcopy.ERR_SHAPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:  # NZ of [300, 300] fp16 needs 184 KiB > 64 KiB
        dcopy.nd_to_nz(out, buf, [300, 300], 2, 16)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    dcopy.nd_to_nz(out, buf, [0, 16], 2, 16)  # empty: success, nothing written
