"""GPU parity: GE Transpose (format_transfer_transpose.cc:142-197) through the C ABI
vs the oracle's restatement, bit-exact, on the permuted-copy kernels: row copies
(innermost axis kept), tiled transposes with 16-byte vectors (aligned rows) and
with element accesses (odd extents), every element width, 2-D to 5-D, ragged
tiles, and a 256 MiB 2-D transpose checked against torch."""
import itertools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DT = {1: 4, 2: 1, 4: 0, 8: 9, 16: 17}  # element bytes -> a GE data type of that size


def _case(torch, dcopy, oracle, shape, perm, eb, seed):
    n = int(np.prod(shape))
    src_np = np.random.default_rng(seed).integers(0, 256, size=n * eb, dtype=np.uint8)
    expect = np.empty_like(src_np)
    assert oracle.transpose(expect, src_np, shape, perm, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((n * eb + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    dcopy.transpose(dst, src, shape, perm, DT[eb])
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[:n * eb].tobytes() == expect.tobytes(), (shape, perm, eb)
    assert (out[n * eb:] == 0xA5).all()


@pytest.mark.parametrize("eb", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("shape,perm", [
    ([64, 64], [1, 0]), ([100, 37], [1, 0]), ([128, 200], [1, 0]), ([3, 1000], [1, 0]),
    ([8, 16, 24, 32], [0, 2, 3, 1]), ([8, 24, 32, 16], [0, 3, 1, 2]), ([5, 7, 9, 11], [3, 2, 1, 0]),
    ([16, 16, 16, 16], [0, 2, 1, 3]), ([4, 6, 8, 10, 12], [4, 0, 3, 1, 2]),
    ([2, 3, 5, 7, 64], [1, 3, 0, 2, 4]), ([33, 65, 2], [2, 1, 0]), ([256, 256, 3, 3], [2, 3, 1, 0]),
    ([5, 7, 37], [1, 0, 2]), ([3, 4, 5, 33], [2, 0, 1, 3]),  # odd rows kept innermost
])
def test_permutes(torch_cuda, dcopy, oracle, eb, shape, perm):
    _case(torch_cuda, dcopy, oracle, shape, perm, eb, sum(shape) + eb)


def test_every_4d_perm(torch_cuda, dcopy, oracle):
    for i, perm in enumerate(itertools.permutations(range(4))):
        _case(torch_cuda, dcopy, oracle, [6, 10, 12, 20], list(perm), 2, i)


def test_unaligned_base(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    shape, perm, eb = [64, 96], [1, 0], 2
    n = int(np.prod(shape))
    src_np = np.random.default_rng(3).integers(0, 256, size=n * eb, dtype=np.uint8)
    expect = np.empty_like(src_np)
    oracle.transpose(expect, src_np, shape, perm, eb)
    src = torch.from_numpy(np.concatenate([np.zeros(2, np.uint8), src_np])).cuda()
    dst = torch.full((n * eb + 6,), 0xA5, dtype=torch.uint8, device="cuda")
    dcopy.transpose(dst.data_ptr() + 6, src.data_ptr() + 2, shape, perm, DT[eb])
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    assert out[6:].tobytes() == expect.tobytes() and (out[:6] == 0xA5).all()


def test_large_against_torch(torch_cuda, dcopy):
    torch = torch_cuda
    a = torch.randint(-2**31, 2**31 - 1, (8192, 8192), dtype=torch.int32, device="cuda")
    out = torch.empty_like(a)
    dcopy.transpose(out, a, [8192, 8192], [1, 0], 0)
    b = torch.randint(-32768, 32767, (32, 256, 56, 56), dtype=torch.int16, device="cuda")
    out2 = torch.empty_like(b)
    dcopy.transpose(out2, b, list(b.shape), [0, 2, 3, 1], 1)
    torch.cuda.synchronize()
    assert torch.equal(out, a.t().contiguous())
    assert torch.equal(out2.view(32, 56, 56, 256), b.permute(0, 2, 3, 1).contiguous())
