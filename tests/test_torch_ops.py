"""torch.library operators over libdcopy: registration and fake shapes on CPU,
results against torch's own reshuffles on the GPU."""
import pytest
import torch


@pytest.fixture(scope="module")
def ops(dcopy):
    from dcopy import torch_ops  # noqa: F401  (registers torch.ops.dcopy.*)
    return torch.ops.dcopy


def test_fake_shapes_without_a_gpu(ops):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(16, 4096, 4096, dtype=torch.float16)
        assert list(ops.nd_to_nz(x, 16).shape) == [16, 256, 256, 16, 16]
        nz = torch.empty(2, 1, 2, 16, 16, dtype=torch.float32)
        assert list(ops.nz_to_nd(nz, [2, 17, 4], 16).shape) == [2, 17, 4]
        assert list(ops.transpose(torch.empty(2, 3, 4, 5), [0, 2, 3, 1]).shape) == [2, 4, 5, 3]
        assert list(ops.datacopy_transpose(torch.empty(8, 5, dtype=torch.int32)).shape) == [5, 8]
        assert list(ops.strided_gather(torch.empty(100), 10, 3, 7).shape) == [30]


@pytest.mark.gpu
def test_ops_match_torch(ops, torch_cuda):
    x = torch.randn(3, 40, 70, device="cuda", dtype=torch.float16)
    nz = ops.nd_to_nz(x, 16)
    assert torch.equal(ops.nz_to_nd(nz, [3, 40, 70], 16), x)
    y = torch.randn(2, 3, 4, 5, device="cuda")
    assert torch.equal(ops.transpose(y, [0, 2, 3, 1]), y.permute(0, 2, 3, 1))
    a = torch.randint(-2**31, 2**31 - 1, (64, 300), dtype=torch.int32, device="cuda")
    assert torch.equal(ops.datacopy_transpose(a), a.t())
    src = torch.randn(4096, 4096, device="cuda")
    g = ops.strided_gather(src[:, 1024:].contiguous().view(-1)[: 4096 * 3072], 4096, 1024, 2048)
    assert torch.equal(g.view(4096, 1024), src[:, 1024:2048])
    dst = torch.zeros(10 * 8, device="cuda")
    s = torch.arange(10 * 12, dtype=torch.float32, device="cuda")
    ops.copy_ext_(dst, s, 10, 4, 8, 4)
    assert torch.equal(dst.view(10, 8)[:, :4], s.view(10, 12)[:, :4])
    assert int((dst.view(10, 8)[:, 4:] != 0).sum()) == 0


@pytest.mark.gpu
def test_opcheck(ops, torch_cuda):
    x = torch.randn(2, 33, 47, device="cuda", dtype=torch.float16)
    torch.library.opcheck(ops.nd_to_nz, (x, 16), test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(ops.transpose, (torch.randn(2, 3, 4, 5, device="cuda"), [3, 1, 2, 0]),
                          test_utils=("test_schema", "test_faketensor"))
