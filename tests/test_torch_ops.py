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
        assert list(ops.box(torch.empty(1000), [3, 4, 5], [200, 30, 1], 7).shape) == [3, 4, 5]
        assert list(ops.nd_to_zz(torch.empty(2, 40, 70, dtype=torch.float16), 16).shape) == \
            [2, 3, 5, 16, 16]
        assert list(ops.zz_to_nd(torch.empty(2, 3, 5, 16, 16), [2, 40, 70], 16).shape) == \
            [2, 40, 70]
        w = torch.empty(20, 24, 3, 3, dtype=torch.float16)
        assert list(ops.to_fractal_z(w, "NCHW", 16).shape) == [18, 2, 16, 16]
        assert list(ops.from_fractal_z(torch.empty(18, 2, 16, 16), "NCHW", [20, 24, 3, 3],
                                       16).shape) == [20, 24, 3, 3]


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
    big = torch.randn(8, 64, 72, device="cuda", dtype=torch.float16)
    assert torch.equal(ops.box(big, [8, 40, 55], [64 * 72, 72, 1], 3),
                       torch.as_strided(big, [8, 40, 55], [64 * 72, 72, 1], 3).contiguous())
    zz = ops.nd_to_zz(x, 16)
    assert torch.equal(ops.zz_to_nd(zz, [3, 40, 70], 16), x)
    w = torch.randn(20, 24, 3, 3, device="cuda", dtype=torch.float16)
    for fmt, t in (("NCHW", w), ("NHWC", w.permute(0, 2, 3, 1).contiguous()),
                   ("HWCN", w.permute(2, 3, 1, 0).contiguous())):
        fz = ops.to_fractal_z(t, fmt, 16)
        assert torch.equal(ops.from_fractal_z(fz, fmt, list(t.shape), 16), t)
    # FRACTAL_Z of NCHW: [C1*H*W, N1, 16, C0] with zero padding of N and C.
    fz = ops.to_fractal_z(w, "NCHW", 16)
    wp = torch.zeros(32, 32, 3, 3, dtype=w.dtype, device="cuda")
    wp[:20, :24] = w
    expect = wp.view(2, 16, 2, 16, 3, 3)  # [N1, N0, C1, C0, H, W]
    expect = expect.permute(2, 4, 5, 0, 1, 3).reshape(2 * 9, 2, 16, 16)  # [C1 H W, N1, N0, C0]
    assert torch.equal(fz, expect)
    assert int((dst.view(10, 8)[:, 4:] != 0).sum()) == 0


@pytest.mark.gpu
def test_opcheck(ops, torch_cuda):
    x = torch.randn(2, 33, 47, device="cuda", dtype=torch.float16)
    torch.library.opcheck(ops.nd_to_nz, (x, 16), test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(ops.transpose, (torch.randn(2, 3, 4, 5, device="cuda"), [3, 1, 2, 0]),
                          test_utils=("test_schema", "test_faketensor"))
