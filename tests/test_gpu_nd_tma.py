"""GPU parity: DataCopyNddma boxes on the TMA tensor-copy path (and, for rows that
are not whole 16-byte granules, on the load/store path), vs the oracle,
bit-exact, with canary-filled destinations (gaps between destination rows must
keep their canary).  Shapes cover 3-, 4- and 5-D boxes, every element width,
boxes that split into many TMA boxes with ragged edges on every axis, padded
source and destination pitches, and a 256 MiB box timed against the byte count.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5


def _strides(shape, pad_elems):
    """Row-major strides of `shape` with the innermost rows padded by pad_elems."""
    st = [1] * len(shape)
    for k in range(len(shape) - 2, -1, -1):
        st[k] = st[k + 1] * (shape[k + 1] + (pad_elems if k == len(shape) - 2 else 0))
    return st


CASES = [  # (sizes, src pad, dst pad, elem bytes)
    ([4, 8, 64], 0, 0, 4), ([3, 17, 300], 4, 12, 4), ([5, 33, 129], 8, 0, 2),
    ([2, 3, 5, 400], 16, 32, 1), ([2, 2, 3, 7, 96], 0, 16, 2), ([3, 70, 70], 2, 6, 8),
    ([6, 5, 40], 1, 3, 16), ([7, 300, 260], 12, 4, 2), ([2, 600, 8], 0, 8, 4),
    ([257, 3, 16], 0, 0, 1),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-e{c[3]}")
def test_tma_boxes_match_oracle(torch_cuda, dcopy, oracle, case):
    torch = torch_cuda
    sizes, sp, dp, eb = case
    ss, ds = _strides(sizes, sp), _strides(sizes, dp)
    src_elems = sizes[0] * ss[0]
    dst_elems = sizes[0] * ds[0]
    src_np = np.random.default_rng(sum(sizes) + eb).integers(0, 256, size=src_elems * eb,
                                                             dtype=np.uint8)
    expect = np.full(dst_elems * eb, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(expect, src_np, sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((dst_elems * eb,), CANARY, dtype=torch.uint8, device="cuda")
    assert dcopy.tma_error() == 0
    dcopy.copy_nd(dst, src, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dcopy.tma_error() == 0
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


def test_large_box_and_throughput(torch_cuda, dcopy):
    """[64, 2048, 1024] fp16 (256 MiB) out of a row-padded source, checked in torch."""
    torch = torch_cuda
    a = torch.randint(-32768, 32767, (64, 2048, 1024 + 64), dtype=torch.int16, device="cuda")
    out = torch.empty(64, 2048, 1024, dtype=torch.int16, device="cuda")
    sizes = [64, 2048, 1024]
    ss = [2048 * 1088, 1088, 1]
    ds = [2048 * 1024, 1024, 1]
    dcopy.copy_nd(out, a, sizes, ss, ds, 2)
    torch.cuda.synchronize()
    assert torch.equal(out, a[:, :, :1024])
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(5):
        dcopy.copy_nd(out, a, sizes, ss, ds, 2)
    e.record()
    e.synchronize()
    gbps = 5 * 2 * out.numel() * 2 / (s.elapsed_time(e) / 1e3) / 1e9
    assert dcopy.tma_error() == 0
    assert gbps > 1000, gbps  # a functional floor, not the performance target
