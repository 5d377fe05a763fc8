"""GPU parity: DataCopyNddma boxes on both box paths — the TMA tensor-copy path
(selected with set_nd_tma; rows that are not whole 16-byte granules still take
the row kernel) and the default row kernel — vs the oracle,
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


@pytest.fixture(params=[True, False], ids=["tma", "rows"])
def box_path(request, dcopy):
    prev = dcopy.set_nd_tma(request.param)
    yield request.param
    dcopy.set_nd_tma(prev)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-e{c[3]}")
def test_tma_boxes_match_oracle(torch_cuda, dcopy, oracle, case, box_path):
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


def test_large_box_and_throughput(torch_cuda, dcopy, box_path):
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


ROW_CASES = [  # (sizes, src strides, dst strides, elem bytes): boxes outside the TMA conditions
    ([7, 300, 260], [300 * 272, 272, 1], [300 * 264, 264, 1], 2),  # 520-byte rows
    ([3, 5, 7, 33], [5 * 7 * 41, 7 * 41, 41, 1], [5 * 7 * 35, 7 * 35, 35, 1], 1),  # odd strides
    ([4, 9, 100], [0, 104, 1], [900, 100, 1], 4),  # broadcast outer source axis
    ([2, 3, 4, 5, 37], [3 * 4 * 5 * 40, 4 * 5 * 40, 5 * 40, 40, 1],
     [3 * 4 * 5 * 42, 4 * 5 * 42, 5 * 42, 42, 1], 2),
    ([6, 1000], [500, 1], [1000, 1], 4),  # source rows overlap (reads only)
    ([5, 7, 24], [7 * 25, 25, 1], [7 * 24, 24, 1], 8),
    ([3, 4, 6], [4 * 7, 7, 1], [4 * 8, 8, 1], 16),
    ([2, 5, 3], [15, 3, 1], [40, 8, 1], 4),  # 12-byte rows, 16-byte aligned destination pitch
]


@pytest.mark.parametrize("case", ROW_CASES, ids=lambda c: f"{c[0]}-e{c[3]}")
def test_row_boxes_match_oracle(torch_cuda, dcopy, oracle, case):
    """Boxes with a contiguous innermost axis that the TMA path declines (ragged or
    unaligned rows, odd strides, broadcast or overlapping source rows): the row
    kernel with a strided destination."""
    torch = torch_cuda
    sizes, ss, ds, eb = case
    src_elems = sum((s - 1) * st for s, st in zip(sizes, ss)) + 1
    dst_elems = sum((s - 1) * st for s, st in zip(sizes, ds)) + 1
    src_np = np.random.default_rng(len(sizes) * 31 + eb).integers(0, 256, size=src_elems * eb,
                                                                  dtype=np.uint8)
    expect = np.full(dst_elems * eb, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(expect, src_np, sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((dst_elems * eb,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_nd(dst, src, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


def _shift_case(seed):
    """Random box whose rows need byte shifts: 1- or 2-byte elements, odd pads, and
    base addresses at any element offset within 16 bytes."""
    rng = np.random.default_rng(1000 + seed)
    eb = int(rng.choice([1, 2]))
    m = int(rng.integers(2, 6))
    L = int(rng.integers(16 // eb, 300 // eb))
    outer = [int(rng.integers(1, 6)) for _ in range(m - 1)]
    sizes = outer + [L]
    sp, dp = int(rng.integers(0, 9)), int(rng.integers(0, 9))
    ss, ds = [1] * m, [1] * m
    for k in range(m - 2, -1, -1):
        ss[k] = ss[k + 1] * (sizes[k + 1] + (sp if k == m - 2 else 0))
        ds[k] = ds[k + 1] * (sizes[k + 1] + (dp if k == m - 2 else 0))
    soff = int(rng.integers(0, 16 // eb)) * eb
    doff = int(rng.integers(0, 16 // eb)) * eb
    return sizes, ss, ds, eb, soff, doff


@pytest.mark.parametrize("seed", range(24))
def test_shifted_rows_match_oracle(torch_cuda, dcopy, oracle, seed):
    """Rows whose length, bases or strides are not 16-byte multiples go through the
    funnel-shift row kernel: bit-exact, bytes outside every row untouched."""
    torch = torch_cuda
    sizes, ss, ds, eb, soff, doff = _shift_case(seed)
    src_bytes = (sum((s - 1) * st for s, st in zip(sizes, ss)) + 1) * eb + soff + 32
    dst_bytes = (sum((s - 1) * st for s, st in zip(sizes, ds)) + 1) * eb + doff + 32
    src_np = np.random.default_rng(seed).integers(0, 256, size=src_bytes, dtype=np.uint8)
    expect = np.full(dst_bytes, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(expect[doff:], src_np[soff:], sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((dst_bytes,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_nd(dst.data_ptr() + doff, src.data_ptr() + soff, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


PERMUTED = [  # (sizes, src memory order outermost first, src pad, dst pad, elem bytes)
    ([4, 14, 14, 40], [0, 3, 1, 2], 0, 0, 2), ([4, 14, 14, 40], [0, 3, 1, 2], 3, 5, 2),
    ([30, 70], [1, 0], 2, 3, 4), ([3, 33, 65], [0, 2, 1], 1, 0, 1), ([5, 6, 7, 8, 9], [4, 3, 2, 1, 0], 0, 2, 8),
    ([2, 3, 40, 24], [1, 0, 3, 2], 4, 1, 16),
]


@pytest.mark.parametrize("case", PERMUTED, ids=lambda c: f"{c[0]}-{c[1]}-e{c[4]}")
def test_permuted_source_boxes(torch_cuda, dcopy, oracle, case):
    """Boxes whose source's unit-stride axis is not the innermost box axis and whose
    destination rows are contiguous (packed or padded): the Transpose tile kernels."""
    torch = torch_cuda
    sizes, order, sp, dp, eb = case
    m = len(sizes)
    ss = [0] * m
    step = 1
    for i in range(m - 1, -1, -1):
        ss[order[i]] = step
        step *= sizes[order[i]] + (sp if i < m - 1 else 0)
    ds = _strides(sizes, dp)
    src_elems = sum((s - 1) * st for s, st in zip(sizes, ss)) + 1
    dst_elems = sum((s - 1) * st for s, st in zip(sizes, ds)) + 1
    src_np = np.random.default_rng(sum(sizes) * eb).integers(0, 256, size=src_elems * eb,
                                                             dtype=np.uint8)
    expect = np.full(dst_elems * eb, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(expect, src_np, sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = torch.full((dst_elems * eb,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_nd(dst, src, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()
