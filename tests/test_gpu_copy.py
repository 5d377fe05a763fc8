"""GPU parity: DataCopyExt strided copies and DataCopyNddma boxes vs the oracle, bit-exact.

Destinations are pre-filled with a canary so bytes in the destination gaps must
stay untouched, as in the oracle.  BASELINE configs 1-3 and 5 run at full size
through size-independent checks (the strided view of the source equals the
packed destination), and at reduced size against the oracle byte for byte.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5


def _canary(torch, n):
    return torch.full((n,), CANARY, dtype=torch.uint8, device="cuda")


def _rand_bytes(n, seed):
    return np.random.default_rng(seed).integers(0, 256, size=n, dtype=np.uint8)


CASES = [  # (blockCount, blockLen, srcGap, dstGap, src_offset, dst_offset)
    (1, 1, 0, 0, 0, 0), (7, 3, 5, 1, 1, 2), (64, 4, 28, 0, 0, 0), (33, 16, 16, 16, 0, 0),
    (33, 16, 16, 16, 4, 8), (100, 32, 0, 0, 0, 0), (100, 32, 32, 0, 0, 0),
    (257, 48, 80, 16, 0, 0), (1000, 64, 192, 0, 16, 0), (300, 100, 3, 7, 5, 1),
    (1023, 128, 512, 0, 0, 0), (64, 512, 2048, 512, 0, 0), (17, 4096, 12288, 0, 0, 0),
    (5, 65536, 65536, 32, 0, 0), (3, 1 << 20, 1 << 16, 0, 0, 0), (1, 1 << 22, 0, 0, 3, 7),
    (4096, 4, 4092, 0, 0, 0), (65536, 2, 6, 0, 2, 0),
    (2000, 77, 13, 5, 3, 9), (500, 1000, 24, 8, 6, 2), (4096, 20, 12, 0, 0, 4),
    (129, 4099, 1, 3, 1, 0), (3000, 18, 0, 14, 15, 1),  # bursts of 1/2/4-byte units
]


@pytest.fixture(params=[False, True], ids=["lsu", "tma"])
def burst_path(request, dcopy):
    """False: the default load/store kernels.  True: the TMA paths selected
    (set_nd_tma), under which 16-byte-granular bursts from 512 bytes take the
    bulk-copy kernel and gapped granular bursts under 128 bytes the 2-D tensor copy."""
    prev = dcopy.set_nd_tma(request.param)
    yield request.param
    dcopy.set_nd_tma(prev)


TMA_BURST_CASES = [  # 16-byte granular: (blockCount, blockLen, srcGap, dstGap, soff, doff)
    (100, 32, 32, 0, 0, 0), (1000, 64, 192, 0, 16, 0), (257, 48, 80, 16, 0, 0),
    (4096, 16, 1008, 32, 0, 0), (300, 112, 16, 0, 0, 16),
    (64, 512, 2048, 512, 0, 0), (17, 4096, 12288, 0, 0, 0), (5, 65536, 65536, 32, 0, 0),
    (3, 1 << 20, 1 << 16, 0, 0, 0), (7, 16400, 16, 48, 32, 16), (1000, 528, 0, 16, 0, 0),
]


@pytest.mark.parametrize("case", CASES + TMA_BURST_CASES, ids=lambda c: "x".join(map(str, c)))
def test_copy_ext_matches_oracle(torch_cuda, dcopy, oracle, case, burst_path):
    torch = torch_cuda
    count, blen, sgap, dgap, soff, doff = case
    src_span = (count - 1) * (blen + sgap) + blen
    dst_span = (count - 1) * (blen + dgap) + blen
    src_np = _rand_bytes(src_span + soff, seed=count * 31 + blen)
    dst_np = np.full(dst_span + doff + 64, CANARY, dtype=np.uint8)
    oracle.copy_ext(dst_np[doff:], src_np[soff:], count, blen, sgap, dgap)
    src = torch.from_numpy(src_np).cuda()
    dst = _canary(torch, dst_span + doff + 64)
    dcopy.copy_ext(dst.data_ptr() + doff, src.data_ptr() + soff, count, blen, sgap, dgap)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == dst_np.tobytes()
    if burst_path:
        assert dcopy.tma_error() == 0  # no bounded wait gave up


def test_copy_ext_32b_units(torch_cuda, dcopy):
    torch = torch_cuda
    src = torch.from_numpy(_rand_bytes(1 << 20, 1)).cuda()
    a = _canary(torch, 1 << 19)
    b = _canary(torch, 1 << 19)
    dcopy.copy_ext_32b(a, src, 100, 4, 12, 2)
    dcopy.copy_ext(b, src, 100, 128, 384, 64)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_config1_contiguous_fp16(torch_cuda, dcopy):
    """262,144 fp16, 8 'cores' x 16 tiles of blockLen 4 KiB."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(262144, generator=g, device="cuda") * 2 - 1).half()
    y = torch.full_like(x, float("nan"))
    # As one DataCopyExt call (blockCount=128 tiles, blockLen=128 x 32 B, gaps 0) ...
    dcopy.copy_ext_32b(y, x, 128, 128, 0, 0)
    torch.cuda.synchronize()
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    # ... and as the per-core tiles of the reference's tiling (8 cores x 16 tiles x 2,048 elems).
    y2 = torch.full_like(x, float("nan"))
    for core in range(8):
        off = core * 16 * 2048
        for tile in range(16):
            o = off + tile * 2048
            dcopy.copy_ext(y2[o:], x[o:], 1, 4096, 0, 0)
    torch.cuda.synchronize()
    assert torch.equal(x.view(torch.int16), y2.view(torch.int16))


def test_config2_strided_gather_fp32(torch_cuda, dcopy):
    """fp32 [4096, 4096] cols 1024..2047 -> [4096, 1024]."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(1)
    src = torch.rand(4096, 4096, generator=g, device="cuda")
    dst = torch.full((4096, 1024), float("nan"), device="cuda")
    dcopy.copy_ext_32b(dst, src[:, 1024:], 4096, 128, 384, 0)
    torch.cuda.synchronize()
    assert torch.equal(dst.view(torch.int32), src[:, 1024:2048].contiguous().view(torch.int32))


@pytest.mark.parametrize("blen", [32, 64, 128, 512, 4096, 65536])
@pytest.mark.parametrize("gapx", [0, 1, 4, 16])
def test_config3_sweep_point(torch_cuda, dcopy, blen, gapx):
    """BASELINE config 3 point at 1/16 size (16 MiB moved); int32 element-index source."""
    torch = torch_cuda
    moved = 16 << 20
    count = moved // blen
    gap = gapx * blen
    src = torch.arange((count * (blen + gap)) // 4, dtype=torch.int32, device="cuda")
    dst = torch.full((moved // 4,), -1, dtype=torch.int32, device="cuda")
    dcopy.copy_ext(dst, src, count, blen, gap, 0)
    torch.cuda.synchronize()
    expect = src.view(count, (blen + gap) // 4)[:, : blen // 4].reshape(-1)
    assert torch.equal(dst, expect)


def test_config3_full_size_point(torch_cuda, dcopy):
    """One full-size config 3 point (256 MiB moved, gap 16x, 4.25 GiB source)."""
    torch = torch_cuda
    blen, gap = 4096, 16 * 4096
    count = (256 << 20) // blen
    src = torch.empty((count * (blen + gap)) // 4, dtype=torch.int32, device="cuda")
    src.copy_(torch.arange(src.numel(), dtype=torch.int32, device="cuda"))
    dst = torch.full(((256 << 20) // 4,), -1, dtype=torch.int32, device="cuda")
    dcopy.copy_ext(dst, src, count, blen, gap, 0)
    torch.cuda.synchronize()
    expect = src.view(count, (blen + gap) // 4)[:, : blen // 4].reshape(-1)
    assert torch.equal(dst, expect)
    del src, dst, expect
    torch.cuda.empty_cache()


def test_overlap_and_extent_refused(torch_cuda, dcopy, cuda_malloc):
    torch = torch_cuda
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext(buf.data_ptr() + 100, buf.data_ptr(), 10, 64, 0, 0)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with cuda_malloc(4096) as p:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.copy_ext(buf, p, 2, 4096, 0, 0)  # source runs past its 4 KiB allocation
        assert e.value.code == dcopy.ERR_PARAM_INVALID
    dcopy.copy_ext(buf, buf, 0, 64, 0, 0)  # empty copies are a no-op


ND_CASES = [  # (sizes, src_strides, dst_strides, elem_bytes)
    ([9, 6, 7], [1, 63, 9], [42, 7, 1], 4),
    ([3, 5], [8, 1], [5, 1], 2),
    ([2, 3, 4, 5, 6], [360, 120, 30, 6, 1], [1, 2, 6, 24, 120], 1),
    ([100, 33], [40, 1], [33, 1], 8),
    ([7, 9, 11], [1, 7, 63], [99, 11, 1], 16),
    ([4, 4], [0, 1], [4, 1], 4),  # broadcast source rows
]


@pytest.mark.parametrize("case", ND_CASES, ids=lambda c: str(c[0]))
def test_copy_nd_matches_oracle(torch_cuda, dcopy, oracle, case):
    torch = torch_cuda
    sizes, ss, ds, eb = case
    src_elems = sum((s - 1) * st for s, st in zip(sizes, ss)) + 1
    dst_elems = sum((s - 1) * st for s, st in zip(sizes, ds)) + 1
    src_np = _rand_bytes(src_elems * eb, seed=len(sizes))
    dst_np = np.full(dst_elems * eb, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(dst_np, src_np, sizes, ss, ds, eb) == 0
    src = torch.from_numpy(src_np).cuda()
    dst = _canary(torch, dst_elems * eb)
    dcopy.copy_nd(dst, src, sizes, ss, ds, eb)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == dst_np.tobytes()


def test_pinned_host_buffers(torch_cuda, dcopy, oracle):
    """Source and destination in pinned host memory: the kernels read and write them
    over PCIe (the end-to-end path of the bench); pageable tensors are refused."""
    torch = torch_cuda
    count, blen, sgap = 300, 4096, 12288
    src_np = _rand_bytes(count * (blen + sgap), seed=11)
    expect = np.full(count * blen, CANARY, dtype=np.uint8)
    oracle.copy_ext(expect, src_np, count, blen, sgap, 0)
    h_src = torch.from_numpy(src_np).pin_memory()
    h_dst = torch.full((count * blen,), CANARY, dtype=torch.uint8).pin_memory()
    dcopy.copy_ext(h_dst, h_src, count, blen, sgap, 0)
    torch.cuda.synchronize()
    assert h_dst.numpy().tobytes() == expect.tobytes()
    # An NDDMA box from device memory into a pinned host buffer (odd rows: shift kernel).
    sizes, ss, ds = [4, 9, 55], [9 * 60, 60, 1], [9 * 55, 55, 1]
    box_np = _rand_bytes(4 * 9 * 60 * 2, seed=12)
    box_exp = np.full(4 * 9 * 55 * 2, CANARY, dtype=np.uint8)
    assert oracle.copy_nd(box_exp, box_np, sizes, ss, ds, 2) == 0
    h_box = torch.full((box_exp.size,), CANARY, dtype=torch.uint8).pin_memory()
    dcopy.copy_nd(h_box, torch.from_numpy(box_np).cuda(), sizes, ss, ds, 2)
    torch.cuda.synchronize()
    assert h_box.numpy().tobytes() == box_exp.tobytes()
    with pytest.raises(ValueError):
        dcopy.copy_ext(torch.empty(16, dtype=torch.uint8), h_src, 1, 16, 0, 0)


@pytest.mark.parametrize("n_copies", [1, 7, 128, 300])
def test_copy_ext_batch_matches_oracle(torch_cuda, dcopy, oracle, n_copies):
    """Independent copies of random shapes (aligned and unaligned) in one batch; 300
    copies take two launches.  Each destination region is checked with the oracle and
    the bytes between regions must keep their canary."""
    torch = torch_cuda
    rng = np.random.default_rng(n_copies)
    src_np = _rand_bytes(1 << 22, seed=n_copies + 1)
    src = torch.from_numpy(src_np).cuda()
    expect = np.full(1 << 23, CANARY, dtype=np.uint8)
    dst = _canary(torch, expect.size)
    copies, at = [], 0
    for _ in range(n_copies):
        count = int(rng.integers(1, 40))
        blen = int(rng.choice([int(rng.integers(1, 200)), 16 * int(rng.integers(1, 40))]))
        sgap, dgap = int(rng.integers(0, 100)), int(rng.integers(0, 20))
        src_span = (count - 1) * (blen + sgap) + blen
        dst_span = (count - 1) * (blen + dgap) + blen
        soff = int(rng.integers(0, src_np.size - src_span))
        at += int(rng.integers(0, 40))
        oracle.copy_ext(expect[at:], src_np[soff:], count, blen, sgap, dgap)
        copies.append((dst.data_ptr() + at, src.data_ptr() + soff, count, blen, sgap, dgap))
        at += dst_span
    assert at < expect.size
    dcopy.copy_ext_batch(copies)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


def test_copy_ext_batch_refuses_overlaps(torch_cuda, dcopy):
    torch = torch_cuda
    a = _canary(torch, 1 << 16)
    b = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    base_a, base_b = a.data_ptr(), b.data_ptr()
    # Two destinations overlapping: refused, nothing written.
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext_batch([(base_a, base_b, 1, 256, 0, 0), (base_a + 128, base_b + 4096, 1, 256, 0, 0)])
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    # A destination overlapping another copy's source: refused.
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext_batch([(base_a, base_b, 1, 256, 0, 0), (base_b + 8192, base_a + 64, 1, 64, 0, 0)])
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    torch.cuda.synchronize()
    assert (a.cpu().numpy() == CANARY).all()
    # Sources may overlap each other.
    dcopy.copy_ext_batch([(base_a, base_b, 4, 64, 0, 0), (base_a + 1024, base_b + 32, 4, 64, 0, 0)])
    torch.cuda.synchronize()
    out = a.cpu().numpy()
    assert (out[:256] == 0).all() and (out[1024:1280] == 0).all() and (out[256:1024] == CANARY).all()


@pytest.mark.parametrize("seed", range(12))
def test_copy_ext_loop_matches_oracle(torch_cuda, dcopy, oracle, seed):
    """LoopModeParams: the DataCopyExt copy inside two outer loops
    (reg_api_call_utils.h:17-25), against the oracle's restatement of the loop nest."""
    torch = torch_cuda
    rng = np.random.default_rng(300 + seed)
    count, blen = int(rng.integers(1, 20)), int(rng.choice([int(rng.integers(1, 90)), 64, 256]))
    sgap, dgap = int(rng.integers(0, 40)), int(rng.integers(0, 12))
    inner_src = (count - 1) * (blen + sgap) + blen
    inner_dst = (count - 1) * (blen + dgap) + blen
    l1, l2 = int(rng.integers(1, 5)), int(rng.integers(1, 4))
    l1s = int(rng.choice([0, inner_src + int(rng.integers(0, 50)), int(rng.integers(1, 30))]))
    l1d = inner_dst + int(rng.integers(0, 20))
    l2s = l1 * max(l1s, 1) + inner_src + int(rng.integers(0, 64))
    l2d = l1 * l1d + int(rng.integers(0, 32))
    soff, doff = int(rng.integers(0, 16)), int(rng.integers(0, 16))
    src_np = _rand_bytes((l2 - 1) * l2s + (l1 - 1) * l1s + inner_src + soff, seed=seed)
    expect = np.full((l2 - 1) * l2d + (l1 - 1) * l1d + inner_dst + doff + 32, CANARY, dtype=np.uint8)
    oracle.copy_ext_loop(expect[doff:], src_np[soff:], count, blen, sgap, dgap, (l1, l1s, l1d),
                         (l2, l2s, l2d))
    src = torch.from_numpy(src_np).cuda()
    dst = _canary(torch, expect.size)
    dcopy.copy_ext_loop(dst.data_ptr() + doff, src.data_ptr() + soff, count, blen, sgap, dgap,
                        (l1, l1s, l1d), (l2, l2s, l2d))
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == expect.tobytes()


@pytest.mark.parametrize("ce_return", [False, True])
@pytest.mark.parametrize("staging_bursts", [1000, 3, 7])
def test_copy_ext_staged_matches_oracle(torch_cuda, dcopy, oracle, ce_return, staging_bursts):
    """Host -> host DataCopyExt through a device staging buffer: the copy engine gathers
    chunks, the kernel (or the copy engine) writes them back; a staging buffer of a few
    bursts runs as a ring of two slots."""
    torch = torch_cuda
    count, blen, sgap, dgap = 300, 96, 160, 32
    src_np = _rand_bytes((count - 1) * (blen + sgap) + blen, seed=21)
    expect = np.full((count - 1) * (blen + dgap) + blen + 16, CANARY, dtype=np.uint8)
    oracle.copy_ext(expect, src_np, count, blen, sgap, dgap)
    h_src = torch.from_numpy(src_np).pin_memory()
    h_dst = torch.full((expect.size,), CANARY, dtype=torch.uint8).pin_memory()
    staging = torch.empty(staging_bursts * blen, dtype=torch.uint8, device="cuda")
    flags = dcopy.STAGED_COPY_ENGINE_RETURN if ce_return else 0
    dcopy.copy_ext_staged(h_dst, h_src, count, blen, sgap, dgap, staging, flags=flags)
    torch.cuda.current_stream().synchronize()
    assert h_dst.numpy().tobytes() == expect.tobytes()


def test_copy_ext_staged_pageable_and_refusals(torch_cuda, dcopy, oracle):
    torch = torch_cuda
    count, blen, sgap = 64, 4096, 12288
    src_np = _rand_bytes((count - 1) * (blen + sgap) + blen, seed=22)
    expect = np.zeros(count * blen, dtype=np.uint8)
    oracle.copy_ext(expect, src_np, count, blen, sgap, 0)
    staging = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    pageable = np.zeros(count * blen, dtype=np.uint8)
    # Pageable host memory both ways: the copy engine writes the result back.
    dcopy.copy_ext_staged(pageable, src_np, count, blen, sgap, 0, staging,
                          flags=dcopy.STAGED_COPY_ENGINE_RETURN)
    torch.cuda.current_stream().synchronize()
    assert pageable.tobytes() == expect.tobytes()
    # The kernel cannot write pageable memory: refused before anything runs.
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext_staged(np.zeros(count * blen, dtype=np.uint8), src_np, count, blen, sgap,
                              0, staging)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:  # staging smaller than two bursts
        dcopy.copy_ext_staged(pageable, src_np, count, blen, sgap, 0, staging, staging_bytes=blen,
                              flags=dcopy.STAGED_COPY_ENGINE_RETURN)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


@pytest.mark.parametrize("sizes,ds", [([2, 4], [1, 1]), ([3, 4], [2, 1]), ([4, 16], [8, 1])])
def test_copy_nd_refuses_repeating_destinations(torch_cuda, dcopy, sizes, ds):
    """A destination box whose elements repeat is PARAM_INVALID and leaves dst untouched."""
    torch = torch_cuda
    src = torch.arange(256, dtype=torch.uint8, device="cuda")
    dst = _canary(torch, 256)
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_nd(dst, src, sizes, [sizes[1], 1], ds, 1)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    torch.cuda.synchronize()
    assert bool((dst == CANARY).all())
