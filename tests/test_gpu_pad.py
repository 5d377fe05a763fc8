"""DataCopyPad with the Unified-Buffer side conventions on the GPU, bit for bit against
the oracle (oracle_copy_pad_gm_to_ub / oracle_copy_pad_ub_to_gm): fp16, fp32 and int8
blocks whose length is not a multiple of 32 bytes, Normal and Compact modes, UB strides
in 32-byte blocks, padding elements and values, and DataCopyPadExtend's element-unit
entry points.  Destinations are canary-filled: bytes the reference does not write must
keep the canary."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0xA5

CASES = [  # (eb, count, blen bytes, gm gap bytes, ub gap blocks, mode, (isPad, left, right, value))
    (2, 37, 6, 10, 0, 0, (True, 0, 0, 0)),            # fp16, 3 elements per block
    (2, 5, 70, 2, 1, 0, (True, 1, 2, 0x3C00)),         # fp16, padding elements of 1.0
    (4, 129, 12, 20, 2, 0, (True, 0, 0, 0)),           # fp32, 3 elements
    (4, 64, 100, 0, 0, 0, (False, 0, 0, 0)),           # fp32, no padding values
    (4, 33, 44, 4, 0, 1, (True, 0, 0, 0x7FC00000)),    # fp32 Compact, NaN rounds the end
    (1, 300, 31, 1, 0, 0, (True, 3, 5, 0x5A)),         # int8
    (1, 1000, 33, 95, 3, 1, (True, 0, 0, 0)),          # int8 Compact, UB gaps
    (1, 2, 4096 + 7, 0, 0, 0, (True, 0, 0, 0x11)),     # long blocks (bulk and shift paths)
    (8, 17, 24, 8, 1, 0, (True, 1, 0, 0x0123456789ABCDEF)),  # 8-byte elements
]


def _rand(n, seed):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"eb{c[0]}-n{c[1]}-L{c[2]}-m{c[5]}")
def test_gm_to_ub_and_back_match_oracle(torch_cuda, dcopy, oracle, case):
    torch = torch_cuda
    eb, n, blen, sgap, ublocks, mode, pad = case
    gm_np = _rand((n - 1) * (blen + sgap) + blen, seed=n + blen)
    span = oracle.pad_ub_span(n, blen, ublocks, mode, pad[1], pad[2], eb)
    ub_expect = np.full(span + 64, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub_expect, gm_np, n, blen, sgap, ublocks, mode, pad, eb) == 0
    gm = torch.from_numpy(gm_np).cuda()
    ub = torch.full((ub_expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_pad_gm_to_ub(ub, gm, n, blen, sgap, ublocks, mode, pad, eb)
    torch.cuda.synchronize()
    assert ub.cpu().numpy().tobytes() == ub_expect.tobytes()
    if pad[1] or pad[2]:
        return  # UB -> GM has no padding elements: the slot layouts differ
    # UB -> GM from the same UB image, into a GM layout with its own gaps.
    dgap = 3 * eb
    back_expect = np.full((n - 1) * (blen + dgap) + blen + 16, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_ub_to_gm(back_expect, ub_expect, n, blen, ublocks, dgap, mode) == 0
    back = torch.full((back_expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.copy_pad_ub_to_gm(back, ub, n, blen, ublocks, dgap, mode)
    torch.cuda.synchronize()
    assert back.cpu().numpy().tobytes() == back_expect.tobytes()
    for i in range(n):  # the round trip gives every block back
        assert back_expect[i * (blen + dgap):i * (blen + dgap) + blen].tobytes() == \
            gm_np[i * (blen + sgap):i * (blen + sgap) + blen].tobytes()


@pytest.mark.parametrize("dtype,eb", [("float16", 2), ("float32", 4), ("int8", 1)])
@pytest.mark.parametrize("mode", [0, 1])
def test_datacopy_pad_extend_units(torch_cuda, dcopy, oracle, dtype, eb, mode):
    """DataCopyPadExtend in elements (datacopy.h:14-40): the GM -> UB overload converts
    dst_stride to 32-byte blocks rounding down and pads with zeros; UB -> GM converts
    src_stride the same way."""
    torch = torch_cuda
    align_num = 32 // eb
    count, blk, ss, ds = 19, 13, 7, 3 * align_num + (align_num - 1)  # ds -> 3 blocks
    gm_np = _rand((count - 1) * (blk + ss) * eb + blk * eb, seed=eb)
    span = oracle.pad_ub_span(count, blk * eb, ds // align_num, mode, 0, 0, eb)
    ub_expect = np.full(span + 32, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub_expect, gm_np, count, blk * eb, ss * eb, ds // align_num,
                                    mode, (True, 0, 0, 0), eb) == 0
    gm = torch.from_numpy(gm_np).cuda()
    ub = torch.full((ub_expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.datacopy_pad_extend(ub, gm, eb, count, blk, ss, ds, to_ub=True, mode=mode)
    torch.cuda.synchronize()
    assert ub.cpu().numpy().tobytes() == ub_expect.tobytes()
    out_expect = np.full((count - 1) * (blk + 5) * eb + blk * eb, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_ub_to_gm(out_expect, ub_expect, count, blk * eb, ds // align_num,
                                    5 * eb, mode) == 0
    out = torch.full((out_expect.size,), CANARY, dtype=torch.uint8, device="cuda")
    dcopy.datacopy_pad_extend(out, ub, eb, count, blk, ds, 5, to_ub=False, mode=mode)
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == out_expect.tobytes()


def test_refusals(torch_cuda, dcopy, cuda_malloc):
    torch = torch_cuda
    gm = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    ub = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    for kw in (dict(elem_bytes=3), dict(elem_bytes=2, block_len=7), dict(mode=5),
               dict(pad=(True, 9, 0, 0), elem_bytes=4)):
        a = dict(block_len=8, elem_bytes=1, mode=0, pad=(True, 0, 0, 0))
        a.update(kw)
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.copy_pad_gm_to_ub(ub, gm, 4, a["block_len"], 0, 0, a["mode"], a["pad"],
                                    a["elem_bytes"])
        assert e.value.code == dcopy.ERR_PARAM_INVALID
    # The UB image of 200 blocks (200 x 32 bytes) would run past an exact-size
    # 4096-byte allocation (torch's caching allocator would hide the overrun inside
    # a larger segment, so the buffer is a raw cudaMalloc).
    with cuda_malloc(4096) as raw_ub:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.copy_pad_gm_to_ub(raw_ub, gm, 200, 8, 0, 0)
        assert e.value.code == dcopy.ERR_PARAM_INVALID
