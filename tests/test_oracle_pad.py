"""The oracle's DataCopyPad with the Unified-Buffer side conventions, checked on the
CPU: the unit conversions of DataCopyPadExtend (ge/compiler/graph/optimize/autofuse/
ascendc/api/datacopy.h:14-40) on the argument lists GE's codegen emits in its own
tests, and the slot layout of Normal and Compact modes on hand-worked cases.

The bytes a real UB holds in its padding positions are not pinned: the reference has
no vectors for them.  What is pinned here is the addressing: where each block lands,
which bytes are padding, and which bytes are never touched."""
import numpy as np
import pytest

CANARY = 0xA5


def _ext_params_load(eb, block_count, block_len, src_stride, dst_stride):
    """DataCopyPadExtend GM -> UB (datacopy.h:16-22): DataCopyExtParams from elements."""
    align_num = 32 // eb
    return block_count, block_len * eb, src_stride * eb, dst_stride // align_num


def _ext_params_store(eb, block_count, block_len, src_stride, dst_stride):
    """DataCopyPadExtend UB -> GM (datacopy.h:31-37)."""
    align_num = 32 // eb
    return block_count, block_len * eb, src_stride // align_num, dst_stride * eb


# Argument lists from GE's codegen tests (T, block_count, block_len, src_stride, dst_stride):
#  - tests/autofuse/ut/codegen/api_call/test_codegen_store_api_call.cpp:131, :139 (store of
#    an int16 output, :87: `DataCopyPadExtend(local_1[0 + 0], local_0, 1, 1, 16 - 1, 0)`, and
#    the same with block_count z0_t_size, taken as 5 here);
#  - tests/autofuse/v35/ut/codegen/reg_api_call/test_codegen_load_reg_api_call.cpp:89, :163
#    (loads of float: `(…, 1, 8, 0, 0)` and `(…, 4, 2, 2, 2 - 2, {loop params})`, whose
#    outer loop is LoopModeParams, covered by the copy_ext_loop tests).
CODEGEN_CASES = [
    ("store", 2, 1, 1, 16 - 1, 0),
    ("store", 2, 5, 1, 16 - 1, 0),
    ("load", 4, 1, 8, 0, 0),
    ("load", 4, 4, 2, 2, 2 - 2),
]


@pytest.mark.parametrize("case", CODEGEN_CASES, ids=lambda c: f"{c[0]}-{c[2]}x{c[3]}")
def test_codegen_call_sites_through_the_oracle(oracle, case):
    kind, eb, count, blen, ss, ds = case
    rng = np.random.default_rng(count * 100 + blen)
    if kind == "load":
        n, L, sgap, ublocks = _ext_params_load(eb, count, blen, ss, ds)
        gm = rng.integers(0, 256, (n - 1) * (L + sgap) + L, dtype=np.uint8)
        span = oracle.pad_ub_span(n, L, ublocks, 0, 0, 0, eb)
        ub = np.full(span + 64, CANARY, dtype=np.uint8)
        assert oracle.copy_pad_gm_to_ub(ub, gm, n, L, sgap, ublocks, 0, (True, 0, 0, 0), eb) == 0
        slot = (L + 31) // 32 * 32
        for i in range(n):  # block i at i*(slot + 32*ublocks); zero padding to the slot end
            b = ub[i * (slot + 32 * ublocks):]
            assert b[:L].tobytes() == gm[i * (L + sgap):i * (L + sgap) + L].tobytes()
            assert (b[L:slot] == 0).all()
        assert (ub[span:] == CANARY).all()
        if (count, blen, ss, ds) == (4, 2, 2, 0):  # four 8-byte blocks, one 32-byte slot each
            assert (n, L, sgap, ublocks) == (4, 8, 8, 0) and span == 4 * 32
    else:
        n, L, ublocks, dgap = _ext_params_store(eb, count, blen, ss, ds)
        # `16 - 1` int16 elements = 30 bytes: 0 whole 32-byte blocks (rounded down).
        assert (L, ublocks, dgap) == (2, 0, 0)
        ub = rng.integers(0, 256, n * 32, dtype=np.uint8)
        gm = np.full(n * L + 16, CANARY, dtype=np.uint8)
        assert oracle.copy_pad_ub_to_gm(gm, ub, n, L, ublocks, dgap, 0) == 0
        for i in range(n):  # UB slot pitch = 32: the 2-byte block rounded up, no stride block
            assert gm[i * L:(i + 1) * L].tobytes() == ub[i * 32:i * 32 + L].tobytes()
        assert (gm[n * L:] == CANARY).all()


def test_normal_mode_padding_layout(oracle):
    """fp16 blocks of 3 elements, 1 left and 2 right padding elements, value 0x1234:
    slot = round_up(2 + 6 + 4, 32) = 32; the UB stride gap is 1 block."""
    gm = np.arange(64, dtype=np.uint8)
    ub = np.full(200, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub, gm, 3, 6, 4, 1, 0, (True, 1, 2, 0x1234), 2) == 0
    for i in range(3):
        b = ub[i * 64:i * 64 + 64]
        assert b[:2].tolist() == [0x34, 0x12]                     # left padding element
        assert b[2:8].tolist() == list(range(i * 10, i * 10 + 6))  # the block
        assert b[8:32].tolist() == [0x34, 0x12] * 12               # right padding + round-up
        assert (b[32:64] == CANARY).all() or i == 2                # the stride gap: untouched
    assert oracle.pad_ub_span(3, 6, 1, 0, 1, 2, 2) == 2 * 64 + 32
    assert (ub[160:] == CANARY).all()


def test_compact_mode_packs_blocks_and_rounds_the_end(oracle):
    """int32 blocks of 12 bytes, Compact: blocks packed at 12-byte pitch, then the
    transfer's end (36 bytes) rounded up to 64 with the padding value."""
    gm = np.arange(100, dtype=np.uint8)
    ub = np.full(96, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub, gm, 3, 12, 20, 0, 1, (True, 0, 0, 0xDEADBEEF), 4) == 0
    for i in range(3):
        assert ub[i * 12:i * 12 + 12].tolist() == list(range(i * 32, i * 32 + 12))
    assert ub[36:64].tolist() == [0xEF, 0xBE, 0xAD, 0xDE] * 7
    assert (ub[64:] == CANARY).all()
    assert oracle.pad_ub_span(3, 12, 0, 1, 0, 0, 4) == 64
    # Without isPad nothing but the blocks is written.
    ub2 = np.full(96, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub2, gm, 3, 12, 20, 0, 1, (False, 0, 0, 7), 4) == 0
    assert (ub2[36:] == CANARY).all()
    # And back: UB -> GM in Compact mode reads 12-byte slots.
    back = np.full(3 * 16, CANARY, dtype=np.uint8)
    assert oracle.copy_pad_ub_to_gm(back, ub, 3, 12, 0, 4, 1) == 0
    for i in range(3):
        assert back[i * 16:i * 16 + 12].tolist() == list(range(i * 32, i * 32 + 12))
        assert (back[i * 16 + 12:i * 16 + 16] == CANARY).all()


@pytest.mark.parametrize("bad", [
    dict(eb=3), dict(blen=7, eb=2), dict(left=9, eb=4), dict(right=33, eb=1), dict(mode=2)])
def test_refusals(oracle, bad):
    a = dict(blen=8, eb=1, left=0, right=0, mode=0)
    a.update(bad)
    gm = np.zeros(64, dtype=np.uint8)
    ub = np.zeros(256, dtype=np.uint8)
    assert oracle.copy_pad_gm_to_ub(ub, gm, 2, a["blen"], 0, 0, a["mode"],
                                    (True, a["left"], a["right"], 0), a["eb"]) == -1
