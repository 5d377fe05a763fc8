"""Pins the oracle's standalone_datacopy restatement to the reference's own Python twin.

Fixtures: tests/golden/standalone_plans.json (profile.py:88-99 tile_plan over a
grid of shapes) and tests/golden/address_model.json (test_address_model.py:13-34
model() digests), both written by tests/golden/make_golden.py.
"""
import hashlib
import importlib.util
import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN


def _plans():
    return json.loads((GOLDEN / "standalone_plans.json").read_text())["cases"]


def _models():
    return json.loads((GOLDEN / "address_model.json").read_text())["cases"]


def test_plan_matches_reference_tile_plan(oracle):
    cases = _plans()
    assert len(cases) > 1000
    for rows, cols, kib, tile_cols, tile_bytes, tile_count in cases:
        rc, t = oracle.plan_tiling(rows, cols, kib, 1)
        if tile_cols is None:
            assert rc == oracle.EPARAM, (rows, cols, kib)
        else:
            assert rc == oracle.OK, (rows, cols, kib)
            assert (t.tile_cols, t.ub_bytes) == (tile_cols, tile_bytes)
            assert (cols + t.tile_cols - 1) // t.tile_cols == tile_count


def test_reference_budget_cases(oracle):
    # test_address_model.py:46-52
    assert oracle.plan_tiling(256, 768, 8)[1].tile_cols == 8
    rc, t = oracle.plan_tiling(256, 768, 240)
    assert rc == 0 and (768 + t.tile_cols - 1) // t.tile_cols == 4
    for shape in [(7, 100, 8), (256, 768, 256), (4096, 100, 8), (512, 768, 1), (8, 0, 8)]:
        assert oracle.plan_tiling(*shape)[0] == oracle.EPARAM


@pytest.mark.parametrize("case", _models(), ids=lambda c: f"{c['rows']}x{c['cols']}k{c['kib']}"
                         f"{'p' if c['pretranspose'] else ''}")
def test_run_tiles_matches_address_model(oracle, case):
    rows, cols, kib = case["rows"], case["cols"], case["kib"]
    a = np.arange(rows * cols, dtype=np.int32)
    rc, t = oracle.plan_tiling(rows, cols, kib, 1)
    assert rc == 0
    y = np.full(rows * cols, -0x5A5A5A5B, dtype=np.int32)
    if case["pretranspose"]:
        b = np.empty_like(a)
        assert oracle.run_tiles(1, a, b, t) == 0
        assert oracle.run_tiles(2, b, y, t) == 0
    else:
        assert oracle.run_tiles(0, a, y, t) == 0
    assert y.size == case["len"]
    assert y[:16].tolist() == case["head"]
    assert hashlib.sha256(y.astype("<i4").tobytes()).hexdigest() == case["sha256"]


def test_store0_writes_nothing(oracle):
    rc, t = oracle.plan_tiling(128, 513, 4, 0)
    assert rc == 0
    a = oracle.fill_pattern(128 * 513)
    y = np.full(128 * 513, 0x7A7A7A7A, dtype=np.int32)
    assert oracle.run_tiles(0, a, y, t) == 0
    assert (y == 0x7A7A7A7A).all()
    # pretranspose ignores store (asc:52): B is always written.
    b = np.zeros_like(a)
    assert oracle.run_tiles(1, a, b, t) == 0
    assert (b.reshape(513, 128) == a.reshape(128, 513).T).all()


def test_demo_verification_rule(oracle):
    # asc:124-125 input pattern and asc:151-154 check: output[c*rows + r] == input[r*cols + c].
    rows, cols = 256, 768
    a = oracle.fill_pattern(rows * cols)
    assert a[1] == 20 and a[2] == 37
    rc, t = oracle.plan_tiling(rows, cols, 8, 1)
    y = np.empty_like(a)
    assert oracle.run_tiles(0, a, y, t) == 0
    assert (y.reshape(cols, rows) == a.reshape(rows, cols).T).all()


def test_check_tiling_rejects_unrunnable(oracle):
    rc, t = oracle.plan_tiling(64, 100, 8, 1)
    assert rc == 0 and oracle.check_tiling(t) == 0
    for field, value in [("tile_cols", 0), ("tile_cols", 101), ("ub_bytes", t.ub_bytes - 4),
                         ("ub_bytes", 240 * 1024 + 4), ("rows", 60), ("store", 2), ("cols", 0)]:
        bad = oracle.Tiling(t.rows, t.cols, t.tile_cols, t.ub_bytes, t.store)
        setattr(bad, field, value)
        assert oracle.check_tiling(bad) == oracle.EPARAM, field


def test_live_reference_python(oracle, reference_root):
    """Re-runs the reference's own tile_plan/model() on shapes outside the fixture."""
    src = reference_root / "standalone_datacopy"
    spec = importlib.util.spec_from_file_location("profile", src / "profile.py")
    profile = importlib.util.module_from_spec(spec)
    saved = sys.modules.get("profile")
    sys.modules["profile"] = profile
    try:
        spec.loader.exec_module(profile)
        spec2 = importlib.util.spec_from_file_location("ref_tam", src / "test_address_model.py")
        tam = importlib.util.module_from_spec(spec2)
        spec2.loader.exec_module(tam)
        rng = np.random.default_rng(7)
        for _ in range(12):
            rows = int(rng.integers(1, 40)) * 8
            cols = int(rng.integers(1, 300))
            kib = int(rng.integers(1, 241))
            try:
                plan = profile.tile_plan(rows, cols, kib)
            except ValueError:
                assert oracle.plan_tiling(rows, cols, kib)[0] == oracle.EPARAM
                continue
            rc, t = oracle.plan_tiling(rows, cols, kib)
            assert rc == 0 and t.tile_cols == plan["tile_cols"]
            for pre in (False, True):
                expect = np.asarray(tam.model(rows, cols, kib, pre), dtype=np.int32)
                a = np.arange(rows * cols, dtype=np.int32)
                y = np.empty_like(a)
                if pre:
                    b = np.empty_like(a)
                    oracle.run_tiles(1, a, b, t)
                    oracle.run_tiles(2, b, y, t)
                else:
                    oracle.run_tiles(0, a, y, t)
                assert (y == expect).all()
    finally:
        if saved is not None:
            sys.modules["profile"] = saved
        else:
            sys.modules.pop("profile", None)


def test_copy_ext_gap_addressing(oracle):
    # The RunTiles gather is a DataCopyExt with blockLen=4, gap=(cols-1)*4 (asc:32-35):
    # one column of A, gathered with the generic gap copy, equals that column.
    rows, cols = 24, 37
    a = np.arange(rows * cols, dtype=np.int32)
    for c in (0, 5, cols - 1):
        col = np.empty(rows, dtype=np.int32)
        oracle.copy_ext(col, a[c:], rows, 4, (cols - 1) * 4, 0)
        assert (col == a.reshape(rows, cols)[:, c]).all()
    # Destination gaps are skipped, not written.
    src = np.arange(64, dtype=np.uint8)
    dst = np.full(96, 0xEE, dtype=np.uint8)
    oracle.copy_ext(dst, src, 4, 16, 0, 8)
    for i in range(4):
        assert (dst[i * 24:i * 24 + 16] == src[i * 16:(i + 1) * 16]).all()
        if i < 3:
            assert (dst[i * 24 + 16:i * 24 + 24] == 0xEE).all()


def test_copy_ext_threads_agree(oracle):
    rng = np.random.default_rng(3)
    src = rng.integers(0, 255, size=1 << 20, dtype=np.uint8)
    d1 = np.zeros(1 << 19, dtype=np.uint8)
    d2 = np.zeros_like(d1)
    oracle.copy_ext(d1, src, 1000, 300, 700, 100)
    oracle.copy_ext(d2, src, 1000, 300, 700, 100, threads=7)
    assert (d1 == d2).all()


def test_copy_nd_matches_numpy(oracle):
    rng = np.random.default_rng(5)
    src = rng.integers(0, 1 << 30, size=(6, 7, 9), dtype=np.int32)
    # Permute axes (2, 0, 1) into a contiguous destination.
    dst = np.empty((9, 6, 7), dtype=np.int32)
    sizes = [9, 6, 7]
    s_strides = [1, 63, 9]
    d_strides = [42, 7, 1]
    assert oracle.copy_nd(dst, src, sizes, s_strides, d_strides, 4) == 0
    assert (dst == np.transpose(src, (2, 0, 1))).all()


def test_copy_ext_loop_is_the_loop_nest(oracle):
    """oracle_copy_ext_loop equals GE codegen's documented loop nest around the gap copy,
    checked against a numpy restatement of the same addresses."""
    rng = np.random.default_rng(77)
    count, blen, sgap, dgap = 5, 24, 8, 4
    l1, l1s, l1d = 3, 200, 150
    l2, l2s, l2d = 2, 700, 500
    src = rng.integers(0, 256, size=2000, dtype=np.uint8)
    got = np.zeros(1200, dtype=np.uint8)
    oracle.copy_ext_loop(got, src, count, blen, sgap, dgap, (l1, l1s, l1d), (l2, l2s, l2d))
    want = np.zeros_like(got)
    for i in range(l2):
        for j in range(l1):
            for b in range(count):
                s0 = i * l2s + j * l1s + b * (blen + sgap)
                d0 = i * l2d + j * l1d + b * (blen + dgap)
                want[d0:d0 + blen] = src[s0:s0 + blen]
    assert got.tobytes() == want.tobytes()
