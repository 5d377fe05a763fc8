"""CPU checks of the C ABI: the library loads, exports every declared symbol, and its
host-only entry points (planner, NZ shape rules, status mapping, argument
validation that precedes any launch) agree with the oracle and the reference.
No kernel is launched here."""
import json
import os
import re

import pytest

from conftest import GOLDEN, ROOT


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").rglob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(dcopy_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol(dcopy):
    names = _declared_symbols()
    assert len(names) >= 14
    lib = dcopy.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_status_mapping(dcopy):
    assert dcopy.lib().dcopy_version() >= 100
    assert dcopy.status_to_ge(0) == 0
    assert dcopy.status_to_ge(dcopy.ERR_PARAM_INVALID) == 145000
    assert dcopy.status_to_ge(dcopy.ERR_SHAPE_INVALID) == 145021
    assert dcopy.status_to_ge(dcopy.ERR_DATATYPE_INVALID) == 145022
    assert dcopy.status_to_ge(dcopy.ERR_FORMAT_INVALID) == 145020


def test_plan_tiling_matches_reference_fixture(dcopy):
    cases = json.loads((GOLDEN / "standalone_plans.json").read_text())["cases"]
    for rows, cols, kib, tile_cols, tile_bytes, _count in cases:
        if tile_cols is None:
            with pytest.raises(dcopy.DcopyError) as e:
                dcopy.plan_tiling(rows, cols, kib, 1)
            assert e.value.code == dcopy.ERR_PARAM_INVALID
        else:
            t = dcopy.plan_tiling(rows, cols, kib, 1)
            assert (t.rows, t.cols, t.tile_cols, t.ub_bytes, t.store) == \
                (rows, cols, tile_cols, tile_bytes, 1)


def test_plan_tiling_messages_follow_reference(dcopy):
    with pytest.raises(dcopy.DcopyError, match="Tile budget must hold a complete transposed row"):
        dcopy.plan_tiling(512, 768, 1, 1)
    with pytest.raises(dcopy.DcopyError, match="64 MiB"):
        dcopy.plan_tiling(4088, 65535, 240, 1)
    with pytest.raises(dcopy.DcopyError, match="store: 0/1"):
        dcopy.plan_tiling(8, 8, 8, 2)


@pytest.mark.parametrize("shape", [[1], [100], [0], [2, 2, 17, 4], [5, 33], [3, 0, 7],
                                   [16, 4096, 4096], [1, 1, 1, 1, 1, 1, 31, 17]])
@pytest.mark.parametrize("w0", [1, 8, 16, 32, 0, -1])
def test_nz_shape_matches_oracle(dcopy, oracle, shape, w0):
    rc, nz, hw = oracle.nz_shape(shape, w0)
    if rc:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.nz_shape(shape, w0)
        assert e.value.code == dcopy.ERR_SHAPE_INVALID
    else:
        assert dcopy.nz_shape(shape, w0) == (nz, hw)


@pytest.mark.parametrize("shape", [[1], [100], [0], [2, 2, 17, 4], [30, 33], [3, 0, 7],
                                   [8, 4096, 4096], [1, 1, 1, 1, 1, 1, 31, 17]])
@pytest.mark.parametrize("c0", [1, 8, 16, 32, 0, -1])
def test_zz_shape_matches_oracle(dcopy, oracle, shape, c0):
    rc, zz, hw = oracle.zz_shape(shape, c0)
    if rc:
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.zz_shape(shape, c0)
        assert e.value.code == dcopy.ERR_SHAPE_INVALID
    else:
        assert dcopy.zz_shape(shape, c0) == (zz, hw)


def test_zz_validation_before_launch(dcopy):
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_zz(0, 0, [4, 4], 3, 16)  # element size not in {1,2,4,8,16}
    assert e.value.code == dcopy.ERR_DATATYPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.zz_to_nd(0, 0, [4, 4], 2, 0)  # the ZZ -> ND loops divide by c0
    assert e.value.code == dcopy.ERR_SHAPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_zz(0, 0, [4, 4], 2, 16)  # NULL buffers with bytes to move
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    dcopy.nd_to_zz(0, 0, [0, 16], 2, 16)  # empty: nothing to move
    f, d = dcopy.FORMAT, dcopy.DATA_TYPE
    assert dcopy.trans_shape(4, f["ND"], [2, 3, 4, 33], d["UINT8"], f["FRACTAL_ZZ"], 32) == \
        [2, 3, 1, 2, 32, 32]
    assert dcopy.trans_tensor_shape(f["NCHW"], [1, 2, 4, 17], d["FLOAT"], f["FRACTAL_ZZ"], 16) \
        == [1, 2, 1, 2, 16, 16]
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.trans_tensor_shape(f["FRACTAL_ZZ"], [1, 1, 16, 16], d["FLOAT"], f["ND"], 16)
    assert e.value.code == dcopy.ERR_FORMAT_INVALID
    # Sizing query without data movement.
    args = dict(src_c0=16, dst_c0=16)
    assert dcopy.trans_format_check(0, 0x1000, f["ND"], f["FRACTAL_ZZ"], [15, 17],
                                    [1, 2, 16, 16], d["FLOAT16"], **args) == 1024


def test_validation_before_launch(dcopy):
    # Each of these fails on the host before any device work.
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_nz(0, 0, [4, 4], 0, 16)
    assert e.value.code == dcopy.ERR_DATATYPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_nz(0, 0, [4, -1], 2, 16)
    assert e.value.code == dcopy.ERR_SHAPE_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.nd_to_nz(0, 0, [4, 4], 2, 16)  # NULL buffers with bytes to move
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext(0, 0, 4, 16, 0, 0)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_nd(0, 0, [2, 2], [2, 1], [0, 1], 4)  # dst stride 0 aliases
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_nd(0, 0, [2, 2], [2, 1], [2, 1], 3)
    assert e.value.code == dcopy.ERR_DATATYPE_INVALID
    dcopy.copy_ext(0, 0, 0, 16, 0, 0)  # nothing to move: OK without touching memory
    dcopy.nd_to_nz(0, 0, [0, 16], 2, 16)
    bad = dcopy.DataCopyTiling(60, 100, 8, 1920, 1)
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.datacopy_small(0, 0, bad)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


def test_error_message_is_thread_local(dcopy):
    import threading
    with pytest.raises(dcopy.DcopyError):
        dcopy.plan_tiling(7, 7, 7, 1)
    seen = []
    t = threading.Thread(target=lambda: seen.append(dcopy.lib().dcopy_last_error_message()))
    t.start()
    t.join()
    assert seen == [b""]
    assert b"rows" in dcopy.lib().dcopy_last_error_message()


def test_nd_tma_selection_round_trips(dcopy):
    """dcopy_set_nd_tma is host state only: it reports the former setting."""
    first = dcopy.set_nd_tma(True)
    assert dcopy.set_nd_tma(False) is True
    assert dcopy.set_nd_tma(first) is False


def test_p2p_engine_selection(dcopy):
    """dcopy_set_p2p_engine is host state only: it reports the former setting and
    refuses an unknown engine without changing the current one."""
    first = dcopy.set_p2p_engine(dcopy.P2P_ENGINE_SM)
    assert dcopy.set_p2p_engine(dcopy.P2P_ENGINE_COPY) == dcopy.P2P_ENGINE_SM
    with pytest.raises(dcopy.DcopyError):
        dcopy.set_p2p_engine(3)
    assert dcopy.set_p2p_engine(first) == dcopy.P2P_ENGINE_COPY


def test_p2p_route_follows_the_engine(dcopy):
    """The route query needs no GPU for the forced engines: COPY routes every copy
    to the copy engine; with SM, memory that is not this GPU's (here: none is)
    takes the load/store kernel."""
    prev = dcopy.set_p2p_engine(dcopy.P2P_ENGINE_COPY)
    try:
        assert dcopy.p2p_route(0x1000, 0x2000, 1 << 30) == dcopy.P2P_ROUTE_COPY_ENGINE
        dcopy.set_p2p_engine(dcopy.P2P_ENGINE_SM)
        assert dcopy.p2p_route(0x1000, 0x2000, 1 << 30) == dcopy.P2P_ROUTE_SM_LOAD_STORE
    finally:
        dcopy.set_p2p_engine(prev)
    assert dcopy.lib().dcopy_p2p_route(None, None, 0, None) == dcopy.ERR_PARAM_INVALID


@pytest.mark.parametrize("value,engine", [(None, 0), ("sm", 1), ("copy", 2), ("2", 2),
                                          ("bogus", 0)])
def test_p2p_engine_from_environment(value, engine):
    """DCOPY_P2P_ENGINE sets the initial engine; unset or unknown means automatic."""
    import subprocess
    import sys
    env = {k: v for k, v in os.environ.items() if k != "DCOPY_P2P_ENGINE"}
    if value is not None:
        env["DCOPY_P2P_ENGINE"] = value
    code = ("import sys; sys.path.insert(0, sys.argv[1]); import dcopy; "
            "print(dcopy.set_p2p_engine(0))")
    out = subprocess.run([sys.executable, "-c", code, str(ROOT / "data-copy_b200")], env=env, check=True,
                         capture_output=True, text=True).stdout
    assert int(out.strip()) == engine


def test_copy_ext_batch_argument_checks(dcopy):
    """Decided on the host before any device work: an empty batch is a no-op, a NULL
    array with a count is refused."""
    dcopy.copy_ext_batch([])
    assert dcopy.lib().dcopy_copy_ext_batch(None, 3, None) == dcopy.ERR_PARAM_INVALID


def test_datacopy_tiles_argument_checks(dcopy):
    t = dcopy.plan_tiling(256, 768, 8, 1)
    for phase, count in ((3, 1), (-1, 1), (0, 0xFFFFFFFF)):
        with pytest.raises(dcopy.DcopyError) as e:
            dcopy.datacopy_tiles(phase, 0x1000, 0x2000, t, 0, count)
        assert e.value.code == dcopy.ERR_PARAM_INVALID


def test_copy_ext_loop_argument_checks(dcopy):
    import ctypes
    p = dcopy.DcopyExtParams(1, 16, 0, 0)
    assert dcopy.lib().dcopy_copy_ext_loop(None, None, ctypes.byref(p), None, None) == \
        dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext_loop(0x1000, 0x2000, 1, 16, 0, 0, (2, 1 << 50, 64))
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    dcopy.copy_ext_loop(0x1000, 0x2000, 0, 16, 0, 0, (2, 64, 64))  # nothing to copy


def test_copy_ext_staged_argument_checks(dcopy):
    import ctypes
    assert dcopy.lib().dcopy_copy_ext_staged(None, None, None, None, 0, 0, None) == \
        dcopy.ERR_PARAM_INVALID
    p = dcopy.DcopyExtParams(4, 64, 0, 0)
    assert dcopy.lib().dcopy_copy_ext_staged(0x1000, 0x2000, ctypes.byref(p), 0x3000, 1 << 20, 6,
                                             None) == dcopy.ERR_PARAM_INVALID  # unknown flags
    assert dcopy.lib().dcopy_copy_ext_staged(0x1000, 0x2000, ctypes.byref(p), None, 1 << 20, 0,
                                             None) == dcopy.ERR_PARAM_INVALID  # no staging


def test_spans_that_would_wrap_are_refused(dcopy):
    """Spans are computed without wrapping: a copy whose span reaches 2^62 bytes is
    refused on the host before any pointer is looked at."""
    big_count, big_gap = 0xFFFFFFFF, 1 << 48
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext(0x1000, 0x2000, big_count, 16, big_gap, 0)
    assert e.value.code == dcopy.ERR_PARAM_INVALID and "2^62" in str(e.value)
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_ext_batch([(0x1000, 0x2000, big_count, 16, big_gap, 0)])
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_nd(0x1000, 0x2000, [0xFFFFFFFF, 0xFFFFFFFF, 4], [1 << 40, 1 << 20, 1],
                      [1 << 24, 4, 1], 4)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.transpose(0x1000, 0x2000, [1 << 31, 1 << 31, 1 << 10], [2, 1, 0], 0)
    assert e.value.code == dcopy.ERR_PARAM_INVALID


@pytest.mark.parametrize("sizes,ds", [
    ([2, 4], [1, 1]),          # two axes on the same stride
    ([3, 4], [2, 1]),          # outer stride inside the inner axis's extent
    ([2, 3, 8], [8, 24, 2]),   # a middle stride of 8 inside the 15 elements dim 2 covers
])
def test_copy_nd_refuses_repeating_destinations_on_host(dcopy, sizes, ds):
    """Boxes whose destination elements repeat are refused before any device memory is
    touched: the kernels write the box concurrently, so the result would not be that of
    the reference's sequential loop."""
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.copy_nd(0x10000, 0x90000, sizes, [1] * len(sizes), ds, 1)
    assert e.value.code == dcopy.ERR_PARAM_INVALID and "destinations would repeat" in str(e.value)
