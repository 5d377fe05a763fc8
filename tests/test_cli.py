"""The C++ host tools: demo_datacopy (the reference host driver's CLI contract,
datacopy_data_collection.asc:97-181) and dcopy_bench (sweep / standalone / nz)."""
import json
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT

BIN = ROOT / "data-copy_b200" / "bin"


def _run(*args, **kw):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=600,
                          **kw)


@pytest.fixture(scope="module")
def demo(dcopy):
    exe = BIN / "demo_datacopy"
    if not exe.exists():
        pytest.fail("demo_datacopy is not built (run __graft_entry__.build())")
    return exe


@pytest.mark.parametrize("args,message", [
    ([], "Usage: demo_datacopy"),
    (["tiny", 256, 768, 8, 1, 0], "Unknown mode"),
    (["small", 7, 768, 8, 1, 0], "rows: 8..4088 multiple of 8"),
    (["small", 4096, 768, 8, 1, 0], "rows: 8..4088 multiple of 8"),
    (["small", 256, 0, 8, 1, 0], "rows: 8..4088"),
    (["small", 256, 768, 241, 1, 0], "tile: 1..240 KiB"),
    (["small", 256, 768, 8, 2, 0], "store: 0/1"),
    (["small", 256, 768, 8, 1, 256], "device: 0..255"),
    (["small", 512, 768, 1, 1, 0], "Tile budget must hold a complete transposed row"),
    (["small", 4088, 65535, 240, 1, 0], "Experiment GM input limit: 64 MiB"),
    (["small", "-8", 768, 8, 1, 0], "Expected a nonnegative integer"),
    (["small", 99999999999, 768, 8, 1, 0], "Integer overflow"),
    (["small", 256, 768, 8, 0, 0, "/tmp/x"], "VERIFICATION_FILE requires STORE=1"),
])
def test_demo_rejects_like_the_reference(demo, args, message, tmp_path):
    r = _run(demo, *args)
    assert r.returncode == 1 and message in r.stderr, (r.stdout, r.stderr)


@pytest.mark.gpu
@pytest.mark.parametrize("mode,kib", [("small", 8), ("large", 240), ("pretranspose", 240)])
def test_demo_runs_and_verifies(demo, torch_cuda, mode, kib, tmp_path):
    report = tmp_path / "verification.txt"
    r = _run(demo, mode, 256, 768, kib, 1, 0, report)
    assert r.returncode == 0, r.stderr
    assert f"mode={mode} rows=256 cols=768 input_bytes=786432" in r.stdout
    assert "verification=PASS" in r.stdout
    assert report.read_text() == "verification=PASS\n"
    r = _run(demo, mode, 4088, 19, 16, 0, 0)
    assert r.returncode == 0 and "verification=not_requested" in r.stdout


@pytest.mark.gpu
def test_bench_standalone_writes_profile_outputs(dcopy, torch_cuda, tmp_path):
    out = tmp_path / "results"
    r = _run(BIN / "dcopy_bench", "standalone", 256, 768, 8, 240, "--trials", 2, "--output", out)
    assert r.returncode == 0, r.stderr
    summary = json.loads((out / "summary.json").read_text())
    assert set(summary["results"]) == {"small", "large", "pretranspose"}
    assert summary["verification"] == "PASS" and summary["small_over_large_duration"] > 0
    assert (out / "raw.csv").read_text().count("\n") == 1 + 3 * 2
    assert "datacopy_contiguous" in (out / "stages.csv").read_text()
    r = _run(BIN / "dcopy_bench", "standalone", 256, 768, 8, 240, "--output", out)
    assert r.returncode == 1  # refuses an existing output directory, like profile.py


@pytest.mark.gpu
def test_bench_sweep_and_nz(dcopy, torch_cuda):
    r = _run(BIN / "dcopy_bench", "sweep", "--moved-mib", 16, "--reps", 2)
    assert r.returncode == 0, r.stderr
    pts = [json.loads(line) for line in r.stdout.splitlines()]
    assert len(pts) == 24 and all(p["verified"] for p in pts)
    r = _run(BIN / "dcopy_bench", "nz", "--batch", 2, "--h", 1024, "--w", 1024, "--reps", 2)
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)["round_trip_bit_exact"] is True
    r = _run(BIN / "dcopy_bench", "nz", "--format", "zz", "--batch", 2, "--h", 1000, "--w", 1000,
             "--reps", 2)
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert out["round_trip_bit_exact"] is True and out["format"] == "zz"
