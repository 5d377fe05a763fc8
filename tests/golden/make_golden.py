#!/usr/bin/env python3
"""Generate the standalone-datacopy golden fixtures from the reference's Python twin.

The reference ships an executable Python model of its tiling and DMA addressing:
``standalone_datacopy/profile.py:88-99`` (``tile_plan``) and
``standalone_datacopy/test_address_model.py:13-34`` (``model``, a byte-level model
of the ``DataCopyPad`` Compact gather).  This script imports both from a reference
checkout and records their outputs as fixtures, so that the oracle and the CUDA
library are checked against the reference's own code on machines that do not
have the reference:

* ``standalone_plans.json`` -- ``tile_plan(rows, cols, kib)`` (or the fact that it
  raised ``ValueError``) over a grid of shapes that covers every limit;
* ``address_model.json`` -- for each shape of ``test_three_paths_and_tail`` plus a
  few ragged shapes, the SHA-256 of ``model(rows, cols, kib, pre)`` packed as
  little-endian int32, its length and its first values.

Usage: python tests/golden/make_golden.py [--reference DIR]
(DIR defaults to $DCOPY_REFERENCE, else the standard checkout location.)
"""
import argparse
import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# The reference checkout: DCOPY_REFERENCE, else `reference` beside this repository.
DEFAULT_REFERENCE = os.environ.get("DCOPY_REFERENCE") or str(HERE.parents[2] / "reference")


def load_reference(ref_root: Path):
    src = ref_root / "standalone_datacopy"
    # The reference's module is named `profile` (shadowing the stdlib module) and
    # test_address_model.py imports it by that name.
    spec = importlib.util.spec_from_file_location("profile", src / "profile.py")
    profile = importlib.util.module_from_spec(spec)
    sys.modules["profile"] = profile
    spec.loader.exec_module(profile)
    spec2 = importlib.util.spec_from_file_location("ref_test_address_model",
                                                   src / "test_address_model.py")
    tam = importlib.util.module_from_spec(spec2)
    spec2.loader.exec_module(tam)
    return profile, tam


PLAN_ROWS = [0, 7, 8, 16, 24, 120, 256, 512, 1024, 2048, 4088, 4095, 4096]
PLAN_COLS = [0, 1, 19, 37, 100, 513, 768, 4096, 16384, 65535, 65536]
PLAN_KIB = [0, 1, 2, 4, 8, 16, 128, 240, 241, 256]

# test_address_model.py:39-40 shapes (rows, cols, small_kib, large_kib), plus ragged ones.
MODEL_SHAPES = [(256, 768, 8, 240), (8, 37, 1, 2), (128, 513, 4, 128), (4088, 19, 16, 240),
                (8, 1, 1, 240), (24, 100, 1, 7), (16, 255, 3, 5), (64, 1000, 1, 3)]


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    args = ap.parse_args()
    profile, tam = load_reference(Path(args.reference))

    plans = []
    for rows in PLAN_ROWS:
        for cols in PLAN_COLS:
            for kib in PLAN_KIB:
                try:
                    plan = profile.tile_plan(rows, cols, kib)
                    plans.append([rows, cols, kib, plan["tile_cols"], plan["tile_bytes"],
                                  plan["tile_count"]])
                except ValueError:
                    plans.append([rows, cols, kib, None, None, None])
    (HERE / "standalone_plans.json").write_text(json.dumps(
        {"source": "standalone_datacopy/profile.py:88-99 tile_plan",
         "columns": ["rows", "cols", "kib", "tile_cols", "tile_bytes", "tile_count"],
         "note": "null plan = tile_plan raised ValueError", "cases": plans},
        separators=(",", ":")) + "\n")

    models = []
    for rows, cols, small, large in MODEL_SHAPES:
        for kib, pre in [(small, False), (large, False), (large, True)]:
            out = np.asarray(tam.model(rows, cols, kib, pre), dtype="<i4")
            models.append({"rows": rows, "cols": cols, "kib": kib, "pretranspose": pre,
                           "len": int(out.size), "head": out[:16].tolist(),
                           "sha256": hashlib.sha256(out.tobytes()).hexdigest()})
    (HERE / "address_model.json").write_text(json.dumps(
        {"source": "standalone_datacopy/test_address_model.py:13-34 model(); input a[i] = i",
         "cases": models}, indent=1) + "\n")
    print(f"wrote {len(plans)} plans and {len(models)} model digests to {HERE}")


if __name__ == "__main__":
    main()
