"""
The tuner end to end on a GPU: `autotune.main` with the reference's flags
(autotune.py:596-640 of the reference) generates softmax variants, compiles
each with nvcc for sm_100a, verifies it against NumPy in a spawned GPU worker,
times it through the C ABI and writes the reference's result files
(`{kernel}_tuning.json`, `_failures.json`, `_convergence.json`,
`live_progress.json`; the reference writes them at autotune.py:285-375).
"""

from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_autotune_softmax_sha_end_to_end(dev, lib, tmp_path):
    import autotune

    rc = autotune.main(["--kernel", "softmax", "--strategy", "sha", "--budget", "6", "--size", "small",
                        "--gpus", "1", "--samples", "10", "--warmup", "3", "--ptx-analysis",
                        "--results-dir", str(tmp_path)])
    assert rc == 0
    tuning = json.loads((tmp_path / "softmax_tuning.json").read_text())
    best = tuning["best"]
    assert best is not None and tuning["n_results"] >= 1
    assert best["correctness_checked"] and best["is_correct"]
    assert best["mean_ms"] > 0 and best["n_samples"] >= 2
    assert best["achieved_gbps"] > 0 and 0 < best["roofline_efficiency_pct"] < 200
    assert best["occupancy"] is not None and best["registers_per_thread"] > 0
    assert best["speedup"] is not None and best["p_value"] is not None
    for name in ("softmax_failures.json", "softmax_convergence.json", "live_progress.json"):
        assert (tmp_path / name).exists(), name
    # every evaluated variant is a library built for this run and its params are baked in
    for v in tuning["variants"]:
        assert v["library"].startswith(str(tmp_path))
