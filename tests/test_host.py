"""
Host-side logic on CPU: statistics, timing-line parsing, search strategies,
roofline and occupancy models, search spaces, variant generation, workloads.
"""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

import benchmark
import generator
import occupancy
import parser as kparser
import roofline
import search
import sharding
import workloads


# --- statistics (src/benchmark.py:192-244) ----------------------------------------

def test_compute_stats_bessel_and_ci():
    s = [1.0, 2.0, 3.0, 4.0]
    mean, std, ci, mn, mx = benchmark._compute_stats(s)
    assert mean == 2.5 and mn == 1.0 and mx == 4.0
    assert std == pytest.approx(np.std(s, ddof=1))
    assert ci == pytest.approx(1.96 * np.std(s, ddof=1) / 2.0)
    assert benchmark._compute_stats([]) == (0.0, 0.0, 0.0, 0.0, 0.0)
    assert benchmark._compute_stats([5.0]) == (5.0, 0.0, 0.0, 5.0, 5.0)


def test_welch_matches_scipy():
    from scipy import stats
    rng = np.random.default_rng(1)
    base = list(rng.normal(2.0, 0.05, 30))
    var = list(rng.normal(1.0, 0.02, 30))
    sp, p, sig, bm = benchmark.compute_significance(var, base)
    assert sp == pytest.approx(np.mean(base) / np.mean(var))
    assert p == pytest.approx(stats.ttest_ind(base, var, equal_var=False).pvalue)
    assert sig and bm == pytest.approx(np.mean(base))
    sp, p, sig, _ = benchmark.compute_significance(base, var)  # slower variant: never significant
    assert sp < 1 and not sig
    assert benchmark.compute_significance(var, []) == (None, None, False, None)


def test_parse_and_format_timing_lines_round_trip():
    text = benchmark.format_timing_output("softmax_x", [0.1, 0.2, 0.3])
    t = benchmark.parse_timing_output(text + "noise line\n")
    assert t["softmax_x"]["samples"] == [0.1, 0.2, 0.3]
    assert t["softmax_x"]["mean_ms"] == pytest.approx(0.2) and t["softmax_x"]["iters"] == 3


def test_benchmark_result_to_dict_drops_samples():
    r = benchmark.BenchmarkResult(kernel="softmax", variant="v", raw_samples=[1.0, 2.0])
    d = r.to_dict()
    assert "raw_samples" not in d and d["kernel"] == "softmax"
    json.dumps(d)


# --- search strategies ---------------------------------------------------------------

def _space():
    return kparser.build_search_space(kparser.build_kernel_profile("softmax"))


def _objective(p):
    # smooth synthetic latency, minimum at block 256, vec 4, min_blocks 1, stages 3
    return (1.0 + (math.log2(p["block_size"]) - 8) ** 2 + (math.log2(p["vec_per_thread"]) - 2) ** 2
            + 0.5 * math.log2(p["min_blocks"]) ** 2 + 0.25 * (p["stages"] - 3) ** 2
            + 0.3 * math.log2(p.get("cluster_size", 1)) + 0.1 * p.get("tma_box", 0) / 4096)


def test_grid_strategy_covers_valid_points():
    sp = _space()
    g = search.GridSearchStrategy(sp, "softmax")
    pts = g.suggest(10_000)
    assert len(pts) == g.total == len(generator.enumerate_variants("softmax", sp))
    assert all(kparser.is_valid("softmax", p) for p in pts)
    for p in pts:
        g.update(p, _objective(p))
    assert g.best() == {"block_size": 256, "vec_per_thread": 4, "min_blocks": 1, "stages": 3, "cluster_size": 1,
                        "tma_box": 0}


def test_bayesian_strategy_finds_optimum_within_budget():
    sp = _space()
    bo = search.BayesianOptStrategy(sp, "softmax", n_calls=30, seed=3)
    n = 0
    while True:
        batch = bo.suggest(1)
        if not batch:
            break
        for p in batch:
            bo.update(p, _objective(p))
            n += 1
    assert n == 30
    assert _objective(bo.best()) <= 1.5  # at or next to the optimum after 30 of the grid's points


def test_bayesian_strategy_handles_failures():
    sp = _space()
    bo = search.BayesianOptStrategy(sp, "softmax", n_calls=12, seed=1)
    for _ in range(12):
        for p in bo.suggest(1):
            bo.update(p, math.inf if p["block_size"] == 1024 else _objective(p))
    assert bo.best()["block_size"] != 1024


def test_sha_halves_and_grows_budget():
    sp = _space()
    sha = search.SuccessiveHalvingStrategy(sp, "softmax", n_configs=16, eta=2, r_min=3, seed=0)
    sizes, budgets = [], []
    while True:
        batch = sha.suggest(100)
        if not batch:
            break
        sizes.append(len(batch))
        budgets.append(sha.budget())
        for p in batch:
            sha.update(p, _objective(p))
    # the last survivor is re-measured once more with the largest budget
    assert sizes == [16, 8, 4, 2, 1]
    assert budgets == [3, 6, 12, 24, 48]
    assert sha.best() is not None


@pytest.mark.parametrize("kernel", list(kparser.FAMILIES))
def test_default_points_are_the_library_defaults(kernel):
    """The default library's configuration is a valid point of the family's
    space, and every axis value of it equals the header default of the macro
    the axis sets (for the macros whose default is a plain number)."""
    import re
    from pathlib import Path
    space = kparser.build_search_space(kparser.build_kernel_profile(kernel))
    pts = kparser.default_points(kernel, space)
    assert pts, kernel
    csrc = Path(generator.__file__).resolve().parent.parent / "csrc"
    text = "\n".join(f.read_text() for f in csrc.glob("*.cuh"))
    fam = kparser.family_of(kernel)
    for base in kparser.DEFAULTS[fam]:
        for axis, macro in generator.MACROS[fam].items():
            if axis not in base:
                continue
            if fam == "matmul" and base["variant"] == "tf32" and axis not in ("cta_tile", "stages"):
                continue  # FFMA-only axes at representative values in the TF32 point
            if fam == "matmul" and base["variant"] == "ffma" and axis in ("cta_tile", "stages", "bk", "min_blocks"):
                continue  # tcgen05-only axes; the wide kernel's k tile (8 when bk is unset) and launch
                          # bounds are its own
            m = re.search(rf"^#define {macro} (\S+)", text, re.M)
            assert m, macro
            if not re.fullmatch(r"-?\d+", m.group(1)):
                continue  # a derived default (an expression of other macros)
            assert generator._macro_value(axis, base[axis]) == m.group(1), (axis, macro)


def test_strategies_evaluate_anchors_first():
    sp = {"a": [1, 2, 3, 4], "b": [0, 1, 2, 3]}
    anchors = [{"a": 3, "b": 2}, {"a": 1, "b": 1}]
    sha = search.make_strategy("sha", sp, n_configs=4, seed=5, anchors=anchors)
    assert sha.suggest(2) == anchors
    bo = search.make_strategy("bayesian", sp, n_calls=6, seed=5, anchors=anchors)
    assert bo.suggest(2) == anchors
    # an anchor outside the space is ignored
    sha = search.make_strategy("sha", sp, n_configs=4, seed=5, anchors=[{"a": 9, "b": 0}])
    assert {"a": 9, "b": 0} not in sha.suggest(10)


def test_make_strategy_names():
    sp = _space()
    assert isinstance(search.make_strategy("grid", sp), search.GridSearchStrategy)
    assert isinstance(search.make_strategy("bo", sp), search.BayesianOptStrategy)
    assert isinstance(search.make_strategy("halving", sp), search.SuccessiveHalvingStrategy)
    with pytest.raises(ValueError):
        search.make_strategy("random", sp)


def test_convergence_logger(tmp_path):
    c = search.ConvergenceLogger("softmax", tmp_path)
    for ms in (3.0, 2.0, 2.5, 1.0):
        c.record({"a": 1}, ms)
    c.save()
    d = json.loads((tmp_path / "softmax_convergence.json").read_text())
    assert [e["best_ms"] for e in d["curve"]] == [3.0, 2.0, 2.0, 1.0] and d["n_evals"] == 4


# --- roofline ------------------------------------------------------------------------

def test_roofline_algorithmic_counts():
    ra = roofline.RooflineAnalyzer()
    assert ra.total_bytes("softmax", {"rows": 4096, "cols": 4096}) == 134_217_728
    assert ra.total_bytes("reduction", {"n": 1 << 28}) == 1_073_741_824
    assert ra.total_bytes("layernorm", {"rows": 16384, "cols": 4096}) == 536_903_680
    assert ra.total_flops("matmul", {"M": 8192, "N": 8192, "K": 8192}) == 1_099_511_627_776
    d = {"B": 8, "H": 32, "S": 4096, "D": 128}
    assert ra.total_flops("attention", d) == 2_199_023_255_552
    assert ra.total_flops("attention", d, causal=True) == 1_099_780_063_232


def test_roofline_fractions():
    peaks = dict(roofline.PEAKS)
    peaks["hbm_gbs"] = 8000.0
    ra = roofline.RooflineAnalyzer(peaks)
    pt = ra.analyze("reduction", {"n": 1 << 28}, elapsed_ms=1_073_741_824 / 8e9)  # exactly 8 TB/s
    assert pt.bound_type == "memory" and pt.efficiency_pct == pytest.approx(100.0)
    assert pt.achieved_gbps == pytest.approx(8000.0)
    assert ra.bound_type("matmul", {"M": 8192, "N": 8192, "K": 8192}) == "compute"
    assert roofline.get_dims("softmax") == {"rows": 4096, "cols": 4096}


def test_measured_peaks_are_used():
    src = roofline.PEAKS["source"]
    if src["hbm_gbs"] == "measured":
        assert roofline.PEAKS["hbm_gbs"] < 8000.0
    assert roofline.PEAKS["fp32_tflops"] == pytest.approx(148 * 128 * 2 * 1.965e9 / 1e12)


# --- occupancy -----------------------------------------------------------------------

PTXAS = """ptxas info    : Compiling entry function '_ZN2kt7softmax8rows_vecILi256ELi4ELi1EEEvPKfPfli' for 'sm_100a'
ptxas info    : Function properties for _ZN2kt7softmax8rows_vecILi256ELi4ELi1EEEvPKfPfli
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 40 registers, used 1 barriers, 256 bytes smem, 400 bytes cmem[0]
ptxas info    : Compiling entry function '_Z3fooPf' for 'sm_100a'
ptxas info    : Function properties for _Z3fooPf
    16 bytes stack frame, 8 bytes spill stores, 4 bytes spill loads
ptxas info    : Used 255 registers, used 0 barriers, 380 bytes cmem[0]
"""


def test_parse_ptxas():
    p = occupancy.parse_ptxas_stderr(PTXAS)
    k = p["_ZN2kt7softmax8rows_vecILi256ELi4ELi1EEEvPKfPfli"]
    assert k == {"registers": 40, "smem_bytes": 256, "spill_stores": 0, "spill_loads": 0, "barriers": 1}
    assert p["_Z3fooPf"]["spill_stores"] == 8 and p["_Z3fooPf"]["registers"] == 255


def test_occupancy_sm100_limits():
    # 40 regs x 256 threads: 1280 regs/warp -> 51 warps by regs -> 6 blocks of 8 warps
    occ, warps = occupancy.compute_occupancy(40, 256, 256)
    assert warps == 48 and occ == pytest.approx(48 / 64)
    # 32 regs x 256: register-unlimited, warp-limited at 64
    assert occupancy.compute_occupancy(32, 0, 256) == (1.0, 64)
    # 200 KiB dynamic smem: one block per SM
    o = occupancy.occupancy_detail(64, 0, 128, dynamic_smem_bytes=200 * 1024)
    assert o[2] == 1 and o[3] == "smem"
    # TMEM: 512 columns per CTA -> one CTA
    assert occupancy.occupancy_detail(64, 0, 128, tmem_columns=512)[2] == 1
    assert occupancy.occupancy_detail(64, 300 * 1024, 128)[3] == "smem>227KiB"


def test_occupancy_analyzer_substring_match():
    info = occupancy.OccupancyAnalyzer().analyze_from_stderr(PTXAS, "rows_vec", 256)
    assert info.registers_per_thread == 40 and info.active_blocks == 6


# --- search spaces and generated sources --------------------------------------------

def test_generic_space_is_the_references():
    prof = kparser.KernelProfile(name="custom", src_path=None, block_dim=16, uses_shared=False, loop_depth=2,
                                 memory=kparser.MemoryAccessPattern(has_strided_access=True, has_reduction=True))
    sp = kparser.build_search_space(prof)
    assert sp["block_size"] == [64, 128, 192, 256] and sp["unroll"] == [1, 2, 4, 8]
    assert sp["_total_variants"] == 4 * 4 * 2 * 2 * 2 * 2
    assert sp["_kernel"] == "custom"


@pytest.mark.parametrize("kernel", kparser.FAMILIES)
def test_family_spaces_generate_valid_sources(kernel):
    sp = kparser.build_search_space(kparser.build_kernel_profile(kernel))
    variants = generator.enumerate_variants(kernel, sp)
    assert variants
    tags = {generator._variant_tag(kernel, p) for p, _ in variants}
    assert len(tags) == len(variants)
    src = generator.generate_source(kernel, {k: v for k, v in variants[0][0].items()
                                             if k not in generator.RUNTIME_PARAMS.get(kernel, ())})
    assert '#include "kt_entry.cuh"' in src and generator.ONLY[kernel] in src
    meta = src.split("KT_VARIANT_JSON ", 1)[1].split("\n", 1)[0]
    assert json.loads(json.loads(meta))["kernel"] == kernel


def test_variant_tag_is_the_references_format():
    assert generator._variant_tag("matmul", {"tile_x": 16, "block_size": 64}) == "matmul_block_size64_tile_x16"


def test_regex_parser_finds_kernels():
    prof = kparser.RegexKernelParser().parse_to_profiles(kparser.build_kernel_profile("softmax").src_path)
    names = {p.name for p in prof}
    assert {"rows_vec", "rows_scalar", "rows_warp", "rows_stream"} <= names


# --- workloads and sharding ---------------------------------------------------------

def test_workloads_are_seeded_and_shaped():
    a = workloads.make_inputs("layernorm", "small", seed=7)
    b = workloads.make_inputs("layernorm", "small", seed=7)
    assert np.array_equal(a["x"], b["x"]) and a["x"].shape == (513, 4096)
    assert abs(a["gamma"].mean() - 1.0) < 0.02 and abs(a["beta"].mean()) < 0.02
    r = workloads.make_inputs("reduction", d={"n": 1 << 16})
    assert r["x"].dtype == np.float32 and r["x"].min() >= -1.0 and r["x"].max() < 1.0
    att = workloads.make_inputs("attention", "kat")
    assert att["q"].dtype == np.uint16 and att["scale"] == pytest.approx(0.125)


@pytest.mark.parametrize("n,world", [(0, 1), (7, 8), (1 << 28, 8), (1000003, 3)])
def test_shard_ranges_partition(n, world):
    ranges = [sharding.shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    sizes = [hi - lo for lo, hi in ranges]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(n, world, world)


def test_tuner_ranks_by_work_and_sizes_resources():
    import autotune
    d = {"B": 8, "H": 32, "S": 4096, "D": 128}
    assert autotune.work_scale("attention", d, {"causal": True}) == pytest.approx(2.0, rel=1e-3)
    assert autotune.work_scale("attention", d, {"causal": False}) == 1.0
    assert autotune.work_scale("matmul", {"M": 8, "N": 8, "K": 8}, {"transpose_b": True}) == 1.0
    # dynamic shared memory of the staged softmax (3 rows of 4096 floats) and the FA kernel
    assert autotune.launch_resources("softmax", {"stages": 3}, {"cols": 4096})[0] == 3 * 4096 * 4 + 3 * 8 + 16
    assert autotune.launch_resources("attention", {"kind": 1, "stages": 2, "v_stages": 2}, d) == (201984, 512)
    assert autotune.kernel_function("attention", {"kind": 2, "causal": True})[1] == 512
    assert autotune.kernel_function("softmax", {"cluster_size": 2})[0] == "rows_kernel"


def test_report_generator_sections(tmp_path):
    import reporter
    from benchmark import BenchmarkResult
    res = [BenchmarkResult(kernel="softmax", variant=f"v{i}", params={"block_size": 256, "stages": s},
                           mean_ms=0.025 + 0.001 * i, ci_95_ms=0.0002, n_samples=10, speedup=200.0 - i,
                           p_value=1e-30, is_significant=True, roofline_efficiency_pct=80.0 - i,
                           occupancy=0.75, registers_per_thread=40, shared_mem_bytes=32784, normalized_ms=0.025,
                           correctness_checked=True, is_correct=True, library="/x/softmax_v.so")
           for i, s in enumerate((2, 3, 4))]
    rg = reporter.ReportGenerator("softmax", "sha", tmp_path)
    rg.set_results(res, baseline_ms=6.7)
    rg.set_roofline_points({"arithmetic_intensity": 0.6, "achieved_gbps": 20.0, "achieved_gflops": 12.0,
                            "bound_type": "memory", "efficiency_pct": 0.3, "ceiling": "HBM"},
                           {"arithmetic_intensity": 0.6, "achieved_gbps": 5300.0, "achieved_gflops": 3300.0,
                            "bound_type": "memory", "efficiency_pct": 81.0, "ceiling": "HBM"})
    rg.set_correctness(3, 1)
    rg.set_resource_report({"_ZN2kt6staged12softmax_rows": {"registers": 40, "smem_bytes": 256, "spill_stores": 0,
                                                             "spill_loads": 0, "barriers": 1}})
    rg.set_convergence({"kernel": "softmax", "n_evals": 15, "best_ms": 0.025, "curve": []})
    path = rg.generate()
    text = path.read_text()
    assert path.name == "softmax_report.md"
    for section in ("# Kernel auto-tuner report", "## Roofline", "## Top configurations", "## Occupancy",
                    "## Resources of the best variant", "## Correctness", "## Convergence",
                    "## Recommended configuration", "B200", "5300 GB/s", "stages"):
        assert section in text, section
    reporter.print_terminal_summary("softmax", res, 6.7, "sha")
    reporter.print_final_summary({"softmax": res, "reduction": []}, {"softmax": 6.7})


def test_tuned_layers_load_params_and_keep_weights(tmp_path):
    import json as _json
    import torch
    import tuned_modules as tm
    assert tm.load_best_params("layernorm", tmp_path) == {}
    (tmp_path / "layernorm_tuning.json").write_text(_json.dumps(
        {"best": {"params": {"stages": 2, "tma_box": 4096}, "library": str(tmp_path / "missing.so")}}))
    assert tm.load_best_params("layernorm", tmp_path) == {"stages": 2, "tma_box": 4096}
    assert tm.tuned_library("layernorm", tmp_path).path.name == "libkt.so"  # the tuned file is gone: default
    model = torch.nn.Sequential(torch.nn.Linear(64, 32), torch.nn.LayerNorm(32), torch.nn.Linear(32, 8, bias=False))
    w0 = model[0].weight.detach().clone()
    tm.apply_tuned_layers(model, "all", results_dir=tmp_path)
    assert isinstance(model[0], tm.TunedLinear) and isinstance(model[1], tm.TunedLayerNorm)
    assert isinstance(model[2], tm.TunedLinear) and model[2].bias is None
    assert torch.equal(model[0].weight, w0)
    assert model[1].tuned_params == {"stages": 2, "tma_box": 4096}
    with pytest.raises(ValueError):
        tm.TunedMultiheadAttention(96, 3)  # head dim 32 is not built
