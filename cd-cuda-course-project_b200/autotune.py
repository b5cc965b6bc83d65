"""
autotune.py — the tuner's command line (B200, sm_100a).

    python autotune.py --kernel=softmax
    python autotune.py --kernel=all --strategy=bayesian
    python autotune.py --kernel=reduction --strategy=sha --gpus=8
    python autotune.py --baseline-only
    python autotune.py --kernel=matmul --skip-verification --workers=8
    python autotune.py --kernel=all --strategy=sha --budget=8 --compile-only   # host cores only

Same flags as the reference's CLI (autotune.py:596-640: --kernel, --baseline-only,
--workers, --warmup, --samples, --iters, --strategy, --skip-verification,
--ptx-analysis, --cuda-graphs, --matrix-size) plus --gpus, --size, --budget,
--results-dir. Pipeline per kernel family:

  1. profile -> search space (parser.build_search_space, Blackwell axes)
  2. the strategy suggests the next points (it decides what runs)
  3. generate + nvcc each point into a shared library (host cores in parallel;
     identical compile keys are reused)
  4. verify it against NumPy (verifier.CorrectnessVerifier) on a GPU worker
  5. time it in-process through the C ABI (kt_time, L2 evicted per sample)
  6. Welch t-test vs the naive GPU baseline, roofline (B200), occupancy
     (ptxas -v report), results JSON (the reference's schemas)

GPU work runs in one worker process per GPU (spawned, CUDA_VISIBLE_DEVICES
pinned); a worker that dies takes only its current variant down: the variant
is recorded as failed and the worker restarted. --ptx-analysis reports the
ptxas resource lines of the winner (registers, shared memory, spills,
barriers); compiler-written PTX/SASS is not read.
"""

from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import queue
import sys
import time
import traceback
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Optional

ROOT = Path(__file__).resolve().parent
SRC_DIR = ROOT / "src"
for _p in (str(ROOT), str(SRC_DIR)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from benchmark import (BenchmarkResult, N_SAMPLES_DEFAULT, N_WARMUP_DEFAULT, _compute_stats,  # noqa: E402
                       compute_significance, run_baseline_benchmark)
from generator import compile_key, ensure_variant  # noqa: E402
from occupancy import OccupancyAnalyzer  # noqa: E402
from parser import FAMILIES, build_kernel_profile, build_search_space, default_points  # noqa: E402
from roofline import RooflineAnalyzer  # noqa: E402
from search import ConvergenceLogger, make_strategy  # noqa: E402

SUPPORTED_KERNELS = list(FAMILIES)
RECYCLE_AFTER = 48  # variant libraries loaded per worker before it is replaced

def work_scale(kernel: str, dims: dict, p: dict) -> float:
    """Work of the family's reference problem over the work of this point's
    problem: runtime axes that change the amount of work (the causal mask
    halves attention's) must not make a point look faster. Layout axes
    (transpose_b) keep the work and give 1."""
    import workloads
    if kernel == "attention" and p.get("causal"):
        d = {k: dims[k] for k in ("B", "H", "S", "D")}
        return workloads.work("attention", d, causal=False).flops / workloads.work("attention", d, causal=True).flops
    return 1.0


def launch_resources(kernel: str, p: dict, dims: dict) -> tuple[int, int]:
    """(dynamic shared memory bytes, TMEM columns) one CTA of the point's kernel
    takes at the tuned problem size, for the occupancy analysis (ptxas reports
    only static shared memory). Mirrors the Cfg/smem_bytes formulas of csrc/."""
    if kernel in ("softmax", "layernorm"):
        cols = int(dims.get("cols", 4096))
        c = int(p.get("cluster_size", 1))
        st = int(p.get("stages", 3))
        if c > 1:
            return (st if st > 0 else 2) * (cols // c) * 4 + (st if st > 0 else 2) * 8 + 16, 0
        return (st * cols * 4 + st * 8 + 16 if st > 0 else 0), 0
    if kernel == "matmul":
        if p.get("variant") == "ffma":
            if int(p.get("ffma_x2", 0)):
                bk = int(p.get("bk", 16))
                return 4 * 2 * bk * ((2 * 128 + 4) + (128 + 4)), 0
            return 0, 0
        bn = int(str(p.get("cta_tile", "128x256")).split("x")[1])
        stages = int(p.get("stages", 4))
        return stages * (128 * 32 + bn * 32) * 4 + 1024 + 256, 2 * bn
    if kernel == "attention":
        d = int(dims.get("D", 128))
        if p.get("kind", 1) == 2:
            return 2 * 128 * d * 2 + 8 * 64 * d * 2 + 1024 + 2048, 512
        st, vst = int(p.get("stages", 2)), int(p.get("v_stages", 2))
        return (2 + st + vst) * 128 * d * 2 + 4096 + 1024 + 256, 512
    return 0, 0


def kernel_function(kernel: str, p: dict) -> tuple[str, int]:
    """The __global__ function a variant of `kernel` launches at the tuned size
    (a substring of its mangled name in the ptxas resource lines) and its block
    size, for the occupancy analysis."""
    if kernel in ("softmax", "layernorm"):
        # cluster_size > 1: rows split across a cluster; stages > 0: the persistent TMA
        # bulk-copy ring kernel; 0: one row per CTA in registers
        if p.get("cluster_size", 1) > 1:
            return "rows_kernel", int(p.get("block_size", 256))
        if p.get("stages", 3) > 0:
            return ("softmax_rows" if kernel == "softmax" else "layernorm_rows"), int(p.get("block_size", 256))
        return "rows_vec", int(p.get("block_size", 256))
    if kernel == "reduction":
        return "sum_f32", int(p.get("block_size", 512))
    if kernel == "matmul":
        if p.get("variant") == "ffma":
            return ("sgemm_128x256" if int(p.get("ffma_wide", 1)) else "sgemm_128x128"), 256
        return "gemm_tf32_kernel", 192
    if kernel == "attention":
        # the library holds D=64 and D=128 instances; the tuned size has D=128
        c = int(bool(p.get("causal")))
        if p.get("kind", 1) == 2:
            # loaders, MMA lane, 2 x 4 softmax warps, 4 epilogue warps
            return f"fa2_fwd_kernelILi128ELi4ELi4ELb{c}", 512
        # 3 loader/MMA warps + 8 softmax warps + 4 epilogue warps (+ 1 P·V-issuing warp with two issuers)
        return f"fa_fwd_kernelILi128ELi{int(p.get('stages', 2))}ELb{c}", 512 if int(p.get("issuers", 2)) == 2 else 480
    raise ValueError(f"unknown kernel {kernel!r}")


def results_dir() -> Path:
    d = Path(os.environ.get("KT_RESULTS_DIR", ROOT / "results"))
    d.mkdir(parents=True, exist_ok=True)
    return d


# ---------------------------------------------------------------------------
# GPU worker process
# ---------------------------------------------------------------------------

def _worker_main(gpu: int, jobs, results) -> None:
    """Verify + time variants on one GPU until a None job arrives."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    for p in (str(ROOT), str(SRC_DIR)):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch

    import kt_lib
    import problems
    from verifier import CorrectnessVerifier

    torch.cuda.set_device(0)
    cache: dict = {}
    verifier = CorrectnessVerifier()
    while True:
        job = jobs.get()
        if job is None:
            return
        jid = job["id"]
        try:
            lib = kt_lib.load(job["so"])
            params = job["params"]
            kernel = job["kernel"]
            out = {"id": jid, "gpu": gpu, "ok": True}
            if job["verify"]:
                vr = verifier.check(kernel, job["so"], params)
                out["verify"] = {"is_correct": vr.is_correct, "max_diff": vr.max_diff,
                                 "normwise": vr.normwise_rel_err, "error": vr.error_msg}
                if not vr.is_correct:
                    results.put({**out, "ok": False, "error": "verification: " + vr.error_msg})
                    continue
            tb = bool(params.get("transpose_b", False))
            causal = bool(params.get("causal", False))
            var = kt_lib.KT_GEMM_FFMA if params.get("variant") == "ffma" else kt_lib.KT_GEMM_TF32
            key = (kernel, job["size"], json.dumps(job.get("dims"), sort_keys=True), tb, causal)
            prob = cache.get(key)
            if prob is None:
                cache.clear()
                torch.cuda.empty_cache()
                prob = problems.make_problem(kernel, job["size"], dims=job.get("dims"), transpose_b=tb,
                                             causal=causal, variant=var, lib=lib)
                cache[key] = prob
            prob.variant = var
            samples = prob.time(lib, job["warmup"], job["samples"])
            graph_ms = None
            if job.get("cuda_graphs"):
                graph_ms = _graph_time(lib, prob)
            out.update(samples=samples, dims=dict(prob.dims), graph_ms=graph_ms,
                       gpu_name=torch.cuda.get_device_name(0))
            results.put(out)
        except Exception as exc:  # noqa: BLE001 - reported per variant
            results.put({"id": jid, "gpu": gpu, "ok": False,
                         "error": f"{type(exc).__name__}: {exc}", "trace": traceback.format_exc()[-2000:]})


def _graph_time(lib, prob, reps: int = 20) -> Optional[float]:
    """Mean time per launch of `reps` launches replayed from one captured CUDA graph."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    args = prob.args()
    with torch.cuda.stream(s):
        lib.run(prob.op(), args, s.cuda_stream)  # warm-up outside capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                lib.run(prob.op(), args, s.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g.replay()
    torch.cuda.synchronize()
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


class GpuPool:
    """One spawned worker per GPU; jobs go to whichever worker is free."""

    def __init__(self, gpus: list[int]):
        self.ctx = mp.get_context("spawn")
        self.gpus = gpus
        self.results = self.ctx.Queue()
        self.workers: dict[int, tuple] = {}
        self.loaded: dict[int, int] = {}
        for g in gpus:
            self._start(g)

    def _start(self, g: int) -> None:
        jobs = self.ctx.Queue()
        p = self.ctx.Process(target=_worker_main, args=(g, jobs, self.results), daemon=True)
        p.start()
        self.workers[g] = (p, jobs)
        self.loaded[g] = 0

    def _stop(self, g: int) -> None:
        p, jobs = self.workers[g]
        try:
            jobs.put(None)
            p.join(timeout=20)
        finally:
            if p.is_alive():
                p.kill()

    def run(self, jobs: list[dict], timeout_s: float = 900.0) -> dict[int, dict]:
        """Run jobs across the workers; returns {job id: result}."""
        pending = list(jobs)
        busy: dict[int, tuple[dict, float]] = {}
        done: dict[int, dict] = {}
        while pending or busy:
            for g in self.gpus:
                if g not in busy and pending:
                    if self.loaded[g] >= RECYCLE_AFTER:
                        self._stop(g)
                        self._start(g)
                    job = pending.pop(0)
                    self.workers[g][1].put(job)
                    self.loaded[g] += 1
                    busy[g] = (job, time.time())
            try:
                r = self.results.get(timeout=1.0)
                done[r["id"]] = r
                for g, (job, _) in list(busy.items()):
                    if job["id"] == r["id"]:
                        del busy[g]
            except queue.Empty:
                pass
            for g, (job, t0) in list(busy.items()):
                p = self.workers[g][0]
                if not p.is_alive() or time.time() - t0 > timeout_s:
                    why = "worker died" if not p.is_alive() else f"timed out after {timeout_s:.0f}s"
                    done[job["id"]] = {"id": job["id"], "gpu": g, "ok": False, "error": why}
                    del busy[g]
                    if p.is_alive():
                        p.kill()
                    self._start(g)
        return done

    def close(self) -> None:
        for g in list(self.workers):
            self._stop(g)


def _visible_gpus(n: int) -> list[int]:
    env = os.environ.get("CUDA_VISIBLE_DEVICES")
    if env:
        ids = [int(x) for x in env.split(",") if x.strip().isdigit()]
        return ids[:n]
    return list(range(n))


# ---------------------------------------------------------------------------
# Tuning loop
# ---------------------------------------------------------------------------

def _size_dims(kernel: str, size: str, matrix_size: Optional[int]) -> Optional[dict]:
    """--matrix-size keeps the reference's meaning: N for matmul, rows for
    softmax/layernorm, 1024·N elements for the reduction, S for attention."""
    import workloads
    if matrix_size is None:
        return None
    d = workloads.dims(kernel, size)
    if kernel == "matmul":
        d.update(M=matrix_size, N=matrix_size, K=matrix_size)
    elif kernel in ("softmax", "layernorm"):
        d["rows"] = matrix_size
    elif kernel == "reduction":
        d["n"] = matrix_size * 1024
    elif kernel == "attention":
        d["S"] = matrix_size
    return d


def autotune_kernel(kernel: str, baseline_data: dict, pool: GpuPool, strategy_name: str = "grid",
                    max_workers: int = 4, warmup: int = N_WARMUP_DEFAULT, n_samples: int = N_SAMPLES_DEFAULT,
                    skip_verification: bool = False, run_ptx_analysis: bool = False, run_cuda_graphs: bool = False,
                    size: str = "config", matrix_size: Optional[int] = None, budget: Optional[int] = None,
                    seed: int = 0) -> list[BenchmarkResult]:
    """Tune one family; returns results sorted best first and writes results/{kernel}_*.json."""
    profile = build_kernel_profile(kernel)
    space = build_search_space(profile)
    strategy = make_strategy(strategy_name, space, kernel=kernel, n_calls=budget or 40,
                             n_configs=budget or 80, seed=seed, anchors=default_points(kernel, space))
    rdir = results_dir()
    conv = ConvergenceLogger(kernel, rdir)
    roof = RooflineAnalyzer()
    occ = OccupancyAnalyzer()
    dims = _size_dims(kernel, size, matrix_size)
    base_samples = baseline_data.get("samples", [])
    base_ms = baseline_data.get("mean_ms")
    live = rdir / "live_progress.json"
    results: list[BenchmarkResult] = []
    failures: list[dict] = []
    n_eval = 0
    t0 = time.time()
    batch_n = max(len(pool.gpus), 1) * 2
    print(f"\n[TUNE] {kernel}: {space['_total_variants']} grid points, strategy={strategy.name}, "
          f"gpus={pool.gpus}, compile workers={max_workers}")
    while True:
        batch = strategy.suggest(batch_n)
        if not batch:
            break
        samples_now = strategy.budget() or n_samples
        # compile the batch on host cores (identical compile keys share one library)
        keys = {compile_key(kernel, p): p for p in batch}
        with ThreadPoolExecutor(max_workers=max_workers) as ex:
            built = dict(zip(keys, ex.map(lambda p: ensure_variant(kernel, p), keys.values())))
        jobs = []
        for i, p in enumerate(batch):
            ok, log, so = built[compile_key(kernel, p)]
            if not ok:
                failures.append({"variant": compile_key(kernel, p), "error": "compile: " + log[-400:]})
                strategy.update(p, float("inf"))
                continue
            jobs.append({"id": n_eval + i, "kernel": kernel, "params": p, "so": str(so), "size": size,
                         "dims": dims, "warmup": warmup, "samples": samples_now, "verify": not skip_verification,
                         "cuda_graphs": run_cuda_graphs, "log": log})
        out = pool.run(jobs)
        for job in jobs:
            r = out.get(job["id"], {"ok": False, "error": "no result"})
            p = job["params"]
            tag = compile_key(kernel, p) + "".join(f"_{k}{p[k]}" for k in ("variant", "transpose_b", "causal")
                                                   if k in p)
            if not r.get("ok"):
                failures.append({"variant": tag, "error": r.get("error", "")})
                strategy.update(p, float("inf"))
                continue
            mean, std, ci, mn, mx = _compute_stats(r["samples"])
            sp, pv, sig, _ = compute_significance(r["samples"], base_samples)
            res = BenchmarkResult(kernel=kernel, variant=tag, params=p, mean_ms=mean, std_ms=std, ci_95_ms=ci,
                                  min_ms=mn, max_ms=mx, n_samples=len(r["samples"]), raw_samples=r["samples"],
                                  speedup=sp, p_value=pv, is_significant=sig, ptx_info=job["log"][-4000:],
                                  library=job["so"], problem=r["dims"], gpu=r["gpu"],
                                  graph_launch_ms=r.get("graph_ms"))
            if "verify" in r:
                res.correctness_checked = True
                res.is_correct = r["verify"]["is_correct"]
                res.max_diff = r["verify"]["max_diff"]
            variant = "ffma" if p.get("variant") == "ffma" else ""
            pt = roof.analyze(kernel, r["dims"], mean, causal=bool(p.get("causal")), variant=variant)
            res.arithmetic_intensity = pt.arithmetic_intensity
            res.achieved_gflops = pt.achieved_gflops
            res.achieved_gbps = pt.achieved_gbps
            res.bound_type = pt.bound_type
            res.roofline_efficiency_pct = pt.efficiency_pct
            res.roofline_ceiling = pt.ceiling_name
            fn, bs = kernel_function(kernel, p)
            dyn, tmem = launch_resources(kernel, p, r["dims"])
            info = occ.analyze_from_stderr(job["log"], fn, bs, dynamic_smem_bytes=dyn, tmem_columns=tmem)
            if info:
                res.occupancy = info.occupancy
                res.registers_per_thread = info.registers_per_thread
                res.shared_mem_bytes = info.shared_mem_bytes
                res.has_register_spill = info.has_register_spill
                res.spill_stores = info.spill_stores
                res.spill_loads = info.spill_loads
            res.normalized_ms = mean * work_scale(kernel, r["dims"], p)
            results.append(res)
            strategy.update(p, res.normalized_ms)
            conv.record(p, res.normalized_ms)
        n_eval += len(batch)
        best = min(results, key=lambda x: x.normalized_ms) if results else None
        elapsed = time.time() - t0
        print(f"  [{n_eval:4d}] best {best.mean_ms:.4f} ms ({best.roofline_efficiency_pct:.1f}% roofline)"
              if best else f"  [{n_eval:4d}] no passing variant yet", f" {elapsed:.0f}s")
        live.write_text(json.dumps({
            "kernel": kernel, "strategy": strategy_name, "done": n_eval, "total": space["_total_variants"],
            "best_ms": round(best.mean_ms, 5) if best else None, "baseline_ms": base_ms,
            "best_speedup": round(best.speedup, 3) if best and best.speedup else None,
            "best_params": best.params if best else None,
            "recent": [{"variant": x.variant, "mean_ms": round(x.mean_ms, 5),
                        "speedup": round(x.speedup, 3) if x.speedup else None, "passed": x.is_significant}
                       for x in sorted(results, key=lambda x: x.mean_ms)[:5]],
        }, indent=2))
    results.sort(key=lambda x: x.normalized_ms)
    conv.save()
    (rdir / f"{kernel}_failures.json").write_text(json.dumps(failures, indent=2))
    (rdir / f"{kernel}_tuning.json").write_text(json.dumps({
        "kernel": kernel, "strategy": strategy_name, "n_variants": space["_total_variants"], "n_evaluated": n_eval,
        "n_results": len(results), "baseline_ms": base_ms, "best": results[0].to_dict() if results else None,
        "variants": [x.to_dict() for x in results[:50]],
    }, indent=2, default=str))
    if not results:
        print(f"[ERROR] {kernel}: no variant compiled, verified and timed successfully")
        return []
    b = results[0]
    print(f"[BEST] {kernel}: {b.variant}  {b.mean_ms:.4f} ms ±{b.ci_95_ms:.4f}  "
          f"{b.achieved_gbps:.0f} GB/s  {b.achieved_gflops / 1e3:.2f} TFLOP/s  "
          f"{b.roofline_efficiency_pct:.1f}% of {b.roofline_ceiling}"
          + (f"  speedup {b.speedup:.1f}x vs naive (p={b.p_value:.2g})" if b.speedup and b.p_value else ""))
    if run_ptx_analysis:
        from occupancy import parse_ptxas_stderr
        print(f"[RESOURCES] ptxas report of {b.variant}:")
        for name, e in parse_ptxas_stderr(b.ptx_info).items():
            print(f"    {name[:70]:70s} regs={e['registers']} smem={e['smem_bytes']} "
                  f"spills={e['spill_stores']}/{e['spill_loads']} barriers={e['barriers']}")
    occ_rows = [r for r in results[:10] if r.occupancy is not None]
    if occ_rows:
        OccupancyAnalyzer.print_table(occ_rows, title=f"Occupancy — {kernel} top 10")
    write_report(kernel, strategy_name, results, base_ms, dims or (results[0].problem if results else None),
                 failures, conv, roof)
    return results


def write_report(kernel: str, strategy_name: str, results: list[BenchmarkResult], base_ms: Optional[float],
                 dims: Optional[dict], failures: list[dict], conv: ConvergenceLogger, roof: RooflineAnalyzer) -> None:
    """results/{kernel}_report.md and the terminal summary (the reference's reporter.py)."""
    from occupancy import parse_ptxas_stderr
    from reporter import ReportGenerator, print_terminal_summary

    def point(ms: float, causal: bool, variant: str) -> dict:
        pt = roof.analyze(kernel, dims, ms, causal=causal, variant=variant)
        return {"arithmetic_intensity": pt.arithmetic_intensity, "achieved_gflops": pt.achieved_gflops,
                "achieved_gbps": pt.achieved_gbps, "bound_type": pt.bound_type, "efficiency_pct": pt.efficiency_pct,
                "ceiling": pt.ceiling_name}

    rg = ReportGenerator(kernel, strategy_name, results_dir())
    rg.set_results(results, base_ms)
    if results and dims:
        b = results[0]
        v = "ffma" if b.params.get("variant") == "ffma" else ""
        rg.set_roofline_points(point(base_ms, False, v) if base_ms else None,
                               point(b.mean_ms, bool(b.params.get("causal")), v))
        rg.set_resource_report(parse_ptxas_stderr(b.ptx_info) or None)
    n_failed = sum(1 for f in failures if str(f.get("error", "")).startswith("verification"))
    n_ok = sum(1 for r in results if r.correctness_checked and r.is_correct)
    rg.set_correctness(n_ok, n_failed)
    conv_file = results_dir() / f"{kernel}_convergence.json"
    if conv_file.exists():
        rg.set_convergence(json.loads(conv_file.read_text()))
    rg.generate()
    print_terminal_summary(kernel, results, base_ms, strategy_name)


def compile_only(kernels: list[str], strategy_name: str, budget: Optional[int], seed: int, workers: int) -> int:
    """Generate and nvcc the variants each strategy suggests first, on host cores.

    Grid and successive halving suggest their whole first round up front (later
    halving rounds re-time a subset of it), so every library those runs load is
    built here; the Bayesian strategy's first batch only. Returns 0 when every
    variant compiled."""
    failed = 0
    for k in kernels:
        space = build_search_space(build_kernel_profile(k))
        strategy = make_strategy(strategy_name, space, kernel=k, n_calls=budget or 40, n_configs=budget or 80,
                                 seed=seed, anchors=default_points(k, space))
        pts = strategy.suggest(1 << 30)
        keys = {compile_key(k, p): p for p in pts}
        t0 = time.time()
        with ThreadPoolExecutor(max_workers=workers) as ex:
            built = list(ex.map(lambda p: ensure_variant(k, p), keys.values()))
        bad = [key for key, (ok, _, _) in zip(keys, built) if not ok]
        failed += len(bad)
        print(f"[COMPILE] {k}: {len(keys)} libraries for {len(pts)} points in {time.time() - t0:.0f}s"
              + (f", {len(bad)} failed: {bad}" if bad else ""))
    print(f"[DONE] libraries in {results_dir() / 'variants'}")
    return 0 if failed == 0 else 1


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Kernel auto-tuner — NVIDIA B200 (sm_100a)")
    ap.add_argument("--kernel", choices=SUPPORTED_KERNELS + ["all"], default="matmul")
    ap.add_argument("--baseline-only", action="store_true")
    ap.add_argument("--workers", type=int, default=max(1, min(8, (os.cpu_count() or 2))),
                    help="parallel nvcc compile workers (host cores)")
    ap.add_argument("--warmup", type=int, default=N_WARMUP_DEFAULT)
    ap.add_argument("--samples", type=int, default=N_SAMPLES_DEFAULT)
    ap.add_argument("--iters", type=int, default=None, help="alias for --samples")
    ap.add_argument("--strategy", choices=["grid", "bayesian", "sha"], default="grid")
    ap.add_argument("--skip-verification", action="store_true")
    ap.add_argument("--ptx-analysis", action="store_true",
                    help="print the ptxas resource report of each winner (no PTX/SASS reading)")
    ap.add_argument("--cuda-graphs", action="store_true", help="also time launches replayed from a CUDA graph")
    ap.add_argument("--matrix-size", type=int, default=None,
                    help="N for matmul, rows for softmax/layernorm, 1024·N for reduction, S for attention")
    ap.add_argument("--size", choices=["kat", "small", "config"], default="config")
    ap.add_argument("--gpus", type=int, default=1, help="GPU workers (one process per GPU)")
    ap.add_argument("--budget", type=int, default=None, help="max evaluations (bayesian) / initial configs (sha)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--results-dir", default=None)
    ap.add_argument("--compile-only", action="store_true",
                    help="only generate and compile the variants the strategy starts with (no GPU needed); a later "
                         "run with the same --results-dir, strategy, budget and seed reuses the libraries")
    a = ap.parse_args(argv)
    if a.results_dir:
        os.environ["KT_RESULTS_DIR"] = a.results_dir
    n_samples = a.iters if a.iters is not None else a.samples
    kernels = SUPPORTED_KERNELS if a.kernel == "all" else [a.kernel]

    if a.compile_only:
        return compile_only(kernels, a.strategy, a.budget, a.seed, a.workers)

    print("[BASELINE] naive GPU kernels ...")
    baselines = run_baseline_benchmark(a.warmup, n_samples, kernels=kernels, size=a.size)
    for tag, r in baselines.items():
        print(f"  {tag:<32} {r['mean_ms']:>10.4f} ms ± {r['ci_95_ms']:.4f}")
    if a.baseline_only:
        return 0
    pool = GpuPool(_visible_gpus(a.gpus))
    try:
        all_results = {}
        for k in kernels:
            bdata = next((v for v in baselines.values() if v["kernel"] == k), {})
            all_results[k] = autotune_kernel(k, bdata, pool, a.strategy, a.workers, a.warmup, n_samples,
                                             a.skip_verification, a.ptx_analysis, a.cuda_graphs, a.size,
                                             a.matrix_size, a.budget, a.seed)
    finally:
        pool.close()
    from reporter import print_final_summary
    print_final_summary(all_results, {k: next((v["mean_ms"] for v in baselines.values() if v["kernel"] == k), None)
                                      for k in kernels})
    print(f"[DONE] results in {results_dir()}")
    return 0 if all(all_results.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
