"""
benchmark.py — statistically rigorous timing of kernel-library variants.

Keeps the reference's measurement API and statistics (src/benchmark.py):
`BenchmarkResult` (:46-104), `compile_kernel` (:109-130), `run_binary`
(:135-152), `parse_timing_output` (:157-187), `_compute_stats` (:192-208),
`compute_significance` (:211-244), `run_statistical_benchmark` (:249-325),
`run_baseline_benchmark` (:330-400) and the ncu CSV helpers (:405-449).

What changed: the reference runs one executable per variant and parses its
SAMPLE/TIMING stdout lines; here a variant is a shared library timed
in-process through `kt_time` (CUDA events on the launching stream, L2
evicted before every sample by reading a buffer of twice the L2 size). The
samples feed the same statistics: Bessel-corrected std, 95 % CI =
1.96·s/√n, two-sided Welch t-test against the naive GPU baseline; a variant
is significant iff p < 0.05 and speedup > 1.
"""

from __future__ import annotations

import json
import math
import os
import subprocess
import warnings
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import List, Optional

try:
    from scipy import stats as _scipy_stats
    _SCIPY_OK = True
except ImportError:  # pragma: no cover
    _scipy_stats = None  # type: ignore
    _SCIPY_OK = False
    warnings.warn("scipy not installed — Welch t-test significance will be skipped.", RuntimeWarning, stacklevel=2)

import build as kt_build

PKG = Path(__file__).resolve().parent.parent
N_WARMUP_DEFAULT = 5
N_SAMPLES_DEFAULT = 30


def results_dir() -> Path:
    d = Path(os.environ.get("KT_RESULTS_DIR", PKG / "results"))
    d.mkdir(parents=True, exist_ok=True)
    return d


@dataclass
class BenchmarkResult:
    """
    Complete benchmark result for one kernel variant (the reference's record,
    src/benchmark.py:46-104, with B200 roofline fields added).
    """
    kernel: str
    variant: str
    params: dict = field(default_factory=dict)

    mean_ms: float = 0.0
    std_ms: float = 0.0
    ci_95_ms: float = 0.0
    min_ms: float = 0.0
    max_ms: float = 0.0
    n_samples: int = 0
    raw_samples: List[float] = field(default_factory=list)

    speedup: Optional[float] = None
    p_value: Optional[float] = None
    is_significant: bool = False

    compile_ok: bool = True
    ptx_info: str = ""

    arithmetic_intensity: Optional[float] = None
    achieved_gflops: Optional[float] = None
    bound_type: Optional[str] = None
    roofline_efficiency_pct: Optional[float] = None
    achieved_gbps: Optional[float] = None
    roofline_ceiling: Optional[str] = None

    occupancy: Optional[float] = None
    registers_per_thread: Optional[int] = None
    shared_mem_bytes: Optional[int] = None
    has_register_spill: bool = False
    spill_stores: int = 0
    spill_loads: int = 0

    graph_launch_ms: Optional[float] = None

    correctness_checked: bool = False
    is_correct: bool = True
    max_diff: Optional[float] = None

    library: str = ""
    problem: dict = field(default_factory=dict)
    gpu: Optional[int] = None
    # mean_ms scaled to the work of the family's reference problem (a causal
    # attention call does half the work of a non-causal one): what the tuner ranks by
    normalized_ms: Optional[float] = None

    def to_dict(self) -> dict:
        """Serialise for JSON (raw_samples excluded, as in the reference)."""
        d = asdict(self)
        d.pop("raw_samples", None)
        return d


# ---------------------------------------------------------------------------
# Compilation and process helpers
# ---------------------------------------------------------------------------

def compile_kernel(src_path: Path, out_path: Path, arch: str = kt_build.ARCH,
                   extra_flags: Optional[List[str]] = None) -> tuple[bool, str]:
    """nvcc a kernel-library translation unit into a shared library for sm_100a
    (always with -Xptxas -v; never fast-math). Returns (ok, stderr)."""
    if arch != kt_build.ARCH:
        raise ValueError(f"only {kt_build.ARCH} is built (asked for {arch})")
    return kt_build.compile_shared(Path(src_path), Path(out_path), extra_flags=extra_flags)


def run_binary(binary: Path, env_overrides: Optional[dict] = None, timeout: int = 120) -> tuple[bool, str, str]:
    """Run an executable with env overrides; (ok, stdout, stderr)."""
    env = os.environ.copy()
    if env_overrides:
        env.update({k: str(v) for k, v in env_overrides.items()})
    r = subprocess.run([str(binary)], capture_output=True, text=True, env=env, timeout=timeout)
    return r.returncode == 0, r.stdout, r.stderr


def parse_timing_output(stdout: str) -> dict[str, dict]:
    """
    Parse `SAMPLE <tag> <ms>` and `TIMING <tag> <mean> <min> <max> <iters>`
    lines into {tag: {"mean_ms", "min_ms", "max_ms", "iters", "samples"}}.
    """
    timings: dict[str, dict] = {}
    for line in stdout.splitlines():
        parts = line.split()
        if not parts:
            continue
        if parts[0] == "SAMPLE" and len(parts) >= 3:
            timings.setdefault(parts[1], {"samples": []})["samples"].append(float(parts[2]))
        elif parts[0] == "TIMING" and len(parts) >= 5:
            t = timings.setdefault(parts[1], {"samples": []})
            t["mean_ms"] = float(parts[2])
            t["min_ms"] = float(parts[3])
            t["max_ms"] = float(parts[4])
            t["iters"] = int(parts[5]) if len(parts) > 5 else 0
    return timings


def format_timing_output(tag: str, samples: List[float]) -> str:
    """The SAMPLE/TIMING text of a sample list (log format of the reference's executables)."""
    lines = [f"SAMPLE {tag} {s:.4f}" for s in samples]
    if samples:
        lines.append(f"TIMING {tag} {sum(samples) / len(samples):.4f} {min(samples):.4f} {max(samples):.4f} "
                     f"{len(samples)}")
    return "\n".join(lines) + "\n"


# ---------------------------------------------------------------------------
# Statistics (unchanged semantics)
# ---------------------------------------------------------------------------

def _compute_stats(samples: List[float]) -> tuple[float, float, float, float, float]:
    """(mean, std with Bessel's correction, 95 % CI half-width 1.96·s/√n, min, max)."""
    n = len(samples)
    if n == 0:
        return 0.0, 0.0, 0.0, 0.0, 0.0
    mean = sum(samples) / n
    if n == 1:
        return mean, 0.0, 0.0, samples[0], samples[0]
    variance = sum((x - mean) ** 2 for x in samples) / (n - 1)
    std = math.sqrt(variance)
    return mean, std, 1.96 * std / math.sqrt(n), min(samples), max(samples)


def compute_significance(variant_samples: List[float], baseline_samples: List[float]
                         ) -> tuple[Optional[float], Optional[float], bool, Optional[float]]:
    """
    Welch's t-test of variant vs baseline: (speedup, p_value, is_significant,
    baseline_mean). speedup > 1 means the variant is faster; significant
    requires p < 0.05 and speedup > 1 (heuristic speedup > 1 without scipy).
    """
    if not baseline_samples:
        return None, None, False, None
    baseline_mean = sum(baseline_samples) / len(baseline_samples)
    variant_mean = sum(variant_samples) / len(variant_samples) if variant_samples else 0.0
    speedup = (baseline_mean / variant_mean) if variant_mean > 0 else None
    p_value: Optional[float] = None
    is_significant = False
    if _SCIPY_OK and len(variant_samples) >= 2 and len(baseline_samples) >= 2:
        try:
            _, pv = _scipy_stats.ttest_ind(baseline_samples, variant_samples, equal_var=False)
            p_value = float(pv)
            if math.isnan(p_value):
                p_value = None
            is_significant = p_value is not None and p_value < 0.05 and speedup is not None and speedup > 1.0
        except Exception:  # noqa: BLE001
            pass
    elif speedup is not None:
        is_significant = speedup > 1.0
    return speedup, p_value, is_significant, baseline_mean


# ---------------------------------------------------------------------------
# In-process benchmarking through the C ABI
# ---------------------------------------------------------------------------

def time_problem(lib, problem, warmup: int, n_samples: int, naive: bool = False, flush: bool = True) -> List[float]:
    """`n_samples` CUDA-event samples (ms) of the problem's op on `lib`."""
    return problem.time(lib, warmup, n_samples, naive=naive, flush=flush)


def run_statistical_benchmark(binary, kernel_tag: str, baseline_samples: Optional[List[float]] = None,
                              warmup: int = N_WARMUP_DEFAULT, n_samples: int = N_SAMPLES_DEFAULT,
                              timeout: int = 180, problem=None) -> Optional["BenchmarkResult"]:
    """
    Time one variant with statistical rigour.

    `binary` is the variant's shared library (path or loaded KtLibrary);
    `problem` a problems.Problem on the current device (default: the
    family's full configuration). Returns None if the library fails.
    """
    import kt_lib
    import problems

    kernel = kernel_tag.split("_")[0]
    try:
        lib = binary if isinstance(binary, kt_lib.KtLibrary) else kt_lib.load(binary)
        prob = problem or problems.make_problem(kernel, "config", lib=lib)
        samples = time_problem(lib, prob, warmup, n_samples)
    except (kt_lib.KtError, OSError, RuntimeError) as exc:
        warnings.warn(f"{kernel_tag}: benchmark failed: {exc}")
        return None
    mean, std, ci, mn, mx = _compute_stats(samples)
    speedup, p_value, sig, _ = compute_significance(samples, baseline_samples or [])
    return BenchmarkResult(kernel=kernel, variant=kernel_tag, params={}, mean_ms=mean, std_ms=std, ci_95_ms=ci,
                           min_ms=mn, max_ms=mx, n_samples=len(samples), raw_samples=samples, speedup=speedup,
                           p_value=p_value, is_significant=sig, library=str(getattr(lib, "path", binary)),
                           problem=dict(prob.dims))


BASELINE_TAGS = {
    "matmul": lambda d: f"matmul_{d['M']}" if d["M"] == d["N"] == d["K"] else f"matmul_{d['M']}x{d['N']}x{d['K']}",
    "softmax": lambda d: f"softmax_{d['rows']}x{d['cols']}",
    "reduction": lambda d: f"reduction_{d['n']}",
    "layernorm": lambda d: f"layernorm_{d['rows']}x{d['cols']}",
    "attention": lambda d: f"attention_{d['B']}x{d['H']}x{d['S']}x{d['D']}",
}

# Naive kernels at full size take seconds per call (one thread per row or
# output); their sample counts are capped to keep the baseline bounded.
_NAIVE_SAMPLE_CAP = {"matmul": 5, "attention": 2}
_NAIVE_SIZE = {"attention": "small"}


def run_baseline_benchmark(warmup: int = N_WARMUP_DEFAULT, n_samples: int = N_SAMPLES_DEFAULT,
                           kernels=("matmul", "softmax", "reduction", "layernorm", "attention"),
                           size: str = "config", lib=None) -> dict[str, dict]:
    """
    Time the naive GPU kernels of the default library (the reference's
    baseline runner, src/kernels/benchmark_runner.cu:236-359) and save
    results/baseline.json. Returns {tag: {mean_ms, std_ms, ci_95_ms, min_ms,
    max_ms, samples, kernel, dims}}.
    """
    import kt_lib
    import problems

    lib = lib or kt_lib.load()
    out: dict[str, dict] = {}
    for k in kernels:
        sz = _NAIVE_SIZE.get(k, size) if size == "config" else size
        prob = problems.make_problem(k, sz, lib=lib)
        n = min(n_samples, _NAIVE_SAMPLE_CAP.get(k, n_samples)) if sz == "config" else n_samples
        w = min(warmup, 1) if k in _NAIVE_SAMPLE_CAP else warmup
        try:
            samples = time_problem(lib, prob, w, n, naive=True)
        except kt_lib.KtError as exc:
            warnings.warn(f"baseline {k}: {exc}")
            continue
        mean, std, ci, mn, mx = _compute_stats(samples)
        out[BASELINE_TAGS[k](prob.dims)] = {"mean_ms": mean, "std_ms": std, "ci_95_ms": ci, "min_ms": mn,
                                             "max_ms": mx, "samples": samples, "kernel": k,
                                             "dims": dict(prob.dims)}
        del prob
    save = {t: {kk: vv for kk, vv in d.items() if kk != "samples"} for t, d in out.items()}
    (results_dir() / "baseline.json").write_text(json.dumps(save, indent=2))
    return out


# ---------------------------------------------------------------------------
# Nsight Compute helpers (kept; the tuner does not call them by default)
# ---------------------------------------------------------------------------

def collect_ncu_metrics(binary: Path, metrics: Optional[List[str]] = None, args: Optional[List[str]] = None) -> dict:
    """Run `ncu --metrics … --csv --clock-control none` on a command; {} if ncu is unavailable."""
    if metrics is None:
        metrics = ["dram__bytes_read.sum", "dram__bytes_write.sum", "gpu__time_duration.sum",
                   "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active"]
    cmd = ["ncu", "--metrics", ",".join(metrics), "--csv", "--clock-control", "none", str(binary), *(args or [])]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            return {}
        return _parse_ncu_csv(r.stdout)
    except (FileNotFoundError, subprocess.TimeoutExpired):
        return {}


def _parse_ncu_csv(csv_text: str) -> dict:
    """Parse `ncu --csv` output into {metric_name: value}."""
    import csv
    import io
    metrics: dict = {}
    rows = [r for r in csv.reader(io.StringIO(csv_text.strip())) if r]
    if len(rows) < 2:
        return metrics
    hdr = rows[0]
    for r in rows[1:]:
        if len(r) < len(hdr):
            continue
        row = dict(zip(hdr, r))
        name = row.get("Metric Name", "")
        val = row.get("Metric Value", "")
        if name:
            try:
                metrics[name] = float(val.replace(",", ""))
            except ValueError:
                metrics[name] = val
    return metrics


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description="Naive GPU baseline timings")
    ap.add_argument("--warmup", type=int, default=N_WARMUP_DEFAULT)
    ap.add_argument("--samples", type=int, default=N_SAMPLES_DEFAULT)
    ap.add_argument("--size", default="config", choices=["kat", "small", "config"])
    a = ap.parse_args()
    res = run_baseline_benchmark(a.warmup, a.samples, size=a.size)
    for tag, r in res.items():
        print(f"{tag:<32} {r['mean_ms']:>10.4f} ms ± {r['ci_95_ms']:.4f}")
