"""
reporter.py — Markdown tuning reports and terminal summaries.

Rebuilds the reference's `ReportGenerator` (src/reporter.py:61-300) and its
`print_terminal_summary` / `print_final_summary` (:305-420) for the B200
tuner. The report keeps the reference's sections and file name
(results/{kernel}_report.md):

  1. header: kernel, date, hardware, strategy
  2. roofline: naive baseline against the best variant, each as achieved
     GB/s or TFLOP/s and as a fraction of the B200 ceiling it is bound by
     (measured copy bandwidth / cuBLAS throughput when MEASURED_PEAKS.json
     exists, nominal otherwise; the source is printed)
  3. top configurations: mean ± 95 % CI, work-normalised time, speed-up over
     the naive kernel, Welch p-value, significance
  4. occupancy: registers, static + dynamic shared memory, spills
  5. resources: the ptxas lines of the winner (registers, shared memory,
     spills, barriers per kernel) in place of the reference's PTX/SASS
     instruction analysis, which is not done here
  6. correctness: variants verified / passed / failed
  7. convergence (bayesian / sha)
  8. recommended configuration and the library file that holds it

Only the standard library is used for formatting.
"""

from __future__ import annotations

import json
from datetime import datetime
from pathlib import Path
from typing import Iterable, Optional, Sequence

from benchmark import BenchmarkResult, results_dir


def hardware_label() -> str:
    """One line naming the GPU and the ceilings the fractions use."""
    from roofline import PEAKS
    src = PEAKS.get("source", {})
    return (f"NVIDIA B200 (sm_100a), HBM3e {PEAKS['hbm_gbs']:.0f} GB/s ({src.get('hbm_gbs', 'nominal')}), "
            f"BF16 tensor {PEAKS['bf16_tflops']:.0f} TFLOP/s ({src.get('bf16_tflops', 'nominal')}), "
            f"FP32 FFMA {PEAKS['fp32_tflops']:.1f} TFLOP/s (nominal)")


def md_table(headers: Sequence[str], rows: Iterable[Sequence[object]]) -> str:
    """GitHub-flavoured Markdown table with padded columns."""
    rows = [[str(c) for c in r] for r in rows]
    widths = [max([len(h)] + [len(r[i]) for r in rows]) for i, h in enumerate(headers)]
    line = lambda cells: "| " + " | ".join(c.ljust(widths[i]) for i, c in enumerate(cells)) + " |"  # noqa: E731
    return "\n".join([line(headers), "| " + " | ".join("-" * w for w in widths) + " |"] + [line(r) for r in rows])


def fmt(v: Optional[float], nd: int = 3, suffix: str = "") -> str:
    return "—" if v is None else f"{v:.{nd}f}{suffix}"


def short_params(params: dict, width: int = 60) -> str:
    """Compact one-line rendering of a parameter point (keys sorted)."""
    abbrev = {"block_size": "blk", "vec_per_thread": "vpt", "min_blocks": "minb", "blocks_per_sm": "bpsm",
              "cluster_size": "cl", "transpose_b": "T", "poly_exp2": "poly", "v_stages": "vst"}
    s = " ".join(f"{abbrev.get(k, k)}={v}" for k, v in sorted(params.items()))
    return s if len(s) <= width else s[:width - 1] + "…"


class ReportGenerator:
    """
    Markdown report of one family's tuning run.

        rg = ReportGenerator("softmax", strategy="sha")
        rg.set_results(sorted_results, baseline_ms=3.21)
        rg.set_roofline_points(baseline_point, best_point)
        rg.set_correctness(n_passed=14, n_failed=1)
        rg.set_resource_report(ptxas_entries)
        rg.set_convergence(convergence_dict)
        path = rg.generate()          # results/softmax_report.md
    """

    def __init__(self, kernel: str, strategy: str = "grid", results_dir_: Optional[Path] = None) -> None:
        self.kernel = kernel
        self.strategy = strategy
        self.dir = Path(results_dir_) if results_dir_ is not None else results_dir()
        self.path = self.dir / f"{kernel}_report.md"
        self.results: list[BenchmarkResult] = []
        self.baseline_ms: Optional[float] = None
        self.roof_base: Optional[dict] = None
        self.roof_best: Optional[dict] = None
        self.n_passed = self.n_failed = self.n_checked = 0
        self.resources: Optional[dict] = None
        self.convergence: Optional[dict] = None

    # -- inputs (the reference's setters) --------------------------------------
    def set_results(self, results: list[BenchmarkResult], baseline_ms: Optional[float] = None) -> None:
        self.results = list(results)
        self.baseline_ms = baseline_ms

    def set_roofline_points(self, baseline_pt: Optional[dict], best_pt: Optional[dict]) -> None:
        """Dicts with arithmetic_intensity, achieved_gflops, achieved_gbps, bound_type, efficiency_pct, ceiling."""
        self.roof_base, self.roof_best = baseline_pt, best_pt

    def set_correctness(self, n_passed: int, n_failed: int, n_checked: int = 0) -> None:
        self.n_passed, self.n_failed = n_passed, n_failed
        self.n_checked = n_checked or (n_passed + n_failed)

    def set_resource_report(self, entries: Optional[dict]) -> None:
        """{kernel name: {registers, smem_bytes, spill_stores, spill_loads, barriers}} (occupancy.parse_ptxas_stderr)."""
        self.resources = entries

    def set_ptx_data(self, data: Optional[dict]) -> None:
        """Kept for callers of the reference's API; PTX is not analysed here, so this is the resource report."""
        self.set_resource_report(data)

    def set_convergence(self, convergence: Optional[dict]) -> None:
        """The ConvergenceLogger file: {kernel, n_evals, best_ms, curve}."""
        self.convergence = convergence

    # -- sections --------------------------------------------------------------
    def _header(self) -> list[str]:
        return [f"# Kernel auto-tuner report — `{self.kernel}`", "",
                md_table(["Field", "Value"], [["Kernel", f"`{self.kernel}`"],
                                              ["Date", datetime.now().strftime("%Y-%m-%d %H:%M:%S")],
                                              ["Hardware", hardware_label()],
                                              ["Strategy", f"`{self.strategy}`"]]), ""]

    @staticmethod
    def _roof_row(name: str, p: dict) -> list[str]:
        memory = p.get("bound_type") == "memory"
        achieved = f"{p.get('achieved_gbps', 0):.0f} GB/s" if memory else f"{p.get('achieved_gflops', 0) / 1e3:.1f} TFLOP/s"
        return [name, f"{p.get('arithmetic_intensity', 0):.2f}", p.get("bound_type", "—"), achieved,
                f"{p.get('efficiency_pct', 0):.1f} %", p.get("ceiling", "—")]

    def _roofline(self) -> list[str]:
        out = ["## Roofline", ""]
        rows = []
        if self.roof_base:
            rows.append(self._roof_row("naive baseline", self.roof_base))
        if self.roof_best:
            rows.append(self._roof_row("best variant", self.roof_best))
        if not rows:
            return out + ["*(no roofline data in this run)*", ""]
        return out + [md_table(["Config", "AI (FLOP/byte)", "Bound", "Achieved", "of ceiling", "Ceiling"], rows), ""]

    def _top(self) -> list[str]:
        out = ["## Top configurations", ""]
        top = self.results[:10]
        if not top:
            return out + ["*(no variant compiled, verified and timed)*", ""]
        rows = [[short_params(r.params), f"{r.mean_ms:.4f} ms", f"±{r.ci_95_ms:.4f}",
                 fmt(r.normalized_ms, 4, " ms"), fmt(r.speedup, 2, "x"),
                 "—" if r.p_value is None else f"{r.p_value:.2g}", "yes" if r.is_significant else "no",
                 fmt(r.roofline_efficiency_pct, 1, " %")] for r in top]
        return out + [md_table(["Config", "mean", "95 % CI", "normalised", "speed-up", "p", "significant",
                                "of ceiling"], rows), ""]

    def _occupancy(self) -> list[str]:
        occ = [r for r in self.results[:10] if r.occupancy is not None]
        if not occ:
            return []
        rows = [[short_params(r.params), f"{100 * r.occupancy:.1f} %", r.registers_per_thread or "—",
                 r.shared_mem_bytes or 0, "yes" if r.has_register_spill else "no"] for r in occ]
        return ["## Occupancy", "", md_table(["Config", "Occupancy", "Registers", "Shared memory (B)", "Spills"],
                                             rows), ""]

    def _resources(self) -> list[str]:
        if not self.resources:
            return []
        rows = [[f"`{name[:70]}`", e.get("registers", "—"), e.get("smem_bytes", "—"),
                 f"{e.get('spill_stores', 0)}/{e.get('spill_loads', 0)}", e.get("barriers", "—")]
                for name, e in self.resources.items()]
        return ["## Resources of the best variant (ptxas)", "",
                md_table(["Kernel", "Registers", "Static smem (B)", "Spill st/ld (B)", "Barriers"], rows), ""]

    def _correctness(self) -> list[str]:
        out = ["## Correctness", ""]
        if self.n_checked == 0:
            return out + ["*(verification skipped in this run)*", ""]
        return out + [md_table(["Metric", "Count"], [["variants verified", self.n_checked],
                                                     ["passed", self.n_passed], ["failed", self.n_failed]]), ""]

    def _convergence(self) -> list[str]:
        c = self.convergence
        if not c or self.strategy not in ("bayesian", "sha"):
            return []
        best = c.get("best_ms")
        best_s = f"{best:.4f} ms" if isinstance(best, (int, float)) else "—"
        return ["## Convergence", "",
                f"Strategy **{self.strategy}** reached its best configuration ({best_s}) "
                f"after **{c.get('n_evals', '—')}** evaluations.", ""]

    def _recommended(self) -> list[str]:
        out = ["## Recommended configuration", ""]
        if not self.results:
            return out + ["*(no successful variant)*", ""]
        b = self.results[0]
        out += [f"**Kernel:** `{self.kernel}`", "", "**Parameters:**", ""]
        out += [f"  - `{k}` = `{v}`" for k, v in b.params.items()]
        out += ["", f"**Mean latency:** {b.mean_ms:.4f} ms ±{b.ci_95_ms:.4f} ms (95 % CI, n={b.n_samples})"]
        if b.speedup:
            sig = "statistically significant" if b.is_significant else "not significant"
            out += ["", f"**Speed-up:** {b.speedup:.2f}x over the naive kernel ({sig})"]
        if b.library:
            out += ["", f"**Library:** `{b.library}`"]
        return out + [""]

    def render(self) -> str:
        lines: list[str] = []
        for sec in (self._header, self._roofline, self._top, self._occupancy, self._resources, self._correctness,
                    self._convergence, self._recommended):
            lines += sec()
        return "\n".join(lines) + "\n"

    def generate(self) -> Path:
        """Write results/{kernel}_report.md and return its path."""
        self.dir.mkdir(parents=True, exist_ok=True)
        self.path.write_text(self.render(), encoding="utf-8")
        print(f"[REPORT] {self.path}")
        return self.path


def print_terminal_summary(kernel: str, results: list[BenchmarkResult], baseline_ms: Optional[float] = None,
                           strategy: str = "grid", n_show: int = 10) -> None:
    """Top results of one family as a plain-text table."""
    W = 100
    print("\n" + "=" * W)
    print(f"  TUNING COMPLETE — {kernel.upper()}  |  strategy={strategy}  |  B200 (sm_100a)")
    print("=" * W)
    if not results:
        print("  No successful results.")
        print("=" * W)
        return
    print(f"  {'Config':<48} {'mean ms':>10} {'±CI':>9} {'speedup':>8} {'p':>9} {'sig':>4} {'roof%':>6}")
    print("  " + "-" * (W - 2))
    for r in results[:n_show]:
        print(f"  {short_params(r.params, 48):<48} {r.mean_ms:>10.4f} {r.ci_95_ms:>9.4f} "
              f"{fmt(r.speedup, 2, 'x'):>8} {('—' if r.p_value is None else f'{r.p_value:.2g}'):>9} "
              f"{('yes' if r.is_significant else 'no'):>4} {fmt(r.roofline_efficiency_pct, 1):>6}")
    b = results[0]
    print("=" * W)
    if baseline_ms:
        print(f"  BEST {b.mean_ms:.4f} ms  |  naive {baseline_ms:.4f} ms  |  speed-up {baseline_ms / b.mean_ms:.1f}x")
    if b.bound_type:
        print(f"  BOUND {b.bound_type}  |  {fmt(b.roofline_efficiency_pct, 1)} % of {b.roofline_ceiling}")
    if b.occupancy is not None:
        print(f"  OCCUPANCY {100 * b.occupancy:.1f} %  |  {b.registers_per_thread} registers  |  "
              f"{'spills' if b.has_register_spill else 'no spills'}")
    print("=" * W + "\n")


def print_final_summary(all_results: dict[str, list[BenchmarkResult]],
                        baselines: Optional[dict[str, float]] = None) -> None:
    """One line per family: naive baseline, best, speed-up, fraction of ceiling."""
    W = 80
    print("\n" + "=" * W)
    print("  FULL TUNING SUMMARY (B200)")
    print("=" * W)
    print(f"  {'Kernel':<12} {'naive ms':>10} {'best ms':>10} {'speed-up':>9} {'of ceiling':>11}")
    print("  " + "-" * (W - 2))
    for k, res in all_results.items():
        if not res:
            print(f"  {k:<12} {'—':>10} {'—':>10} {'—':>9} {'—':>11}")
            continue
        b = res[0]
        base = (baselines or {}).get(k)
        sp = f"{base / b.mean_ms:.1f}x" if base else "—"
        print(f"  {k:<12} {fmt(base, 4):>10} {b.mean_ms:>10.4f} {sp:>9} {fmt(b.roofline_efficiency_pct, 1, ' %'):>11}")
    print("=" * W + "\n")


def report_from_files(kernel: str, rdir: Optional[Path] = None) -> Path:
    """Rebuild {kernel}_report.md from the tuning, failures and convergence files of a finished run."""
    rdir = Path(rdir) if rdir is not None else results_dir()
    t = json.loads((rdir / f"{kernel}_tuning.json").read_text())
    fields = set(BenchmarkResult.__dataclass_fields__)
    results = [BenchmarkResult(**{k: v for k, v in d.items() if k in fields}) for d in t.get("variants", [])]
    rg = ReportGenerator(kernel, t.get("strategy", "grid"), rdir)
    rg.set_results(results, t.get("baseline_ms"))
    fails = rdir / f"{kernel}_failures.json"
    n_failed = len(json.loads(fails.read_text())) if fails.exists() else 0
    n_ok = sum(1 for r in results if r.correctness_checked and r.is_correct)
    rg.set_correctness(n_ok, n_failed)
    conv = rdir / f"{kernel}_convergence.json"
    if conv.exists():
        rg.set_convergence(json.loads(conv.read_text()))
    if results:
        b = results[0]
        rg.set_roofline_points(None, {"arithmetic_intensity": b.arithmetic_intensity or 0.0,
                                      "achieved_gflops": b.achieved_gflops or 0.0,
                                      "achieved_gbps": b.achieved_gbps or 0.0, "bound_type": b.bound_type,
                                      "efficiency_pct": b.roofline_efficiency_pct or 0.0,
                                      "ceiling": b.roofline_ceiling})
    return rg.generate()
