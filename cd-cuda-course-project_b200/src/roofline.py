"""
roofline.py — roofline model for NVIDIA B200 (sm_100a).

Rebuild of the reference's RTX-2070 model (src/roofline.py:26-276): same
`RooflineAnalyzer` methods (total_flops, total_bytes, arithmetic_intensity,
achieved_gflops, bound_type, peak_performance, efficiency_pct, analyze,
print_summary_table) and `get_dims`, with

  * B200 ceilings: measured HBM copy bandwidth and cuBLAS bf16 throughput
    from MEASURED_PEAKS.json when present (burst / sustained), else nominal
    (HBM3e ~8 TB/s, FP32 SIMT 148 SM × 128 FMA × 2 × 1.965 GHz, TF32 dense
    1.1 PFLOP/s, BF16 dense 2.25 PFLOP/s);
  * per-family ceilings: softmax, reduction and LayerNorm are HBM-bound and
    reported in GB/s; matmul (FFMA → FP32 SIMT, TF32 → TF32 tensor) and
    attention (BF16 tensor) in TFLOP/s;
  * the byte/FLOP models of workloads.work() (BASELINE's algorithmic counts)
    instead of the reference's 3·R·C·4 LayerNorm / 5·R·C softmax models;
  * dims taken from the actual problem (the reference hard-codes them,
    src/roofline.py:281-293).
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Literal, Optional

from workloads import SIZES, Work, work

BoundType = Literal["memory", "compute"]

SM_COUNT = 148
SM_MAX_MHZ = 1965.0

NOMINAL = {
    "hbm_gbs": 8000.0,
    "fp32_tflops": SM_COUNT * 128 * 2 * SM_MAX_MHZ * 1e6 / 1e12,   # ≈ 74.5
    "tf32_tflops": 1100.0,
    "bf16_tflops": 2250.0,
}


def _find_measured_peaks() -> Optional[Path]:
    env = os.environ.get("KT_MEASURED_PEAKS")
    cands = [Path(env)] if env else []
    here = Path(__file__).resolve()
    cands += [p / "MEASURED_PEAKS.json" for p in (here.parent.parent.parent, here.parent.parent, Path.cwd())]
    for c in cands:
        if c.is_file():
            return c
    return None


def load_peaks() -> dict:
    """
    Ceilings used for every fraction, each with its provenance:
    hbm_gbs (measured copy, or nominal), bf16_tflops / bf16_tflops_sustained
    (measured cuBLAS, or nominal), tf32_tflops (half of the bf16 figure, the
    documented dense ratio), fp32_tflops (nominal SIMT FMA peak).
    """
    peaks = dict(NOMINAL)
    src = {k: "nominal" for k in NOMINAL}
    path = _find_measured_peaks()
    if path is not None:
        try:
            m = json.loads(path.read_text())
            if m.get("hbm_gbs"):
                peaks["hbm_gbs"] = float(m["hbm_gbs"])
                src["hbm_gbs"] = "measured"
            if m.get("bf16_tflops"):
                peaks["bf16_tflops"] = float(m["bf16_tflops"])
                src["bf16_tflops"] = "measured"
                peaks["tf32_tflops"] = float(m["bf16_tflops"]) / 2.0
                src["tf32_tflops"] = "measured bf16 / 2"
            if m.get("bf16_tflops_sustained"):
                peaks["bf16_tflops_sustained"] = float(m["bf16_tflops_sustained"])
                src["bf16_tflops_sustained"] = "measured"
        except (OSError, ValueError):
            pass
    peaks["source"] = src
    return peaks


PEAKS = load_peaks()
PEAK_TFLOPS = PEAKS["bf16_tflops"]
MEM_BW_GBPS = PEAKS["hbm_gbs"]
RIDGE_POINT = PEAK_TFLOPS * 1e3 / MEM_BW_GBPS  # FLOP/byte


@dataclass
class RooflinePoint:
    """One kernel's position on the roofline."""
    kernel: str
    dims: tuple
    arithmetic_intensity: float   # FLOP / byte
    achieved_gflops: float
    achieved_gbps: float
    peak_gflops: float            # compute ceiling for compute-bound, AI·BW for memory-bound
    bound_type: BoundType
    efficiency_pct: float         # achieved / ceiling · 100 (not clamped)
    ceiling_name: str = ""


def _dims_dict(kernel: str, dims) -> dict:
    if isinstance(dims, dict):
        return dims
    keys = {"softmax": ("rows", "cols"), "layernorm": ("rows", "cols"), "reduction": ("n",),
            "matmul": ("M", "N", "K"), "attention": ("B", "H", "S", "D")}[kernel]
    if kernel == "matmul" and len(dims) == 1:
        dims = (dims[0],) * 3
    return dict(zip(keys, dims))


class RooflineAnalyzer:
    """
    Roofline metrics for the five tuned families on B200.

        ra = RooflineAnalyzer()
        pt = ra.analyze("softmax", {"rows": 4096, "cols": 4096}, elapsed_ms=0.021)
    """

    def __init__(self, peaks: Optional[dict] = None):
        self.peaks = peaks or PEAKS
        self.peak_tflops = self.peaks["bf16_tflops"]
        self.mem_bw_gbps = self.peaks["hbm_gbs"]
        self.ridge_point = self.peak_tflops * 1e3 / self.mem_bw_gbps

    @staticmethod
    def _base(kernel: str) -> str:
        return kernel.split("_")[0]

    def _work(self, kernel: str, dims, causal: bool = False, variant: str = "") -> Work:
        k = self._base(kernel)
        return work(k, _dims_dict(k, dims), causal=causal, variant=variant)

    def total_flops(self, kernel: str, dims, causal: bool = False) -> int:
        return self._work(kernel, dims, causal).flops

    def total_bytes(self, kernel: str, dims, causal: bool = False) -> int:
        return self._work(kernel, dims, causal).bytes

    def arithmetic_intensity(self, kernel: str, dims, causal: bool = False) -> float:
        w = self._work(kernel, dims, causal)
        return w.flops / w.bytes if w.bytes else 0.0

    def achieved_gflops(self, kernel: str, dims, elapsed_ms: float, causal: bool = False) -> float:
        if elapsed_ms <= 0:
            return 0.0
        return self.total_flops(kernel, dims, causal) / (elapsed_ms * 1e6)

    def achieved_gbps(self, kernel: str, dims, elapsed_ms: float, causal: bool = False) -> float:
        if elapsed_ms <= 0:
            return 0.0
        return self.total_bytes(kernel, dims, causal) / (elapsed_ms * 1e6)

    def bound_type(self, kernel: str, dims, causal: bool = False) -> BoundType:
        return "memory" if self._work(kernel, dims, causal).bound == "hbm" else "compute"

    def compute_ceiling_gflops(self, kernel: str, variant: str = "") -> tuple[float, str]:
        k = self._base(kernel)
        if k == "matmul":
            if variant == "ffma":
                return self.peaks["fp32_tflops"] * 1e3, "FP32 SIMT (nominal)"
            return self.peaks["tf32_tflops"] * 1e3, f"TF32 tensor ({self.peaks['source'].get('tf32_tflops')})"
        return self.peaks["bf16_tflops"] * 1e3, f"BF16 tensor ({self.peaks['source'].get('bf16_tflops')})"

    def peak_performance(self, kernel: str, dims, causal: bool = False, variant: str = "") -> float:
        """Applicable ceiling in GFLOP/s (memory-bound: AI × HBM bandwidth)."""
        if self.bound_type(kernel, dims, causal) == "memory":
            return self.arithmetic_intensity(kernel, dims, causal) * self.mem_bw_gbps
        return self.compute_ceiling_gflops(kernel, variant)[0]

    def efficiency_pct(self, kernel: str, dims, elapsed_ms: float, causal: bool = False,
                       variant: str = "") -> float:
        """Achieved / ceiling × 100. Memory-bound families compare bytes/s
        with the HBM ceiling; compute-bound ones FLOP/s with the tensor or
        SIMT ceiling. Not clamped: a hair above 100 % is possible against
        a measured copy-bandwidth ceiling."""
        if elapsed_ms <= 0:
            return 0.0
        if self.bound_type(kernel, dims, causal) == "memory":
            return self.achieved_gbps(kernel, dims, elapsed_ms, causal) / self.mem_bw_gbps * 100.0
        ceiling = self.compute_ceiling_gflops(kernel, variant)[0]
        return self.achieved_gflops(kernel, dims, elapsed_ms, causal) / ceiling * 100.0

    def analyze(self, kernel: str, dims, elapsed_ms: float, causal: bool = False,
                variant: str = "") -> RooflinePoint:
        dd = _dims_dict(self._base(kernel), dims)
        bound = self.bound_type(kernel, dd, causal)
        if bound == "memory":
            name = f"HBM {self.mem_bw_gbps:.0f} GB/s ({self.peaks['source'].get('hbm_gbs')})"
        else:
            name = self.compute_ceiling_gflops(kernel, variant)[1]
        return RooflinePoint(
            kernel=kernel,
            dims=tuple(dd.values()),
            arithmetic_intensity=self.arithmetic_intensity(kernel, dd, causal),
            achieved_gflops=self.achieved_gflops(kernel, dd, elapsed_ms, causal),
            achieved_gbps=self.achieved_gbps(kernel, dd, elapsed_ms, causal),
            peak_gflops=self.peak_performance(kernel, dd, causal, variant),
            bound_type=bound,
            efficiency_pct=self.efficiency_pct(kernel, dd, elapsed_ms, causal, variant),
            ceiling_name=name,
        )

    def print_summary_table(self, entries: list, title: str = "Roofline Summary") -> None:
        """entries: (kernel, dims, elapsed_ms) tuples."""
        print(f"\n{'=' * 86}")
        print(f"  {title}  |  B200  |  HBM {self.mem_bw_gbps:.0f} GB/s  BF16 {self.peak_tflops:.0f} TFLOP/s")
        print(f"{'=' * 86}")
        print(f"{'Kernel':<20} {'AI':>8} {'Bound':>8} {'GB/s':>10} {'TFLOP/s':>9} {'Eff%':>7}  ceiling")
        print("-" * 86)
        for kernel, dd, ms in entries:
            pt = self.analyze(kernel, dd, ms)
            print(f"{kernel:<20} {pt.arithmetic_intensity:>8.2f} {pt.bound_type:>8} "
                  f"{pt.achieved_gbps:>10.1f} {pt.achieved_gflops / 1e3:>9.2f} {pt.efficiency_pct:>6.1f}%  "
                  f"{pt.ceiling_name}")
        print("=" * 86 + "\n")


KERNEL_DIMS: dict[str, dict] = {k: SIZES[k]["config"] for k in SIZES}


def get_dims(kernel: str, size: str = "config") -> dict:
    """Problem dims for a kernel at a size configuration (default: the full config)."""
    base = kernel.split("_")[0]
    return dict(SIZES.get(base, SIZES["matmul"])[size])
