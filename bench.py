#!/usr/bin/env python
"""
bench.py — throughput of the tuned kernel library on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's CPU (NumPy) path
    python bench.py --only matmul_tf32 ...    # one case alone (profiler captures)

One step is one pass of a kernel family over its full synthetic batch. The
headline workload (the top-level `value`) is the sum reduction: 2^28 fp32
values ~ U[-1,1], sharded contiguously across the ranks (total size fixed:
strong scaling); each rank reduces its shard to an fp64 partial with the
library's kernel and the partials are combined with one NCCL all-reduce.
The same run then measures every other family at its configuration size,
each reported under `families`:

    softmax           fp32 4096x4096, rows sharded
    layernorm         fp32 16384x4096, rows sharded
    matmul_tf32       fp32 8192^3 on tcgen05 (TF32), row-blocks of A sharded
    matmul_tf32_tb    the same with B stored transposed (transpose_b)
    matmul_ffma       fp32 8192^3 on the FP32 FMA pipe
    attention         flash-attention fwd bf16 [8,32,4096,128], (b,h) sharded
    attention_causal  the same with the causal mask

Per case: `value` (whole job, device-resident inputs), `e2e` (pinned host
inputs copied in and the result copied out every step, through the C ABI),
the roofline of its kernel (CUDA events on the launching stream), parity of
the result against the oracle on a bounded sample of every rank's shard, the
CPU baseline (N=1), clocks sampled over its soak and timed steps, and the
number of library kernels launched in its timed region.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field
from datetime import timedelta
from pathlib import Path
from typing import Callable, Optional

REPO = Path(__file__).resolve().parent
PKG = REPO / "cd-cuda-course-project_b200"
sys.path.insert(0, str(PKG / "src"))

METRIC = ("achieved HBM GB/s (softmax/reduce/LN) & TFLOP/s (matmul/attn) vs roofline, 1–8 B200")


@dataclass(frozen=True)
class Case:
    name: str
    kernel: str          # family: reduction | softmax | layernorm | matmul | attention
    variant: str = ""    # matmul: tf32 | ffma
    tb: bool = False     # matmul: B holds Bt (N x K)
    causal: bool = False


CASES = {c.name: c for c in (
    Case("reduction", "reduction"),
    Case("reduction_nccl", "reduction", "nccl"),
    Case("softmax", "softmax"),
    Case("layernorm", "layernorm"),
    Case("matmul_tf32", "matmul", "tf32"),
    Case("matmul_tf32_tb", "matmul", "tf32", tb=True),
    Case("matmul_ffma", "matmul", "ffma"),
    Case("matmul_ffma_tb", "matmul", "ffma", tb=True),
    Case("attention", "attention"),
    Case("attention_causal", "attention", causal=True),
)}
DEFAULT_FAMILIES = ("softmax", "layernorm", "matmul_tf32", "matmul_tf32_tb", "matmul_ffma", "attention",
                    "attention_causal")

# kernel instance (name<template arguments>) each case's dominant launch runs
# with the default library, matched against the `kernel_id:` line of the
# committed ncu summaries under profiles/
KERNEL_ID = {
    "reduction": "sum_f32_xrank<512,4>",
    "reduction_nccl": "sum_f32<512,4>",
    "softmax": "softmax_rows<256,4,2>",
    "layernorm": "layernorm_rows<256,4,2>",
    "matmul_tf32": "gemm_tf32_kernel<256,4,0>",
    "matmul_tf32_tb": "gemm_tf32_kernel<256,4,1>",
    "matmul_ffma": "sgemm_128x256<0,1,8>",
    "matmul_ffma_tb": "sgemm_128x256<1,1,8>",
    "attention": "fa_fwd_kernel<128,2,0>",
    "attention_causal": "fa_fwd_kernel<128,2,1>",
}


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--kernel", choices=["reduction", "softmax", "layernorm", "matmul", "attention"],
                   default="reduction", help="family of the headline (top-level) measurement")
    p.add_argument("--variant", choices=["tf32", "ffma"], default="tf32", help="matmul headline variant")
    p.add_argument("--transpose-b", action="store_true", help="matmul headline: B holds Bt (N×K)")
    p.add_argument("--causal", action="store_true", help="attention headline: causal mask")
    p.add_argument("--families", default="all",
                   help="comma list of cases measured after the headline, 'all' or 'none'")
    p.add_argument("--only", choices=sorted(CASES), default=None,
                   help="measure this case alone as the headline (no families)")
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--soak-s", type=float, default=1.5,
                   help="seconds of untimed steps run under the clock sampler before each case's timed steps")
    p.add_argument("--scale", type=float, default=1.0,
                   help="shrink the leading dim of every workload (small cases for profiler captures)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    return p.parse_args()


def headline_case(args: argparse.Namespace) -> Case:
    if args.only:
        return CASES[args.only]
    k = args.kernel
    if k == "matmul":
        return CASES[f"matmul_{args.variant}{'_tb' if args.transpose_b else ''}"]
    if k == "attention":
        return CASES["attention_causal" if args.causal else "attention"]
    return CASES[k]


def family_cases(args: argparse.Namespace, head: Case) -> list[Case]:
    if args.only or args.families == "none":
        return []
    names = DEFAULT_FAMILIES if args.families == "all" else tuple(x.strip() for x in args.families.split(",") if x.strip())
    for n in names:
        if n not in CASES:
            raise SystemExit(f"unknown case {n!r}; known: {sorted(CASES)}")
    out = [CASES[n] for n in names if n != head.name]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.families == "all" and head.name == "reduction" and world > 1:
        out.insert(0, CASES["reduction_nccl"])  # the same sum with the partials combined by NCCL, for comparison
    return out


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def emit(obj: dict) -> None:
    print(json.dumps(obj), flush=True)


def workload_name(c: Case) -> str:
    if c.kernel == "reduction":
        how = ("fp64 partials combined by one NCCL all-reduce" if c.variant == "nccl"
               else "fp64 partials combined inside the kernel over NVLink peer stores")
        return f"sum reduction fp32 N=2^28 U[-1,1] -> fp64 sum, contiguous shards, {how}"
    return {
        "softmax": "row softmax fp32 4096x4096 N(0,1), rows sharded",
        "layernorm": "layernorm fp32 16384x4096 N(0,1), gamma=1+0.1N, beta=0.1N, eps=1e-5, rows sharded",
        "matmul": f"matmul fp32 8192^3 U[-1,1] {c.variant}{' transpose_b' if c.tb else ''}, row-blocks of A sharded",
        "attention": f"flash-attention fwd bf16 B=8 H=32 S=4096 D=128 N(0,1) "
                     f"{'causal' if c.causal else 'non-causal'}, batch*head sharded",
    }[c.kernel]


def scaled_dims(kernel: str, scale: float) -> dict:
    """The full configuration, with its leading dim multiplied by `scale` (<= 1)."""
    import workloads
    d = workloads.dims(kernel, "config")
    if scale >= 1.0:
        return d
    lead = {"reduction": "n", "softmax": "rows", "layernorm": "rows", "matmul": "M", "attention": "B"}[kernel]
    d[lead] = max(1, int(d[lead] * scale))
    return d


# ---------------------------------------------------------------------------
# Clock sampler (nvidia-smi, read-only queries), windows per case
# ---------------------------------------------------------------------------

SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int, period_ms: int = 100):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.rows: list[tuple[float, list[str]]] = []
        self._t = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [x.strip() for x in line.strip().split(",")]))

    def stop(self) -> None:
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)

    def summary(self, t0: float, t1: float) -> Optional[dict]:
        if self.proc is None:
            return None
        rows = []
        for t, parts in list(self.rows):
            if not (t0 <= t <= t1) or len(parts) < 10:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]),
                             "util": float(parts[4]) if parts[4] not in ("[N/A]", "N/A") else 0.0,
                             "hw": parts[6], "hwt": parts[7], "swt": parts[8], "pcap": parts[9]})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [r for r in rows if r["util"] >= 50.0] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(loaded)}


# ---------------------------------------------------------------------------
# Committed ncu summaries
# ---------------------------------------------------------------------------

def profiled_traffic(kernel_id: str, units_per_launch: int) -> Optional[dict]:
    """DRAM bytes per launch of `kernel_id` from the committed ncu summaries
    (profiles/*.md with `kernel_id:`, `units_per_launch:` and
    `traffic_bytes_per_launch:` lines). A capture of a smaller case of a
    streaming kernel is scaled by the units processed; the summary states
    whether that holds (`traffic_scales: linear`)."""
    best = None
    for p in sorted((REPO / "profiles").glob("*.md")):
        text = p.read_text()
        m_id = re.search(r"^kernel_id:\s*(\S+)", text, re.M)
        m_tr = re.search(r"^traffic_bytes_per_launch:\s*([0-9]+)", text, re.M)
        m_u = re.search(r"^units_per_launch:\s*([0-9]+)", text, re.M)
        if not (m_id and m_tr and m_u) or m_id.group(1) != kernel_id:
            continue
        units, traffic = int(m_u.group(1)), int(m_tr.group(1))
        linear = re.search(r"^traffic_scales:\s*linear", text, re.M) is not None
        if units == units_per_launch:
            return {"bytes": traffic, "source": f"profiles/{p.name}", "scaled": False}
        if linear and best is None:
            best = {"bytes": int(round(traffic * units_per_launch / units)), "source": f"profiles/{p.name}",
                    "scaled": f"x{units_per_launch / units:.4g} from a {units}-unit capture"}
    return best


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU (NumPy) path on the host cores
# ---------------------------------------------------------------------------

class CpuRef:
    """Bounded samples of each case on the host cores: the reference's NumPy
    formulas (oracle/cpu_baseline.py) at the reference's own precision."""

    def __init__(self, seed: int):
        from oracle import cpu_baseline as cb
        self.cb = cb
        self.seed = seed
        self.threads = cb.host_threads()
        self._cache: dict = {}

    def _inputs(self, kernel: str, part=None):
        import workloads
        key = (kernel, part)
        if key not in self._cache:
            self._cache = {k: v for k, v in self._cache.items() if k[0] == kernel}
            self._cache[key] = workloads.make_inputs(kernel, d=workloads.dims(kernel, "config"), seed=self.seed,
                                                     part=part)
        return self._cache[key]

    def step(self, c: Case) -> tuple[float, float, str]:
        """One timed sample: (seconds, units done, sample description); units
        are bytes for the HBM families and FLOPs for matmul/attention."""
        import numpy as np
        import workloads
        cb, th = self.cb, self.threads
        if c.kernel == "reduction":
            x = self._inputs("reduction")["x"]
            r = cb.reduce_sum(x, th, reps=1)
            return r["best_s"], x.nbytes, "whole array n=2^28 (fp64 NumPy sum, chunked over the host threads)"
        if c.kernel == "softmax":
            inp = self._inputs("softmax")
            r = cb.rows_op("softmax", inp["x"], th, 1)
            return r["best_s"], r["bytes"], "whole 4096x4096 batch (fp32 NumPy, rows over the host threads)"
        if c.kernel == "layernorm":
            rows = 2048
            inp = self._inputs("layernorm", (0, rows))
            r = cb.rows_op("layernorm", inp["x"], th, 1, inp["gamma"], inp["beta"], inp["eps"])
            return r["best_s"], r["bytes"], f"{rows} of 16384 rows (fp64 NumPy statistics, rows over the host threads)"
        if c.kernel == "matmul":
            rows = 512
            inp = self._inputs("matmul", (0, rows))
            if c.tb and "Bt" not in inp:
                inp["Bt"] = np.ascontiguousarray(inp["B"].T)
            r = cb.matmul(inp["A"], inp["Bt"] if c.tb else inp["B"], reps=1, transpose_b=c.tb)
            return r["best_s"], r["flops"], f"{rows}x8192 row block of A x full B{'t' if c.tb else ''} (fp32 BLAS)"
        nh = 2
        inp = self._inputs("attention", (0, nh))
        key = ("attention_f32", nh)
        if key not in self._cache:
            self._cache[key] = tuple(workloads.bf16_to_f32(inp[n]) for n in ("q", "k", "v"))
        q, k, v = self._cache[key]
        r = cb.attention_heads(q, k, v, inp["scale"], c.causal, th)
        return r["best_s"], r["flops"], f"{nh} of 256 (b,h) heads, S=4096 D=128 (fp32 NumPy, heads over threads)"

    def measure(self, c: Case, steps: int, warmup: int, budget_s: float) -> dict:
        for _ in range(warmup):
            self.step(c)
        ts, us = [], []
        t_start = time.monotonic()
        sample = ""
        for _ in range(max(1, steps)):
            t, u, sample = self.step(c)
            ts.append(t)
            us.append(u)
            if time.monotonic() - t_start > budget_s:
                break
        unit = "GB/s" if c.kernel in ("reduction", "softmax", "layernorm") else "TFLOP/s"
        value = sum(us) / sum(ts) / (1e9 if unit == "GB/s" else 1e12)
        return {"value": value, "unit": unit, "cores": self.threads, "kind": "port", "sample": sample,
                "steps": len(ts), "ms_per_step": 1e3 * sum(ts) / len(ts)}


def run_reference(args: argparse.Namespace, rank: int, world: int) -> None:
    if rank != 0:
        return
    head = headline_case(args)
    fams = family_cases(args, head)
    cpu = CpuRef(args.seed)

    def line(c: Case, budget_s: float) -> dict:
        r = cpu.measure(c, args.steps, args.warmup, budget_s)
        return {"value": r["value"], "unit": r["unit"], "ms_per_step": r["ms_per_step"], "steps": r["steps"],
                "config": {"workload": workload_name(c), **scaled_dims(c.kernel, 1.0)},
                "cpu_baseline": r, "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0,
                                           "d2h_bytes_per_step": 0}}

    h = line(head, 60.0)
    families = {c.name: line(c, 8.0) for c in fams}
    emit({
        "metric": METRIC, "impl": "reference", "value": h["value"], "unit": h["unit"], "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": h["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32" if head.kernel != "attention" else "bf16", "data": "synthetic", "config": h["config"],
        "cpu_baseline": h["cpu_baseline"], "e2e": h["e2e"], "families": families,
    })


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

@dataclass
class Job:
    """One case set up on this rank: its launch, e2e copies, work counts and checks."""
    case: Case
    dims: dict
    launch: Callable[[object], None]
    dev_src: object
    e2e_src: object
    e2e_in: Callable[[], None]
    e2e_out: Callable[[], None]
    units_job: int              # bytes (HBM families) or FLOPs of the whole job
    units_launch: int           # this rank's share, per launch
    unit: str
    dtype: str
    bound: str                  # hbm | tensor | fp32
    h2d: int
    d2h: int
    dev_bytes: int
    parity: Callable[[], dict]
    collective: Optional[Callable[[], None]] = None   # a step's exchange after the kernel (None: none)
    launches_per_step: int = 1
    tensors: list = field(default_factory=list)


class Ctx:
    def __init__(self, args, rank, world, local, dev, lib, stream):
        self.args, self.rank, self.world, self.local = args, rank, world, local
        self.dev, self.lib, self.stream, self.sh = dev, lib, stream, stream.cuda_stream


def setup_job(ctx: Ctx, c: Case) -> Job:
    import numpy as np
    import torch

    import kt_lib
    import sharding
    import workloads
    from oracle import ref

    lib, dev, sh = ctx.lib, ctx.dev, ctx.sh
    d = scaled_dims(c.kernel, ctx.args.scale)
    e2e = not ctx.args.no_e2e

    def pinned(a: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()

    def shard(n: int) -> tuple[int, int]:
        return sharding.shard_range(n, ctx.world, ctx.rank)

    if c.kernel == "reduction":
        n = d["n"]
        lo, hi = shard(n)
        x_np = workloads.make_inputs("reduction", d=d, seed=ctx.args.seed, part=(lo, hi))["x"]
        x_h = pinned(x_np)
        x_d = x_h.to(dev)
        x_e = torch.empty_like(x_d) if e2e else x_d
        out64 = torch.zeros(1, dtype=torch.float64, device=dev)
        out_h = torch.zeros(1, dtype=torch.float64).pin_memory()
        ws_bytes = lib.reduce_workspace_bytes(hi - lo)
        ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        if c.variant == "nccl":
            def launch(src):
                lib.reduce_sum_f32(src.data_ptr(), hi - lo, out64.data_ptr(), None, ws.data_ptr(), ws_bytes, sh)

            collective = lambda: sharding.combine_partials(out64)  # noqa: E731
        else:
            xsum = sharding.XrankSum(lib, hi - lo, dev)

            def launch(src):
                xsum(src.data_ptr(), hi - lo, out64.data_ptr(), sh)

            collective = None

        def parity():
            import torch.distributed as dist
            part = ref.reduce_sum_ref(x_np)
            parts = [part]
            if ctx.world > 1:
                parts = [None] * ctx.world
                dist.all_gather_object(parts, part)
            want = math.fsum(parts)
            got = float(out64.item())
            rel = abs(got - want) / abs(want)
            return {"gpu_sum": got, "oracle_sum": want, "rel_err": rel, "tol": 1e-4, "ok": rel <= 1e-4,
                    "checked": "whole sum (oracle: fp64 sum of every rank's shard)"}

        return Job(c, d, launch, x_d, x_e, lambda: x_e.copy_(x_h, non_blocking=True),
                   lambda: out_h.copy_(out64, non_blocking=True), n * 4, (hi - lo) * 4, "GB/s", "f32", "hbm",
                   x_h.numel() * 4, 8, x_d.numel() * 4, parity, collective=collective,
                   tensors=[x_h, x_d, x_e, out64, out_h, ws])

    if c.kernel in ("softmax", "layernorm"):
        R, C = d["rows"], d["cols"]
        lo, hi = shard(R)
        inp = workloads.make_inputs(c.kernel, d=d, seed=ctx.args.seed, part=(lo, hi))
        x_h = pinned(inp["x"])
        x_d = x_h.to(dev)
        x_e = torch.empty_like(x_d) if e2e else x_d
        y_d = torch.empty_like(x_d)
        y_h = torch.empty(x_d.shape, dtype=torch.float32).pin_memory()
        extra_h, extra_d = [], []
        if c.kernel == "layernorm":
            g_h, b_h = pinned(inp["gamma"]), pinned(inp["beta"])
            g_d, b_d = g_h.to(dev), b_h.to(dev)
            extra_h, extra_d = [g_h, b_h], [g_d, b_d]
        eps = float(inp.get("eps", 1e-5))

        def launch(src):
            if c.kernel == "softmax":
                lib.softmax_f32(src.data_ptr(), y_d.data_ptr(), hi - lo, C, sh)
            else:
                lib.layernorm_f32(src.data_ptr(), extra_d[0].data_ptr(), extra_d[1].data_ptr(), y_d.data_ptr(),
                                  hi - lo, C, eps, sh)

        def e2e_in():
            x_e.copy_(x_h, non_blocking=True)
            for hh, dd in zip(extra_h, extra_d):
                dd.copy_(hh, non_blocking=True)

        def parity():
            rows = min(256, hi - lo)
            idx = np.unique(np.linspace(0, hi - lo - 1, rows).astype(np.int64)) if hi > lo else np.zeros(0, np.int64)
            xs = inp["x"][idx]
            want = ref.softmax_ref(xs) if c.kernel == "softmax" else ref.layernorm_ref(xs, inp["gamma"], inp["beta"], eps)
            got = y_d[torch.from_numpy(idx).to(dev)].cpu().numpy()
            err = ref.normwise_rel_err(got, want)
            return {"normwise_rel_err": err, "tol": 1e-5, "ok": bool(err <= 1e-5),
                    "checked": f"{len(idx)} rows spread over every rank's shard"}

        extra_bytes = sum(t.numel() * 4 for t in extra_h)
        return Job(c, d, launch, x_d, x_e, e2e_in, lambda: y_h.copy_(y_d, non_blocking=True),
                   workloads.work(c.kernel, d).bytes, workloads.work(c.kernel, {"rows": hi - lo, "cols": C}).bytes,
                   "GB/s", "f32", "hbm", x_h.numel() * 4 + extra_bytes, y_h.numel() * 4, 2 * x_d.numel() * 4, parity,
                   tensors=[x_h, x_d, x_e, y_d, y_h, *extra_h, *extra_d])

    if c.kernel == "matmul":
        M, N, K = d["M"], d["N"], d["K"]
        lo, hi = shard(M)
        inp = workloads.make_inputs("matmul", d=d, seed=ctx.args.seed, part=(lo, hi))
        B_np = np.ascontiguousarray(inp["B"].T) if c.tb else inp["B"]
        A_h, B_h = pinned(inp["A"]), pinned(B_np)
        A_d, B_d = A_h.to(dev), B_h.to(dev)
        A_e = torch.empty_like(A_d) if e2e else A_d
        C_d = torch.empty((hi - lo, N), dtype=torch.float32, device=dev)
        C_h = torch.empty((hi - lo, N), dtype=torch.float32).pin_memory()
        variant = kt_lib.KT_GEMM_TF32 if c.variant == "tf32" else kt_lib.KT_GEMM_FFMA

        def launch(src):
            lib.gemm_f32(src.data_ptr(), B_d.data_ptr(), C_d.data_ptr(), hi - lo, N, K, c.tb, variant, sh)

        def e2e_in():
            A_e.copy_(A_h, non_blocking=True)
            B_d.copy_(B_h, non_blocking=True)

        def parity():
            rows = min(64, hi - lo)
            idx = np.unique(np.linspace(0, hi - lo - 1, rows).astype(np.int64))
            want = ref.matmul_ref(inp["A"][idx], B_np, transpose_b=c.tb)
            got = C_d[torch.from_numpy(idx).to(dev)].cpu().numpy()
            err = ref.normwise_rel_err(got, want)
            tol = 1e-3 if c.variant == "tf32" else 1e-5
            return {"normwise_rel_err": err, "tol": tol, "ok": bool(err <= tol),
                    "checked": f"{len(idx)} rows of C spread over every rank's row block"}

        return Job(c, d, launch, A_d, A_e, e2e_in, lambda: C_h.copy_(C_d, non_blocking=True),
                   2 * M * N * K, 2 * (hi - lo) * N * K, "TFLOP/s", c.variant, "fp32" if c.variant == "ffma" else "tensor",
                   (A_h.numel() + B_h.numel()) * 4, C_h.numel() * 4, (A_d.numel() + B_d.numel() + C_d.numel()) * 4,
                   parity, tensors=[A_h, B_h, A_d, B_d, A_e, C_d, C_h])

    Bb, H, S, D = d["B"], d["H"], d["S"], d["D"]
    lo, hi = shard(Bb * H)
    inp = workloads.make_inputs("attention", d=d, seed=ctx.args.seed, part=(lo, hi))
    q_h, k_h, v_h = (pinned(inp[nm].view(np.int16)) for nm in ("q", "k", "v"))
    q_d, k_d, v_d = (t.to(dev) for t in (q_h, k_h, v_h))
    q_e = torch.empty_like(q_d) if e2e else q_d
    o_d = torch.empty_like(q_d)
    o_h = torch.empty(q_d.shape, dtype=torch.int16).pin_memory()
    scale = float(inp["scale"])

    def launch(src):
        lib.fa_fwd_bf16(src.data_ptr(), k_d.data_ptr(), v_d.data_ptr(), o_d.data_ptr(), 1, hi - lo, S, D, scale,
                        c.causal, sh)

    def e2e_in():
        q_e.copy_(q_h, non_blocking=True)
        k_d.copy_(k_h, non_blocking=True)
        v_d.copy_(v_h, non_blocking=True)

    def parity():
        # one head in fp64 (rows of the score matrix sampled) per rank: the first and last head of its shard
        errs = []
        heads = sorted({0, hi - lo - 1}) if hi > lo else []
        for h in heads:
            q = workloads.bf16_to_f32(inp["q"][h])
            k = workloads.bf16_to_f32(inp["k"][h])
            v = workloads.bf16_to_f32(inp["v"][h])
            rows = np.unique(np.linspace(0, S - 1, 512).astype(np.int64))
            want = ref.attention_rows_ref(q, k, v, rows, scale, c.causal)
            got = workloads.bf16_to_f32(o_d[h].cpu().numpy().view(np.uint16))[rows]
            errs.append(ref.normwise_rel_err(got, want))
        err = max(errs) if errs else 0.0
        return {"normwise_rel_err": err, "tol": 2e-2, "ok": bool(err <= 2e-2),
                "checked": f"{len(heads)} heads per rank (first and last of its shard), 512 query rows each"}

    return Job(c, d, launch, q_d, q_e, e2e_in, lambda: o_h.copy_(o_d, non_blocking=True),
               workloads.work("attention", d, causal=c.causal).flops,
               workloads.work("attention", {"B": 1, "H": hi - lo, "S": S, "D": D}, causal=c.causal).flops,
               "TFLOP/s", "bf16", "tensor", 3 * q_h.numel() * 2, o_h.numel() * 2, 4 * q_d.numel() * 2, parity,
               tensors=[q_h, k_h, v_h, q_d, k_d, v_d, q_e, o_d, o_h])


def cpu_baseline_for(cpu, c: Case, args) -> dict:
    """The oracle port timed on a bounded sample on the host cores (N=1, rank 0)."""
    return cpu.measure(c, 3, 1, 6.0)


def main() -> None:
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import kt_lib
    from roofline import PEAKS

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    lib = kt_lib.load()
    stream = torch.cuda.current_stream()
    ctx = Ctx(args, rank, world, local, dev, lib, stream)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush_buf = torch.empty(int(2 * l2) // 4 + 1024, dtype=torch.float32, device=dev)
    flush_sink = torch.empty(1, dtype=torch.float32, device=dev)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = int(vis.split(",")[local]) if vis and vis.split(",")[local].strip().isdigit() else local
    sampler = ClockSampler(phys) if rank == 0 else None
    if sampler:
        sampler.start()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuRef(args.seed)

    def run(c: Case) -> dict:
        job = setup_job(ctx, c)
        flush_needed = job.dev_bytes < 4 * l2

        def flush():
            if flush_needed:
                torch.sum(flush_buf, dim=0, keepdim=True, out=flush_sink)

        def timed(step_fn, steps: int, inner: bool = True):
            ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(4)) for _ in range(steps)]
            barrier()
            torch.cuda.synchronize()
            for i in range(steps):
                flush()
                step_fn(ev[i])
            torch.cuda.synchronize()
            barrier()
            step = [a.elapsed_time(b) for a, b, _, _ in ev]
            if job.collective is None or not inner:
                return step, list(step)
            return step, [x.elapsed_time(y) for _, _, x, y in ev]

        # A step is bracketed by events e0..e1. With an exchange after the
        # kernel, a second pair e2..e3 brackets the kernel alone; without one
        # the kernel is the whole step and its time is e0..e1 (no extra event
        # records inside the step).
        def dev_step(e):
            e[0].record(stream)
            if job.collective is not None:
                e[2].record(stream)
                job.launch(job.dev_src)
                e[3].record(stream)
                job.collective()
            else:
                job.launch(job.dev_src)
            e[1].record(stream)

        def e2e_step(e):
            e[0].record(stream)
            job.e2e_in()
            job.launch(job.e2e_src)
            if job.collective is not None:
                job.collective()
            job.e2e_out()
            e[1].record(stream)

        warm_ms, _ = timed(dev_step, max(args.warmup, 3))
        # soak: untimed steps under the clock sampler so that the clock record
        # covers the steady state; the count is agreed across ranks (every
        # rank issues the same collectives)
        per_step = max_over_ranks(max(statistics.median(warm_ms), 1e-3))
        n_soak = int(max_over_ranks(float(int(min(max(args.soak_s, 0.0) * 1e3 / per_step, 200000)))))
        t_win0 = time.monotonic()
        dummy = tuple(torch.cuda.Event(enable_timing=True) for _ in range(4))
        for i in range(n_soak):
            flush()
            dev_step(dummy)
            if i % 64 == 63:
                torch.cuda.synchronize()
        step_ms, kern_ms = timed(dev_step, args.steps)
        t_win1 = time.monotonic()
        total_ms = max_over_ranks(sum(step_ms))
        kern_avg_ms = max_over_ranks(sum(kern_ms) / len(kern_ms))
        scale_u = 1e9 if job.unit == "GB/s" else 1e12
        value = job.units_job * args.steps / (total_ms * 1e-3) / scale_u

        e2e = None
        if not args.no_e2e:
            for _ in range(max(3, min(args.warmup, 5))):
                e2e_step(dummy)
            torch.cuda.synchronize()
            e_steps = max(3, min(args.steps, 50))
            e_ms, _ = timed(e2e_step, e_steps, inner=False)
            e_total = max_over_ranks(sum(e_ms))
            e2e = {"value": job.units_job * e_steps / (e_total * 1e-3) / scale_u, "unit": job.unit,
                   "h2d_bytes_per_step": int(sum_over_ranks(job.h2d)),
                   "d2h_bytes_per_step": int(sum_over_ranks(job.d2h)),
                   "ms_per_step": e_total / e_steps, "steps": e_steps}

        parity = None
        if not args.no_parity:
            torch.cuda.synchronize()
            p = job.parity()
            if world > 1:
                allp = [None] * world
                dist.all_gather_object(allp, p)
                if c.kernel == "reduction":
                    p = allp[0]
                else:
                    worst = max(allp, key=lambda q: q.get("normwise_rel_err", 0.0))
                    p = dict(worst, ok=all(q["ok"] for q in allp), ranks_checked=world)
            parity = p

        clocks = sampler.summary(t_win0, t_win1) if sampler else None
        capped = bool(clocks and "sw_power_cap" in clocks.get("reasons", []))
        achieved_units = job.units_launch / (kern_avg_ms * 1e-3)
        if job.bound == "hbm":
            achieved = achieved_units / 1e9
            peak = PEAKS["hbm_gbs"]
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "peak_source": f"{PEAKS['source']['hbm_gbs']} copy bandwidth (MEASURED_PEAKS hbm_gbs)",
                    "algo_bytes_per_launch": job.units_launch}
        else:
            achieved = achieved_units / 1e12
            if job.bound == "fp32":
                peak = burst = PEAKS["fp32_tflops"]
                src = "nominal FP32 SIMT (148 SM x 128 FMA x 2 x 1.965 GHz; no measured figure exists)"
                if clocks and clocks.get("sm_mhz"):
                    roofline_at_clock = peak * clocks["sm_mhz"] / 1965.0
                else:
                    roofline_at_clock = None
            else:
                div = 2.0 if c.kernel == "matmul" else 1.0
                burst = PEAKS["bf16_tflops"] / div
                sust = PEAKS.get("bf16_tflops_sustained", PEAKS["bf16_tflops"]) / div
                peak = sust if capped else burst
                what = "measured bf16 cuBLAS" + (" / 2 (dense TF32 rate)" if div == 2.0 else "")
                src = f"{what}, {'sustained (power cap active)' if capped else 'burst'}"
                roofline_at_clock = None
            roof = {"bound": "tensor" if job.bound == "tensor" else "fp32", "achieved": achieved, "peak": peak,
                    "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": src, "peak_burst": burst,
                    "frac_of_burst": achieved / burst, "algo_flops_per_launch": job.units_launch}
            if roofline_at_clock:
                roof["peak_at_sampled_clock"] = roofline_at_clock
                roof["frac_at_sampled_clock"] = achieved / roofline_at_clock
        roof["kernel_ms"] = kern_avg_ms
        tr = profiled_traffic(KERNEL_ID[c.name], job.units_launch)
        roof["traffic"] = tr["bytes"] if tr else None
        if tr:
            roof["traffic_source"] = tr["source"] + (f" ({tr['scaled']})" if tr["scaled"] else "")
        roof["kernel_id"] = KERNEL_ID[c.name]

        cpu_b = cpu_baseline_for(cpu, c, args) if cpu is not None else None
        res = {
            "value": value, "unit": job.unit, "ms_per_step": total_ms / args.steps, "kernel_ms": kern_avg_ms,
            "dtype": job.dtype, "steps": args.steps,
            "config": {"workload": workload_name(c) + (f" scaled x{args.scale}" if args.scale < 1 else ""), **job.dims,
                       "l2": (f"flushed before every step (read of {2 * l2 >> 20} MiB)" if flush_needed
                              else f"inputs ({job.dev_bytes >> 20} MiB per GPU) larger than L2, no flush"),
                       "parallelism": f"shards x{world}"},
            "roofline": roof, "cpu_baseline": cpu_b, "e2e": e2e, "parity": parity,
            "gpu_launches": job.launches_per_step * args.steps, "clocks": clocks,
        }
        job.tensors.clear()
        del job
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        return res

    head = headline_case(args)
    h = run(head)
    families = {}
    for c in family_cases(args, head):
        families[c.name] = run(c)
    if sampler:
        sampler.stop()

    if rank == 0:
        out = {
            "metric": METRIC, "value": h["value"], "unit": h["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": h["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": h["dtype"], "data": "synthetic",
            "config": dict(h["config"], seed=args.seed, case=head.name,
                           clock_note=f"clocks sampled over a {args.soak_s:.1f} s soak of the same step and the timed steps"),
            "roofline": h["roofline"], "cpu_baseline": h["cpu_baseline"], "e2e": h["e2e"],
            "gpu_launches": h["gpu_launches"], "clocks": h["clocks"], "parity": h["parity"],
            "families": families,
            "library": str(lib.path.relative_to(REPO)) if lib.path.is_relative_to(REPO) else str(lib.path),
        }
        emit(out)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
