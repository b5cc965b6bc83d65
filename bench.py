#!/usr/bin/env python
"""
bench.py — throughput of the tuned kernel library on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--kernel reduction]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's CPU (NumPy) path

One step is one pass of a kernel family over its full synthetic batch. The
default workload is the sum reduction: 2^28 fp32 values ~ U[-1,1], sharded
contiguously across the ranks (total size fixed: strong scaling); each rank
reduces its shard to an fp64 partial with the library's kernel and the
partials are combined with one NCCL all-reduce. Other families
(--kernel softmax|layernorm|matmul|attention) shard rows / row-blocks of A /
batch×head pairs and need no collective.

Printed by rank 0: one JSON line with the metric, whole-job `value`
(device-resident inputs), `e2e` (pinned host inputs copied in and the result
copied out every step, through the C ABI), the roofline of the dominant
kernel, the CPU baseline (N=1), clocks sampled around the timed steps, and
the number of library kernels launched in the timed region.
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
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "cd-cuda-course-project_b200"
sys.path.insert(0, str(PKG / "src"))

METRIC = ("achieved HBM GB/s (softmax/reduce/LN) & TFLOP/s (matmul/attn) vs roofline, 1–8 B200")


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--kernel", choices=["reduction", "softmax", "layernorm", "matmul", "attention"],
                   default="reduction")
    p.add_argument("--variant", choices=["tf32", "ffma"], default="tf32", help="matmul variant")
    p.add_argument("--transpose-b", action="store_true", help="matmul: B holds Bt (N×K)")
    p.add_argument("--causal", action="store_true", help="attention: causal mask")
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--soak-s", type=float, default=2.0,
                   help="seconds of untimed steps run under the clock sampler before the timed steps")
    p.add_argument("--scale", type=float, default=1.0,
                   help="shrink the leading dim of the workload (small cases for profiler captures)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def emit(obj: dict) -> None:
    print(json.dumps(obj), flush=True)


# ---------------------------------------------------------------------------
# Clock sampler (nvidia-smi, read-only queries)
# ---------------------------------------------------------------------------

SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, period_ms: int = 100):
        self.period_ms = period_ms
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 f"-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        rows = []
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append({"idx": int(parts[0]), "sm": float(parts[1]), "max": float(parts[2]),
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
# Reference arm: the reference's CPU (NumPy) path on the host cores
# ---------------------------------------------------------------------------

def run_reference(args: argparse.Namespace, rank: int, world: int) -> None:
    if rank != 0:
        return
    import numpy as np
    import workloads
    from oracle import cpu_baseline as cb

    threads = cb.host_threads()
    k = args.kernel
    d = workloads.dims(k, "config")
    if k == "reduction":
        x = workloads.make_inputs(k, d=d, seed=args.seed)["x"]
        for _ in range(args.warmup):
            cb.reduce_sum(x, threads, reps=1)
        t = [cb.reduce_sum(x, threads, reps=1)["best_s"] for _ in range(args.steps)]
        value, unit, sample = x.nbytes * len(t) / sum(t) / 1e9, "GB/s", f"full array n=2^28 per step"
        dtype = "f32"
    elif k in ("softmax", "layernorm"):
        inp = workloads.make_inputs(k, d=d, seed=args.seed)
        fn = (lambda: cb.rows_op(k, inp["x"], threads, 1)) if k == "softmax" else \
             (lambda: cb.rows_op(k, inp["x"], threads, 1, inp["gamma"], inp["beta"], inp["eps"]))
        for _ in range(args.warmup):
            fn()
        t = [fn()["best_s"] for _ in range(args.steps)]
        nb = workloads.work(k, d).bytes
        value, unit, sample, dtype = nb * len(t) / sum(t) / 1e9, "GB/s", "full batch per step", "f32"
    elif k == "matmul":
        n = 2048  # bounded sample: a 2048-row block of A against the full B
        inp = workloads.make_inputs(k, d=d, seed=args.seed)
        A = inp["A"][:n]
        t = []
        for i in range(args.warmup + args.steps):
            r = cb.matmul(A, inp["B"], reps=1)
            if i >= args.warmup:
                t.append(r["best_s"])
        value = 2 * n * d["N"] * d["K"] * len(t) / sum(t) / 1e12
        unit, sample, dtype = "TFLOP/s", f"{n}x8192 row block of A per step (BLAS fp32)", "f32"
    else:
        nh = 2  # bounded sample: 2 (b,h) heads per step
        S, D = d["S"], d["D"]
        rng = np.random.default_rng(args.seed)
        q, kk, v = (workloads.bf16_to_f32(workloads.bf16_bits(rng.standard_normal((nh, S, D), dtype=np.float32)))
                    for _ in range(3))
        t = []
        for i in range(args.warmup + args.steps):
            r = cb.attention_heads(q, kk, v, 1.0 / math.sqrt(D), args.causal, threads)
            if i >= args.warmup:
                t.append(r["best_s"])
        value = r["flops"] * len(t) / sum(t) / 1e12
        unit, sample, dtype = "TFLOP/s", f"{nh} heads of S=4096 D=128 per step (fp32 NumPy)", "bf16"
    emit({
        "metric": METRIC, "impl": "reference", "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(t) / len(t),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic", "config": {"workload": _workload_name(args), **d},
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def _workload_name(args: argparse.Namespace) -> str:
    return {
        "reduction": "sum reduction fp32 N=2^28 U[-1,1] -> fp64 sum, contiguous shards + NCCL all-reduce",
        "softmax": "row softmax fp32 4096x4096 N(0,1), rows sharded",
        "layernorm": "layernorm fp32 16384x4096 N(0,1), gamma=1+0.1N, beta=0.1N, eps=1e-5, rows sharded",
        "matmul": f"matmul fp32 8192^3 U[-1,1] {args.variant}{' transpose_b' if args.transpose_b else ''}, "
                  "row-blocks of A sharded",
        "attention": f"flash-attention fwd bf16 B=8 H=32 S=4096 D=128 N(0,1) "
                     f"{'causal' if args.causal else 'non-causal'}, batch*head sharded",
    }[args.kernel]


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def main() -> None:
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    import kt_lib
    import sharding
    import workloads
    from roofline import RooflineAnalyzer, PEAKS

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    lib = kt_lib.load()
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    k = args.kernel
    d_full = scaled_dims(k, args.scale)
    inp = workloads.make_inputs(k, d=d_full, seed=args.seed)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    ra = RooflineAnalyzer()

    def shard(n: int) -> tuple[int, int]:
        return sharding.shard_range(n, world, rank)

    def pinned(a: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()

    # --- per-family set-up: device tensors, a device-resident step, an e2e step
    launches_per_step = 1
    algo_bytes_launch = algo_flops_launch = 0
    if k == "reduction":
        n = d_full["n"]
        lo, hi = shard(n)
        xs = inp["x"][lo:hi]
        x_h = pinned(xs)
        x_d = x_h.to(dev)
        x_e = torch.empty_like(x_d) if not args.no_e2e else x_d
        out64 = torch.zeros(1, dtype=torch.float64, device=dev)
        out_h = torch.zeros(1, dtype=torch.float64).pin_memory()
        ws_bytes = lib.reduce_workspace_bytes(hi - lo)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        units_job = n * 4
        algo_bytes_launch = (hi - lo) * 4
        h2d, d2h = x_h.numel() * 4, 8
        unit, dtype = "GB/s", "f32"

        def kernel(src):
            lib.reduce_sum_f32(src.data_ptr(), hi - lo, out64.data_ptr(), None, ws.data_ptr(), ws_bytes, sh)

        def collective():
            sharding.combine_partials(out64)

        def e2e_in():
            x_e.copy_(x_h, non_blocking=True)

        def e2e_out():
            out_h.copy_(out64, non_blocking=True)

        dev_in = x_d
        e2e_src = x_e
        input_bytes_dev = x_d.numel() * 4
    elif k in ("softmax", "layernorm"):
        R, C = d_full["rows"], d_full["cols"]
        lo, hi = shard(R)
        x_h = pinned(inp["x"][lo:hi])
        x_d = x_h.to(dev)
        x_e = torch.empty_like(x_d) if not args.no_e2e else x_d
        y_d = torch.empty_like(x_d)
        y_h = torch.empty(x_d.shape, dtype=torch.float32).pin_memory()
        if k == "layernorm":
            g_d = torch.from_numpy(inp["gamma"]).to(dev)
            b_d = torch.from_numpy(inp["beta"]).to(dev)
        units_job = workloads.work(k, d_full).bytes
        algo_bytes_launch = workloads.work(k, {"rows": hi - lo, "cols": C}).bytes
        h2d, d2h = x_h.numel() * 4, x_h.numel() * 4
        unit, dtype = "GB/s", "f32"

        def kernel(src):
            if k == "softmax":
                lib.softmax_f32(src.data_ptr(), y_d.data_ptr(), hi - lo, C, sh)
            else:
                lib.layernorm_f32(src.data_ptr(), g_d.data_ptr(), b_d.data_ptr(), y_d.data_ptr(), hi - lo, C,
                                  float(inp["eps"]), sh)

        def collective():
            pass

        def e2e_in():
            x_e.copy_(x_h, non_blocking=True)

        def e2e_out():
            y_h.copy_(y_d, non_blocking=True)

        dev_in = x_d
        e2e_src = x_e
        input_bytes_dev = 2 * x_d.numel() * 4
    elif k == "matmul":
        M, N, K = d_full["M"], d_full["N"], d_full["K"]
        lo, hi = shard(M)
        Bnp = np.ascontiguousarray(inp["B"].T) if args.transpose_b else inp["B"]
        A_h = pinned(inp["A"][lo:hi])
        B_h = pinned(Bnp)
        A_d, B_d = A_h.to(dev), B_h.to(dev)
        A_e = torch.empty_like(A_d) if not args.no_e2e else A_d
        C_d = torch.empty((hi - lo, N), dtype=torch.float32, device=dev)
        C_h = torch.empty((hi - lo, N), dtype=torch.float32).pin_memory()
        variant = kt_lib.KT_GEMM_TF32 if args.variant == "tf32" else kt_lib.KT_GEMM_FFMA
        units_job = 2 * M * N * K
        algo_flops_launch = 2 * (hi - lo) * N * K
        h2d, d2h = A_h.numel() * 4, C_h.numel() * 4
        unit, dtype = "TFLOP/s", args.variant

        def kernel(src):
            lib.gemm_f32(src.data_ptr(), B_d.data_ptr(), C_d.data_ptr(), hi - lo, N, K, args.transpose_b, variant, sh)

        def collective():
            pass

        def e2e_in():
            A_e.copy_(A_h, non_blocking=True)

        def e2e_out():
            C_h.copy_(C_d, non_blocking=True)

        dev_in = A_d
        e2e_src = A_e
        input_bytes_dev = (A_d.numel() + B_d.numel() + C_d.numel()) * 4
    else:
        Bb, H, S, D = d_full["B"], d_full["H"], d_full["S"], d_full["D"]
        lo, hi = shard(Bb * H)
        def heads(a):
            return np.ascontiguousarray(a.reshape(Bb * H, S, D)[lo:hi])
        q_h, k_h, v_h = (pinned(heads(inp[nm]).view(np.int16)) for nm in ("q", "k", "v"))
        q_d, k_d, v_d = (t.to(dev) for t in (q_h, k_h, v_h))
        q_e = torch.empty_like(q_d) if not args.no_e2e else q_d
        o_d = torch.empty_like(q_d)
        o_h = torch.empty(q_d.shape, dtype=torch.int16).pin_memory()
        units_job = workloads.work(k, d_full, causal=args.causal).flops
        algo_flops_launch = workloads.work(k, {"B": 1, "H": hi - lo, "S": S, "D": D}, causal=args.causal).flops
        h2d, d2h = 3 * q_h.numel() * 2, o_h.numel() * 2
        unit, dtype = "TFLOP/s", "bf16"

        def kernel(src):
            lib.fa_fwd_bf16(src.data_ptr(), k_d.data_ptr(), v_d.data_ptr(), o_d.data_ptr(), 1, hi - lo, S, D,
                            float(inp["scale"]), args.causal, sh)

        def collective():
            pass

        def e2e_in():
            q_e.copy_(q_h, non_blocking=True)
            k_d.copy_(k_h, non_blocking=True)
            v_d.copy_(v_h, non_blocking=True)

        def e2e_out():
            o_h.copy_(o_d, non_blocking=True)

        dev_in = q_d
        e2e_src = q_e
        input_bytes_dev = 4 * q_d.numel() * 2

    flush_needed = input_bytes_dev < 4 * l2
    flush_buf = torch.empty(int(2 * l2) // 4 + 1024, dtype=torch.float32, device=dev) if flush_needed else None
    flush_sink = torch.empty(1, dtype=torch.float32, device=dev)

    def flush():
        if flush_buf is not None:
            torch.sum(flush_buf, dim=0, keepdim=True, out=flush_sink)

    # --- device-resident timed loop --------------------------------------
    def timed(step_fn, steps: int):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
               torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            flush()
            step_fn(ev[i])
        torch.cuda.synchronize()
        barrier()
        step_ms = [a.elapsed_time(b) for a, b, _, _ in ev]
        kern_ms = [c.elapsed_time(e) for _, _, c, e in ev]
        return step_ms, kern_ms

    def dev_step(e):
        e[0].record(stream)
        e[2].record(stream)
        kernel(dev_in)
        e[3].record(stream)
        collective()
        e[1].record(stream)

    def e2e_step(e):
        e[0].record(stream)
        e2e_in()
        e[2].record(stream)
        kernel(e2e_src)
        e[3].record(stream)
        collective()
        e2e_out()
        e[1].record(stream)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    warm_ms, _ = timed(dev_step, max(args.warmup, 3))
    # soak: untimed steps under the clock sampler, so that the clock record
    # covers the steady state of the timed steps. The count is agreed across
    # ranks (every rank must issue the same collectives).
    per_step = max_over_ranks(max(statistics.median(warm_ms), 1e-3))
    n_soak = int(min(max(args.soak_s, 0.0) * 1e3 / per_step, 200000))
    n_soak = int(max_over_ranks(float(n_soak)))
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for i in range(n_soak):
        flush()
        dev_step((torch.cuda.Event(enable_timing=True),) * 4)
        if i % 64 == 63:
            torch.cuda.synchronize()
    step_ms, kern_ms = timed(dev_step, args.steps)
    clocks = sampler.stop() if sampler else None

    total_ms = max_over_ranks(sum(step_ms))
    kern_avg_ms = max_over_ranks(sum(kern_ms) / len(kern_ms))
    value = units_job * args.steps / (total_ms * 1e-3) / (1e9 if unit == "GB/s" else 1e12)

    e2e = None
    if not args.no_e2e:
        for _ in range(max(3, min(args.warmup, 5))):
            e2e_step((torch.cuda.Event(enable_timing=True),) * 4)
        torch.cuda.synchronize()
        e2e_steps = max(3, min(args.steps, 50))
        e_ms, _ = timed(e2e_step, e2e_steps)
        e_total = max_over_ranks(sum(e_ms))
        e2e = {"value": units_job * e2e_steps / (e_total * 1e-3) / (1e9 if unit == "GB/s" else 1e12),
               "unit": unit, "h2d_bytes_per_step": int(h2d) * world, "d2h_bytes_per_step": int(d2h) * world,
               "ms_per_step": e_total / e2e_steps, "steps": e2e_steps}

    # roofline of the dominant kernel (per launch, this rank's share). Tensor
    # kernels are compared with the measured sustained cuBLAS figure when the
    # clock record shows the power cap engaged during the timed steps (the
    # regime actually measured), else with the burst figure; both are reported.
    power_capped = bool(clocks and "sw_power_cap" in clocks.get("reasons", []))
    if unit == "GB/s":
        achieved = algo_bytes_launch / (kern_avg_ms * 1e-3) / 1e9
        peak = PEAKS["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": PEAKS["source"]["hbm_gbs"] + " copy bandwidth (MEASURED_PEAKS hbm_gbs)",
                "algo_bytes_per_launch": algo_bytes_launch, "kernel_ms": kern_avg_ms}
    else:
        achieved = algo_flops_launch / (kern_avg_ms * 1e-3) / 1e12
        bf16_burst = PEAKS["bf16_tflops"]
        bf16_sust = PEAKS.get("bf16_tflops_sustained", bf16_burst)
        if k == "matmul" and args.variant == "ffma":
            peak, burst, src = PEAKS["fp32_tflops"], PEAKS["fp32_tflops"], "nominal FP32 SIMT (148 SM x 128 FMA x 2 x 1.965 GHz)"
        elif k == "matmul":
            burst = bf16_burst / 2.0
            peak = (bf16_sust / 2.0) if power_capped else burst
            src = ("measured bf16 sustained / 2 (power cap active)" if power_capped else "measured bf16 burst / 2")
        else:
            burst = bf16_burst
            peak = bf16_sust if power_capped else burst
            src = "measured bf16 sustained (power cap active)" if power_capped else "measured bf16 burst"
        roof = {"bound": "tensor" if not (k == "matmul" and args.variant == "ffma") else "fp32",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": src, "peak_burst": burst, "frac_of_burst": achieved / burst,
                "algo_flops_per_launch": algo_flops_launch, "kernel_ms": kern_avg_ms}
    roof["traffic"] = profiled_traffic(k)

    # parity of the result (device result vs the oracle's value from the CPU-baseline leg)
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, parity = cpu_baseline_leg(args, inp, k, locals())

    if rank == 0:
        emit({
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": _workload_name(args) + (f" scaled x{args.scale}" if args.scale < 1 else ""), **d_full,
                       "l2": (f"flushed before every step (read of {2 * l2 >> 20} MiB)" if flush_needed
                              else f"inputs ({input_bytes_dev >> 20} MiB per GPU) larger than L2, no flush"),
                       "parallelism": f"shards x{world}", "seed": args.seed,
                       "clock_note": f"clocks sampled over a {args.soak_s:.1f} s soak of the same step and the timed steps"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps, "clocks": clocks, "parity": parity,
            "library": str(lib.path.relative_to(REPO)) if lib.path.is_relative_to(REPO) else str(lib.path),
        })
    if world > 1:
        dist.destroy_process_group()


def scaled_dims(kernel: str, scale: float) -> dict:
    """The full configuration, with its leading dim multiplied by `scale` (<= 1)."""
    import workloads
    d = workloads.dims(kernel, "config")
    if scale >= 1.0:
        return d
    lead = {"reduction": "n", "softmax": "rows", "layernorm": "rows", "matmul": "M", "attention": "B"}[kernel]
    d[lead] = max(1, int(d[lead] * scale))
    return d


def profiled_traffic(kernel: str):
    """DRAM bytes per launch from the committed ncu summary of this family's
    kernel, if one records it (a `traffic_bytes_per_launch:` line)."""
    for p in sorted((REPO / "profiles").glob(f"{kernel}*.md")):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
        if m:
            return int(m.group(1))
    return None


def cpu_baseline_leg(args, inp, k, env):
    """Time the oracle (NumPy restatement of the reference's CPU path) on a
    bounded sample of this workload; also return the parity of the GPU result."""
    import numpy as np
    import torch
    from oracle import cpu_baseline as cb
    from oracle import ref

    threads = cb.host_threads()
    if k == "reduction":
        x = inp["x"]
        r = cb.reduce_sum(x, threads, reps=5)
        gpu = float(env["out64"].item())
        rel = abs(gpu - r["result"]) / abs(r["result"])
        cpu = {"value": x.nbytes / r["best_s"] / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": "full array n=2^28, best of 5 (NumPy fp64 sum, chunked over threads)"}
        return cpu, {"gpu_sum": gpu, "oracle_sum": r["result"], "rel_err": rel, "tol": 1e-4, "ok": rel <= 1e-4}
    if k in ("softmax", "layernorm"):
        rows = min(1024, inp["x"].shape[0])
        xs = inp["x"][:rows]
        if k == "softmax":
            r = cb.rows_op(k, xs, threads, 3)
            want = ref.softmax_ref(xs)
        else:
            r = cb.rows_op(k, xs, threads, 3, inp["gamma"], inp["beta"], inp["eps"])
            want = ref.layernorm_ref(xs, inp["gamma"], inp["beta"], inp["eps"])
        got = env["y_d"][:rows].cpu().numpy()
        err = ref.normwise_rel_err(got, want)
        cpu = {"value": r["bytes"] / r["best_s"] / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"first {rows} rows, best of 3"}
        return cpu, {"normwise_rel_err": err, "tol": 1e-5, "ok": err <= 1e-5, "rows_checked": rows}
    if k == "matmul":
        n = 256
        A = inp["A"][:n]
        r = cb.matmul(A, inp["B"], reps=2)
        want = ref.matmul_ref(A, inp["B"])
        got = env["C_d"][:n].cpu().numpy()
        err = ref.normwise_rel_err(got, want)
        tol = 1e-3 if args.variant == "tf32" else 1e-5
        cpu = {"value": r["flops"] / r["best_s"] / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{n}x8192 rows of A x full B, best of 2 (BLAS fp32)"}
        return cpu, {"normwise_rel_err": err, "tol": tol, "ok": err <= tol, "rows_checked": n}
    S, D = inp["S"], inp["D"]
    import workloads
    q = workloads.bf16_to_f32(inp["q"].reshape(-1, S, D)[:1])
    kk = workloads.bf16_to_f32(inp["k"].reshape(-1, S, D)[:1])
    v = workloads.bf16_to_f32(inp["v"].reshape(-1, S, D)[:1])
    r = cb.attention_heads(q, kk, v, float(inp["scale"]), args.causal, threads)
    want = ref.attention_ref(q, kk, v, float(inp["scale"]), args.causal)
    got = workloads.bf16_to_f32(env["o_d"][:1].cpu().numpy().view(np.uint16))
    err = ref.normwise_rel_err(got, want)
    cpu = {"value": r["flops"] / r["best_s"] / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
           "sample": "1 head S=4096 D=128 (fp32 NumPy), best of 1"}
    return cpu, {"normwise_rel_err": err, "tol": 2e-2, "ok": err <= 2e-2, "heads_checked": 1}


if __name__ == "__main__":
    main()
