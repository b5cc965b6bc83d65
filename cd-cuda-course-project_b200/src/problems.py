"""
problems.py — device-resident problem instances for one kernel family.

Replaces the per-variant `main()` set-up of the reference (cudaMalloc +
rand() fill + launch configuration, src/generator.py:218-281, and the fixed
inputs of the verify mains, src/verifier.py:60-209): a `Problem` owns the
device tensors (torch provides the memory), builds the `kt_args` block of
the C ABI for the family's op, reads the output back, and carries an L2
flush buffer for timing.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

import kt_lib
import workloads


@dataclass
class Problem:
    kernel: str
    dims: dict
    host: dict                 # numpy inputs
    dev: dict                  # torch device tensors
    causal: bool = False
    transpose_b: bool = False
    variant: int = kt_lib.KT_GEMM_TF32
    extra: dict = field(default_factory=dict)

    # ----------------------------------------------------------------------
    def args(self, naive: bool = False) -> kt_lib.KtArgs:
        d, t = self.dims, self.dev
        k = self.kernel
        if k == "softmax":
            return kt_lib.make_args(in0=t["x"].data_ptr(), out0=t["y"].data_ptr(), d0=d["rows"], d1=d["cols"])
        if k == "layernorm":
            return kt_lib.make_args(in0=t["x"].data_ptr(), in1=t["gamma"].data_ptr(), in2=t["beta"].data_ptr(),
                                    out0=t["y"].data_ptr(), d0=d["rows"], d1=d["cols"], f0=self.host["eps"])
        if k == "reduction":
            ws = t["ws_naive"] if naive else t["ws"]
            return kt_lib.make_args(in0=t["x"].data_ptr(), out0=t["out64"].data_ptr(), out1=t["out32"].data_ptr(),
                                    workspace=ws.data_ptr(), ws_bytes=ws.numel(), d0=d["n"])
        if k == "matmul":
            return kt_lib.make_args(in0=t["A"].data_ptr(), in1=t["B"].data_ptr(), out0=t["C"].data_ptr(),
                                    d0=d["M"], d1=d["N"], d2=d["K"], i0=int(self.transpose_b), i1=self.variant)
        if k == "attention":
            return kt_lib.make_args(in0=t["q"].data_ptr(), in1=t["k"].data_ptr(), in2=t["v"].data_ptr(),
                                    out0=t["o"].data_ptr(), d0=d["B"], d1=d["H"], d2=d["S"], d3=d["D"],
                                    f0=self.host["scale"], i0=int(self.causal))
        raise ValueError(k)

    def op(self, naive: bool = False) -> str:
        return ("naive_" if naive else "") + self.kernel

    def output(self) -> np.ndarray:
        """Copy the result back (fp64 scalar for the reduction, fp32 arrays otherwise)."""
        import torch
        torch.cuda.synchronize()
        t = self.dev
        if self.kernel == "reduction":
            return np.array([t["out64"].item()])
        if self.kernel in ("softmax", "layernorm"):
            return t["y"].cpu().numpy()
        if self.kernel == "matmul":
            return t["C"].cpu().numpy()
        o = t["o"].cpu().numpy().view(np.uint16)
        return workloads.bf16_to_f32(o)

    def run(self, lib: kt_lib.KtLibrary, naive: bool = False, stream: Optional[int] = None) -> None:
        lib.run(self.op(naive), self.args(naive), stream)

    def time(self, lib: kt_lib.KtLibrary, warmup: int, iters: int, naive: bool = False,
             flush: bool = True) -> list[float]:
        fb = self.extra.get("flush")
        if flush and fb is not None:
            return lib.time(self.op(naive), self.args(naive), warmup, iters, fb.data_ptr(), fb.numel() * 4)
        return lib.time(self.op(naive), self.args(naive), warmup, iters)

    @property
    def work(self) -> workloads.Work:
        var = "ffma" if (self.kernel == "matmul" and self.variant == kt_lib.KT_GEMM_FFMA) else ""
        return workloads.work(self.kernel, self.dims, causal=self.causal, variant=var)


def make_problem(kernel: str, size: str = "config", seed: int = workloads.DEFAULT_SEED,
                 dims: Optional[dict] = None, host: Optional[dict] = None, device=None,
                 causal: bool = False, transpose_b: bool = False, variant: int = kt_lib.KT_GEMM_TF32,
                 lib: Optional[kt_lib.KtLibrary] = None, flush: bool = True) -> Problem:
    """Allocate a problem on `device` (default: current CUDA device) from seeded inputs."""
    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    h = host if host is not None else workloads.make_inputs(kernel, size, seed, d=dims)
    d = {key: h[key] for key in workloads.SIZES[kernel]["config"]}
    t: dict = {}

    def up(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    if kernel in ("softmax", "layernorm"):
        t["x"] = up(h["x"])
        t["y"] = torch.empty_like(t["x"])
        if kernel == "layernorm":
            t["gamma"] = up(h["gamma"])
            t["beta"] = up(h["beta"])
    elif kernel == "reduction":
        lib = lib or kt_lib.load()
        t["x"] = up(h["x"])
        t["out64"] = torch.zeros(1, dtype=torch.float64, device=dev)
        t["out32"] = torch.zeros(1, dtype=torch.float32, device=dev)
        t["ws"] = torch.empty(max(16, lib.reduce_workspace_bytes(d["n"])), dtype=torch.uint8, device=dev)
        t["ws_naive"] = torch.empty(max(16, 4 * ((d["n"] + 255) // 256)), dtype=torch.uint8, device=dev)
    elif kernel == "matmul":
        t["A"] = up(h["A"])
        t["B"] = up(np.ascontiguousarray(h["B"].T) if transpose_b else h["B"])
        t["C"] = torch.empty((d["M"], d["N"]), dtype=torch.float32, device=dev)
    elif kernel == "attention":
        for nm in ("q", "k", "v"):
            t[nm] = up(np.asarray(h[nm], dtype=np.uint16).view(np.int16))
        t["o"] = torch.empty_like(t["q"])
    else:
        raise ValueError(kernel)
    p = Problem(kernel, d, h, t, causal=causal, transpose_b=transpose_b, variant=variant)
    if flush:
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        p.extra["flush"] = torch.empty(int(2 * l2) // 4 + 256, dtype=torch.float32, device=dev)
    return p
