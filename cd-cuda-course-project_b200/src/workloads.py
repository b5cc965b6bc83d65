"""
workloads.py — seeded synthetic inputs with the shapes and value
distributions of the five tuned kernel families.

The reference fills its benchmark inputs with `rand()/RAND_MAX`
(src/generator.py:231-243) and its verification inputs with closed forms at
tiny sizes (src/verifier.py:66-191). Here every family has three size
configurations:

  kat     — the reference verifier's own problem size;
  small   — a multi-tile size that the CPU checks in well under a second;
  config  — the full benchmark configuration:
              softmax   fp32 4096×4096, x ~ N(0,1)
              reduction fp32 2^28, x ~ U[-1,1]  (fp64 sum)
              layernorm fp32 16384×4096, x ~ N(0,1), gamma = 1+0.1·N(0,1),
                        beta = 0.1·N(0,1), eps = 1e-5
              matmul    fp32 8192×8192×8192, A, B ~ U[-1,1], ±transpose_b
              attention bf16 [8, 32, 4096, 128], Q, K, V ~ N(0,1),
                        scale 1/sqrt(128), causal and non-causal
All generators use numpy.random.default_rng(seed).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

DEFAULT_SEED = 2024

SIZES: dict[str, dict[str, dict]] = {
    "softmax": {
        "kat": {"rows": 4, "cols": 16},
        "small": {"rows": 257, "cols": 4096},
        "config": {"rows": 4096, "cols": 4096},
    },
    "reduction": {
        "kat": {"n": 256},
        "small": {"n": (1 << 22) + 3},
        "config": {"n": 1 << 28},
    },
    "layernorm": {
        "kat": {"rows": 4, "cols": 16},
        "small": {"rows": 513, "cols": 4096},
        "config": {"rows": 16384, "cols": 4096},
    },
    "matmul": {
        "kat": {"M": 64, "N": 64, "K": 64},
        "small": {"M": 512, "N": 384, "K": 1024},
        "config": {"M": 8192, "N": 8192, "K": 8192},
    },
    "attention": {
        "kat": {"B": 1, "H": 1, "S": 512, "D": 64},
        "small": {"B": 2, "H": 3, "S": 1024, "D": 128},
        "config": {"B": 8, "H": 32, "S": 4096, "D": 128},
    },
}

KERNELS = tuple(SIZES)


def dims(kernel: str, size: str = "config") -> dict:
    """Problem dims of a family at a named size configuration."""
    return dict(SIZES[kernel][size])


@dataclass
class Work:
    """Algorithmic work of one call: bytes moved (HBM) and FLOPs."""
    bytes: int
    flops: int
    bound: str  # "hbm" | "tensor" | "fp32"
    notes: str = ""
    extra: dict = field(default_factory=dict)


def work(kernel: str, d: dict, causal: bool = False, variant: str = "") -> Work:
    """
    Algorithmic bytes/FLOPs per call, the numerator of the roofline fraction.

    softmax: read x + write y = 2·R·C·4 bytes.  reduction: N·4.  layernorm:
    2·R·C·4 + 2·C·4.  matmul: 2·M·N·K FLOPs.  attention: 4·B·H·S²·D
    (non-causal) or 4·B·H·D·S(S+1)/2 (causal, unmasked pairs only).
    """
    if kernel == "softmax":
        R, C = d["rows"], d["cols"]
        return Work(2 * R * C * 4, 5 * R * C, "hbm")
    if kernel == "reduction":
        return Work(d["n"] * 4, d["n"], "hbm")
    if kernel == "layernorm":
        R, C = d["rows"], d["cols"]
        return Work(2 * R * C * 4 + 2 * C * 4, 8 * R * C, "hbm")
    if kernel == "matmul":
        M, N, K = d["M"], d["N"], d["K"]
        bound = "fp32" if variant == "ffma" else "tensor"
        return Work((M * K + K * N + M * N) * 4, 2 * M * N * K, bound)
    if kernel == "attention":
        B, H, S, D = d["B"], d["H"], d["S"], d["D"]
        pairs = S * (S + 1) // 2 if causal else S * S
        return Work(4 * B * H * S * D * 2, 4 * B * H * pairs * D, "tensor")
    raise ValueError(f"unknown kernel {kernel!r}")


def make_inputs(kernel: str, size: str = "config", seed: int = DEFAULT_SEED, d: dict | None = None) -> dict:
    """
    Seeded inputs as numpy arrays (fp32; attention as bf16 bit patterns in
    uint16 plus their exact fp32 values). `d` overrides the named size.
    """
    d = dict(d) if d is not None else dims(kernel, size)
    rng = np.random.default_rng(seed)
    if kernel == "softmax":
        return {"x": rng.standard_normal((d["rows"], d["cols"]), dtype=np.float32), **d}
    if kernel == "reduction":
        return {"x": uniform_pm1(rng, d["n"]), **d}
    if kernel == "layernorm":
        R, C = d["rows"], d["cols"]
        x = rng.standard_normal((R, C), dtype=np.float32)
        gamma = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
        beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
        return {"x": x, "gamma": gamma, "beta": beta, "eps": 1e-5, **d}
    if kernel == "matmul":
        M, N, K = d["M"], d["N"], d["K"]
        A = uniform_pm1(rng, M * K).reshape(M, K)
        B = uniform_pm1(rng, K * N).reshape(K, N)
        return {"A": A, "B": B, **d}
    if kernel == "attention":
        B, H, S, D = d["B"], d["H"], d["S"], d["D"]
        out = dict(d)
        for name in ("q", "k", "v"):
            f = rng.standard_normal((B, H, S, D), dtype=np.float32)
            bits = bf16_bits(f)
            out[name] = bits
        out["scale"] = 1.0 / math.sqrt(D)
        return out
    raise ValueError(f"unknown kernel {kernel!r}")


def uniform_pm1(rng: np.random.Generator, n: int) -> np.ndarray:
    """n fp32 values uniform on [-1, 1), drawn natively in fp32 (2^28 values in ~3 s)."""
    x = rng.random(n, dtype=np.float32)
    x *= 2.0
    x -= 1.0
    return x


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> fp32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
