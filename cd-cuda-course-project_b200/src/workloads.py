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
All generators are numpy.random.default_rng streams seeded per block from
(seed, family, tensor, block) (see make_inputs).
"""

from __future__ import annotations

import math
import os
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


# Inputs are drawn in fixed blocks along the sharded dimension, each block from
# its own generator seeded by (seed, family, tensor, block). Any contiguous
# part of the batch can therefore be generated alone and matches the same
# slice of the whole batch, so every rank builds only its shard and the data
# does not depend on the number of GPUs.
_BLOCK = {"reduction": 1 << 20, "softmax": 64, "layernorm": 64, "matmul": 64, "attention": 1}
_TAG = {"softmax": 1, "layernorm": 2, "reduction": 3, "matmul": 4, "attention": 5}
_PARAMS_BLOCK = 1 << 40  # block id of the per-family parameters (gamma/beta, matmul B)


def _rng(seed: int, kernel: str, tensor: int, block: int) -> np.random.Generator:
    return np.random.default_rng([int(seed), _TAG[kernel], int(tensor), int(block)])


def _blocks(kernel: str, seed: int, tensor: int, lo: int, hi: int, row_shape: tuple, dtype, fill_fn) -> np.ndarray:
    """Units [lo, hi) of the sharded dimension, each unit of shape row_shape,
    filled block by block (threads: NumPy's generators release the GIL).
    fill_fn(rng, dst) fills dst in place from rng."""
    bs = _BLOCK[kernel]
    out = np.empty((hi - lo, *row_shape), dtype=dtype)
    if hi <= lo:
        return out
    blocks = range(lo // bs, (hi - 1) // bs + 1)

    def fill(b: int) -> None:
        b0, b1 = b * bs, (b + 1) * bs
        a0, a1 = max(lo, b0), min(hi, b1)
        rng = _rng(seed, kernel, tensor, b)
        if a0 == b0 and a1 == b1:
            fill_fn(rng, out[a0 - lo:a1 - lo])
        else:  # a block cut by the part's edge: draw it whole, keep the overlap
            tmp = np.empty((b1 - b0, *row_shape), dtype=dtype)
            fill_fn(rng, tmp)
            out[a0 - lo:a1 - lo] = tmp[a0 - b0:a1 - b0]

    if len(blocks) > 4 and out.nbytes > (8 << 20):
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
            list(ex.map(fill, blocks))
    else:
        for b in blocks:
            fill(b)
    return out


def _normal(rng: np.random.Generator, dst: np.ndarray) -> None:
    rng.standard_normal(out=dst, dtype=np.float32)


def _uniform(rng: np.random.Generator, dst: np.ndarray) -> None:
    rng.random(out=dst, dtype=np.float32)
    dst *= 2.0
    dst -= 1.0


def _normal_bf16(rng: np.random.Generator, dst: np.ndarray) -> None:
    f = np.empty(dst.shape, dtype=np.float32)
    rng.standard_normal(out=f, dtype=np.float32)
    dst[...] = bf16_bits(f)


def shard_unit(kernel: str) -> str:
    """Name of the dimension a family is sharded along (and `part` counts)."""
    return {"reduction": "n", "softmax": "rows", "layernorm": "rows", "matmul": "M", "attention": "B*H"}[kernel]


def make_inputs(kernel: str, size: str = "config", seed: int = DEFAULT_SEED, d: dict | None = None,
                part: tuple[int, int] | None = None) -> dict:
    """
    Seeded inputs as numpy arrays (fp32; attention as bf16 bit patterns in
    uint16). `d` overrides the named size. `part` = (lo, hi) generates only
    units [lo, hi) of the sharded dimension (elements, rows, rows of A, or
    (batch, head) pairs as a [hi-lo, S, D] array), equal to that slice of the
    whole batch; replicated tensors (gamma, beta, matmul B) are always whole.
    """
    d = dict(d) if d is not None else dims(kernel, size)
    if kernel == "reduction":
        n = d["n"]
        lo, hi = part if part is not None else (0, n)
        return {"x": _blocks(kernel, seed, 0, lo, hi, (), np.float32, _uniform), **d}
    if kernel in ("softmax", "layernorm"):
        R, C = d["rows"], d["cols"]
        lo, hi = part if part is not None else (0, R)
        x = _blocks(kernel, seed, 0, lo, hi, (C,), np.float32, _normal)
        if kernel == "softmax":
            return {"x": x, **d}
        rng = _rng(seed, kernel, 1, _PARAMS_BLOCK)
        gamma = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
        beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
        return {"x": x, "gamma": gamma, "beta": beta, "eps": 1e-5, **d}
    if kernel == "matmul":
        M, N, K = d["M"], d["N"], d["K"]
        lo, hi = part if part is not None else (0, M)
        A = _blocks(kernel, seed, 0, lo, hi, (K,), np.float32, _uniform)
        B = np.empty((K, N), dtype=np.float32)
        _uniform(_rng(seed, kernel, 1, _PARAMS_BLOCK), B)
        return {"A": A, "B": B, **d}
    if kernel == "attention":
        B, H, S, D = d["B"], d["H"], d["S"], d["D"]
        out = dict(d)
        lo, hi = part if part is not None else (0, B * H)
        for t, name in enumerate(("q", "k", "v")):
            bits = _blocks(kernel, seed, t, lo, hi, (S, D), np.uint16, _normal_bf16)
            out[name] = bits if part is not None else bits.reshape(B, H, S, D)
        out["scale"] = 1.0 / math.sqrt(D)
        return out
    raise ValueError(f"unknown kernel {kernel!r}")


def uniform_pm1(rng: np.random.Generator, n: int) -> np.ndarray:
    """n fp32 values uniform on [-1, 1), drawn natively in fp32."""
    x = np.empty(n, dtype=np.float32)
    _uniform(rng, x)
    return x


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> fp32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
