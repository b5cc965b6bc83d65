"""
oracle/cpu_baseline.py — times the reference's CPU path (its NumPy verifier
formulas, restated in oracle/ref.py) on this machine's host cores.

Test/benchmark infrastructure only: used by bench.py's CPU-baseline leg and
its `--impl reference` arm, never by the library or the tuner.

NumPy's elementwise and reduction loops run on one thread; the work is split
into contiguous chunks over a thread pool (NumPy releases the GIL inside
those loops), so `threads` host cores are in use. BLAS matmul uses its own
thread pool.
"""

from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor
from typing import Callable

import numpy as np

from . import ref


def host_threads() -> int:
    """Cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


def _time(fn: Callable[[], object], reps: int) -> tuple[float, float, object]:
    times = []
    out = None
    for _ in range(max(1, reps)):
        t0 = time.perf_counter()
        out = fn()
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[0], times[len(times) // 2], out


def reduce_sum(x: np.ndarray, threads: int, reps: int = 3) -> dict:
    """fp64 sum of fp32 x (`x.sum(dtype=float64)`), chunked over `threads`."""
    chunks = np.array_split(np.asarray(x).ravel(), max(1, threads))
    with ThreadPoolExecutor(max(1, threads)) as ex:
        def run():
            return float(sum(ex.map(lambda c: c.sum(dtype=np.float64), chunks)))
        best, median, out = _time(run, reps)
    return {"best_s": best, "median_s": median, "result": out, "bytes": x.nbytes, "threads": threads}


def softmax_f32(x: np.ndarray) -> np.ndarray:
    """Row softmax evaluated in fp32, as the reference's `_ref_softmax` does
    (src/verifier.py:245-250): subtract the row max, np.exp, divide by the row sum."""
    e = np.exp(x - x.max(axis=1, keepdims=True))
    e /= e.sum(axis=1, keepdims=True)
    return e


def rows_op(kind: str, x: np.ndarray, threads: int, reps: int = 3, gamma=None, beta=None, eps: float = 1e-5) -> dict:
    """Row softmax or LayerNorm in the reference's own precision (softmax in
    fp32, src/verifier.py:245-250; LayerNorm statistics in fp64, :267-274),
    rows chunked over threads."""
    chunks = np.array_split(np.arange(x.shape[0]), max(1, threads))

    def part(idx):
        rows = x[idx[0]:idx[-1] + 1] if idx.size else x[:0]
        if kind == "softmax":
            return softmax_f32(rows)
        return ref.layernorm_ref(rows, gamma, beta, eps).astype(np.float32)

    with ThreadPoolExecutor(max(1, threads)) as ex:
        def run():
            return list(ex.map(part, chunks))
        best, median, _ = _time(run, reps)
    nbytes = 2 * x.nbytes + (0 if gamma is None else 2 * np.asarray(gamma).nbytes)
    return {"best_s": best, "median_s": median, "bytes": nbytes, "threads": threads}


def matmul(A: np.ndarray, B: np.ndarray, reps: int = 2, transpose_b: bool = False) -> dict:
    """fp32 BLAS matmul A @ B (the reference's `np.matmul` path), BLAS threads."""
    Bm = B.T if transpose_b else B

    def run():
        return A @ Bm
    best, median, _ = _time(run, reps)
    M, K = A.shape
    N = Bm.shape[1]
    return {"best_s": best, "median_s": median, "flops": 2 * M * N * K}


def attention_heads(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool,
                    threads: int, reps: int = 1) -> dict:
    """Per-head fp32 attention (src/verifier.py:277-294 evaluated in fp32) over the
    given heads ([h, S, D] arrays), heads spread over threads."""
    def head(i):
        s = (q[i] @ k[i].T) * np.float32(scale)
        if causal:
            s = np.where(np.triu(np.ones(s.shape, dtype=bool), 1), np.float32(-np.inf), s)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        return p @ v[i]

    with ThreadPoolExecutor(max(1, threads)) as ex:
        def run():
            return list(ex.map(head, range(q.shape[0])))
        best, median, _ = _time(run, reps)
    S, D = q.shape[1], q.shape[2]
    pairs = S * (S + 1) // 2 if causal else S * S
    return {"best_s": best, "median_s": median, "flops": 4 * q.shape[0] * pairs * D, "heads": q.shape[0]}
