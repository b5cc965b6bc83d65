"""
oracle/ref.py — CPU restatement of the reference's NumPy verifier, used ONLY as
test infrastructure (tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg). Nothing in the shipped library or tuner imports this module.

Parity is pinned: tests/golden/reference_kat.npz holds the outputs of the
reference's own `_ref_*` functions (src/verifier.py:221-294), produced by
tests/golden/make_golden.py, and tests/test_oracle.py checks every function
here against them.

Each function names the reference lines it restates. Where BASELINE's
configurations go beyond the reference (seeded inputs, gamma/beta, fp64
reduction, transpose_b, bf16 batched causal attention) the extension is
stated in the docstring.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# Deterministic known-answer inputs of the reference's verify mains
# ---------------------------------------------------------------------------


def kat_pattern(n: int, modulus: int = 97, offset: float = 0.5) -> np.ndarray:
    """(i % modulus) * 0.01 - offset as fp32 (src/verifier.py:66-72, :97-101, :122-127, :154)."""
    i = np.arange(n, dtype=np.float64)
    return ((i % modulus) * 0.01 - offset).astype(np.float32)


def kat_matmul_inputs(N: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """A[i]=(i%97)*0.01-0.5, B[i]=(i%89)*0.01-0.3, N×N fp32 (src/verifier.py:66-72, :234-238)."""
    A = kat_pattern(N * N, 97, 0.5).reshape(N, N)
    B = kat_pattern(N * N, 89, 0.3).reshape(N, N)
    return A, B


def kat_attention_inputs(S: int = 512, D: int = 64) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Q=sin(0.01 i), K=cos(0.01 i), V=sin(0.007 i), S×D fp32 (src/verifier.py:181-191, :284-287)."""
    i = np.arange(S * D, dtype=np.float64)
    Q = np.sin(i * 0.01).reshape(S, D).astype(np.float32)
    K = np.cos(i * 0.01).reshape(S, D).astype(np.float32)
    V = np.sin(i * 0.007).reshape(S, D).astype(np.float32)
    return Q, K, V


# ---------------------------------------------------------------------------
# Reference formulas (fp64 restatements)
# ---------------------------------------------------------------------------


def softmax_ref(x: np.ndarray) -> np.ndarray:
    """Row softmax exp(x - max)/sum along the last axis, in fp64
    (src/verifier.py:245-250; the reference evaluates it in fp32)."""
    x64 = np.asarray(x, dtype=np.float64)
    m = x64.max(axis=-1, keepdims=True)
    e = np.exp(x64 - m)
    return e / e.sum(axis=-1, keepdims=True)


def layernorm_ref(x: np.ndarray, gamma: np.ndarray | None = None, beta: np.ndarray | None = None,
                  eps: float = 1e-5) -> np.ndarray:
    """gamma*(x-mean)/sqrt(var+eps)+beta with the biased variance, in fp64
    (src/verifier.py:267-274; gamma=1, beta=0 there, per-column gamma/beta here)."""
    x64 = np.asarray(x, dtype=np.float64)
    mean = x64.mean(axis=-1, keepdims=True)
    var = x64.var(axis=-1, keepdims=True)
    y = (x64 - mean) / np.sqrt(var + eps)
    if gamma is not None:
        y = y * np.asarray(gamma, dtype=np.float64)
    if beta is not None:
        y = y + np.asarray(beta, dtype=np.float64)
    return y


def reduction_partials_ref(x: np.ndarray, block_size: int) -> np.ndarray:
    """Per-block partial sums over 2*block_size consecutive fp32 values, the
    reference's reduction oracle (src/verifier.py:253-264)."""
    x32 = np.asarray(x, dtype=np.float32)
    stride = 2 * block_size
    grid = (x32.size + stride - 1) // stride
    out = np.zeros(grid, dtype=np.float32)
    for b in range(grid):
        out[b] = x32[b * stride:(b + 1) * stride].sum()
    return out


def reduce_sum_ref(x: np.ndarray) -> float:
    """Whole sum accumulated in fp64: `x.sum(dtype=float64)` (BASELINE's oracle for
    the reduction; the reference only checks partials, src/verifier.py:253-264)."""
    return float(np.asarray(x).sum(dtype=np.float64))


def matmul_ref(A: np.ndarray, B: np.ndarray, transpose_b: bool = False) -> np.ndarray:
    """fp64 matmul (src/verifier.py:234-242). transpose_b: B holds Bt (N×K) and the
    product is A @ Bt.T — the layout the reference's transpose_b load reads
    (src/generator.py:286-293)."""
    A64 = np.asarray(A, dtype=np.float64)
    B64 = np.asarray(B, dtype=np.float64)
    return A64 @ (B64.T if transpose_b else B64)


def attention_ref(Q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float | None = None,
                  causal: bool = False) -> np.ndarray:
    """softmax(Q K^T * scale) V per head in fp64 (src/verifier.py:277-294), over any
    leading batch dims, with an optional causal mask (key j > query i excluded)."""
    Q64 = np.asarray(Q, dtype=np.float64)
    K64 = np.asarray(K, dtype=np.float64)
    V64 = np.asarray(V, dtype=np.float64)
    D = Q64.shape[-1]
    sc = 1.0 / np.sqrt(D) if scale is None else float(scale)
    scores = (Q64 @ np.swapaxes(K64, -1, -2)) * sc
    if causal:
        S_q, S_k = scores.shape[-2], scores.shape[-1]
        mask = np.triu(np.ones((S_q, S_k), dtype=bool), k=1)
        scores = np.where(mask, -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    return p @ V64


def attention_rows_ref(Q: np.ndarray, K: np.ndarray, V: np.ndarray, rows: np.ndarray, scale: float,
                       causal: bool = False) -> np.ndarray:
    """attention_ref for the query rows `rows` of one head ([S, D] arrays) only:
    the same formula (src/verifier.py:277-294), with the causal mask of the
    full sequence (key j excluded from query row i when j > i). Lets a test
    check a long sequence at a fraction of the cost of every row."""
    rows = np.asarray(rows, dtype=np.int64)
    K64 = np.asarray(K, dtype=np.float64)
    V64 = np.asarray(V, dtype=np.float64)
    out = np.empty((rows.size, K64.shape[-1] if V64.ndim == 2 else V64.shape[-1]), dtype=np.float64)
    for i0 in range(0, rows.size, 256):
        r = rows[i0:i0 + 256]
        s = (np.asarray(Q, dtype=np.float64)[r] @ K64.T) * float(scale)
        if causal:
            s = np.where(np.arange(K64.shape[0])[None, :] > r[:, None], -np.inf, s)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        out[i0:i0 + r.size] = p @ V64
    return out


# ---------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as __float2bfloat16_rn)
# ---------------------------------------------------------------------------


def bf16_bits_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even; NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = np.uint16(0x7FC0)
    return out


def f32_from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> exact fp32 values."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Tolerance metrics (BASELINE: softmax/LN 1e-5 rel, reduction 1e-4, TF32 1e-3, bf16 attention 2e-2)
# ---------------------------------------------------------------------------


def normwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got-ref| / max|ref| (the normwise metric for every family)."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(r))) if r.size else 0.0
    if r.size == 0:
        return 0.0
    num = float(np.max(np.abs(g - r)))
    return num / denom if denom > 0 else num


def product_scaled_err(got: np.ndarray, A: np.ndarray, B: np.ndarray) -> float:
    """max|C - A·B| / max(|A|·|B|): the error of a matmul measured against the
    magnitude of its products. Rounding each operand to tf32 (10 explicit
    mantissa bits) moves every product by at most ~2^-10 of its size, so this
    ratio stays below 1e-3 even when a short dot product cancels to a small
    value, where max|C - A·B| / max|A·B| need not."""
    A64 = np.asarray(A, dtype=np.float64)
    B64 = np.asarray(B, dtype=np.float64)
    exact = A64 @ B64
    scale = float(np.max(np.abs(A64) @ np.abs(B64))) if exact.size else 0.0
    num = float(np.max(np.abs(np.asarray(got, dtype=np.float64) - exact))) if exact.size else 0.0
    return num / scale if scale > 0 else num


def max_abs_diff(got: np.ndarray, ref: np.ndarray) -> float:
    """The reference's metric: max absolute difference (src/verifier.py:558-569)."""
    g = np.asarray(got, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    if g.size == 0 or r.size == 0:
        return 0.0
    return float(np.max(np.abs(g - r)))
