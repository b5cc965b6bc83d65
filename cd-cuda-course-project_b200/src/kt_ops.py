"""
kt_ops.py — torch-facing wrappers over the C ABI.

torch provides device memory and streams only; every computation goes
through the loaded kernel library. Each wrapper checks device, dtype and
contiguity, allocates the output, and launches on torch's current stream.
There is no CPU or torch fallback: a missing library raises.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

import kt_lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def softmax(x: torch.Tensor, out: Optional[torch.Tensor] = None, lib: Optional[kt_lib.KtLibrary] = None) -> torch.Tensor:
    """Row softmax over the last dim of a 2-D fp32 tensor."""
    _check(x, "x", torch.float32)
    if x.dim() != 2:
        raise ValueError("x must be 2-D (rows, cols)")
    lib = lib or kt_lib.load()
    y = out if out is not None else torch.empty_like(x)
    lib.softmax_f32(x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1], _stream())
    return y


def layernorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
              out: Optional[torch.Tensor] = None, lib: Optional[kt_lib.KtLibrary] = None) -> torch.Tensor:
    """LayerNorm over the last dim of a 2-D fp32 tensor (biased variance)."""
    for t, n in ((x, "x"), (gamma, "gamma"), (beta, "beta")):
        _check(t, n, torch.float32)
    if x.dim() != 2 or gamma.numel() != x.shape[1] or beta.numel() != x.shape[1]:
        raise ValueError("layernorm: x (rows, cols), gamma/beta (cols,)")
    lib = lib or kt_lib.load()
    y = out if out is not None else torch.empty_like(x)
    lib.layernorm_f32(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(),
                      x.shape[0], x.shape[1], float(eps), _stream())
    return y


class ReduceWorkspace:
    """Caller-owned scratch for kt_reduce_sum_f32, reusable across calls."""

    def __init__(self, n: int, device: torch.device | str = "cuda", lib: Optional[kt_lib.KtLibrary] = None):
        lib = lib or kt_lib.load()
        self.bytes = lib.reduce_workspace_bytes(n)
        self.buf = torch.empty(max(self.bytes, 16), dtype=torch.uint8, device=device)


def reduce_sum(x: torch.Tensor, out64: Optional[torch.Tensor] = None, out32: Optional[torch.Tensor] = None,
               workspace: Optional[ReduceWorkspace] = None,
               lib: Optional[kt_lib.KtLibrary] = None) -> torch.Tensor:
    """Sum of all elements of an fp32 tensor, accumulated in fp64 (returns a 1-element fp64 tensor)."""
    _check(x, "x", torch.float32)
    lib = lib or kt_lib.load()
    n = x.numel()
    if out64 is None:
        out64 = torch.empty(1, dtype=torch.float64, device=x.device)
    ws = workspace or ReduceWorkspace(n, x.device, lib)
    lib.reduce_sum_f32(x.data_ptr(), n, out64.data_ptr(), out32.data_ptr() if out32 is not None else None,
                       ws.buf.data_ptr(), ws.bytes, _stream())
    return out64


def gemm(A: torch.Tensor, B: torch.Tensor, transpose_b: bool = False, variant: int = kt_lib.KT_GEMM_TF32,
         out: Optional[torch.Tensor] = None, lib: Optional[kt_lib.KtLibrary] = None) -> torch.Tensor:
    """C = A·B, or A·Bt^T when transpose_b (B then holds Bt, shape N×K)."""
    _check(A, "A", torch.float32)
    _check(B, "B", torch.float32)
    M, K = A.shape
    if transpose_b:
        N, K2 = B.shape
    else:
        K2, N = B.shape
    if K2 != K:
        raise ValueError(f"gemm: inner dims differ ({K} vs {K2})")
    lib = lib or kt_lib.load()
    C = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=A.device)
    lib.gemm_f32(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, transpose_b, variant, _stream())
    return C


def fa_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
           causal: bool = False, out: Optional[torch.Tensor] = None,
           lib: Optional[kt_lib.KtLibrary] = None) -> torch.Tensor:
    """Flash-attention forward on bf16 [B, H, S, D] tensors."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check(t, n, torch.bfloat16)
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("fa_fwd: q, k, v must share shape [B, H, S, D]")
    B, H, S, D = q.shape
    lib = lib or kt_lib.load()
    o = out if out is not None else torch.empty_like(q)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    lib.fa_fwd_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, D, sc, causal, _stream())
    return o
