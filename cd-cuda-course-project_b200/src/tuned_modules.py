"""
tuned_modules.py — PyTorch layers that run on the tuned B200 kernels.

The reference's `TunedLinear`, `TunedLayerNorm` and `TunedMultiheadAttention`
(src/pytorch_integration.py:314-378) only attach the tuner's best parameters
to the stock torch layers as metadata and compute with cuBLAS / SDPA. Here
the same three layers compute with the kernel library: each one loads the
variant library the tuner picked (results/{kernel}_tuning.json, field
`best.library`), or the default library when no tuning result exists, and
calls it through the C ABI on the current CUDA stream:

  TunedLinear             y = x·W^T (+ b): kt_gemm_f32 with transpose_b (the
                          nn.Linear weight is already the N×K "Bt" layout);
                          TF32 tensor cores by default, exact FFMA on request
                          or when the tuned winner is the FFMA variant
  TunedLayerNorm          kt_layernorm_f32 over the last dimension
  TunedMultiheadAttention q/k/v/out projections as TunedLinear, the attention
                          core as kt_fa_fwd_bf16 (bf16 Q/K/V, fp32 softmax and
                          accumulation), optionally causal

They are inference layers (the library has forward kernels only): a call
with autograd recording raises instead of silently computing something else.
`apply_tuned_layers` swaps them into a model, copying the weights (the
reference's version builds fresh layers and drops the trained weights).
`sdpa_comparison` checks and times the attention core against
torch.nn.functional.scaled_dot_product_attention (the reference's SDPA vs
manual-attention benchmark, src/pytorch_integration.py:120-192).
"""

from __future__ import annotations

import json
import math
import os
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

import kt_lib
import kt_ops


def _results_dir(results_dir: Optional[os.PathLike] = None) -> Path:
    if results_dir is not None:
        return Path(results_dir)
    env = os.environ.get("KT_RESULTS_DIR")
    return Path(env) if env else Path(__file__).resolve().parent.parent / "results"


def load_best_params(kernel: str, results_dir: Optional[os.PathLike] = None) -> Dict[str, Any]:
    """Parameters of the tuner's best variant of `kernel` ({} without a tuning result)."""
    f = _results_dir(results_dir) / f"{kernel}_tuning.json"
    if not f.exists():
        return {}
    best = json.loads(f.read_text()).get("best") or {}
    return dict(best.get("params") or {})


def tuned_library(kernel: str, results_dir: Optional[os.PathLike] = None) -> kt_lib.KtLibrary:
    """The library of the tuner's best variant of `kernel` if it exists, else the default library."""
    f = _results_dir(results_dir) / f"{kernel}_tuning.json"
    if f.exists():
        best = json.loads(f.read_text()).get("best") or {}
        so = best.get("library")
        if so and Path(so).exists():
            return kt_lib.load(so)
    return kt_lib.load()


def _no_autograd(name: str, *tensors: torch.Tensor) -> None:
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise RuntimeError(f"{name} runs forward-only B200 kernels; call it under torch.no_grad() "
                           "or torch.inference_mode()")


class TunedLinear(nn.Linear):
    """nn.Linear computed by the library's GEMM (x·W^T with W as the transpose_b operand)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, kernel: str = "matmul",
                 variant: Optional[str] = None, results_dir: Optional[os.PathLike] = None,
                 device=None, dtype=None) -> None:
        super().__init__(in_features, out_features, bias, device=device, dtype=dtype)
        self.tuned_params = load_best_params(kernel, results_dir)
        self._lib = tuned_library(kernel, results_dir)
        v = variant or self.tuned_params.get("variant", "tf32")
        self.gemm_variant = kt_lib.KT_GEMM_FFMA if v == "ffma" else kt_lib.KT_GEMM_TF32

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _no_autograd("TunedLinear", x, self.weight, self.bias)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).contiguous()
        y = kt_ops.gemm(x2, self.weight.contiguous(), transpose_b=True, variant=self.gemm_variant, lib=self._lib)
        if self.bias is not None:
            y.add_(self.bias)
        return y.view(*lead, self.out_features)


class TunedLayerNorm(nn.LayerNorm):
    """nn.LayerNorm over the last dimension computed by the library's LayerNorm kernel."""

    def __init__(self, normalized_shape: int, eps: float = 1e-5, results_dir: Optional[os.PathLike] = None,
                 device=None, dtype=None) -> None:
        super().__init__(normalized_shape, eps=eps, elementwise_affine=True, device=device, dtype=dtype)
        if len(self.normalized_shape) != 1:
            raise ValueError("TunedLayerNorm normalises the last dimension only")
        self.tuned_params = load_best_params("layernorm", results_dir)
        self._lib = tuned_library("layernorm", results_dir)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _no_autograd("TunedLayerNorm", x, self.weight, self.bias)
        c = self.normalized_shape[0]
        y = kt_ops.layernorm(x.reshape(-1, c).contiguous(), self.weight, self.bias, self.eps, lib=self._lib)
        return y.view(x.shape)


class TunedMultiheadAttention(nn.Module):
    """Multi-head attention (batch_first) with the flash-attention kernel as its core."""

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0, bias: bool = True,
                 results_dir: Optional[os.PathLike] = None, device=None, dtype=None) -> None:
        super().__init__()
        if embed_dim % num_heads:
            raise ValueError("embed_dim must be divisible by num_heads")
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        if self.head_dim not in (64, 128):
            raise ValueError(f"head dim {self.head_dim}: the attention kernel supports 64 and 128")
        self.scale = self.head_dim ** -0.5
        self.dropout = dropout
        self.tuned_params = load_best_params("attention", results_dir)
        self._lib = tuned_library("attention", results_dir)
        kw = dict(bias=bias, results_dir=results_dir, device=device, dtype=dtype)
        self.q_proj = TunedLinear(embed_dim, embed_dim, **kw)
        self.k_proj = TunedLinear(embed_dim, embed_dim, **kw)
        self.v_proj = TunedLinear(embed_dim, embed_dim, **kw)
        self.out_proj = TunedLinear(embed_dim, embed_dim, **kw)

    def _heads(self, t: torch.Tensor, B: int, S: int) -> torch.Tensor:
        return t.view(B, S, self.num_heads, self.head_dim).transpose(1, 2).contiguous().to(torch.bfloat16)

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                key_padding_mask: Optional[torch.Tensor] = None, need_weights: bool = False,
                is_causal: bool = False) -> Tuple[torch.Tensor, None]:
        if key_padding_mask is not None:
            raise NotImplementedError("key_padding_mask is not supported by the attention kernel")
        if need_weights:
            raise NotImplementedError("the attention kernel does not form the weight matrix")
        if self.training and self.dropout > 0:
            raise NotImplementedError("attention dropout is not supported (inference layer)")
        B, S, _ = query.shape
        if key.shape[1] != S or value.shape[1] != S:
            raise NotImplementedError("query and key/value sequences of different lengths")
        q = self._heads(self.q_proj(query), B, S)
        k = self._heads(self.k_proj(key), B, S)
        v = self._heads(self.v_proj(value), B, S)
        o = kt_ops.fa_fwd(q, k, v, scale=self.scale, causal=is_causal, lib=self._lib)
        o = o.to(query.dtype).transpose(1, 2).reshape(B, S, self.embed_dim)
        return self.out_proj(o), None


def apply_tuned_layers(model: nn.Module, kernel: str = "matmul", results_dir: Optional[os.PathLike] = None) -> nn.Module:
    """Replace nn.Linear (kernel "matmul" or "all") and nn.LayerNorm ("layernorm" or "all")
    in `model` by their tuned versions, in place, keeping the weights."""
    for name, module in list(model.named_modules()):
        if not name:
            continue
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        new = None
        if kernel in ("matmul", "all") and type(module) is nn.Linear:
            new = TunedLinear(module.in_features, module.out_features, module.bias is not None,
                              results_dir=results_dir, device=module.weight.device, dtype=module.weight.dtype)
        elif kernel in ("layernorm", "all") and type(module) is nn.LayerNorm and module.elementwise_affine \
                and len(module.normalized_shape) == 1:
            new = TunedLayerNorm(module.normalized_shape[0], module.eps, results_dir=results_dir,
                                 device=module.weight.device, dtype=module.weight.dtype)
        if new is not None:
            new.load_state_dict(module.state_dict())
            setattr(parent, child, new)
    return model


@torch.no_grad()
def sdpa_comparison(batch: int = 4, heads: int = 8, seq_len: int = 1024, head_dim: int = 128, causal: bool = False,
                    warmup: int = 3, samples: int = 20, seed: int = 0, lib: Optional[kt_lib.KtLibrary] = None) -> dict:
    """The attention kernel against torch's scaled_dot_product_attention on the
    same bf16 inputs: normwise difference and mean CUDA-event times."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(batch, heads, seq_len, head_dim, device="cuda", dtype=torch.bfloat16, generator=g)
               for _ in range(3))
    scale = 1.0 / math.sqrt(head_dim)
    lib = lib or kt_lib.load()

    def ours():
        return kt_ops.fa_fwd(q, k, v, scale=scale, causal=causal, lib=lib)

    def sdpa():
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)

    def time_ms(fn) -> float:
        for _ in range(warmup):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(samples)]
        for a, b in ev:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / samples

    a, b = ours().float(), sdpa().float()
    err = float((a - b).abs().max() / b.abs().max())
    t_ours, t_sdpa = time_ms(ours), time_ms(sdpa)
    pairs = seq_len * (seq_len + 1) // 2 if causal else seq_len * seq_len
    flops = 4 * batch * heads * pairs * head_dim
    return {"shape": [batch, heads, seq_len, head_dim], "causal": causal, "normwise_diff": err,
            "kt_ms": t_ours, "sdpa_ms": t_sdpa, "kt_tflops": flops / t_ours / 1e9, "sdpa_tflops": flops / t_sdpa / 1e9}
