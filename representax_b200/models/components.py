"""Reusable numerical components (PyTorch reference path).

Parity: src/representax/models/components.py:28-258 — HF ``[out, in]`` linear
layout, fp32-statistics LayerNorm / RMSNorm, activations, dropout, masked
dot-product attention with local windows, padding-aware mean pooling and L2
normalisation. These run on any device and serve as the oracle of the native
kernels in ``representax_b200.ops``.
"""

from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn.functional as F

Activation = Literal["gelu", "gelu_new", "gelu_pytorch_tanh", "relu", "silu"]


def activate(x: torch.Tensor, name: str) -> torch.Tensor:
    if name == "gelu":
        return F.gelu(x)
    if name in {"gelu_new", "gelu_pytorch_tanh", "gelu_tanh"}:
        return F.gelu(x, approximate="tanh")
    if name == "relu":
        return F.relu(x)
    if name in {"silu", "swish"}:
        return F.silu(x)
    raise ValueError(f"unsupported activation {name!r}")


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, eps: float) -> torch.Tensor:
    out = F.layer_norm(x.float(), (x.shape[-1],), weight.float(), None if bias is None else bias.float(), eps)
    return out.to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return out.to(x.dtype)


def dropout(x: torch.Tensor, p: float, generator: torch.Generator | None) -> torch.Tensor:
    """Dropout driven by an explicit generator (None means evaluation)."""

    if generator is None or p <= 0.0:
        return x
    keep = torch.rand(x.shape, generator=generator, device=x.device) >= p
    return torch.where(keep, x / (1.0 - p), torch.zeros((), dtype=x.dtype, device=x.device))


def dot_product_attention(q, k, v, *, key_mask=None, bias=None, causal=False, window: int | None = None,
                          dropout_p: float = 0.0, generator=None):
    """Masked attention on [batch, seq, heads, head_dim] tensors (fp32 softmax)."""

    b, s, h, d = q.shape
    kv_heads = k.shape[2]
    if kv_heads != h:
        rep = h // kv_heads
        k = k.repeat_interleave(rep, dim=2)
        v = v.repeat_interleave(rep, dim=2)
    scores = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) / math.sqrt(d)
    if bias is not None:
        scores = scores + bias.float()
    mask = torch.ones((b, 1, s, k.shape[1]), dtype=torch.bool, device=q.device)
    if key_mask is not None:
        mask = mask & key_mask[:, None, None, :].bool()
    i = torch.arange(s, device=q.device)[:, None]
    j = torch.arange(k.shape[1], device=q.device)[None, :]
    if causal:
        mask = mask & (j <= i)
    if window is not None and window >= 0:
        mask = mask & ((j - i).abs() <= window)
    scores = scores.masked_fill(~mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    probs = torch.nan_to_num(probs, nan=0.0)
    probs = dropout(probs, dropout_p, generator)
    out = torch.einsum("bhqk,bkhd->bqhd", probs, v.float())
    return out.to(q.dtype)


def mean_pool(hidden: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    m = mask.to(torch.float32)[..., None]
    total = (hidden.float() * m).sum(-2)
    count = torch.clamp(m.sum(-2), min=1.0)
    return total / count


def l2_normalize(x: torch.Tensor) -> torch.Tensor:
    x = x.float()
    return x / torch.clamp(torch.linalg.vector_norm(x, dim=-1, keepdim=True), min=1e-12)


def last_token_pool(hidden: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    idx = torch.clamp(mask.long().sum(-1) - 1, min=0)
    # Right-padded: the last valid token sits at (length - 1).
    return hidden[torch.arange(hidden.shape[0], device=hidden.device), idx].float()


def init_linear(out_features: int, in_features: int, scale: float, generator: torch.Generator | None,
                bias: bool = True) -> tuple[torch.nn.Parameter, torch.nn.Parameter | None]:
    w = torch.nn.Parameter(torch.randn(out_features, in_features, generator=generator) * scale)
    b = torch.nn.Parameter(torch.zeros(out_features)) if bias else None
    return w, b


__all__ = [
    "activate",
    "dot_product_attention",
    "dropout",
    "init_linear",
    "l2_normalize",
    "last_token_pool",
    "layer_norm",
    "mean_pool",
    "rms_norm",
]
