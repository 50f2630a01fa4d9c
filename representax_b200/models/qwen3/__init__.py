"""Qwen3-style causal decoder tower shared by Jina v5 (text) and Qwen3-VL.

Pre-RMSNorm blocks: fused q/k/v projection -> per-head q/k RMSNorm -> RoPE
(1-D positions, or interleaved / sectioned M-RoPE from 3-axis positions)
-> causal grouped-query attention -> o_proj (+ residual); RMSNorm ->
fused gate/up projection -> SwiGLU -> down_proj (+ residual). Every op runs
on packed rows through ``ops.nn`` (sm_100a kernels on bf16 CUDA tensors:
the q/k norm and rotation are one fused kernel, attention is the packed
causal GQA kernel).

Parity: src/representax/models/jina_v5/model.py:79-227 and
src/representax/models/qwen3_vl/text.py:65-367 (decoder block, q/k norm,
GQA, M-RoPE with ``mrope_section`` interleaving, DeepStack injection into
the first layers).
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any

import torch
from pydantic import model_validator
from torch import nn

from representax_b200._config import FrozenConfig
from representax_b200.ops import nn as N


class Qwen3TextConfig(FrozenConfig):
    vocab_size: int = 151936
    hidden_size: int = 2048
    intermediate_size: int = 6144
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dimension: int = 128
    max_position_embeddings: int = 32768
    rope_theta: float = 1_000_000.0
    mrope_section: tuple[int, int, int] | None = None
    mrope_interleaved: bool = True
    norm_epsilon: float = 1e-6
    pad_token_id: int = 151643
    initializer_range: float = 0.02
    tie_word_embeddings: bool = True
    qkv_bias: bool = False        # Qwen2 / Qwen2.5 projections carry biases
    qk_norm: bool = True          # Qwen3 per-head RMSNorm on q and k

    @model_validator(mode="after")
    def _validate(self):
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")
        if self.head_dimension % 2:
            raise ValueError("head_dimension must be even")
        return self

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any], **overrides: Any) -> "Qwen3TextConfig":
        text = value.get("text_config", value)
        rope = text.get("rope_parameters") or text.get("rope_scaling") or {}
        theta = float(rope.get("rope_theta", text.get("rope_theta", 1_000_000.0)))
        section = rope.get("mrope_section")
        hidden, heads = int(text["hidden_size"]), int(text["num_attention_heads"])
        fields = dict(
            vocab_size=int(text["vocab_size"]), hidden_size=hidden, intermediate_size=int(text["intermediate_size"]),
            num_hidden_layers=int(text["num_hidden_layers"]), num_attention_heads=heads,
            num_key_value_heads=int(text.get("num_key_value_heads", heads)),
            head_dimension=int(text.get("head_dim") or hidden // heads),
            max_position_embeddings=int(text.get("max_position_embeddings", 32768)), rope_theta=theta,
            mrope_section=None if section is None else tuple(int(s) for s in section),
            mrope_interleaved=bool(rope.get("mrope_interleaved", True)),
            norm_epsilon=float(text.get("rms_norm_eps", 1e-6)),
            pad_token_id=int(text.get("pad_token_id") or 151643),
            tie_word_embeddings=bool(value.get("tie_word_embeddings", text.get("tie_word_embeddings", True))),
        )
        fields.update(overrides)
        return cls(**fields)

    def to_hf_config(self) -> dict[str, Any]:
        rope: dict[str, Any] = {"rope_type": "default", "rope_theta": self.rope_theta}
        if self.mrope_section is not None:
            rope.update(mrope_section=list(self.mrope_section), mrope_interleaved=self.mrope_interleaved)
        return {"vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
                "intermediate_size": self.intermediate_size, "num_hidden_layers": self.num_hidden_layers,
                "num_attention_heads": self.num_attention_heads, "num_key_value_heads": self.num_key_value_heads,
                "head_dim": self.head_dimension, "max_position_embeddings": self.max_position_embeddings,
                "rope_parameters": rope, "rms_norm_eps": self.norm_epsilon, "pad_token_id": self.pad_token_id,
                "tie_word_embeddings": self.tie_word_embeddings, "hidden_act": "silu"}


def _normal(shape, std, g):
    return nn.Parameter(torch.randn(*shape, generator=g) * std)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, cfg: Qwen3TextConfig, g: torch.Generator) -> None:
        super().__init__()
        h, d, std = cfg.hidden_size, cfg.head_dimension, cfg.initializer_range
        qd, kd = cfg.num_attention_heads * d, cfg.num_key_value_heads * d
        self.input_norm = nn.Parameter(torch.ones(h))
        self.qkv = _normal((qd + 2 * kd, h), std, g)       # [q; k; v] rows
        self.qkv_bias = nn.Parameter(torch.zeros(qd + 2 * kd)) if cfg.qkv_bias else None
        self.q_norm = nn.Parameter(torch.ones(d)) if cfg.qk_norm else None
        self.k_norm = nn.Parameter(torch.ones(d)) if cfg.qk_norm else None
        self.o_proj = _normal((h, qd), std, g)
        self.post_norm = nn.Parameter(torch.ones(h))
        self.gate_up = _normal((2 * cfg.intermediate_size, h), std, g)  # [gate; up] rows
        self.down = _normal((h, cfg.intermediate_size), std, g)

    def forward(self, h, seg, pos, axis_of, inv_freq, cfg: Qwen3TextConfig):
        x = N.rms_norm(h, self.input_norm, cfg.norm_epsilon)
        a = N.qkv_attention(N.linear(x, self.qkv, self.qkv_bias), seg, heads=cfg.num_attention_heads,
                            kv_heads=cfg.num_key_value_heads, pos=pos, inv_freq=inv_freq, axis_of=axis_of,
                            q_norm=self.q_norm, k_norm=self.k_norm, norm_eps=cfg.norm_epsilon, causal=True)
        h = N.linear(a, self.o_proj, residual=h)
        x = N.rms_norm(h, self.post_norm, cfg.norm_epsilon)
        g = N.gated_activation(N.linear(x, self.gate_up), "silu")
        return N.linear(g, self.down, residual=h)


class Qwen3TextTower(nn.Module):
    def __init__(self, cfg: Qwen3TextConfig, g: torch.Generator) -> None:
        super().__init__()
        self.config = cfg
        self.embed_tokens = _normal((cfg.vocab_size, cfg.hidden_size), cfg.initializer_range, g)
        self.layers = nn.ModuleList(Qwen3DecoderLayer(cfg, g) for _ in range(cfg.num_hidden_layers))
        self.norm = nn.Parameter(torch.ones(cfg.hidden_size))
        self.register_buffer("inv_freq", N.rope_inv_freq(cfg.head_dimension, cfg.rope_theta), persistent=False)
        axis = None
        if cfg.mrope_section is not None:
            axis = torch.tensor(N.mrope_axis_table(cfg.head_dimension, cfg.mrope_section,
                                                   interleaved=cfg.mrope_interleaved), dtype=torch.int32)
        self.register_buffer("axis_of", axis, persistent=False)

    def token_embeddings(self, ids: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        return torch.nn.functional.embedding(ids.long(), self.embed_tokens).to(dtype)

    def forward(self, emb: torch.Tensor, seg: N.Segments, pos: torch.Tensor, *,
                deepstack: Sequence[torch.Tensor] = (), visual_rows: torch.Tensor | None = None,
                all_layers: bool = False):
        """``pos``: int [T] or [3, T]; ``deepstack[i]`` is added to ``visual_rows`` after layer i."""

        cfg = self.config
        pos = pos if pos.dim() == 2 else pos[None]
        axis = self.axis_of if pos.shape[0] > 1 else None
        h = emb
        states = [h]
        for i, layer in enumerate(self.layers):
            h = layer(h, seg, pos, axis, self.inv_freq, cfg)
            if i < len(deepstack):
                h = h.index_add(0, visual_rows, deepstack[i].to(h.dtype))
            if all_layers:
                states.append(h)
        h = N.rms_norm(h, self.norm, cfg.norm_epsilon)
        if all_layers:
            states[-1] = h
            return states
        return h


def qwen3_layer_state(layer: Qwen3DecoderLayer, cfg: Qwen3TextConfig, prefix: str) -> dict[str, torch.Tensor]:
    """Hugging Face names of one decoder layer (q/k/v and gate/up split)."""

    d = cfg.head_dimension
    qd, kd, inter = cfg.num_attention_heads * d, cfg.num_key_value_heads * d, cfg.intermediate_size
    w = layer.qkv.detach()
    gu = layer.gate_up.detach()
    out = {
        prefix + "input_layernorm.weight": layer.input_norm.detach(),
        prefix + "self_attn.q_proj.weight": w[:qd], prefix + "self_attn.k_proj.weight": w[qd:qd + kd],
        prefix + "self_attn.v_proj.weight": w[qd + kd:], prefix + "self_attn.o_proj.weight": layer.o_proj.detach(),
        prefix + "post_attention_layernorm.weight": layer.post_norm.detach(),
        prefix + "mlp.gate_proj.weight": gu[:inter], prefix + "mlp.up_proj.weight": gu[inter:],
        prefix + "mlp.down_proj.weight": layer.down.detach(),
    }
    if layer.q_norm is not None:
        out[prefix + "self_attn.q_norm.weight"] = layer.q_norm.detach()
        out[prefix + "self_attn.k_norm.weight"] = layer.k_norm.detach()
    if layer.qkv_bias is not None:
        b = layer.qkv_bias.detach()
        out[prefix + "self_attn.q_proj.bias"] = b[:qd]
        out[prefix + "self_attn.k_proj.bias"] = b[qd:qd + kd]
        out[prefix + "self_attn.v_proj.bias"] = b[qd + kd:]
    return out


def load_qwen3_layer(layer: Qwen3DecoderLayer, tensors: Mapping[str, torch.Tensor], prefix: str) -> None:
    t = lambda n: tensors[prefix + n]  # noqa: E731
    with torch.no_grad():
        layer.input_norm.copy_(t("input_layernorm.weight"))
        layer.qkv.copy_(torch.cat([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                                   t("self_attn.v_proj.weight")]))
        layer.o_proj.copy_(t("self_attn.o_proj.weight"))
        if layer.q_norm is not None:
            layer.q_norm.copy_(t("self_attn.q_norm.weight"))
            layer.k_norm.copy_(t("self_attn.k_norm.weight"))
        if layer.qkv_bias is not None:
            layer.qkv_bias.copy_(torch.cat([t("self_attn.q_proj.bias"), t("self_attn.k_proj.bias"),
                                            t("self_attn.v_proj.bias")]))
        layer.post_norm.copy_(t("post_attention_layernorm.weight"))
        layer.gate_up.copy_(torch.cat([t("mlp.gate_proj.weight"), t("mlp.up_proj.weight")]))
        layer.down.copy_(t("mlp.down_proj.weight"))


def qwen3_tower_state(tower: Qwen3TextTower, prefix: str) -> dict[str, torch.Tensor]:
    out = {prefix + "embed_tokens.weight": tower.embed_tokens.detach(), prefix + "norm.weight": tower.norm.detach()}
    for i, layer in enumerate(tower.layers):
        out.update(qwen3_layer_state(layer, tower.config, f"{prefix}layers.{i}."))
    return out


def load_qwen3_tower(tower: Qwen3TextTower, tensors: Mapping[str, torch.Tensor], prefix: str) -> None:
    with torch.no_grad():
        tower.embed_tokens.copy_(tensors[prefix + "embed_tokens.weight"])
        tower.norm.copy_(tensors[prefix + "norm.weight"])
    for i, layer in enumerate(tower.layers):
        load_qwen3_layer(layer, tensors, f"{prefix}layers.{i}.")


def last_token_rows(seg: N.Segments) -> torch.Tensor:
    """Packed row index of each sequence's final token."""

    return (seg.cu_seqlens[1:] - 1).long().clamp_min(0)


__all__ = ["Qwen3DecoderLayer", "Qwen3TextConfig", "Qwen3TextTower", "last_token_rows", "load_qwen3_layer",
           "load_qwen3_tower", "qwen3_layer_state", "qwen3_tower_state"]
