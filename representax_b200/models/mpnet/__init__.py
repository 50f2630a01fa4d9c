"""MPNet encoder: post-LN BERT layers with a shared relative-position bias.

Parity: ``create_mpnet_position_ids``, ``mpnet_relative_position_bucket``,
``MPNetConfig``, ``MPNetEncoder`` and ``MPNetCheckpointAdapter`` of
src/representax/models/mpnet/{model,config,checkpoint}.py: padding-aware
position ids (cumulative count of non-padding tokens offset by the padding
index), a [buckets, heads] relative-attention bias shared by every layer and
added to the attention scores, GELU MLP, mean pooling + L2, Hugging Face
tensor names (``encoder.layer.{i}.attention.attn.q.weight`` ...).

The relative bias depends only on ``j - i``, so the native path turns the
bucket table into a per-head lookup over signed distances and the attention
kernels add it to the scores in-kernel (and reduce its gradient per CTA).
"""

from __future__ import annotations

import json
import math
import os
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch
from torch import nn

from representax_b200._config import FrozenConfig
from representax_b200.core import EncoderMetadata, Modality, Route
from representax_b200.models import components as cmp
from representax_b200.models.text_batch import TokenBatch
from representax_b200.precision import active_compute_dtype


class MPNetConfig(FrozenConfig):
    vocab_size: int = 30527
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    max_position_embeddings: int = 514
    relative_attention_num_buckets: int = 32
    hidden_activation: str = "gelu"
    hidden_dropout_probability: float = 0.1
    attention_dropout_probability: float = 0.1
    norm_epsilon: float = 1e-5
    initializer_range: float = 0.02
    pad_token_id: int = 1

    @property
    def head_dimension(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "MPNetConfig":
        return cls(vocab_size=int(value["vocab_size"]), hidden_size=int(value["hidden_size"]),
                   intermediate_size=int(value["intermediate_size"]),
                   num_hidden_layers=int(value["num_hidden_layers"]),
                   num_attention_heads=int(value["num_attention_heads"]),
                   max_position_embeddings=int(value["max_position_embeddings"]),
                   relative_attention_num_buckets=int(value.get("relative_attention_num_buckets", 32)),
                   hidden_activation=str(value.get("hidden_act", "gelu")),
                   hidden_dropout_probability=float(value.get("hidden_dropout_prob", 0.1)),
                   attention_dropout_probability=float(value.get("attention_probs_dropout_prob", 0.1)),
                   norm_epsilon=float(value.get("layer_norm_eps", 1e-5)),
                   initializer_range=float(value.get("initializer_range", 0.02)),
                   pad_token_id=int(value.get("pad_token_id", 1)))

    def to_hf_config(self) -> dict[str, Any]:
        return {"architectures": ["MPNetModel"], "model_type": "mpnet", "vocab_size": self.vocab_size,
                "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
                "num_hidden_layers": self.num_hidden_layers, "num_attention_heads": self.num_attention_heads,
                "max_position_embeddings": self.max_position_embeddings,
                "relative_attention_num_buckets": self.relative_attention_num_buckets,
                "hidden_act": self.hidden_activation, "hidden_dropout_prob": self.hidden_dropout_probability,
                "attention_probs_dropout_prob": self.attention_dropout_probability,
                "layer_norm_eps": self.norm_epsilon, "initializer_range": self.initializer_range,
                "pad_token_id": self.pad_token_id}


def create_mpnet_position_ids(input_ids: torch.Tensor, *, padding_index: int = 1) -> torch.Tensor:
    mask = (input_ids != padding_index).to(input_ids.dtype)
    return torch.cumsum(mask, dim=1) * mask + padding_index


def mpnet_relative_position_bucket(relative_position: torch.Tensor, *, num_buckets: int = 32,
                                   max_distance: int = 128) -> torch.Tensor:
    if num_buckets < 4 or num_buckets % 2:
        raise ValueError("num_buckets must be even and >= 4")
    if max_distance <= num_buckets // 4:
        raise ValueError("max_distance must exceed the exact bucket range")
    distance = -relative_position
    half = num_buckets // 2
    direction = (distance < 0).to(torch.int64) * half
    distance = distance.abs()
    max_exact = half // 2
    small = distance < max_exact
    safe = torch.clamp(distance, min=max_exact).to(torch.float32)
    log = max_exact + (torch.log(safe / max_exact) / math.log(max_distance / max_exact)
                       * (half - max_exact)).to(torch.int64)
    log = torch.clamp(log, max=half - 1)
    return direction + torch.where(small, distance, log)


def relative_bias_lut(table: torch.Tensor, max_len: int, num_buckets: int) -> torch.Tensor:
    """[heads, 2 * max_len - 1] bias over signed distances d = j - i (index d + max_len - 1)."""

    d = torch.arange(-(max_len - 1), max_len, device=table.device)
    buckets = mpnet_relative_position_bucket(d, num_buckets=num_buckets)
    return table[buckets].T.contiguous().float()


class MPNetLayer(nn.Module):
    def __init__(self, config: MPNetConfig, generator=None) -> None:
        super().__init__()
        h, f, r = config.hidden_size, config.intermediate_size, config.initializer_range
        p = lambda t: nn.Parameter(t)  # noqa: E731
        self.qkv_weight = p(torch.randn(3 * h, h, generator=generator) * r)
        self.qkv_bias = p(torch.zeros(3 * h))
        self.out_weight = p(torch.randn(h, h, generator=generator) * r)
        self.out_bias = p(torch.zeros(h))
        self.attn_norm_weight = p(torch.ones(h))
        self.attn_norm_bias = p(torch.zeros(h))
        self.ffn_in_weight = p(torch.randn(f, h, generator=generator) * r)
        self.ffn_in_bias = p(torch.zeros(f))
        self.ffn_out_weight = p(torch.randn(h, f, generator=generator) * r)
        self.ffn_out_bias = p(torch.zeros(h))
        self.out_norm_weight = p(torch.ones(h))
        self.out_norm_bias = p(torch.zeros(h))


class MPNetEncoder(nn.Module):
    def __init__(self, config: MPNetConfig, *, seed: int = 0, model_id: str = "representax/mpnet",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32,
                 pooling: str = "mean", normalize: bool = True) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        r, h = config.initializer_range, config.hidden_size
        self.config = config
        word = torch.randn(config.vocab_size, h, generator=g) * r
        word[config.pad_token_id] = 0
        self.word = nn.Parameter(word)
        self.position = nn.Parameter(torch.randn(config.max_position_embeddings, h, generator=g) * r)
        self.emb_norm_weight = nn.Parameter(torch.ones(h))
        self.emb_norm_bias = nn.Parameter(torch.zeros(h))
        self.relative_attention_bias = nn.Parameter(
            torch.randn(config.relative_attention_num_buckets, config.num_attention_heads, generator=g) * r)
        self.layers = nn.ModuleList(MPNetLayer(config, g) for _ in range(config.num_hidden_layers))
        self.pooler_weight = nn.Parameter(torch.randn(h, h, generator=g) * r)
        self.pooler_bias = nn.Parameter(torch.zeros(h))
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision, output_dimension=h,
                                        routes=frozenset(Route), modalities=frozenset({Modality.TEXT}))
        self.compute_dtype = compute_dtype
        self.pooling = pooling
        self.normalize = normalize

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None) -> TokenBatch:
        del token_type_ids  # MPNet has no segment embeddings
        return TokenBatch.from_arrays(input_ids=input_ids, attention_mask=attention_mask)

    def _dtype(self):
        return active_compute_dtype(self.compute_dtype)

    # ------------------------------------------------------------ native path
    def _native(self, batch: TokenBatch) -> bool:
        pk = batch.packed
        return (pk is not None and pk.input_ids.is_cuda and self._dtype() == torch.bfloat16
                and self.config.head_dimension == 64 and self.config.hidden_activation == "gelu")

    def _rel_buckets(self, max_len: int, device) -> torch.Tensor:
        cache = getattr(self, "_bucket_cache", {})
        key = (max_len, str(device))
        if key not in cache:
            d = torch.arange(-(max_len - 1), max_len, device=device)
            cache[key] = mpnet_relative_position_bucket(d, num_buckets=self.config.relative_attention_num_buckets)
            self._bucket_cache = cache
        return cache[key]

    def _native_hidden(self, batch: TokenBatch, generator=None):
        """Packed rows through the fused BERT-style blocks with the relative bias in the attention kernel."""

        from representax_b200.ops import functional as Fn

        cfg = self.config
        pk = batch.packed
        packed = Fn.Packed(cu_seqlens=pk.cu_seqlens, max_len=pk.max_len, total=pk.total)
        # MPNet positions count valid tokens from padding_index + 1 (right padding: column + 2)
        pos = pk.position_ids if batch.position_ids is not None else pk.position_ids + (cfg.pad_token_id + 1)
        if not hasattr(self, "_zero_types") or self._zero_types.device != pk.input_ids.device:
            self._zero_types = torch.zeros(1, cfg.hidden_size, device=pk.input_ids.device)
        p_h, p_a = cfg.hidden_dropout_probability, cfg.attention_dropout_probability
        seed = generator.initial_seed() if generator is not None and (p_h > 0 or p_a > 0) else None
        drop = (lambda site: None if seed is None else Fn.Dropout(seed, site, p_a, p_h))  # noqa: E731
        h = Fn.embed_layer_norm(pk.input_ids, pos, None, self.word, self.position, self._zero_types,
                                self.emb_norm_weight, self.emb_norm_bias, cfg.norm_epsilon, cfg.pad_token_id,
                                dropout=drop(0))
        buckets = self._rel_buckets(max(pk.max_len, 1), pk.input_ids.device)
        fused_bias = seed is None or p_h == 0
        for i, layer in enumerate(self.layers):
            s1 = Fn.attention_block(h, layer.qkv_weight, layer.qkv_bias, layer.out_weight, layer.out_bias, packed,
                                    heads=cfg.num_attention_heads, out_bias_grad_fused=fused_bias,
                                    dropout=drop(16 * (i + 1)), rel_table=self.relative_attention_bias,
                                    rel_buckets=buckets)
            h1 = Fn.layer_norm(s1, layer.attn_norm_weight, layer.attn_norm_bias, cfg.norm_epsilon,
                               producer_bias=layer.out_bias if fused_bias else None)
            s2 = Fn.mlp_block(h1, layer.ffn_in_weight, layer.ffn_in_bias, layer.ffn_out_weight, layer.ffn_out_bias,
                              out_bias_grad_fused=fused_bias, dropout=drop(16 * (i + 1)))
            h = Fn.layer_norm(s2, layer.out_norm_weight, layer.out_norm_bias, cfg.norm_epsilon,
                              producer_bias=layer.ffn_out_bias if fused_bias else None)
        return h, packed

    def hidden_states(self, batch: TokenBatch, *, generator=None) -> torch.Tensor:
        if self._native(batch):
            h, _ = self._native_hidden(batch, generator)
            m = batch.attention_mask.to(h.device).bool()
            out = h.new_zeros(m.shape + (h.shape[-1],))
            out[m] = h
            return out
        cfg = self.config
        dtype = self._dtype()
        ids = batch.input_ids.long()
        mask = batch.attention_mask.bool()
        s = ids.shape[1]
        pos = batch.position_ids.long() if batch.position_ids is not None else create_mpnet_position_ids(
            ids, padding_index=cfg.pad_token_id)
        word = self.word[ids]
        word = torch.where((ids == cfg.pad_token_id)[..., None], word.detach(), word)
        hidden = cmp.layer_norm(word + self.position[pos], self.emb_norm_weight, self.emb_norm_bias, cfg.norm_epsilon)
        hidden = cmp.dropout(hidden, cfg.hidden_dropout_probability, generator).to(dtype)
        idx = torch.arange(s, device=ids.device)
        buckets = mpnet_relative_position_bucket(idx[None, :] - idx[:, None],
                                                 num_buckets=cfg.relative_attention_num_buckets)
        bias = self.relative_attention_bias[buckets].permute(2, 0, 1)[None]
        b, heads, hd = ids.shape[0], cfg.num_attention_heads, cfg.head_dimension
        for layer in self.layers:
            w = lambda t: t.to(dtype)  # noqa: E731
            qkv = torch.nn.functional.linear(hidden, w(layer.qkv_weight), w(layer.qkv_bias))
            q, k, v = qkv.split(cfg.hidden_size, -1)
            shape = (b, s, heads, hd)
            att = cmp.dot_product_attention(q.reshape(shape), k.reshape(shape), v.reshape(shape), key_mask=mask,
                                            bias=bias, dropout_p=cfg.attention_dropout_probability,
                                            generator=generator)
            att = torch.nn.functional.linear(att.reshape(b, s, -1), w(layer.out_weight), w(layer.out_bias))
            att = cmp.dropout(att, cfg.hidden_dropout_probability, generator)
            hidden = cmp.layer_norm(hidden + att, w(layer.attn_norm_weight), w(layer.attn_norm_bias), cfg.norm_epsilon)
            mid = cmp.activate(torch.nn.functional.linear(hidden, w(layer.ffn_in_weight), w(layer.ffn_in_bias)),
                               cfg.hidden_activation)
            out = torch.nn.functional.linear(mid, w(layer.ffn_out_weight), w(layer.ffn_out_bias))
            out = cmp.dropout(out, cfg.hidden_dropout_probability, generator)
            hidden = cmp.layer_norm(hidden + out, w(layer.out_norm_weight), w(layer.out_norm_bias), cfg.norm_epsilon)
        return hidden

    def encode(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        del route
        if self._native(inputs) and self.pooling in ("mean", "cls", "first", "last", "lasttoken"):
            from representax_b200.ops import functional as Fn

            h, packed = self._native_hidden(inputs, generator)
            return Fn.pool(h, packed, self.pooling, self.normalize)
        hidden = self.hidden_states(inputs, generator=generator)
        mask = inputs.attention_mask
        if self.pooling == "mean":
            pooled = cmp.mean_pool(hidden, mask)
        elif self.pooling in {"cls", "first"}:
            pooled = hidden[:, 0].float()
        else:
            pooled = cmp.last_token_pool(hidden, mask)
        return cmp.l2_normalize(pooled) if self.normalize else pooled


_LAYER = {"out_weight": "attention.attn.o.weight", "out_bias": "attention.attn.o.bias",
          "attn_norm_weight": "attention.LayerNorm.weight", "attn_norm_bias": "attention.LayerNorm.bias",
          "ffn_in_weight": "intermediate.dense.weight", "ffn_in_bias": "intermediate.dense.bias",
          "ffn_out_weight": "output.dense.weight", "ffn_out_bias": "output.dense.bias",
          "out_norm_weight": "output.LayerNorm.weight", "out_norm_bias": "output.LayerNorm.bias"}
_TOP = {"word": "embeddings.word_embeddings.weight", "position": "embeddings.position_embeddings.weight",
        "emb_norm_weight": "embeddings.LayerNorm.weight", "emb_norm_bias": "embeddings.LayerNorm.bias",
        "pooler_weight": "pooler.dense.weight", "pooler_bias": "pooler.dense.bias"}


class MPNetCheckpointAdapter:
    @staticmethod
    def state_dict(model: MPNetEncoder) -> dict[str, torch.Tensor]:
        out = {name: getattr(model, attr).detach().float().cpu().contiguous() for attr, name in _TOP.items()}
        out["encoder.relative_attention_bias.weight"] = model.relative_attention_bias.detach().float().cpu()
        h = model.config.hidden_size
        for i, layer in enumerate(model.layers):
            p = f"encoder.layer.{i}."
            w, b = layer.qkv_weight.detach().float().cpu(), layer.qkv_bias.detach().float().cpu()
            for j, part in enumerate("qkv"):
                out[f"{p}attention.attn.{part}.weight"] = w[j * h:(j + 1) * h].contiguous()
                out[f"{p}attention.attn.{part}.bias"] = b[j * h:(j + 1) * h].contiguous()
            for attr, name in _LAYER.items():
                out[p + name] = getattr(layer, attr).detach().float().cpu().contiguous()
        return out

    @staticmethod
    def from_state_dict(model: MPNetEncoder, tensors: Mapping[str, torch.Tensor]) -> MPNetEncoder:
        with torch.no_grad():
            for attr, name in _TOP.items():
                getattr(model, attr).copy_(tensors[name])
            model.relative_attention_bias.copy_(tensors["encoder.relative_attention_bias.weight"])
            for i, layer in enumerate(model.layers):
                p = f"encoder.layer.{i}."
                layer.qkv_weight.copy_(torch.cat([tensors[f"{p}attention.attn.{x}.weight"] for x in "qkv"]))
                layer.qkv_bias.copy_(torch.cat([tensors[f"{p}attention.attn.{x}.bias"] for x in "qkv"]))
                for attr, name in _LAYER.items():
                    getattr(layer, attr).copy_(tensors[p + name])
        return model

    @classmethod
    def load(cls, path, **kwargs) -> MPNetEncoder:
        from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset

        config = MPNetConfig.from_hf_config(load_hf_config(path))
        kwargs.setdefault("model_id", Path(path).name)
        model = MPNetEncoder(config, **kwargs)
        names = set(cls.state_dict(model))
        return cls.from_state_dict(model, load_safetensor_subset(path, names, prefixes=("", "mpnet.")))

    @classmethod
    def save(cls, model: MPNetEncoder, path) -> None:
        from representax_b200.integrations.huggingface import save_safetensors

        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        (path / "config.json").write_text(json.dumps(model.config.to_hf_config(), indent=2, sort_keys=True))
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


def build_mpnet(*, seed: int = 0, compute_dtype: str = "float32", **config) -> MPNetEncoder:
    return MPNetEncoder(MPNetConfig(**config), seed=seed, compute_dtype=getattr(torch, compute_dtype))


__all__ = ["MPNetCheckpointAdapter", "MPNetConfig", "MPNetEncoder", "build_mpnet", "create_mpnet_position_ids",
           "mpnet_relative_position_bucket", "relative_bias_lut"]
