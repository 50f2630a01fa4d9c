"""Sentence-Transformers module chain over token-level backbones.

Parity: src/representax/models/sentence.py:38-294 — ``SentencePooling``
(cls, max, mean, mean_sqrt_len_tokens, weightedmean, lasttoken; several
modes concatenate), ``SentenceDense`` (Linear + identity/tanh/relu/gelu/silu),
``SentenceNormalize``, ``SentenceBatch`` (backbone inputs plus a prompt-aware
pooling mask) and ``SentenceEncoder`` (backbone -> pooling ->
postprocessors -> optional Matryoshka truncation; ``encode_layers`` applies
the chain at every depth). The numerics follow Sentence-Transformers 5.x:
means divide by max(count, 1e-9); the last-token mode zeroes padding and
falls back to the final position when a row has no valid token.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch import nn

from representax_b200.core.model import EncoderMetadata, Route

POOLING_MODES = ("cls", "max", "mean", "mean_sqrt_len_tokens", "weightedmean", "lasttoken")
DENSE_ACTIVATIONS = ("identity", "tanh", "relu", "gelu", "silu")


class SentencePooling(nn.Module):
    """Padded-token pooling with Sentence-Transformers semantics."""

    def __init__(self, input_dimension: int, modes: tuple[str, ...] = ("mean",), include_prompt: bool = True) -> None:
        super().__init__()
        modes = (modes,) if isinstance(modes, str) else tuple(modes)
        unknown = [m for m in modes if m not in POOLING_MODES]
        if input_dimension < 1 or not modes or unknown:
            raise ValueError(f"SentencePooling({input_dimension}, {modes}): width >= 1 and modes from "
                             f"{sorted(POOLING_MODES)} required")
        self.input_dimension = input_dimension
        self.modes = modes
        self.include_prompt = include_prompt

    @property
    def output_dimension(self) -> int:
        return self.input_dimension * len(self.modes)

    def forward(self, hidden: torch.Tensor, attention_mask: torch.Tensor) -> torch.Tensor:
        expected = (*attention_mask.shape, self.input_dimension)
        if tuple(hidden.shape) != expected:
            raise ValueError(f"pooling got token states {tuple(hidden.shape)} for a mask of "
                             f"{tuple(attention_mask.shape)}; expected {expected}")
        valid = attention_mask.to(hidden.device).bool()
        mask = valid[..., None].to(hidden.dtype)
        b, s, _ = hidden.shape
        rows = torch.arange(b, device=hidden.device)
        outs = []
        mean_sum = mean_count = None
        for mode in self.modes:
            if mode == "cls":
                outs.append(hidden[rows, valid.int().argmax(1)])
            elif mode == "max":
                outs.append(hidden.masked_fill(~valid[..., None], float("-inf")).amax(1))
            elif mode in ("mean", "mean_sqrt_len_tokens"):
                if mean_sum is None:
                    mean_sum = (hidden * mask).sum(1)
                    mean_count = mask.sum(1).clamp_min(1e-9)
                div = mean_count if mode == "mean" else mean_count.float().sqrt().to(hidden.dtype)
                outs.append(mean_sum / div)
            elif mode == "weightedmean":
                weights = torch.arange(1, s + 1, device=hidden.device, dtype=hidden.dtype)[None, :, None]
                wm = mask * weights
                outs.append((hidden * wm).sum(1) / wm.sum(1).clamp_min(1e-9))
            else:  # lasttoken
                rev = valid.flip(1)
                found = rev.any(1)
                last = s - 1 - rev.int().argmax(1)
                last = torch.where(found, last, torch.full_like(last, s - 1))
                outs.append((hidden * mask)[rows, last])
        return torch.cat(outs, dim=-1)


class SentenceDense(nn.Module):
    """One Dense postprocessor (``linear.weight`` in [out, in] layout)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, activation: str = "tanh") -> None:
        super().__init__()
        if activation not in DENSE_ACTIVATIONS:
            raise ValueError(f"Dense activation {activation!r} is not implemented")
        self.weight = nn.Parameter(weight.detach().clone().float())
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone().float())
        self.activation = activation

    @property
    def output_dimension(self) -> int:
        return self.weight.shape[0]

    def forward(self, value: torch.Tensor) -> torch.Tensor:
        b = None if self.bias is None else self.bias.to(value.dtype)
        value = torch.nn.functional.linear(value, self.weight.to(value.dtype), b)
        if self.activation == "tanh":
            return torch.tanh(value)
        if self.activation == "relu":
            return torch.relu(value)
        if self.activation == "gelu":
            return torch.nn.functional.gelu(value)
        if self.activation == "silu":
            return torch.nn.functional.silu(value)
        return value


class SentenceNormalize(nn.Module):
    def forward(self, value: torch.Tensor) -> torch.Tensor:
        v = value.float()
        return v / v.norm(dim=-1, keepdim=True).clamp_min(1e-12)


@dataclass
class SentenceBatch:
    """Backbone inputs plus the pooling mask (prompt tokens removed)."""

    backbone_inputs: Any
    pooling_mask: Any

    def __post_init__(self) -> None:
        if not isinstance(self.pooling_mask, torch.Tensor):
            self.pooling_mask = torch.as_tensor(self.pooling_mask)

    @property
    def batch_size(self) -> int:
        return int(self.pooling_mask.shape[0])

    def map_tensors(self, fn) -> "SentenceBatch":
        inner = self.backbone_inputs
        inner = inner.map_tensors(fn) if hasattr(inner, "map_tensors") else fn(inner)
        return SentenceBatch(inner, fn(self.pooling_mask))

    def rows(self, start: int, stop: int) -> "SentenceBatch":
        return SentenceBatch(self.backbone_inputs.rows(start, stop), self.pooling_mask[start:stop])


class SentenceEncoder(nn.Module):
    """A token backbone plus serialized dense sentence modules."""

    def __init__(self, backbone: nn.Module, pooling: SentencePooling, postprocessors=(),
                 metadata: EncoderMetadata | None = None, truncate_dimension: int | None = None) -> None:
        super().__init__()
        self.backbone = backbone
        self.pooling = pooling
        self.postprocessors = nn.ModuleList(postprocessors)
        out = pooling.output_dimension
        for module in postprocessors:
            out = getattr(module, "output_dimension", out)
        if truncate_dimension is not None and not 0 < truncate_dimension <= out:
            raise ValueError("truncate_dimension is larger than the embedding or below 1")
        self.truncate_dimension = truncate_dimension
        if metadata is None:
            base = backbone.metadata
            metadata = EncoderMetadata(model_id=base.model_id, revision=base.revision,
                                       output_dimension=truncate_dimension or out, routes=base.routes,
                                       modalities=base.modalities)
        self.metadata = metadata

    @classmethod
    def load_from_hf(cls, model_name_or_path: str | Path, **options: Any):
        """Load weights and preprocessing from a local Sentence-Transformers directory."""

        from representax_b200.integrations.sentence_transformers import load_sentence_transformer

        for name in ("parameter_dtype", "compute_dtype"):
            if isinstance(options.get(name), str):
                options[name] = getattr(torch, options[name])
        loaded = load_sentence_transformer(model_name_or_path, **options)
        return loaded.model, loaded.processor

    def make_batch(self, *, input_ids, attention_mask, token_type_ids=None):
        builder = getattr(self.backbone, "make_batch", None)
        if not callable(builder):
            raise TypeError(f"{type(self.backbone).__name__} has no make_batch(); it cannot build token batches")
        return builder(input_ids=input_ids, attention_mask=attention_mask, token_type_ids=token_type_ids)

    @staticmethod
    def _split(inputs):
        if isinstance(inputs, SentenceBatch):
            return inputs.backbone_inputs, inputs.pooling_mask
        mask = getattr(inputs, "attention_mask", None)
        if mask is None:
            raise TypeError(f"{type(inputs).__name__} has no attention_mask to pool with")
        return inputs, mask

    def _post(self, value: torch.Tensor) -> torch.Tensor:
        for module in self.postprocessors:
            value = module(value)
        if self.truncate_dimension is not None:
            value = value[..., : self.truncate_dimension]
        return value

    def encode(self, inputs: Any, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        del route
        hidden_states = getattr(self.backbone, "hidden_states", None)
        if not callable(hidden_states):
            raise TypeError(f"{type(self.backbone).__name__} has no hidden_states(); nothing to pool")
        backbone_inputs, mask = self._split(inputs)
        return self._post(self.pooling(hidden_states(backbone_inputs, generator=generator), mask))

    def encode_layers(self, inputs: Any, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        del route
        layer_states = getattr(self.backbone, "hidden_states_by_layer", None)
        if not callable(layer_states):
            raise TypeError(f"{type(self.backbone).__name__} has no hidden_states_by_layer()")
        backbone_inputs, mask = self._split(inputs)
        states = layer_states(backbone_inputs, generator=generator)
        return torch.stack([self._post(self.pooling(h, mask)) for h in states])


SentencePostprocessor = SentenceDense | SentenceNormalize

__all__ = ["DENSE_ACTIVATIONS", "POOLING_MODES", "SentenceBatch", "SentenceDense", "SentenceEncoder",
           "SentenceNormalize", "SentencePooling", "SentencePostprocessor"]
