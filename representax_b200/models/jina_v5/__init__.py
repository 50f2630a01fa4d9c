"""Jina v5 Omni Small, text path: Qwen3 decoder, last-token pooling, Matryoshka output.

Parity: src/representax/models/jina_v5/{config,model,checkpoint}.py and the
pinned loader of src/representax/integrations/jina.py:33-70 — checkpoint
tensors under ``language_model.`` (Qwen3 layout), causal attention, the
final valid token pooled, truncated to ``output_dimension`` and
L2-normalised.
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch
from torch import nn

from representax_b200.core.model import EncoderMetadata, Modality, Route
from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset, save_safetensors
from representax_b200.models.qwen3 import (
    Qwen3TextConfig,
    Qwen3TextTower,
    last_token_rows,
    load_qwen3_tower,
    qwen3_tower_state,
)
from representax_b200.models.text_batch import TokenBatch, packed_segments
from representax_b200.ops import nn as N
from representax_b200.precision import active_compute_dtype

JINA_V5_MODEL_ID = "jinaai/jina-embeddings-v5-omni-small"
_PREFIXES = ("language_model.", "model.language_model.", "model.", "")


class JinaV5TextEncoder(nn.Module):
    def __init__(self, config: Qwen3TextConfig, *, output_dimension: int | None = None, seed: int = 0,
                 model_id: str = "representax/jina-v5-text", revision: str = "random-init",
                 compute_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        self.config = config
        self.tower = Qwen3TextTower(config, torch.Generator().manual_seed(seed))
        out = output_dimension or config.hidden_size
        if not 0 < out <= config.hidden_size:
            raise ValueError("output_dimension must be in (0, hidden_size]")
        self.compute_dtype = compute_dtype
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision, output_dimension=out,
                                        routes=frozenset(Route), modalities=frozenset({Modality.TEXT}))

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None) -> TokenBatch:
        del token_type_ids
        return TokenBatch.from_arrays(input_ids=input_ids, attention_mask=attention_mask)

    def packed_hidden(self, batch: TokenBatch, *, all_layers: bool = False):
        dtype = active_compute_dtype(self.compute_dtype)
        pk, seg = packed_segments(batch, self.tower.embed_tokens.device)
        emb = self.tower.token_embeddings(pk.input_ids, dtype)
        return self.tower(emb, seg, pk.position_ids, all_layers=all_layers), seg

    def hidden_states(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        h, _ = self.packed_hidden(inputs)
        m = inputs.attention_mask.to(h.device).bool()
        out = h.new_zeros(m.shape + (h.shape[-1],))
        out[m] = h
        return out

    def _pool(self, h, seg):
        pooled = h[last_token_rows(seg), : self.metadata.output_dimension].float()
        return pooled / pooled.norm(dim=-1, keepdim=True).clamp_min(1e-12)

    def encode(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        return self._pool(h, seg)

    def encode_layers(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        states, seg = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([self._pool(s, seg) for s in states])


class JinaV5CheckpointAdapter:
    @staticmethod
    def state_dict(model: JinaV5TextEncoder) -> dict[str, torch.Tensor]:
        return {k: v.float().cpu().contiguous() for k, v in qwen3_tower_state(model.tower, "language_model.").items()}

    @classmethod
    def from_state_dict(cls, model: JinaV5TextEncoder, tensors: Mapping[str, torch.Tensor]) -> JinaV5TextEncoder:
        for prefix in _PREFIXES:
            if prefix + "embed_tokens.weight" in tensors:
                load_qwen3_tower(model.tower, tensors, prefix)
                return model
        raise KeyError("checkpoint has no Qwen3 text tower")

    @classmethod
    def load(cls, path: str | os.PathLike, *, output_dimension: int | None = None,
             compute_dtype: torch.dtype = torch.float32, **kwargs) -> JinaV5TextEncoder:
        path = Path(path)
        hf = load_hf_config(path)
        cfg = Qwen3TextConfig.from_hf_config(hf)
        kwargs.setdefault("model_id", path.name)
        kwargs.setdefault("revision", "local")
        model = JinaV5TextEncoder(cfg, output_dimension=output_dimension or hf.get("output_dimension"),
                                  compute_dtype=compute_dtype, **kwargs)
        names = set()
        for prefix in _PREFIXES:
            names |= set(qwen3_tower_state(model.tower, prefix))
        return cls.from_state_dict(model, load_safetensor_subset(path, names))

    @classmethod
    def save(cls, model: JinaV5TextEncoder, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        cfg: dict[str, Any] = {"model_type": "qwen3", **model.config.to_hf_config(),
                               "output_dimension": model.metadata.output_dimension}
        with open(path / "config.json", "w") as handle:
            json.dump(cfg, handle, indent=2, sort_keys=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


def load_jina_v5_small_text_encoder(path: str | os.PathLike, **kwargs) -> JinaV5TextEncoder:
    """Pinned loader for a local Jina v5 Omni Small directory (text path)."""

    return JinaV5CheckpointAdapter.load(path, **kwargs)


__all__ = ["JINA_V5_MODEL_ID", "JinaV5CheckpointAdapter", "JinaV5TextEncoder", "load_jina_v5_small_text_encoder"]
