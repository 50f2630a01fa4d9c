"""Hugging Face safetensors <-> native BERT parameters.

Parity: ``bert_weight_names`` and ``BertCheckpointAdapter`` of
src/representax/models/bert/checkpoint.py:32-333. Files use the upstream
tensor names (``encoder.layer.{i}.attention.self.query.weight`` ...) so a
checkpoint written here loads in Transformers and vice versa; the fused QKV
parameter is split / concatenated at this boundary.
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping
from pathlib import Path

import torch

from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset, save_safetensors

from .config import BertConfig
from .model import BertEncoder

_LAYER_MAP = {
    "out_weight": "attention.output.dense.weight",
    "out_bias": "attention.output.dense.bias",
    "attn_norm_weight": "attention.output.LayerNorm.weight",
    "attn_norm_bias": "attention.output.LayerNorm.bias",
    "ffn_in_weight": "intermediate.dense.weight",
    "ffn_in_bias": "intermediate.dense.bias",
    "ffn_out_weight": "output.dense.weight",
    "ffn_out_bias": "output.dense.bias",
    "out_norm_weight": "output.LayerNorm.weight",
    "out_norm_bias": "output.LayerNorm.bias",
}
_EMB_MAP = {
    "word": "embeddings.word_embeddings.weight",
    "position": "embeddings.position_embeddings.weight",
    "token_type": "embeddings.token_type_embeddings.weight",
    "norm_weight": "embeddings.LayerNorm.weight",
    "norm_bias": "embeddings.LayerNorm.bias",
}


def bert_weight_names(config: BertConfig) -> frozenset[str]:
    names = set(_EMB_MAP.values()) | {"pooler.dense.weight", "pooler.dense.bias"}
    for i in range(config.num_hidden_layers):
        p = f"encoder.layer.{i}."
        names.update(p + n for n in _LAYER_MAP.values())
        for part in ("query", "key", "value"):
            names.update({f"{p}attention.self.{part}.weight", f"{p}attention.self.{part}.bias"})
    return frozenset(names)


class BertCheckpointAdapter:
    """Load / save native BERT encoders in the upstream safetensors layout."""

    @staticmethod
    def state_dict(model: BertEncoder) -> dict[str, torch.Tensor]:
        out: dict[str, torch.Tensor] = {}
        e = model.embeddings
        for attr, name in _EMB_MAP.items():
            out[name] = getattr(e, attr).detach().float().cpu().contiguous()
        h = model.config.hidden_size
        for i, layer in enumerate(model.layers):
            p = f"encoder.layer.{i}."
            w = layer.qkv_weight.detach().float().cpu()
            b = layer.qkv_bias.detach().float().cpu()
            for j, part in enumerate(("query", "key", "value")):
                out[f"{p}attention.self.{part}.weight"] = w[j * h:(j + 1) * h].contiguous()
                out[f"{p}attention.self.{part}.bias"] = b[j * h:(j + 1) * h].contiguous()
            for attr, name in _LAYER_MAP.items():
                out[p + name] = getattr(layer, attr).detach().float().cpu().contiguous()
        out["pooler.dense.weight"] = model.pooler_weight.detach().float().cpu().contiguous()
        out["pooler.dense.bias"] = model.pooler_bias.detach().float().cpu().contiguous()
        return out

    @staticmethod
    def from_state_dict(model: BertEncoder, tensors: Mapping[str, torch.Tensor], *, strict: bool = True) -> BertEncoder:
        expected = bert_weight_names(model.config)
        present = set(tensors)
        missing = sorted(expected - present)
        if strict and missing:
            raise KeyError(f"checkpoint is missing tensors: {missing[:5]}{'...' if len(missing) > 5 else ''}")

        def put(param: torch.nn.Parameter, value: torch.Tensor) -> None:
            if tuple(value.shape) != tuple(param.shape):
                raise ValueError(f"shape mismatch {tuple(value.shape)} vs {tuple(param.shape)}")
            with torch.no_grad():
                param.copy_(value.to(param.dtype))

        e = model.embeddings
        for attr, name in _EMB_MAP.items():
            if name in tensors:
                put(getattr(e, attr), tensors[name])
        for i, layer in enumerate(model.layers):
            p = f"encoder.layer.{i}."
            parts = [p + f"attention.self.{x}" for x in ("query", "key", "value")]
            if all(n + ".weight" in tensors for n in parts):
                put(layer.qkv_weight, torch.cat([tensors[n + ".weight"] for n in parts]))
                put(layer.qkv_bias, torch.cat([tensors[n + ".bias"] for n in parts]))
            for attr, name in _LAYER_MAP.items():
                if p + name in tensors:
                    put(getattr(layer, attr), tensors[p + name])
        if "pooler.dense.weight" in tensors:
            put(model.pooler_weight, tensors["pooler.dense.weight"])
            put(model.pooler_bias, tensors["pooler.dense.bias"])
        return model

    @classmethod
    def load(cls, path: str | os.PathLike, *, model_id: str | None = None, revision: str = "local",
             compute_dtype: torch.dtype = torch.float32, **kwargs) -> BertEncoder:
        path = Path(path)
        config = BertConfig.from_hf_config(load_hf_config(path))
        model = BertEncoder(config, model_id=model_id or path.name, revision=revision,
                            compute_dtype=compute_dtype, **kwargs)
        names = bert_weight_names(config)
        tensors = load_safetensor_subset(path, names, prefixes=("", "bert."))
        return cls.from_state_dict(model, tensors)

    @classmethod
    def save(cls, model: BertEncoder, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        with open(path / "config.json", "w") as handle:
            json.dump(model.config.to_hf_config(), handle, indent=2, sort_keys=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


__all__ = ["BertCheckpointAdapter", "bert_weight_names"]
