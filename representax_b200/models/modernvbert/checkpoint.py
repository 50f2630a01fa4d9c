"""ModernVBERT <-> Hugging Face safetensors (Transformers ``ModernVBertModel`` layout).

Parity: src/representax/models/modernvbert/checkpoint.py (name mapping,
fused / split q-k-v handling, sharded safetensors, config round trip). The
tensor names are the upstream ones so exported bundles load in Transformers.
SigLIP q/k/v projections are fused into one ``[3H, H]`` matrix natively and
split again on save; the patch convolution is stored flattened.
"""

from __future__ import annotations

import json
import os
from collections.abc import Callable, Iterator, Mapping
from pathlib import Path

import torch

from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset, save_safetensors

from .config import ModernVBERTConfig, ModernVBERTTextConfig
from .model import ModernBertTextTower, ModernVBERTEncoder, ModernVBERTTextEncoder, SigLIPVisionTower

# (hf name, getter of the native parameter, split index or None)
Entry = tuple[str, Callable[[], torch.nn.Parameter]]


def _text_entries(tower: ModernBertTextTower, prefix: str) -> Iterator[tuple[str, torch.nn.Parameter]]:
    yield f"{prefix}embeddings.tok_embeddings.weight", tower.tok_embeddings
    yield f"{prefix}embeddings.norm.weight", tower.emb_norm
    for i, layer in enumerate(tower.layers):
        p = f"{prefix}layers.{i}."
        if layer.attn_norm is not None:
            yield p + "attn_norm.weight", layer.attn_norm
        yield p + "attn.Wqkv.weight", layer.Wqkv
        yield p + "attn.Wo.weight", layer.Wo
        yield p + "mlp_norm.weight", layer.mlp_norm
        yield p + "mlp.Wi.weight", layer.Wi
        yield p + "mlp.Wo.weight", layer.mlp_Wo
    yield f"{prefix}final_norm.weight", tower.final_norm


def _vision_state(tower: SigLIPVisionTower, prefix: str) -> dict[str, torch.Tensor]:
    cfg = tower.config
    out: dict[str, torch.Tensor] = {}
    e = f"{prefix}embeddings."
    out[e + "patch_embedding.weight"] = tower.patch_w.detach().reshape(
        cfg.hidden_size, cfg.num_channels, cfg.patch_size, cfg.patch_size)
    out[e + "patch_embedding.bias"] = tower.patch_b.detach()
    out[e + "position_embedding.weight"] = tower.position.detach()
    h = cfg.hidden_size
    for i, layer in enumerate(tower.layers):
        p = f"{prefix}encoder.layers.{i}."
        for j, name in enumerate(("q_proj", "k_proj", "v_proj")):
            out[p + f"self_attn.{name}.weight"] = layer.qkv_w.detach()[j * h:(j + 1) * h]
            out[p + f"self_attn.{name}.bias"] = layer.qkv_b.detach()[j * h:(j + 1) * h]
        for attr, name in (("out", "self_attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2"),
                           ("ln1", "layer_norm1"), ("ln2", "layer_norm2")):
            out[p + name + ".weight"] = getattr(layer, attr + "_w").detach()
            out[p + name + ".bias"] = getattr(layer, attr + "_b").detach()
    out[f"{prefix}post_layernorm.weight"] = tower.post_w.detach()
    out[f"{prefix}post_layernorm.bias"] = tower.post_b.detach()
    return out


def _load_vision(tower: SigLIPVisionTower, tensors: Mapping[str, torch.Tensor], prefix: str) -> None:
    cfg = tower.config
    e = f"{prefix}embeddings."
    with torch.no_grad():
        tower.patch_w.copy_(tensors[e + "patch_embedding.weight"].reshape(cfg.hidden_size, -1))
        tower.patch_b.copy_(tensors[e + "patch_embedding.bias"])
        tower.position.copy_(tensors[e + "position_embedding.weight"])
        for i, layer in enumerate(tower.layers):
            p = f"{prefix}encoder.layers.{i}."
            layer.qkv_w.copy_(torch.cat([tensors[p + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")]))
            layer.qkv_b.copy_(torch.cat([tensors[p + f"self_attn.{n}.bias"] for n in ("q_proj", "k_proj", "v_proj")]))
            for attr, name in (("out", "self_attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2"),
                               ("ln1", "layer_norm1"), ("ln2", "layer_norm2")):
                getattr(layer, attr + "_w").copy_(tensors[p + name + ".weight"])
                getattr(layer, attr + "_b").copy_(tensors[p + name + ".bias"])
        tower.post_w.copy_(tensors[f"{prefix}post_layernorm.weight"])
        tower.post_b.copy_(tensors[f"{prefix}post_layernorm.bias"])


_VISION_PREFIXES = ("vision_model.vision_model.", "vision_model.", "model.vision_model.")
_TEXT_PREFIXES = ("text_model.", "model.text_model.")


class ModernVBERTCheckpointAdapter:
    """Load / save :class:`ModernVBERTEncoder` (and the text-only encoder)."""

    @staticmethod
    def state_dict(model) -> dict[str, torch.Tensor]:
        if isinstance(model, ModernVBERTTextEncoder):
            return {n: p.detach() for n, p in _text_entries(model.tower, "")}
        out = {n: p.detach() for n, p in _text_entries(model.text, "text_model.")}
        out.update(_vision_state(model.vision, "vision_model.vision_model."))
        out["connector.modality_projection.weight"] = model.connector.detach()
        return {k: v.float().cpu().contiguous() for k, v in out.items()}

    @staticmethod
    def _pick(tensors: Mapping[str, torch.Tensor], prefixes, probe: str) -> str:
        for prefix in prefixes:
            if prefix + probe in tensors:
                return prefix
        raise KeyError(f"checkpoint has no tensor ending in {probe!r}")

    @classmethod
    def from_state_dict(cls, model, tensors: Mapping[str, torch.Tensor]):
        text = model.tower if isinstance(model, ModernVBERTTextEncoder) else model.text
        tp = cls._pick(tensors, ("",) + _TEXT_PREFIXES if isinstance(model, ModernVBERTTextEncoder) else _TEXT_PREFIXES,
                       "embeddings.tok_embeddings.weight")
        with torch.no_grad():
            for name, param in _text_entries(text, tp):
                value = tensors[name]
                if tuple(value.shape) != tuple(param.shape):
                    raise ValueError(f"{name}: shape {tuple(value.shape)} != {tuple(param.shape)}")
                param.copy_(value.to(param.dtype))
        if isinstance(model, ModernVBERTEncoder):
            vp = cls._pick(tensors, _VISION_PREFIXES, "post_layernorm.weight")
            _load_vision(model.vision, tensors, vp)
            for name in ("connector.modality_projection.weight", "model.connector.modality_projection.weight"):
                if name in tensors:
                    with torch.no_grad():
                        model.connector.copy_(tensors[name])
                    break
            else:
                raise KeyError("checkpoint has no connector.modality_projection.weight")
        return model

    @classmethod
    def load(cls, path: str | os.PathLike, *, text_only: bool = False, compute_dtype: torch.dtype = torch.float32,
             **kwargs):
        path = Path(path)
        hf = load_hf_config(path)
        kwargs.setdefault("model_id", path.name)
        kwargs.setdefault("revision", "local")
        if text_only or hf.get("model_type") == "modernbert":
            model = ModernVBERTTextEncoder(ModernVBERTTextConfig.from_hf_config(hf), compute_dtype=compute_dtype,
                                           **kwargs)
        else:
            model = ModernVBERTEncoder(ModernVBERTConfig.from_hf_config(hf), compute_dtype=compute_dtype, **kwargs)
        from safetensors import safe_open

        from representax_b200.integrations.huggingface import _weight_files

        names = set()
        for file in _weight_files(path):
            with safe_open(str(file), framework="pt") as handle:
                names |= set(handle.keys())
        return cls.from_state_dict(model, load_safetensor_subset(path, names))

    @classmethod
    def save(cls, model, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        cfg = model.config.to_hf_config()
        with open(path / "config.json", "w") as handle:
            json.dump(cfg, handle, indent=2, sort_keys=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


__all__ = ["ModernVBERTCheckpointAdapter"]
