"""CLIP dual encoder with BGE-VL additive text+image composition.

Text tower: token + absolute position embeddings, causal pre-LN blocks
(quick-GELU MLP), final LayerNorm, pooled at the EOS token (the arg-max id
for legacy configs with ``eos_token_id == 2``), linear projection. Vision
tower: [CLS] + patch embeddings (bias-free patch projection) + positions,
pre-LayerNorm, blocks, post-LayerNorm of the [CLS] row, projection. A
sample may carry text, an image or both; the representation is the sum of
the valid parts, L2-normalised (BGE-VL composition).

Parity: src/representax/models/clip/{config,model,checkpoint}.py (M12).
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch import nn

from representax_b200._config import FrozenConfig
from representax_b200.core.model import EncoderMetadata, Modality, Route
from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset, save_safetensors
from representax_b200.models.modernvbert.model import VisionLayer, patchify
from representax_b200.models.text_batch import TokenBatch, packed_segments
from representax_b200.ops import nn as N
from representax_b200.precision import active_compute_dtype


class CLIPTextConfig(FrozenConfig):
    vocab_size: int = 49408
    hidden_size: int = 512
    intermediate_size: int = 2048
    num_hidden_layers: int = 12
    num_attention_heads: int = 8
    max_position_embeddings: int = 77
    hidden_activation: str = "quick_gelu"
    norm_epsilon: float = 1e-5
    eos_token_id: int = 2


class CLIPVisionConfig(FrozenConfig):
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    num_channels: int = 3
    image_size: int = 224
    patch_size: int = 32
    hidden_activation: str = "quick_gelu"
    norm_epsilon: float = 1e-5

    @property
    def num_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2


class CLIPConfig(FrozenConfig):
    text: CLIPTextConfig = CLIPTextConfig()
    vision: CLIPVisionConfig = CLIPVisionConfig()
    projection_dimension: int = 512
    logit_scale_init: float = 2.6592
    normalize_output: bool = True

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "CLIPConfig":
        t, v = value["text_config"], value["vision_config"]
        return cls(
            text=CLIPTextConfig(vocab_size=int(t["vocab_size"]), hidden_size=int(t["hidden_size"]),
                                intermediate_size=int(t["intermediate_size"]),
                                num_hidden_layers=int(t["num_hidden_layers"]),
                                num_attention_heads=int(t["num_attention_heads"]),
                                max_position_embeddings=int(t.get("max_position_embeddings", 77)),
                                hidden_activation=str(t.get("hidden_act", "quick_gelu")),
                                norm_epsilon=float(t.get("layer_norm_eps", 1e-5)),
                                eos_token_id=int(t.get("eos_token_id", 2))),
            vision=CLIPVisionConfig(hidden_size=int(v["hidden_size"]), intermediate_size=int(v["intermediate_size"]),
                                    num_hidden_layers=int(v["num_hidden_layers"]),
                                    num_attention_heads=int(v["num_attention_heads"]),
                                    num_channels=int(v.get("num_channels", 3)), image_size=int(v["image_size"]),
                                    patch_size=int(v["patch_size"]),
                                    hidden_activation=str(v.get("hidden_act", "quick_gelu")),
                                    norm_epsilon=float(v.get("layer_norm_eps", 1e-5))),
            projection_dimension=int(value.get("projection_dim", 512)),
            logit_scale_init=float(value.get("logit_scale_init_value", 2.6592)))

    def to_hf_config(self) -> dict[str, Any]:
        t, v = self.text, self.vision
        return {"model_type": "clip", "projection_dim": self.projection_dimension,
                "logit_scale_init_value": self.logit_scale_init,
                "text_config": {"vocab_size": t.vocab_size, "hidden_size": t.hidden_size,
                                "intermediate_size": t.intermediate_size, "num_hidden_layers": t.num_hidden_layers,
                                "num_attention_heads": t.num_attention_heads,
                                "max_position_embeddings": t.max_position_embeddings, "hidden_act": t.hidden_activation,
                                "layer_norm_eps": t.norm_epsilon, "eos_token_id": t.eos_token_id},
                "vision_config": {"hidden_size": v.hidden_size, "intermediate_size": v.intermediate_size,
                                  "num_hidden_layers": v.num_hidden_layers, "num_attention_heads": v.num_attention_heads,
                                  "num_channels": v.num_channels, "image_size": v.image_size,
                                  "patch_size": v.patch_size, "hidden_act": v.hidden_activation,
                                  "layer_norm_eps": v.norm_epsilon}}


@dataclass
class CLIPBatch:
    """Text ([B, S] ids + mask + per-sample validity), images ([B, C, H, W]), or both."""

    input_ids: torch.Tensor | None = None
    attention_mask: torch.Tensor | None = None
    text_valid: torch.Tensor | None = None
    pixel_values: torch.Tensor | None = None
    image_valid: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if self.input_ids is None and self.pixel_values is None:
            raise ValueError("CLIP batches require text, images, or both")
        if self.input_ids is not None:
            if self.attention_mask is None or self.attention_mask.shape != self.input_ids.shape:
                raise ValueError("attention_mask must align with input_ids")
            if self.text_valid is None:
                self.text_valid = torch.ones(self.input_ids.shape[0], dtype=torch.bool)
        if self.pixel_values is not None:
            if self.pixel_values.ndim != 4:
                raise ValueError("pixel_values must have shape [batch, channel, height, width]")
            if self.image_valid is None:
                self.image_valid = torch.ones(self.pixel_values.shape[0], dtype=torch.bool)
        if self.input_ids is not None and self.pixel_values is not None and \
                self.input_ids.shape[0] != self.pixel_values.shape[0]:
            raise ValueError("text and image inputs must share the sample dimension")

    @property
    def batch_size(self) -> int:
        return (self.input_ids if self.input_ids is not None else self.pixel_values).shape[0]

    def map_tensors(self, fn) -> "CLIPBatch":
        opt = lambda t: None if t is None else fn(t)  # noqa: E731
        return CLIPBatch(opt(self.input_ids), opt(self.attention_mask), opt(self.text_valid), opt(self.pixel_values),
                         opt(self.image_valid))


def _normal(shape, std, g):
    return nn.Parameter(torch.randn(*shape, generator=g) * std)


class CLIPEncoder(nn.Module):
    def __init__(self, config: CLIPConfig, *, seed: int = 0, model_id: str = "representax/clip",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = config
        t, v = config.text, config.vision
        self.token_embedding = _normal((t.vocab_size, t.hidden_size), 0.02, g)
        self.text_position = _normal((t.max_position_embeddings, t.hidden_size), 0.01, g)
        self.text_layers = nn.ModuleList(VisionLayer(t.hidden_size, t.intermediate_size, g)
                                         for _ in range(t.num_hidden_layers))
        self.text_final_w, self.text_final_b = nn.Parameter(torch.ones(t.hidden_size)), nn.Parameter(torch.zeros(t.hidden_size))
        self.class_embedding = _normal((v.hidden_size,), 0.02, g)
        self.patch_w = _normal((v.hidden_size, v.num_channels * v.patch_size ** 2), 0.02, g)
        self.vision_position = _normal((v.num_patches + 1, v.hidden_size), 0.02, g)
        self.pre_w, self.pre_b = nn.Parameter(torch.ones(v.hidden_size)), nn.Parameter(torch.zeros(v.hidden_size))
        self.vision_layers = nn.ModuleList(VisionLayer(v.hidden_size, v.intermediate_size, g)
                                           for _ in range(v.num_hidden_layers))
        self.post_w, self.post_b = nn.Parameter(torch.ones(v.hidden_size)), nn.Parameter(torch.zeros(v.hidden_size))
        self.text_projection = _normal((config.projection_dimension, t.hidden_size), 0.02, g)
        self.visual_projection = _normal((config.projection_dimension, v.hidden_size), 0.02, g)
        self.logit_scale = nn.Parameter(torch.tensor(config.logit_scale_init))
        self.compute_dtype = compute_dtype
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision,
                                        output_dimension=config.projection_dimension, routes=frozenset(Route),
                                        modalities=frozenset({Modality.TEXT, Modality.IMAGE}))

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None) -> CLIPBatch:
        return CLIPBatch(torch.as_tensor(input_ids).long(), torch.as_tensor(attention_mask).long())

    def text_features(self, input_ids: torch.Tensor, attention_mask: torch.Tensor) -> torch.Tensor:
        cfg = self.config.text
        dtype = active_compute_dtype(self.compute_dtype)
        dev = self.token_embedding.device
        batch = TokenBatch(attention_mask=attention_mask.cpu(), input_ids=input_ids.cpu())
        pk, seg = packed_segments(batch, dev)
        h = (torch.nn.functional.embedding(pk.input_ids.long(), self.token_embedding)
             + self.text_position[pk.position_ids.long()]).to(dtype)
        for layer in self.text_layers:
            h = layer(h, seg, cfg.num_attention_heads, cfg.norm_epsilon, cfg.hidden_activation, causal=True)
        h = N.layer_norm(h, self.text_final_w, self.text_final_b, cfg.norm_epsilon)
        ids = input_ids.to(dev)
        if cfg.eos_token_id == 2:
            col = ids.argmax(-1)
        else:
            col = (ids == cfg.eos_token_id).int().argmax(-1)
        rows = seg.cu_seqlens[:-1].long() + col
        return N.linear(h[rows], self.text_projection).float()

    def image_features(self, pixel_values: torch.Tensor) -> torch.Tensor:
        cfg = self.config.vision
        dtype = active_compute_dtype(self.compute_dtype)
        dev = self.patch_w.device
        n = pixel_values.shape[0]
        patches = N.linear(patchify(pixel_values.to(dev, dtype), cfg.patch_size), self.patch_w)
        cls = self.class_embedding.to(dtype).expand(n, 1, -1)
        h = torch.cat([cls, patches.reshape(n, cfg.num_patches, -1)], 1) + self.vision_position.to(dtype)
        h = N.layer_norm(h.reshape(n * (cfg.num_patches + 1), -1), self.pre_w, self.pre_b, cfg.norm_epsilon)
        seg = N.Segments.from_lengths([cfg.num_patches + 1] * n, dev)
        for layer in self.vision_layers:
            h = layer(h, seg, cfg.num_attention_heads, cfg.norm_epsilon, cfg.hidden_activation)
        pooled = N.layer_norm(h[seg.cu_seqlens[:-1].long()], self.post_w, self.post_b, cfg.norm_epsilon)
        return N.linear(pooled, self.visual_projection).float()

    def encode(self, inputs: CLIPBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        dev = self.token_embedding.device
        out = torch.zeros(inputs.batch_size, self.config.projection_dimension, device=dev)
        if inputs.input_ids is not None:
            text = self.text_features(inputs.input_ids, inputs.attention_mask)
            out = out + torch.where(inputs.text_valid.to(dev)[:, None], text, torch.zeros_like(text))
        if inputs.pixel_values is not None:
            image = self.image_features(inputs.pixel_values)
            out = out + torch.where(inputs.image_valid.to(dev)[:, None], image, torch.zeros_like(image))
        if self.config.normalize_output:
            out = out / out.norm(dim=-1, keepdim=True).clamp_min(1e-12)
        return out


def _layer_names(prefix: str, i: int):
    p = f"{prefix}encoder.layers.{i}."
    return p


def _layer_state(layer: VisionLayer, p: str, h: int) -> dict[str, torch.Tensor]:
    out = {}
    for j, n in enumerate(("q_proj", "k_proj", "v_proj")):
        out[p + f"self_attn.{n}.weight"] = layer.qkv_w.detach()[j * h:(j + 1) * h]
        out[p + f"self_attn.{n}.bias"] = layer.qkv_b.detach()[j * h:(j + 1) * h]
    for attr, name in (("out", "self_attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2"),
                       ("ln1", "layer_norm1"), ("ln2", "layer_norm2")):
        out[p + name + ".weight"] = getattr(layer, attr + "_w").detach()
        out[p + name + ".bias"] = getattr(layer, attr + "_b").detach()
    return out


def _load_layer(layer: VisionLayer, t: Mapping[str, torch.Tensor], p: str) -> None:
    with torch.no_grad():
        layer.qkv_w.copy_(torch.cat([t[p + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")]))
        layer.qkv_b.copy_(torch.cat([t[p + f"self_attn.{n}.bias"] for n in ("q_proj", "k_proj", "v_proj")]))
        for attr, name in (("out", "self_attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2"),
                           ("ln1", "layer_norm1"), ("ln2", "layer_norm2")):
            getattr(layer, attr + "_w").copy_(t[p + name + ".weight"])
            getattr(layer, attr + "_b").copy_(t[p + name + ".bias"])


class CLIPCheckpointAdapter:
    @staticmethod
    def state_dict(model: CLIPEncoder) -> dict[str, torch.Tensor]:
        c = model.config
        out = {"text_model.embeddings.token_embedding.weight": model.token_embedding.detach(),
               "text_model.embeddings.position_embedding.weight": model.text_position.detach(),
               "text_model.final_layer_norm.weight": model.text_final_w.detach(),
               "text_model.final_layer_norm.bias": model.text_final_b.detach(),
               "vision_model.embeddings.class_embedding": model.class_embedding.detach(),
               "vision_model.embeddings.patch_embedding.weight": model.patch_w.detach().reshape(
                   c.vision.hidden_size, c.vision.num_channels, c.vision.patch_size, c.vision.patch_size),
               "vision_model.embeddings.position_embedding.weight": model.vision_position.detach(),
               "vision_model.pre_layrnorm.weight": model.pre_w.detach(),
               "vision_model.pre_layrnorm.bias": model.pre_b.detach(),
               "vision_model.post_layernorm.weight": model.post_w.detach(),
               "vision_model.post_layernorm.bias": model.post_b.detach(),
               "text_projection.weight": model.text_projection.detach(),
               "visual_projection.weight": model.visual_projection.detach(),
               "logit_scale": model.logit_scale.detach()}
        for i, layer in enumerate(model.text_layers):
            out.update(_layer_state(layer, f"text_model.encoder.layers.{i}.", c.text.hidden_size))
        for i, layer in enumerate(model.vision_layers):
            out.update(_layer_state(layer, f"vision_model.encoder.layers.{i}.", c.vision.hidden_size))
        return {k: v.float().cpu().contiguous() for k, v in out.items()}

    @classmethod
    def from_state_dict(cls, model: CLIPEncoder, t: Mapping[str, torch.Tensor]) -> CLIPEncoder:
        c = model.config
        with torch.no_grad():
            model.token_embedding.copy_(t["text_model.embeddings.token_embedding.weight"])
            model.text_position.copy_(t["text_model.embeddings.position_embedding.weight"])
            model.text_final_w.copy_(t["text_model.final_layer_norm.weight"])
            model.text_final_b.copy_(t["text_model.final_layer_norm.bias"])
            model.class_embedding.copy_(t["vision_model.embeddings.class_embedding"])
            model.patch_w.copy_(t["vision_model.embeddings.patch_embedding.weight"].reshape(c.vision.hidden_size, -1))
            model.vision_position.copy_(t["vision_model.embeddings.position_embedding.weight"])
            model.pre_w.copy_(t["vision_model.pre_layrnorm.weight"])
            model.pre_b.copy_(t["vision_model.pre_layrnorm.bias"])
            model.post_w.copy_(t["vision_model.post_layernorm.weight"])
            model.post_b.copy_(t["vision_model.post_layernorm.bias"])
            model.text_projection.copy_(t["text_projection.weight"])
            model.visual_projection.copy_(t["visual_projection.weight"])
            if "logit_scale" in t:
                model.logit_scale.copy_(t["logit_scale"].reshape(()))
        for i, layer in enumerate(model.text_layers):
            _load_layer(layer, t, f"text_model.encoder.layers.{i}.")
        for i, layer in enumerate(model.vision_layers):
            _load_layer(layer, t, f"vision_model.encoder.layers.{i}.")
        return model

    @classmethod
    def load(cls, path: str | os.PathLike, *, compute_dtype: torch.dtype = torch.float32, **kwargs) -> CLIPEncoder:
        path = Path(path)
        kwargs.setdefault("model_id", path.name)
        kwargs.setdefault("revision", "local")
        model = CLIPEncoder(CLIPConfig.from_hf_config(load_hf_config(path)), compute_dtype=compute_dtype, **kwargs)
        return cls.from_state_dict(model, load_safetensor_subset(path, set(cls.state_dict(model))))

    @classmethod
    def save(cls, model: CLIPEncoder, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        with open(path / "config.json", "w") as handle:
            json.dump(model.config.to_hf_config(), handle, indent=2, sort_keys=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


def build_clip(*, seed: int = 0, compute_dtype: str = "float32", **config) -> CLIPEncoder:
    return CLIPEncoder(CLIPConfig(**config), seed=seed, compute_dtype=getattr(torch, compute_dtype))


__all__ = ["CLIPBatch", "CLIPCheckpointAdapter", "CLIPConfig", "CLIPEncoder", "CLIPTextConfig", "CLIPVisionConfig",
           "build_clip"]
