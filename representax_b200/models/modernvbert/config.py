"""ModernVBERT configuration: ModernBERT text tower + SigLIP vision tower.

Parity: src/representax/models/modernvbert/config.py (text / vision /
composite configs, validation, Transformers config mapping with per-layer
RoPE theta for full and sliding attention).
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from typing import Any, Literal

from pydantic import model_validator

from representax_b200._config import FrozenConfig

AttentionType = Literal["full_attention", "sliding_attention"]
MODERNVBERT_MODEL_ID = "ModernVBERT/modernvbert-embed"


class ModernVBERTTextConfig(FrozenConfig):
    vocab_size: int = 50368
    hidden_size: int = 768
    intermediate_size: int = 1152
    num_hidden_layers: int = 22
    num_attention_heads: int = 12
    layer_types: tuple[AttentionType, ...] | None = None
    global_attn_every_n_layers: int = 3
    local_attention: int = 128
    full_attention_rope_theta: float = 160000.0
    sliding_attention_rope_theta: float = 10000.0
    norm_epsilon: float = 1e-5
    max_position_embeddings: int = 8192
    hidden_activation: str = "gelu"
    pad_token_id: int = 50283
    initializer_range: float = 0.02

    @model_validator(mode="after")
    def _validate(self):
        for name in ("vocab_size", "hidden_size", "intermediate_size", "num_attention_heads",
                     "max_position_embeddings", "local_attention"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        if self.head_dimension % 2:
            raise ValueError("rotary attention needs an even head dimension")
        if self.layer_types is not None and len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("layer_types must contain one entry per layer")
        for name in ("full_attention_rope_theta", "sliding_attention_rope_theta", "norm_epsilon"):
            v = getattr(self, name)
            if not math.isfinite(v) or v <= 0:
                raise ValueError(f"{name} must be finite and positive")
        return self

    @property
    def head_dimension(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def layer_type(self, index: int) -> AttentionType:
        if self.layer_types is not None:
            return self.layer_types[index]
        return "full_attention" if index % self.global_attn_every_n_layers == 0 else "sliding_attention"

    def rope_theta(self, layer_type: AttentionType) -> float:
        return self.full_attention_rope_theta if layer_type == "full_attention" else self.sliding_attention_rope_theta

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "ModernVBERTTextConfig":
        text = value.get("text_config", value)
        rope = text.get("rope_parameters") or {}

        def theta(kind: str, legacy: str, default: float) -> float:
            section = rope.get(kind) if isinstance(rope, Mapping) else None
            if isinstance(section, Mapping) and "rope_theta" in section:
                return float(section["rope_theta"])
            if text.get(legacy) is not None:
                return float(text[legacy])
            return default

        layer_types = text.get("layer_types")
        return cls(
            vocab_size=int(text["vocab_size"]), hidden_size=int(text["hidden_size"]),
            intermediate_size=int(text["intermediate_size"]), num_hidden_layers=int(text["num_hidden_layers"]),
            num_attention_heads=int(text["num_attention_heads"]),
            layer_types=None if layer_types is None else tuple(layer_types),
            global_attn_every_n_layers=int(text.get("global_attn_every_n_layers", 3)),
            local_attention=int(text.get("local_attention", 128)),
            full_attention_rope_theta=theta("full_attention", "global_rope_theta", 160000.0),
            sliding_attention_rope_theta=theta("sliding_attention", "local_rope_theta", 10000.0),
            norm_epsilon=float(text.get("norm_eps", text.get("layer_norm_eps", 1e-5))),
            max_position_embeddings=int(text.get("max_position_embeddings", 8192)),
            hidden_activation=str(text.get("hidden_activation", "gelu")),
            pad_token_id=int(text.get("pad_token_id", 50283) or 0),
            initializer_range=float(text.get("initializer_range", 0.02)),
        )

    def to_hf_config(self) -> dict[str, Any]:
        return {
            "model_type": "modernbert", "vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size, "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "layer_types": [self.layer_type(i) for i in range(self.num_hidden_layers)],
            "global_attn_every_n_layers": self.global_attn_every_n_layers, "local_attention": self.local_attention,
            "rope_parameters": {
                "full_attention": {"rope_type": "default", "rope_theta": self.full_attention_rope_theta},
                "sliding_attention": {"rope_type": "default", "rope_theta": self.sliding_attention_rope_theta},
            },
            "norm_eps": self.norm_epsilon, "norm_bias": False, "mlp_bias": False, "attention_bias": False,
            "max_position_embeddings": self.max_position_embeddings, "hidden_activation": self.hidden_activation,
            "pad_token_id": self.pad_token_id, "initializer_range": self.initializer_range,
        }


class SigLIPVisionConfig(FrozenConfig):
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    num_channels: int = 3
    image_size: int = 512
    patch_size: int = 16
    norm_epsilon: float = 1e-6
    hidden_activation: str = "gelu_pytorch_tanh"

    @model_validator(mode="after")
    def _validate(self):
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("vision hidden_size must be divisible by num_attention_heads")
        if self.image_size % self.patch_size:
            raise ValueError("image_size must be divisible by patch_size")
        return self

    @property
    def head_dimension(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def patch_grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def num_patches(self) -> int:
        return self.patch_grid ** 2

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "SigLIPVisionConfig":
        v = value.get("vision_config", value)
        return cls(hidden_size=int(v["hidden_size"]), intermediate_size=int(v["intermediate_size"]),
                   num_hidden_layers=int(v["num_hidden_layers"]), num_attention_heads=int(v["num_attention_heads"]),
                   num_channels=int(v.get("num_channels", 3)), image_size=int(v["image_size"]),
                   patch_size=int(v["patch_size"]), norm_epsilon=float(v.get("layer_norm_eps", 1e-6)),
                   hidden_activation=str(v.get("hidden_act", "gelu_pytorch_tanh")))

    def to_hf_config(self) -> dict[str, Any]:
        return {"model_type": "siglip_vision_model", "hidden_size": self.hidden_size,
                "intermediate_size": self.intermediate_size, "num_hidden_layers": self.num_hidden_layers,
                "num_attention_heads": self.num_attention_heads, "num_channels": self.num_channels,
                "image_size": self.image_size, "patch_size": self.patch_size, "layer_norm_eps": self.norm_epsilon,
                "hidden_act": self.hidden_activation}


class ModernVBERTConfig(FrozenConfig):
    text: ModernVBERTTextConfig = ModernVBERTTextConfig()
    vision: SigLIPVisionConfig = SigLIPVisionConfig()
    image_token_id: int = 50407
    pixel_shuffle_factor: int = 4

    @model_validator(mode="after")
    def _validate(self):
        if self.vision.patch_grid % self.pixel_shuffle_factor:
            raise ValueError("the patch grid must be divisible by pixel_shuffle_factor")
        return self

    @property
    def image_sequence_length(self) -> int:
        return self.vision.num_patches // self.pixel_shuffle_factor ** 2

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "ModernVBERTConfig":
        return cls(text=ModernVBERTTextConfig.from_hf_config(value),
                   vision=SigLIPVisionConfig.from_hf_config(value),
                   image_token_id=int(value.get("image_token_id", 50407)),
                   pixel_shuffle_factor=int(value.get("pixel_shuffle_factor", 4)))

    def to_hf_config(self) -> dict[str, Any]:
        return {"model_type": "modernvbert", "text_config": self.text.to_hf_config(),
                "vision_config": self.vision.to_hf_config(), "image_token_id": self.image_token_id,
                "pixel_shuffle_factor": self.pixel_shuffle_factor}


__all__ = ["AttentionType", "MODERNVBERT_MODEL_ID", "ModernVBERTConfig", "ModernVBERTTextConfig",
           "SigLIPVisionConfig"]
