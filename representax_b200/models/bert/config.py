"""BERT architecture configuration (HF ``config.json`` mapping).

Parity: ``BertConfig`` of src/representax/models/bert/config.py:17-125.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, Literal

from pydantic import model_validator

from representax_b200._config import FrozenConfig


class BertConfig(FrozenConfig):
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    max_position_embeddings: int
    type_vocab_size: int = 2
    hidden_activation: Literal["gelu", "gelu_new", "relu", "silu"] = "gelu"
    hidden_dropout_probability: float = 0.1
    attention_dropout_probability: float = 0.1
    norm_epsilon: float = 1e-12
    initializer_range: float = 0.02
    pad_token_id: int = 0

    @model_validator(mode="after")
    def _validate(self) -> "BertConfig":
        for name in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                     "num_attention_heads", "max_position_embeddings", "type_vocab_size"):
            if getattr(self, name) <= 0 and name != "num_hidden_layers":
                raise ValueError(f"{name} must be positive")
        if self.num_hidden_layers < 0:
            raise ValueError("num_hidden_layers must be non-negative")
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        for name in ("hidden_dropout_probability", "attention_dropout_probability"):
            value = getattr(self, name)
            if not 0.0 <= value < 1.0:
                raise ValueError(f"{name} must be in [0, 1)")
        return self

    @property
    def head_dimension(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "BertConfig":
        activation = str(value.get("hidden_act", "gelu"))
        return cls(
            vocab_size=int(value["vocab_size"]),
            hidden_size=int(value["hidden_size"]),
            intermediate_size=int(value["intermediate_size"]),
            num_hidden_layers=int(value["num_hidden_layers"]),
            num_attention_heads=int(value["num_attention_heads"]),
            max_position_embeddings=int(value["max_position_embeddings"]),
            type_vocab_size=int(value.get("type_vocab_size", 2)),
            hidden_activation=activation,  # type: ignore[arg-type]
            hidden_dropout_probability=float(value.get("hidden_dropout_prob", 0.1)),
            attention_dropout_probability=float(value.get("attention_probs_dropout_prob", 0.1)),
            norm_epsilon=float(value.get("layer_norm_eps", 1e-12)),
            initializer_range=float(value.get("initializer_range", 0.02)),
            pad_token_id=int(value.get("pad_token_id", 0)),
        )

    def to_hf_config(self) -> dict[str, Any]:
        return {
            "architectures": ["BertModel"],
            "model_type": "bert",
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "max_position_embeddings": self.max_position_embeddings,
            "type_vocab_size": self.type_vocab_size,
            "hidden_act": self.hidden_activation,
            "hidden_dropout_prob": self.hidden_dropout_probability,
            "attention_probs_dropout_prob": self.attention_dropout_probability,
            "layer_norm_eps": self.norm_epsilon,
            "initializer_range": self.initializer_range,
            "pad_token_id": self.pad_token_id,
            "position_embedding_type": "absolute",
        }

    @classmethod
    def base(cls, **overrides) -> "BertConfig":
        values = dict(vocab_size=30522, hidden_size=768, intermediate_size=3072, num_hidden_layers=12,
                      num_attention_heads=12, max_position_embeddings=512)
        values.update(overrides)
        return cls(**values)

    @classmethod
    def small(cls, **overrides) -> "BertConfig":
        values = dict(vocab_size=30522, hidden_size=384, intermediate_size=1536, num_hidden_layers=6,
                      num_attention_heads=12, max_position_embeddings=512)
        values.update(overrides)
        return cls(**values)


__all__ = ["BertConfig"]
