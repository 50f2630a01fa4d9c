"""Loss-modifier configurations (src/representax/tasks/modifiers/config.py)."""

from __future__ import annotations

from typing import Literal

from pydantic import Field, model_validator

from representax_b200.tasks.config import LossModifierConfig


class MatryoshkaModifierConfig(LossModifierConfig):
    kind: Literal["matryoshka"] = "matryoshka"
    dimensions: tuple[int, ...]
    weights: tuple[float, ...] | None = None
    dimensions_per_step: int = -1

    @model_validator(mode="after")
    def _check(self):
        if not self.dimensions or any(d <= 0 for d in self.dimensions):
            raise ValueError("Matryoshka dimensions must be positive and non-empty")
        if self.weights is not None and len(self.weights) != len(self.dimensions):
            raise ValueError("Matryoshka weights must match dimensions")
        return self


class AdaptiveLayerModifierConfig(LossModifierConfig):
    kind: Literal["adaptive_layer"] = "adaptive_layer"
    layers_per_step: int = 1
    final_layer_weight: float = Field(default=1.0, ge=0)
    prior_layer_weight: float = Field(default=1.0, ge=0)
    kl_divergence_weight: float = Field(default=1.0, ge=0)
    kl_temperature: float = Field(default=0.3, ge=0)


class Matryoshka2dModifierConfig(LossModifierConfig):
    kind: Literal["matryoshka_2d"] = "matryoshka_2d"
    dimensions: tuple[int, ...]
    matryoshka_weights: tuple[float, ...] | None = None
    dimensions_per_step: int = -1
    layers_per_step: int = 1
    final_layer_weight: float = 1.0
    prior_layer_weight: float = 1.0
    kl_divergence_weight: float = 1.0
    kl_temperature: float = 0.3


__all__ = ["AdaptiveLayerModifierConfig", "Matryoshka2dModifierConfig", "MatryoshkaModifierConfig"]
