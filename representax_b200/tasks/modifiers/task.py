"""Composable dimensional and layerwise objectives.

Parity: ``MatryoshkaTask``, ``AdaptiveLayerTask`` and ``Matryoshka2dTask`` of
src/representax/tasks/modifiers/task.py:23-398.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import torch

from representax_b200.core import LossOutput, encode, encode_layers


def _selected(count: int, per_step: int, generator) -> torch.Tensor:
    if per_step == -1 or per_step >= count:
        return torch.ones(count, dtype=torch.bool)
    if generator is None:
        raise ValueError("random modifier sampling requires a generator")
    idx = torch.randperm(count, generator=generator, device=generator.device)[:per_step].cpu()
    mask = torch.zeros(count, dtype=torch.bool)
    mask[idx] = True
    return mask


def _shrink(value: torch.Tensor, dimension: int) -> torch.Tensor:
    if not value.is_floating_point() or value.ndim < 2:
        raise TypeError("task representations must be floating tensors of rank >= 2")
    if dimension > value.shape[-1]:
        raise ValueError("Matryoshka dimension exceeds representation dimension")
    t = value[..., :dimension].to(torch.float32)
    return t / torch.clamp(torch.linalg.vector_norm(t, dim=-1, keepdim=True), min=1e-12)


def _map_reps(reps, fn):
    if isinstance(reps, torch.Tensor):
        return fn(reps)
    return type(reps)(_map_reps(r, fn) for r in reps)


def _first(reps) -> torch.Tensor:
    return reps if isinstance(reps, torch.Tensor) else _first(reps[0])


class MatryoshkaTask:
    """Apply one representation task at several normalised prefix dimensions."""

    def __init__(self, task: Any, dimensions, *, weights=None, dimensions_per_step: int = -1) -> None:
        if not hasattr(task, "loss_from_representations"):
            raise TypeError("Matryoshka requires a representation task")
        dimensions = tuple(int(d) for d in dimensions)
        if not dimensions or any(d <= 0 for d in dimensions):
            raise ValueError("Matryoshka dimensions must be positive and non-empty")
        weights = tuple(weights) if weights else tuple(1.0 for _ in dimensions)
        if len(weights) != len(dimensions):
            raise ValueError("Matryoshka weights must match dimensions")
        if any(not math.isfinite(w) or w <= 0 for w in weights):
            raise ValueError("Matryoshka weights must be finite and positive")
        if dimensions_per_step == 0 or dimensions_per_step < -1:
            raise ValueError("dimensions_per_step must be -1 or positive")
        ordered = sorted(zip(dimensions, weights), reverse=True)
        self.task = task
        self.dimensions = tuple(d for d, _ in ordered)
        self.weights = tuple(float(w) for _, w in ordered)
        self.dimensions_per_step = dimensions_per_step

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return self.task.representations(model, batch, generator=generator, encode_fn=encode_fn)

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        reps = self.representations(model, batch, generator=generator)
        return self.loss_from_representations(reps, batch, generator=generator)

    def loss_from_representations(self, representations, batch, *, generator=None,
                                  row_chunk_size: int | None = None) -> LossOutput:
        full = _first(representations).shape[-1]
        if self.dimensions[0] > full:
            raise ValueError("Matryoshka dimension exceeds representation dimension")
        selected = _selected(len(self.dimensions), self.dimensions_per_step, generator)
        losses = []
        for dimension in self.dimensions:
            shrunk = _map_reps(representations, lambda v, d=dimension: _shrink(v, d))
            adapter = getattr(self.task, "dimension_batch", None)
            dim_batch = adapter(batch, dimension=dimension, full_dimension=full) if callable(adapter) else batch
            if row_chunk_size is None:
                out = self.task.loss_from_representations(shrunk, dim_batch)
            else:
                out = self.task.loss_from_representations(shrunk, dim_batch, row_chunk_size=row_chunk_size)
            losses.append(out.loss)
        stacked = torch.stack(losses)
        weights = torch.tensor(self.weights, dtype=torch.float32, device=stacked.device)
        weights = torch.where(selected.to(stacked.device), weights, torch.zeros_like(weights))
        return LossOutput(loss=(weights * stacked).sum(),
                          metrics={"dimension_losses": stacked.detach(),
                                   "selected_dimensions": selected.to(stacked.device)})


@dataclass
class AdaptiveLayerTask:
    """Apply a representation task at the final and selected prior depths."""

    task: Any
    layers_per_step: int = 1
    final_layer_weight: float = 1.0
    prior_layer_weight: float = 1.0
    kl_divergence_weight: float = 1.0
    kl_temperature: float = 0.3

    def __post_init__(self) -> None:
        if self.layers_per_step == 0 or self.layers_per_step < -1:
            raise ValueError("layers_per_step must be -1 or positive")
        for name in ("final_layer_weight", "prior_layer_weight", "kl_divergence_weight", "kl_temperature"):
            value = getattr(self, name)
            if not math.isfinite(value) or value < 0:
                raise ValueError(f"{name} must be finite and non-negative")

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        layered = self.task.representations(model, batch, generator=generator, encode_fn=encode_layers)
        depth = _first(layered).shape[0]
        final = _map_reps(layered, lambda v: v[-1])
        final_out = self.task.loss_from_representations(final, batch)
        prior_count = depth - 1
        selected = _selected(prior_count, self.layers_per_step, generator)
        n_sel = max(int(selected.sum()), 1)
        loss = self.final_layer_weight * final_out.loss
        layer_losses = []
        kl_losses = []
        final_scores = _similarity(final)
        for i in range(prior_count):
            if not bool(selected[i]):
                continue
            prior = _map_reps(layered, lambda v, i=i: v[i])
            out = self.task.loss_from_representations(prior, batch)
            weight = self.prior_layer_weight * (1 + i) / prior_count
            layer_losses.append(weight * out.loss / n_sel)
            if self.kl_divergence_weight > 0:
                kl_losses.append(_kl(final_scores, _similarity(prior), self.kl_temperature) / n_sel)
        if layer_losses:
            loss = loss + torch.stack(layer_losses).sum()
        if kl_losses:
            loss = loss + self.kl_divergence_weight * torch.stack(kl_losses).sum()
        return LossOutput(loss=loss, metrics={"final_loss": final_out.loss.detach()})


def _similarity(reps) -> torch.Tensor:
    flat = torch.cat([r.reshape(-1, r.shape[-1]) for r in (reps if not isinstance(reps, torch.Tensor) else (reps,))])
    return flat @ flat.T


def _kl(teacher: torch.Tensor, student: torch.Tensor, temperature: float) -> torch.Tensor:
    t = torch.log_softmax(teacher.detach() / temperature, -1)
    s = torch.log_softmax(student / temperature, -1)
    return (t.exp() * (t - s)).sum(-1).mean() * temperature * temperature


@dataclass
class Matryoshka2dTask:
    """Joint layer x dimension objective (Matryoshka2dLoss)."""

    task: Any
    dimensions: tuple[int, ...]
    layers_per_step: int = 1
    dimensions_per_step: int = -1
    final_layer_weight: float = 1.0
    prior_layer_weight: float = 1.0
    kl_divergence_weight: float = 1.0
    kl_temperature: float = 0.3
    matryoshka_weights: tuple[float, ...] | None = None

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        inner = MatryoshkaTask(self.task, self.dimensions, weights=self.matryoshka_weights,
                               dimensions_per_step=self.dimensions_per_step)

        class _Wrapped:
            def representations(_s, *a, **k):
                return inner.representations(*a, **k)

            def loss_from_representations(_s, reps, b):
                return inner.loss_from_representations(reps, b, generator=generator)

        adaptive = AdaptiveLayerTask(_Wrapped(), layers_per_step=self.layers_per_step,
                                     final_layer_weight=self.final_layer_weight,
                                     prior_layer_weight=self.prior_layer_weight,
                                     kl_divergence_weight=self.kl_divergence_weight,
                                     kl_temperature=self.kl_temperature)
        return adaptive.loss(model, batch, generator=generator)


__all__ = ["AdaptiveLayerTask", "Matryoshka2dTask", "MatryoshkaTask"]
