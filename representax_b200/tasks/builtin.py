"""Built-in task, loss and modifier definitions registered at import."""

from __future__ import annotations

from .guided import GISTBatch, GISTConfig, GISTTask, GuidedRetrievalConfig
from .modifiers import (
    AdaptiveLayerModifierConfig,
    AdaptiveLayerTask,
    Matryoshka2dModifierConfig,
    Matryoshka2dTask,
    MatryoshkaModifierConfig,
    MatryoshkaTask,
)
from .registry_types import LossDefinition, LossModifierDefinition, TaskDefinition
from .retrieval import MNRConfig, MNRTask, RetrievalBatch, RetrievalConfig


def _mnr(task, loss):
    if not isinstance(task, RetrievalConfig) or not isinstance(loss, MNRConfig):
        raise TypeError("mnr requires RetrievalConfig and MNRConfig")
    return MNRTask(scale=loss.scale, symmetric=loss.symmetric, negative_scope=loss.negative_scope)


def _gist(task, loss):
    if not isinstance(loss, GISTConfig):
        raise TypeError("gist requires GISTConfig")
    return GISTTask(temperature=loss.temperature, margin_strategy=loss.margin_strategy, margin=loss.margin,
                    contrast_anchors=loss.contrast_anchors, contrast_positives=loss.contrast_positives)


TASKS = [
    TaskDefinition("retrieval", RetrievalConfig, RetrievalBatch),
    TaskDefinition("guided_retrieval", GuidedRetrievalConfig, GISTBatch),
]
LOSSES = [
    LossDefinition("mnr", MNRConfig, _mnr, frozenset({"retrieval"}), frozenset({"direct", "grad_cache"})),
    LossDefinition("gist", GISTConfig, _gist, frozenset({"guided_retrieval"}), frozenset({"direct", "grad_cache"})),
]
MODIFIERS = [
    LossModifierDefinition(
        "matryoshka", MatryoshkaModifierConfig,
        lambda task, c: MatryoshkaTask(task, c.dimensions, weights=c.weights, dimensions_per_step=c.dimensions_per_step),
        frozenset({"direct", "grad_cache"})),
    LossModifierDefinition(
        "adaptive_layer", AdaptiveLayerModifierConfig,
        lambda task, c: AdaptiveLayerTask(task, layers_per_step=c.layers_per_step,
                                          final_layer_weight=c.final_layer_weight,
                                          prior_layer_weight=c.prior_layer_weight,
                                          kl_divergence_weight=c.kl_divergence_weight,
                                          kl_temperature=c.kl_temperature),
        frozenset({"direct"})),
    LossModifierDefinition(
        "matryoshka_2d", Matryoshka2dModifierConfig,
        lambda task, c: Matryoshka2dTask(task, c.dimensions, layers_per_step=c.layers_per_step,
                                         dimensions_per_step=c.dimensions_per_step,
                                         final_layer_weight=c.final_layer_weight,
                                         prior_layer_weight=c.prior_layer_weight,
                                         kl_divergence_weight=c.kl_divergence_weight,
                                         kl_temperature=c.kl_temperature,
                                         matryoshka_weights=c.matryoshka_weights),
        frozenset({"direct"})),
]
