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
from . import objectives as O


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
    TaskDefinition("pairwise", O.PairwiseConfig, O.PairwiseBatch),
    TaskDefinition("explicit_triplet", O.ExplicitTripletConfig, O.ExplicitTripletBatch),
    TaskDefinition("labeled_examples", O.LabeledExamplesConfig, O.LabeledExamplesBatch),
    TaskDefinition("embedding_distillation", O.EmbeddingDistillationConfig, O.EmbeddingDistillationBatch),
    TaskDefinition("margin_distillation", O.MarginDistillationConfig, O.MarginDistillationBatch),
    TaskDefinition("distribution_distillation", O.DistributionDistillationConfig, O.DistributionDistillationBatch),
    TaskDefinition("pair_classification", O.PairClassificationConfig, O.PairClassificationBatch),
    TaskDefinition("contrastive_tension_pairs", O.ContrastiveTensionPairsConfig, O.ContrastiveTensionBatch),
    TaskDefinition("contrastive_tension_examples", O.ContrastiveTensionExamplesConfig, O.ContrastiveTensionExamples),
    TaskDefinition("representation_regularization", O.RegularizationConfig, O.RegularizationBatch),
    TaskDefinition("denoising_reconstruction", O.DenoisingConfig, O.DenoisingBatch),
    TaskDefinition("mega_batch", O.MegaBatchConfig, O.MegaBatch),
]


def _routes(task):
    return dict(left_route=task.left_route, right_route=task.right_route) if isinstance(task, O.PairwiseConfig) else {}


DIRECT = frozenset({"direct"})
LOSSES = [
    LossDefinition("mnr", MNRConfig, _mnr, frozenset({"retrieval"}), frozenset({"direct", "grad_cache"})),
    LossDefinition("gist", GISTConfig, _gist, frozenset({"guided_retrieval"}), frozenset({"direct", "grad_cache"})),
    LossDefinition("cosine_regression", O.CosineRegressionConfig, lambda t, c: O.CosineRegressionTask(**_routes(t)),
                   frozenset({"pairwise"}), DIRECT, microbatch_accumulation=True),
    LossDefinition("contrastive", O.ContrastiveConfig,
                   lambda t, c: O.ContrastiveTask(**_routes(t), distance=c.distance, margin=c.margin,
                                                  online=c.mining == "online"), frozenset({"pairwise"}), DIRECT),
    LossDefinition("cosent", O.CoSENTConfig, lambda t, c: O.CoSENTTask(**_routes(t), scale=c.scale),
                   frozenset({"pairwise"}), DIRECT),
    LossDefinition("angle", O.AngleConfig, lambda t, c: O.AnglETask(**_routes(t), scale=c.scale),
                   frozenset({"pairwise"}), DIRECT),
    LossDefinition("triplet", O.ExplicitTripletLossConfig,
                   lambda t, c: O.ExplicitTripletTask(distance=c.distance, margin=c.margin, anchor_route=t.anchor_route,
                                                      positive_route=t.positive_route, negative_route=t.negative_route),
                   frozenset({"explicit_triplet"}), DIRECT),
    LossDefinition("batch_triplet", O.BatchTripletLossConfig,
                   lambda t, c: O.BatchTripletTask(strategy=c.strategy, distance=c.distance, margin=c.margin,
                                                   route=t.route), frozenset({"labeled_examples"}), DIRECT),
    LossDefinition("batch_hard_soft_margin", O.BatchHardSoftMarginLossConfig,
                   lambda t, c: O.BatchTripletTask(strategy="hard_soft_margin", distance=c.distance, route=t.route),
                   frozenset({"labeled_examples"}), DIRECT),
    LossDefinition("embedding_distillation", O.EmbeddingDistillationLossConfig,
                   lambda t, c: O.EmbeddingDistillationTask(metric=c.metric), frozenset({"embedding_distillation"}),
                   DIRECT, microbatch_accumulation=True),
    LossDefinition("margin_mse", O.MarginMSELossConfig, lambda t, c: O.MarginDistillationTask(similarity=c.similarity),
                   frozenset({"margin_distillation"}), DIRECT, microbatch_accumulation=True),
    LossDefinition("distribution_kl", O.DistributionKLLossConfig,
                   lambda t, c: O.DistributionDistillationTask(temperature=c.temperature, similarity=c.similarity),
                   frozenset({"distribution_distillation"}), DIRECT, microbatch_accumulation=True),
    LossDefinition("softmax_classification", O.SoftmaxClassificationConfig,
                   lambda t, c: O.SoftmaxClassificationTask(concatenation=c.concatenation),
                   frozenset({"pair_classification"}), DIRECT),
    LossDefinition("contrastive_tension", O.ContrastiveTensionConfig, lambda t, c: O.ContrastiveTensionTask(),
                   frozenset({"contrastive_tension_pairs"}), DIRECT),
    LossDefinition("contrastive_tension_in_batch", O.ContrastiveTensionInBatchConfig,
                   lambda t, c: O.ContrastiveTensionInBatchTask(scale=c.scale),
                   frozenset({"contrastive_tension_examples"}), DIRECT),
    LossDefinition("global_orthogonal_regularization", O.GORConfig,
                   lambda t, c: O.GORTask(mean_weight=c.mean_weight, second_moment_weight=c.second_moment_weight),
                   frozenset({"representation_regularization"}), DIRECT),
    LossDefinition("denoising_autoencoder", O.DenoisingAutoEncoderConfig, lambda t, c: O.DenoisingAutoEncoderTask(),
                   frozenset({"denoising_reconstruction"}), DIRECT),
    LossDefinition("mega_batch_margin", O.MegaBatchMarginConfig,
                   lambda t, c: O.MegaBatchMarginTask(positive_margin=c.positive_margin,
                                                      negative_margin=c.negative_margin),
                   frozenset({"mega_batch"}), frozenset({"direct", "mega_batch_mining"})),
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
