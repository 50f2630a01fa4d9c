"""Triplet objectives: explicit (anchor, positive, negative) triplets and in-batch mining over labelled examples (all, hard, semi-hard, soft margin).

The import path of this family in the reference package (`representax.tasks.triplet`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    BatchHardSoftMarginLossConfig,
    BatchTripletLossConfig,
    BatchTripletTask,
    ExplicitTripletBatch,
    ExplicitTripletConfig,
    ExplicitTripletLossConfig,
    ExplicitTripletTask,
    LabeledExamplesBatch,
    LabeledExamplesConfig,
    aligned_triplet_distance,
    pairwise_triplet_distances,
    triplet_masks,
    explicit_triplet_loss,
    batch_all_triplet_loss,
    batch_hard_triplet_loss,
    batch_hard_soft_margin_triplet_loss,
    batch_semi_hard_triplet_loss,
)

__all__ = [
    "BatchHardSoftMarginLossConfig",
    "BatchTripletLossConfig",
    "BatchTripletTask",
    "ExplicitTripletBatch",
    "ExplicitTripletConfig",
    "ExplicitTripletLossConfig",
    "ExplicitTripletTask",
    "LabeledExamplesBatch",
    "LabeledExamplesConfig",
    "aligned_triplet_distance",
    "pairwise_triplet_distances",
    "triplet_masks",
    "explicit_triplet_loss",
    "batch_all_triplet_loss",
    "batch_hard_triplet_loss",
    "batch_hard_soft_margin_triplet_loss",
    "batch_semi_hard_triplet_loss",
]
