"""Pairwise objectives: cosine regression, contrastive / online contrastive, CoSENT, AnglE and the pair-ranking form.

The import path of this family in the reference package (`representax.tasks.pairwise`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    AngleConfig,
    AnglETask,
    CoSENTConfig,
    CoSENTTask,
    ContrastiveConfig,
    ContrastiveTask,
    CosineRegressionConfig,
    CosineRegressionTask,
    PairwiseBatch,
    PairwiseConfig,
    pairwise_angle_similarity,
    pairwise_cosine_similarity,
    pairwise_distance,
    cosine_regression_loss,
    contrastive_loss,
    online_contrastive_loss,
    pair_ranking_loss,
)

__all__ = [
    "AngleConfig",
    "AnglETask",
    "CoSENTConfig",
    "CoSENTTask",
    "ContrastiveConfig",
    "ContrastiveTask",
    "CosineRegressionConfig",
    "CosineRegressionTask",
    "PairwiseBatch",
    "PairwiseConfig",
    "pairwise_angle_similarity",
    "pairwise_cosine_similarity",
    "pairwise_distance",
    "cosine_regression_loss",
    "contrastive_loss",
    "online_contrastive_loss",
    "pair_ranking_loss",
]
