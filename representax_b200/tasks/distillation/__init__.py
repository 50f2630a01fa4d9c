"""Distillation objectives: embedding regression (MSE / L2 / cosine) to a teacher, MarginMSE, and KL between score distributions.

The import path of this family in the reference package (`representax.tasks.distillation`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    DistributionDistillationBatch,
    DistributionDistillationConfig,
    DistributionDistillationTask,
    DistributionKLLossConfig,
    EmbeddingDistillationBatch,
    EmbeddingDistillationConfig,
    EmbeddingDistillationLossConfig,
    EmbeddingDistillationTask,
    MarginDistillationBatch,
    MarginDistillationConfig,
    MarginDistillationTask,
    MarginMSELossConfig,
    embedding_distillation_loss,
    margin_mse_loss,
    distribution_kl_loss,
)

__all__ = [
    "DistributionDistillationBatch",
    "DistributionDistillationConfig",
    "DistributionDistillationTask",
    "DistributionKLLossConfig",
    "EmbeddingDistillationBatch",
    "EmbeddingDistillationConfig",
    "EmbeddingDistillationLossConfig",
    "EmbeddingDistillationTask",
    "MarginDistillationBatch",
    "MarginDistillationConfig",
    "MarginDistillationTask",
    "MarginMSELossConfig",
    "embedding_distillation_loss",
    "margin_mse_loss",
    "distribution_kl_loss",
]
