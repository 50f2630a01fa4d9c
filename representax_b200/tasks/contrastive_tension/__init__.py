"""Contrastive tension: two encoders, explicit example pairs or in-batch negatives.

The import path of this family in the reference package (`representax.tasks.contrastive_tension`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    ContrastiveTensionBatch,
    ContrastiveTensionConfig,
    ContrastiveTensionExamples,
    ContrastiveTensionExamplesConfig,
    ContrastiveTensionInBatchConfig,
    ContrastiveTensionInBatchTask,
    ContrastiveTensionPairsConfig,
    ContrastiveTensionTask,
    contrastive_tension_loss,
    contrastive_tension_in_batch_loss,
)

__all__ = [
    "ContrastiveTensionBatch",
    "ContrastiveTensionConfig",
    "ContrastiveTensionExamples",
    "ContrastiveTensionExamplesConfig",
    "ContrastiveTensionInBatchConfig",
    "ContrastiveTensionInBatchTask",
    "ContrastiveTensionPairsConfig",
    "ContrastiveTensionTask",
    "contrastive_tension_loss",
    "contrastive_tension_in_batch_loss",
]
