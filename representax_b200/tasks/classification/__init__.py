"""Pair classification with a softmax head over (u, v, |u - v|, ...) features.

The import path of this family in the reference package (`representax.tasks.classification`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    PairClassificationBatch,
    PairClassificationConfig,
    SoftmaxClassificationConfig,
    SoftmaxClassificationTask,
    softmax_classification_loss,
)

__all__ = [
    "PairClassificationBatch",
    "PairClassificationConfig",
    "SoftmaxClassificationConfig",
    "SoftmaxClassificationTask",
    "softmax_classification_loss",
]
