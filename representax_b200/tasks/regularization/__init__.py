"""Global orthogonal regularisation of anchor / negative embeddings.

The import path of this family in the reference package (`representax.tasks.regularization`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    GORConfig,
    GORTask,
    RegularizationBatch,
    RegularizationConfig,
    global_orthogonal_regularization,
)

GlobalOrthogonalRegularizationTask = GORTask

__all__ = [
    "GORConfig",
    "GORTask",
    "RegularizationBatch",
    "RegularizationConfig",
    "global_orthogonal_regularization",
    "GlobalOrthogonalRegularizationTask",
]
