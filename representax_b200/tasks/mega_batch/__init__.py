"""Mega-batch margin objective with hardest negatives mined across the whole batch.

The import path of this family in the reference package (`representax.tasks.mega_batch`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    MegaBatch,
    MegaBatchConfig,
    MegaBatchMarginConfig,
    MegaBatchMarginTask,
    mega_batch_margin_loss,
    hardest_negative_indices,
)

__all__ = [
    "MegaBatch",
    "MegaBatchConfig",
    "MegaBatchMarginConfig",
    "MegaBatchMarginTask",
    "mega_batch_margin_loss",
    "hardest_negative_indices",
]
