"""Denoising auto-encoder (TSDAE) reconstruction objective.

The import path of this family in the reference package (`representax.tasks.reconstruction`);
the implementations live in `representax_b200.tasks.objectives`.
"""
from representax_b200.tasks.objectives import (  # noqa: F401
    DenoisingAutoEncoderConfig,
    DenoisingAutoEncoderTask,
    DenoisingBatch,
    DenoisingConfig,
)

__all__ = [
    "DenoisingAutoEncoderConfig",
    "DenoisingAutoEncoderTask",
    "DenoisingBatch",
    "DenoisingConfig",
]
