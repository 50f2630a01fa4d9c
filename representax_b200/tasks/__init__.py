"""Representation objectives and their registries."""

from . import guided, modifiers, retrieval
from .config import LossConfig, LossModifierConfig, TaskConfig
from .registry import (
    BUILTIN_LOSS_MODIFIERS,
    BUILTIN_LOSSES,
    BUILTIN_TASKS,
    LossDefinition,
    LossModifierDefinition,
    LossModifierRegistry,
    LossRegistry,
    TaskDefinition,
    TaskRegistry,
    build_task,
)
from .retrieval import MNRConfig, MNRTask, RetrievalBatch, RetrievalCollator, RetrievalConfig, retrieval_batch

__all__ = [
    "BUILTIN_LOSSES", "BUILTIN_LOSS_MODIFIERS", "BUILTIN_TASKS", "LossConfig", "LossDefinition",
    "LossModifierConfig", "LossModifierDefinition", "LossModifierRegistry", "LossRegistry", "MNRConfig",
    "MNRTask", "RetrievalBatch", "RetrievalCollator", "RetrievalConfig", "TaskConfig", "TaskDefinition",
    "TaskRegistry", "build_task", "guided", "modifiers", "retrieval", "retrieval_batch",
]
