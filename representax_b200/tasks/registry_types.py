"""Definition records of the task / loss / modifier registries."""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

from .config import LossConfig, LossModifierConfig, TaskConfig


@dataclass(frozen=True, slots=True)
class TaskDefinition:
    kind: str
    config_type: type[TaskConfig]
    batch_type: type | None = None


@dataclass(frozen=True, slots=True)
class LossDefinition:
    kind: str
    config_type: type[LossConfig]
    build: Callable[[TaskConfig, LossConfig], Any]
    task_kinds: frozenset[str]
    training_strategies: frozenset[str]
    microbatch_accumulation: bool = False

    def __post_init__(self) -> None:
        if not self.task_kinds:
            raise ValueError("a loss must support at least one task")
        if not self.training_strategies:
            raise ValueError("a loss must support at least one training strategy")


@dataclass(frozen=True, slots=True)
class LossModifierDefinition:
    kind: str
    config_type: type[LossModifierConfig]
    build: Callable[[Any, LossModifierConfig], Any]
    training_strategies: frozenset[str]
    microbatch_accumulation: bool = False


__all__ = ["LossDefinition", "LossModifierDefinition", "TaskDefinition"]
