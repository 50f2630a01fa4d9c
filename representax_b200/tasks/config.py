"""The three open config families of a job: task, loss and loss modifier.

Each family is distinguished only by its ``kind`` string; the matching
registry (tasks/registry.py) maps a kind to the concrete config class and the
code that runs it. Parity: src/representax/tasks/config.py (same class names
and field, so job files carry over).
"""

from __future__ import annotations

from representax_b200._config import FrozenConfig, NonEmptyString


class TaskConfig(FrozenConfig):
    """What the batch means (pairs, triplets, labelled examples, ...); ``kind`` picks the task."""

    kind: NonEmptyString


class LossConfig(FrozenConfig):
    """Which objective is optimised on the task's representations; ``kind`` picks the loss."""

    kind: NonEmptyString


class LossModifierConfig(FrozenConfig):
    """A wrapper that reshapes a loss (Matryoshka prefixes, per-layer terms); ``kind`` picks it."""

    kind: NonEmptyString


__all__ = ["LossConfig", "LossModifierConfig", "TaskConfig"]
