"""Retrieval task and MNR loss configuration (src/representax/tasks/retrieval/config.py)."""

from __future__ import annotations

from typing import Literal

from representax_b200._config import FinitePositiveFloat
from representax_b200.tasks.config import LossConfig, TaskConfig


class RetrievalConfig(TaskConfig):
    kind: Literal["retrieval"] = "retrieval"


class MNRConfig(LossConfig):
    kind: Literal["mnr"] = "mnr"
    scale: FinitePositiveFloat = 20.0
    symmetric: bool = False
    negative_scope: Literal["local", "global"] = "global"


__all__ = ["MNRConfig", "RetrievalConfig"]
