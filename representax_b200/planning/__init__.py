"""Execution planning contracts that preserve scientific parameters.

Parity: src/representax/planning/specs.py:10-13 (``ExecutionPlanner``, a
protocol only). ``check_plan`` enforces the contract a planner must keep: a
plan may change execution-role fields (parallelism, chunk sizes, kernels,
overlap) but never a scientific-role field.
"""

from __future__ import annotations

from typing import Protocol

from representax_b200._config import ParameterRole, project_parameters
from representax_b200.config import JobConfig, RematerializationPolicy, TrainingConfig


class ExecutionPlanner(Protocol):
    """A boundary that turns a job into a faster job with the same science."""

    def plan(self, job: JobConfig) -> JobConfig: ...


def check_plan(before: JobConfig, after: JobConfig) -> JobConfig:
    """Raise if ``after`` changed any scientific parameter of ``before``."""

    if project_parameters(before, ParameterRole.SCIENTIFIC) != project_parameters(after, ParameterRole.SCIENTIFIC):
        raise ValueError("an execution plan changed scientific parameters")
    return after


__all__ = ["ExecutionPlanner", "JobConfig", "ParameterRole", "RematerializationPolicy", "TrainingConfig",
           "check_plan"]
