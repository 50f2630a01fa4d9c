"""Task boundary shared by retrieval and the other objectives.

Parity: ``LossOutput``, ``Task``, ``RepresentationTask`` and ``evaluate_loss``
of src/representax/core/task.py:19-81.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

import torch

EncodeFunction = Callable[..., torch.Tensor]


@dataclass
class LossOutput:
    """Scalar optimisation target plus named metric tensors."""

    loss: torch.Tensor
    metrics: Mapping[str, torch.Tensor] = field(default_factory=dict)


@runtime_checkable
class Task(Protocol):
    """Interprets examples and turns model outputs into a loss."""

    def loss(self, model: Any, batch: Any, *, generator: Any = None) -> LossOutput: ...


@runtime_checkable
class RepresentationTask(Task, Protocol):
    """A task whose model work separates from its representation loss.

    The seam lets loss modifiers and cached (GradCache) execution reuse one
    encoder pass.
    """

    def representations(self, model: Any, batch: Any, *, generator: Any = None,
                        encode_fn: EncodeFunction) -> Any: ...

    def loss_from_representations(self, representations: Any, batch: Any) -> LossOutput: ...


def evaluate_loss(task: Task, model: Any, batch: Any, *, generator: Any = None) -> LossOutput:
    """Evaluate a task while validating the optimisation boundary."""

    output = task.loss(model, batch, generator=generator)
    loss = output.loss
    if not isinstance(loss, torch.Tensor) or loss.ndim != 0:
        raise ValueError("task loss must be scalar")
    if not loss.is_floating_point():
        raise TypeError("task loss must have a floating dtype")
    metrics = {name: torch.as_tensor(value).to(torch.float32) for name, value in output.metrics.items()}
    return LossOutput(loss=loss.to(torch.float32), metrics=metrics)


__all__ = ["EncodeFunction", "LossOutput", "RepresentationTask", "Task", "evaluate_loss"]
