"""Optimizer and learning-rate schedules.

Parity: ``build_optimizer`` of src/representax/train/optimizer.py:14-81. The
reference resolves a dotted Optax target; the same targets are accepted here
(``optax.adamw``, ``optax.constant_schedule``, ``optax.linear_schedule``,
``optax.warmup_cosine_decay_schedule``, ``optax.cosine_decay_schedule``,
``optax.warmup_constant_schedule``) and map to one fused AdamW implementation
with identical defaults and update rule (eps outside the square root,
decoupled weight decay scaled by the learning rate).
"""

from __future__ import annotations

import math
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

Schedule = Callable[[int], float]


@dataclass(frozen=True)
class AdamW:
    learning_rate: float | Schedule = 1e-3
    b1: float = 0.9
    b2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 1e-4

    def lr(self, step: int) -> float:
        value = self.learning_rate
        return float(value(step)) if callable(value) else float(value)


def constant_schedule(value: float) -> Schedule:
    return lambda step: value


def linear_schedule(init_value: float, end_value: float, transition_steps: int, transition_begin: int = 0) -> Schedule:
    def fn(step: int) -> float:
        t = min(max(step - transition_begin, 0), transition_steps) / max(transition_steps, 1)
        return init_value + (end_value - init_value) * t

    return fn


def cosine_decay_schedule(init_value: float, decay_steps: int, alpha: float = 0.0, exponent: float = 1.0) -> Schedule:
    def fn(step: int) -> float:
        t = min(step, decay_steps) / max(decay_steps, 1)
        cosine = 0.5 * (1 + math.cos(math.pi * t))
        return init_value * ((1 - alpha) * cosine ** exponent + alpha)

    return fn


def warmup_cosine_decay_schedule(init_value: float, peak_value: float, warmup_steps: int, decay_steps: int,
                                 end_value: float = 0.0, exponent: float = 1.0) -> Schedule:
    def fn(step: int) -> float:
        if step < warmup_steps:
            return init_value + (peak_value - init_value) * step / max(warmup_steps, 1)
        t = min(step - warmup_steps, decay_steps - warmup_steps) / max(decay_steps - warmup_steps, 1)
        cosine = 0.5 * (1 + math.cos(math.pi * t)) ** exponent
        return end_value + (peak_value - end_value) * cosine

    return fn


def warmup_constant_schedule(init_value: float, peak_value: float, warmup_steps: int) -> Schedule:
    return lambda step: (init_value + (peak_value - init_value) * step / max(warmup_steps, 1)
                         if step < warmup_steps else peak_value)


_SCHEDULES = {
    "optax.constant_schedule": constant_schedule,
    "optax.linear_schedule": linear_schedule,
    "optax.cosine_decay_schedule": cosine_decay_schedule,
    "optax.warmup_cosine_decay_schedule": warmup_cosine_decay_schedule,
    "optax.warmup_constant_schedule": warmup_constant_schedule,
}
_OPTIMIZERS = {"optax.adamw", "representax_b200.train.optimizer.AdamW", "adamw"}


def build_schedule(config: Any) -> Schedule:
    target = config.target
    if target.startswith("representax_b200.train.optimizer."):
        target = "optax." + target.rsplit(".", 1)[1]
    try:
        factory = _SCHEDULES[target]
    except KeyError as error:
        raise ValueError(f"unsupported schedule target {config.target!r}") from error
    return factory(**config.parameters)


def build_optimizer(config: Any) -> AdamW:
    """Build the optimizer of an ``OptimizationConfig``."""

    if config.optimizer.target not in _OPTIMIZERS:
        raise ValueError(f"unsupported optimizer target {config.optimizer.target!r}")
    params = dict(config.optimizer.parameters)
    if config.schedule is not None:
        params[config.schedule_parameter] = build_schedule(config.schedule)
    allowed = {"learning_rate", "b1", "b2", "eps", "weight_decay"}
    unknown = set(params) - allowed
    if unknown:
        raise ValueError(f"unsupported AdamW parameters: {sorted(unknown)}")
    return AdamW(**params)


__all__ = ["AdamW", "build_optimizer", "build_schedule", "constant_schedule", "cosine_decay_schedule",
           "linear_schedule", "warmup_constant_schedule", "warmup_cosine_decay_schedule"]
