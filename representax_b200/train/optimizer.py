"""Optimizer and learning-rate schedules.

Parity: ``build_optimizer`` of src/representax/train/optimizer.py:14-81: the
optimizer and schedule come from dotted targets. The Optax spellings of the
common ones map to built-ins over the flat parameter store: ``optax.adamw``
(the fused AdamW kernels, same defaults and update rule: eps outside the
square root, decoupled weight decay scaled by the learning rate),
``optax.adam``, ``optax.sgd``, ``optax.lion`` and the Optax schedules; any other
target is imported and called, and must return a flat optimizer (``lr``,
``init_state``, ``update``) or a schedule.
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


@dataclass(frozen=True)
class SGD:
    """SGD with optional (Nesterov) momentum and decoupled weight decay on the flat store."""

    learning_rate: float | Schedule = 1e-2
    momentum: float | None = None
    nesterov: bool = False
    weight_decay: float = 0.0

    def lr(self, step: int) -> float:
        value = self.learning_rate
        return float(value(step)) if callable(value) else float(value)

    def init_state(self, master):
        import torch

        return {"trace": torch.zeros_like(master)} if self.momentum else {}

    def update(self, master, grad, state, lr: float, step: int) -> None:
        g = grad + self.weight_decay * master if self.weight_decay else grad
        if self.momentum:
            trace = state["trace"]
            trace.mul_(self.momentum).add_(g)
            g = g + self.momentum * trace if self.nesterov else trace
        master.add_(g, alpha=-lr)


@dataclass(frozen=True)
class Lion:
    """Lion (sign of an interpolated momentum) with decoupled weight decay."""

    learning_rate: float | Schedule = 1e-4
    b1: float = 0.9
    b2: float = 0.99
    weight_decay: float = 1e-3

    def lr(self, step: int) -> float:
        value = self.learning_rate
        return float(value(step)) if callable(value) else float(value)

    def init_state(self, master):
        import torch

        return {"exp_avg": torch.zeros_like(master)}

    def update(self, master, grad, state, lr: float, step: int) -> None:
        m = state["exp_avg"]
        direction = (self.b1 * m + (1 - self.b1) * grad).sign_()
        master.add_(direction + self.weight_decay * master, alpha=-lr)
        m.mul_(self.b2).add_(grad, alpha=1 - self.b2)


def is_flat_optimizer(value: Any) -> bool:
    """The protocol the train step drives: ``lr(step)``, ``init_state(master)``,
    ``update(master, clipped_grad, state, lr, step)`` (in place, fp32 flat buffers)."""

    return all(callable(getattr(value, name, None)) for name in ("lr", "init_state", "update"))


_SCHEDULES = {
    "optax.constant_schedule": constant_schedule,
    "optax.linear_schedule": linear_schedule,
    "optax.cosine_decay_schedule": cosine_decay_schedule,
    "optax.warmup_cosine_decay_schedule": warmup_cosine_decay_schedule,
    "optax.warmup_constant_schedule": warmup_constant_schedule,
}
# Optax spellings of the built-in optimizers (job files written for the reference carry them).
_BUILTIN_OPTIMIZERS: dict[str, Callable[..., Any]] = {
    "optax.adamw": AdamW,
    "adamw": AdamW,
    "optax.adam": lambda **kw: AdamW(**{"weight_decay": 0.0, **kw}),
    "optax.sgd": SGD,
    "optax.lion": Lion,
}


def resolve_target(target: str) -> Any:
    """Import ``package.module.attribute`` (trusted configuration: importing runs module code)."""

    module_name, dot, attribute = target.rpartition(".")
    if not dot or not module_name or not attribute:
        raise ValueError(f"target {target!r} is not a dotted import path such as 'optax.adamw'")
    import importlib

    try:
        module = importlib.import_module(module_name)
    except ModuleNotFoundError as error:
        raise ImportError(f"cannot import {module_name!r} for target {target!r}") from error
    if not hasattr(module, attribute):
        raise AttributeError(f"{module_name!r} has no attribute {attribute!r} (target {target!r})")
    return getattr(module, attribute)


def build_schedule(config: Any) -> Schedule:
    """Optax schedule names map to the built-in schedules; any other dotted
    target is imported and called with the parameters, and must return a
    ``step -> value`` callable."""

    target = config.target
    if target.startswith("representax_b200.train.optimizer."):
        target = "optax." + target.rsplit(".", 1)[1]
    factory = _SCHEDULES.get(target) or resolve_target(config.target)
    schedule = factory(**config.parameters)
    if not callable(schedule):
        raise TypeError(f"schedule target {config.target!r} returned {type(schedule).__name__}, not a function "
                        "of the step")
    return schedule


def build_optimizer(config: Any):
    """Build the optimizer of an ``OptimizationConfig`` from its dotted target.

    ``optax.adamw`` (and ``optax.adam``) give the fused AdamW kernels; ``optax.sgd``
    and ``optax.lion`` the flat-store SGD / Lion; any other target is imported
    and called with the parameters and has to return an object implementing
    :func:`is_flat_optimizer`'s protocol.
    """

    target = config.optimizer.target
    factory = _BUILTIN_OPTIMIZERS.get(target)
    if factory is None:
        factory = resolve_target(target)
        if not callable(factory):
            raise TypeError(f"optimizer target {target!r} is not callable")
    params = dict(config.optimizer.parameters)
    if config.schedule is not None:
        if config.schedule_parameter in params:
            raise ValueError(f"{config.schedule_parameter!r} is given both as an optimizer parameter and by the "
                             "schedule")
        params[config.schedule_parameter] = build_schedule(config.schedule)
    try:
        optimizer = factory(**params)
    except TypeError as error:
        raise ValueError(f"optimizer {target!r} rejected its parameters {sorted(params)}: {error}") from error
    if not (isinstance(optimizer, AdamW) or is_flat_optimizer(optimizer)):
        raise TypeError(f"optimizer target {target!r} built a {type(optimizer).__name__}, which has no "
                        "lr / init_state / update methods")
    return optimizer


__all__ = ["AdamW", "Lion", "SGD", "build_optimizer", "build_schedule", "constant_schedule", "cosine_decay_schedule",
           "is_flat_optimizer", "linear_schedule", "resolve_target", "warmup_constant_schedule",
           "warmup_cosine_decay_schedule"]
