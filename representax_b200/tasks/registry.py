"""Immutable task / loss / loss-modifier registries.

Parity: ``TaskRegistry``, ``LossRegistry``, ``LossModifierRegistry``,
``BUILTIN_*`` and ``build_task`` of src/representax/tasks/registry.py:138-873.
Each loss declares the task kinds it supports, its training strategies
(``direct``, ``grad_cache``, ``mega_batch_mining``) and whether it decomposes
exactly over gradient-accumulation microbatches; ``JobConfig`` validation uses
these declarations.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Mapping
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any

from .config import LossConfig, LossModifierConfig, TaskConfig


def _index(definitions: Iterable[Any], label: str) -> Mapping[str, Any]:
    out: dict[str, Any] = {}
    for d in definitions:
        if d.kind in out:
            raise ValueError(f"duplicate {label} kind {d.kind!r}")
        out[d.kind] = d
    return MappingProxyType(out)


def _parse(value: Any, *, base: type, definitions: Mapping[str, Any], label: str):
    if isinstance(value, base):
        definition = definitions.get(value.kind)
        if definition is None:
            raise ValueError(f"{label} kind {value.kind!r} is not registered")
        if not isinstance(value, definition.config_type):
            raise TypeError(f"{label} {value.kind!r} requires {definition.config_type.__name__}, "
                            f"received {type(value).__name__}")
        return value
    if not isinstance(value, Mapping):
        raise TypeError(f"{label} config must be a mapping or {base.__name__}")
    kind = value.get("kind")
    if not isinstance(kind, str):
        raise ValueError(f"{label} config requires a string kind")
    definition = definitions.get(kind)
    if definition is None:
        raise ValueError(f"{label} kind {kind!r} is not registered")
    return definition.config_type.model_validate(value)


from .registry_types import LossDefinition, LossModifierDefinition, TaskDefinition


class _Registry:
    _label = ""
    _base: type = object

    def __init__(self, definitions: Iterable[Any]) -> None:
        self._definitions = _index(definitions, self._label)

    @property
    def definitions(self) -> Mapping[str, Any]:
        return self._definitions

    def definition(self, kind: str):
        try:
            return self._definitions[kind]
        except KeyError as error:
            raise KeyError(f"{self._label} kind {kind!r} is not registered") from error

    def parse(self, value: Any):
        return _parse(value, base=self._base, definitions=self._definitions, label=self._label)

    def extended(self, *definitions):
        return type(self)((*self._definitions.values(), *definitions))


class TaskRegistry(_Registry):
    _label = "task"
    _base = TaskConfig


class LossRegistry(_Registry):
    _label = "loss"
    _base = LossConfig

    def build(self, task: TaskConfig, config: LossConfig) -> Any:
        definition = self.definition(config.kind)
        if not isinstance(config, definition.config_type):
            raise TypeError(f"loss {config.kind!r} requires {definition.config_type.__name__}")
        return definition.build(task, config)


class LossModifierRegistry(_Registry):
    _label = "loss modifier"
    _base = LossModifierConfig

    def build(self, task: Any, config: LossModifierConfig) -> Any:
        definition = self.definition(config.kind)
        if not isinstance(config, definition.config_type):
            raise TypeError(f"loss modifier {config.kind!r} requires {definition.config_type.__name__}")
        return definition.build(task, config)


def _builtin_definitions():
    from . import builtin

    return builtin.TASKS, builtin.LOSSES, builtin.MODIFIERS


_TASKS, _LOSSES, _MODIFIERS = _builtin_definitions()
BUILTIN_TASKS = TaskRegistry(_TASKS)
BUILTIN_LOSSES = LossRegistry(_LOSSES)
BUILTIN_LOSS_MODIFIERS = LossModifierRegistry(_MODIFIERS)


def build_task(task: TaskConfig, loss: LossConfig, modifiers: tuple[LossModifierConfig, ...] = (), *,
               loss_registry: LossRegistry = BUILTIN_LOSSES,
               modifier_registry: LossModifierRegistry = BUILTIN_LOSS_MODIFIERS) -> Any:
    definition = loss_registry.definition(loss.kind)
    if task.kind not in definition.task_kinds:
        raise ValueError(f"loss {loss.kind!r} does not support task {task.kind!r}")
    built = loss_registry.build(task, loss)
    for modifier in modifiers:
        built = modifier_registry.build(built, modifier)
    return built


__all__ = ["BUILTIN_LOSSES", "BUILTIN_LOSS_MODIFIERS", "BUILTIN_TASKS", "LossDefinition", "LossModifierDefinition",
           "LossModifierRegistry", "LossRegistry", "TaskDefinition", "TaskRegistry", "build_task"]
