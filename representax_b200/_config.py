"""Declarative configuration with parameter roles.

Every job-config field may carry one of two roles (parity with the role
system of src/representax/_config.py:17-107, same names and JSON output):

* ``Scientific[T]`` -- changing the value changes what is learned; these
  fields form the resume fingerprint.
* ``Execution[T]`` -- changing the value only changes how the run executes
  (batching, placement, threads); a planner may rewrite them freely.

Design: ``Scientific`` / ``Execution`` are subscriptable marker factories
that expand to ``Annotated[T, RoleTag(role)]``, so the role lands in the
pydantic ``FieldInfo.metadata`` of the field and nowhere else. Each config
class builds its field -> role table once, when pydantic finishes the class
(``__pydantic_init_subclass__``), and rejects a field tagged twice right
there instead of at first projection. Projection walks the config tree with
an explicit work list.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import StrEnum
from typing import Annotated, Any, ClassVar

from pydantic import BaseModel, ConfigDict, Field

NonEmptyString = Annotated[str, Field(min_length=1)]
FinitePositiveFloat = Annotated[float, Field(gt=0, allow_inf_nan=False)]


class ParameterRole(StrEnum):
    SCIENTIFIC = "scientific"
    EXECUTION = "execution"


@dataclass(frozen=True, slots=True)
class RoleTag:
    """Metadata object stored beside a field's other constraints."""

    role: ParameterRole


class _RoleMarker:
    """``Scientific[int]`` -> ``Annotated[int, RoleTag(SCIENTIFIC)]``."""

    __slots__ = ("role",)

    def __init__(self, role: ParameterRole) -> None:
        self.role = role

    def __getitem__(self, annotation: Any) -> Any:
        return Annotated[annotation, RoleTag(self.role)]

    def __repr__(self) -> str:
        return f"{self.role.value.capitalize()}[...]"


Scientific = _RoleMarker(ParameterRole.SCIENTIFIC)
Execution = _RoleMarker(ParameterRole.EXECUTION)


def _roles_from_metadata(cls: type[BaseModel]) -> dict[str, ParameterRole]:
    table: dict[str, ParameterRole] = {}
    for name, info in cls.model_fields.items():
        tags = {item.role for item in info.metadata if isinstance(item, RoleTag)}
        tagged = sum(isinstance(item, RoleTag) for item in info.metadata)
        if tagged > 1:
            kinds = ", ".join(sorted(role.value for role in tags)) or "?"
            raise TypeError(f"{cls.__name__}.{name}: a field takes one parameter role, found {tagged} ({kinds})")
        if tags:
            table[name] = tags.pop()
    return table


class FrozenConfig(BaseModel):
    """Immutable configuration: unknown keys are rejected, defaults validated."""

    model_config = ConfigDict(extra="forbid", frozen=True, validate_default=True)

    _parameter_roles: ClassVar[dict[str, ParameterRole]] = {}

    @classmethod
    def __pydantic_init_subclass__(cls, **kwargs: Any) -> None:
        super().__pydantic_init_subclass__(**kwargs)
        cls._parameter_roles = _roles_from_metadata(cls)


def role_table(cls: type[BaseModel]) -> dict[str, ParameterRole]:
    """Field name -> role for one config class (fields without a role omitted)."""

    table = getattr(cls, "_parameter_roles", None)
    if not isinstance(table, dict):  # a plain BaseModel nested in a config
        table = _roles_from_metadata(cls)
    return table


def field_role(cls: type[BaseModel], name: str) -> ParameterRole | None:
    return role_table(cls).get(name)


def project_parameters(config: BaseModel, role: ParameterRole | str) -> dict[str, Any]:
    """The sub-tree of ``config`` (as JSON values) made of fields with ``role``.

    A field tagged with the role is taken whole. An untagged field holding a
    nested config is searched recursively and kept only when something in it
    carries the role; untagged leaves and fields of the other role are dropped.
    """

    wanted = ParameterRole(role)
    result: dict[str, Any] = {}
    # (model instance, its JSON dump, the output dict for it, parent dict, key in parent)
    work: list[tuple[BaseModel, dict[str, Any], dict[str, Any], dict[str, Any] | None, str]] = [
        (config, config.model_dump(mode="json"), result, None, "")]
    attach: list[tuple[dict[str, Any], str, dict[str, Any]]] = []
    while work:
        model, dumped, out, parent, key = work.pop()
        roles = role_table(type(model))
        for name in type(model).model_fields:
            tag = roles.get(name)
            if tag is wanted:
                out[name] = dumped[name]
                continue
            child = getattr(model, name)
            if tag is None and isinstance(child, BaseModel):
                sub: dict[str, Any] = {}
                work.append((child, dumped[name], sub, out, name))
        if parent is not None:
            attach.append((parent, key, out))
    # Children were processed after their parents; attach the non-empty ones
    # deepest-first so an empty grandchild does not keep its parent alive.
    for parent, key, out in reversed(attach):
        if out:
            parent[key] = out
    return _ordered_like(result, config.model_dump(mode="json"))


def _ordered_like(projected: dict[str, Any], dumped: dict[str, Any]) -> dict[str, Any]:
    """Re-key ``projected`` in the declaration order of ``dumped`` (stable JSON)."""

    ordered: dict[str, Any] = {}
    for name, value in dumped.items():
        if name not in projected:
            continue
        picked = projected[name]
        if isinstance(picked, dict) and isinstance(value, dict) and picked is not value:
            picked = _ordered_like(picked, value)
        ordered[name] = picked
    return ordered


__all__ = [
    "Execution",
    "FinitePositiveFloat",
    "FrozenConfig",
    "NonEmptyString",
    "ParameterRole",
    "RoleTag",
    "Scientific",
    "field_role",
    "project_parameters",
    "role_table",
]
