"""Pydantic boundary for declarative configuration with parameter roles.

Parity: ``FrozenConfig``, ``Scientific`` / ``Execution`` role annotations and
``project_parameters`` of src/representax/_config.py:17-107. A field marked
``Scientific`` changes what is learned (it enters the resume fingerprint); an
``Execution`` field only changes how (planner search space).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import StrEnum
from functools import cache
from typing import Annotated, Any, TypeVar, get_origin, get_type_hints

from pydantic import BaseModel, ConfigDict, Field
from typing_extensions import TypeAliasType

NonEmptyString = Annotated[str, Field(min_length=1)]
FinitePositiveFloat = Annotated[float, Field(gt=0, allow_inf_nan=False)]


class ParameterRole(StrEnum):
    SCIENTIFIC = "scientific"
    EXECUTION = "execution"


@dataclass(frozen=True, slots=True)
class ParameterRoleMetadata:
    role: ParameterRole


_T = TypeVar("_T")
Scientific = TypeAliasType(
    "Scientific",
    Annotated[_T, ParameterRoleMetadata(ParameterRole.SCIENTIFIC)],
    type_params=(_T,),
)
Execution = TypeAliasType(
    "Execution",
    Annotated[_T, ParameterRoleMetadata(ParameterRole.EXECUTION)],
    type_params=(_T,),
)


class FrozenConfig(BaseModel):
    """Immutable, closed configuration."""

    model_config = ConfigDict(extra="forbid", frozen=True, validate_default=True)


@cache
def _alias_roles(model: type[BaseModel]) -> dict[str, ParameterRole]:
    roles: dict[str, ParameterRole] = {}
    for name, annotation in get_type_hints(model, include_extras=True).items():
        origin = get_origin(annotation)
        if origin is Scientific:
            roles[name] = ParameterRole.SCIENTIFIC
        elif origin is Execution:
            roles[name] = ParameterRole.EXECUTION
    return roles


def field_role(model: type[BaseModel], name: str) -> ParameterRole | None:
    markers = [m for m in model.model_fields[name].metadata if isinstance(m, ParameterRoleMetadata)]
    if len(markers) > 1:
        raise TypeError(f"configuration field {model.__name__}.{name} has many roles")
    direct = markers[0].role if markers else None
    alias = _alias_roles(model).get(name)
    if direct is not None and alias is not None:
        raise TypeError(f"configuration field {model.__name__}.{name} has many roles")
    return direct or alias


def _project(model: BaseModel, dumped: dict[str, Any], role: ParameterRole) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for name in type(model).model_fields:
        value = getattr(model, name)
        this_role = field_role(type(model), name)
        if this_role is role:
            out[name] = dumped[name]
        elif this_role is None and isinstance(value, BaseModel):
            nested = _project(value, dumped[name], role)
            if nested:
                out[name] = nested
    return out


def project_parameters(config: FrozenConfig, role: ParameterRole | str) -> dict[str, Any]:
    """Project a config onto the fields carrying one intrinsic role."""

    return _project(config, config.model_dump(mode="json"), ParameterRole(role))


__all__ = [
    "Execution",
    "FinitePositiveFloat",
    "FrozenConfig",
    "NonEmptyString",
    "ParameterRole",
    "Scientific",
    "field_role",
    "project_parameters",
]
