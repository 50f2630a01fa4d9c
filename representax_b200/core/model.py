"""Model-neutral representation-encoder contract.

Parity: ``Route``, ``Modality``, ``EncoderMetadata``, ``Encoder``,
``encode``, ``encode_layers``, ``BoundEncoder`` and ``bind`` of
src/representax/core/model.py:20-212. Encoders here are ``torch.nn.Module``
objects; ``encode`` enforces the same output contract ([batch, dimension],
floating, the declared width) and returns the accumulation dtype (fp32).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from enum import StrEnum
from typing import Any, ClassVar, Protocol, runtime_checkable

import torch

from representax_b200.precision import active_policy


class Route(StrEnum):
    """Semantic route through a representation model."""

    GENERIC = "generic"
    QUERY = "query"
    DOCUMENT = "document"


class Modality(str):
    """Validated, extensible name of one atomic input modality.

    ``fused`` is deliberately not a modality: multimodal inputs are
    compositions of artifacts.
    """

    TEXT: ClassVar["Modality"]
    IMAGE: ClassVar["Modality"]
    AUDIO: ClassVar["Modality"]
    VIDEO: ClassVar["Modality"]

    _NAME = re.compile(r"^[a-z][a-z0-9]*(?:[._/-][a-z0-9]+)*$")

    def __new__(cls, value: str) -> "Modality":
        if not isinstance(value, str) or not cls._NAME.fullmatch(value):
            raise ValueError(
                "modality names must be lowercase identifiers optionally "
                "separated by '.', '/', '_', or '-'"
            )
        return str.__new__(cls, value)

    @property
    def value(self) -> str:
        return str(self)


Modality.TEXT = Modality("text")
Modality.IMAGE = Modality("image")
Modality.AUDIO = Modality("audio")
Modality.VIDEO = Modality("video")
BUILTIN_MODALITIES = frozenset({Modality.TEXT, Modality.IMAGE, Modality.AUDIO, Modality.VIDEO})


@dataclass(frozen=True)
class EncoderMetadata:
    """Static identity and capabilities attached to an encoder."""

    model_id: str
    revision: str
    output_dimension: int
    routes: frozenset = field(default_factory=lambda: frozenset(Route))
    modalities: frozenset = field(default_factory=lambda: frozenset({Modality.TEXT}))

    def __post_init__(self) -> None:
        if not self.model_id:
            raise ValueError("model_id must be non-empty")
        if not self.revision:
            raise ValueError("revision must be non-empty")
        if self.output_dimension <= 0:
            raise ValueError("output_dimension must be positive")
        if not self.routes:
            raise ValueError("an encoder must support at least one route")
        if not self.modalities:
            raise ValueError("an encoder must support at least one modality")


@runtime_checkable
class Encoder(Protocol):
    """Structural boundary implemented by native encoder modules."""

    metadata: EncoderMetadata

    def encode(self, inputs: Any, *, route: Route, generator: Any = None) -> torch.Tensor: ...


@runtime_checkable
class LayerwiseEncoder(Encoder, Protocol):
    """Encoder that exposes postprocessed representations at every depth."""

    def encode_layers(self, inputs: Any, *, route: Route, generator: Any = None) -> torch.Tensor: ...


def _metadata(model: Any) -> EncoderMetadata:
    if not isinstance(model, torch.nn.Module):
        raise TypeError("encoders must be torch.nn.Module trees")
    metadata = getattr(model, "metadata", None)
    if not isinstance(metadata, EncoderMetadata):
        raise TypeError("encoders must expose EncoderMetadata")
    if not callable(getattr(model, "encode", None)):
        raise TypeError("encoders must implement encode")
    return metadata


def _check_route(metadata: EncoderMetadata, route: Route | str) -> Route:
    route = Route(route)
    if route not in metadata.routes:
        raise ValueError(f"{metadata.model_id} does not support route {route.value!r}")
    return route


def encode(model: Encoder, inputs: Any, *, route: Route | str = Route.GENERIC,
           generator: Any = None) -> torch.Tensor:
    """Encode one batch and enforce the shared representation contract."""

    metadata = _metadata(model)
    route = _check_route(metadata, route)
    result = model.encode(inputs, route=route, generator=generator)
    if not isinstance(result, torch.Tensor):
        raise TypeError("encoder output must be a tensor")
    if result.ndim != 2:
        raise ValueError("encoder output must have shape [batch, dimension]")
    if not result.is_floating_point():
        raise TypeError("encoder output must have a floating dtype")
    if result.shape[1] != metadata.output_dimension:
        raise ValueError(
            f"{metadata.model_id} declares output_dimension="
            f"{metadata.output_dimension} but returned {result.shape[1]}"
        )
    return result.to(active_policy().accumulation_dtype)


def encode_layers(model: LayerwiseEncoder, inputs: Any, *, route: Route | str = Route.GENERIC,
                  generator: Any = None) -> torch.Tensor:
    """Encode every available depth with a stable layer-major contract."""

    metadata = _metadata(model)
    route = _check_route(metadata, route)
    layerwise = getattr(model, "encode_layers", None)
    if not callable(layerwise):
        raise TypeError(f"{metadata.model_id} does not expose layerwise representations")
    result = layerwise(inputs, route=route, generator=generator)
    if result.ndim != 3:
        raise ValueError("layerwise encoder output must have shape [layer, batch, dimension]")
    if not result.is_floating_point():
        raise TypeError("layerwise encoder output must have a floating dtype")
    if result.shape[0] < 2:
        raise ValueError("layerwise encoders must expose a prior and final layer")
    if result.shape[2] != metadata.output_dimension:
        raise ValueError(
            f"{metadata.model_id} declares output_dimension="
            f"{metadata.output_dimension} but returned {result.shape[2]}"
        )
    return result.to(active_policy().accumulation_dtype)


class BoundEncoder:
    """An encoder with a fixed semantic route."""

    def __init__(self, model: Encoder, route: Route | str) -> None:
        self.model = model
        self.route = _check_route(_metadata(model), route)

    def __call__(self, inputs: Any, *, generator: Any = None) -> torch.Tensor:
        return encode(self.model, inputs, route=self.route, generator=generator)


def bind(model: Encoder, *, route: Route | str) -> BoundEncoder:
    """Bind one route without creating duplicate query/document APIs."""

    return BoundEncoder(model, route)


__all__ = [
    "BUILTIN_MODALITIES",
    "BoundEncoder",
    "Encoder",
    "EncoderMetadata",
    "LayerwiseEncoder",
    "Modality",
    "Route",
    "bind",
    "encode",
    "encode_layers",
]
