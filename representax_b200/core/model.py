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

    # lowercase word, optionally continued by '.', '/', '_' or '-' separated words
    _NAME = re.compile(r"[a-z][a-z0-9]*(?:[._/-][a-z0-9]+)*")

    def __new__(cls, value: str) -> "Modality":
        if isinstance(value, str) and cls._NAME.fullmatch(value):
            return str.__new__(cls, value)
        raise ValueError(f"{value!r} is not a modality name: use lowercase words such as 'text' or "
                         "'image/depth' (separators '.', '/', '_', '-')")

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
        problems = [text for bad, text in (
            (not self.model_id, "empty model_id"),
            (not self.revision, "empty revision"),
            (self.output_dimension < 1, f"output_dimension {self.output_dimension} < 1"),
            (not self.routes, "no route"),
            (not self.modalities, "no modality"),
        ) if bad]
        if problems:
            raise ValueError("EncoderMetadata: " + ", ".join(problems))


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
    """The metadata of an object that satisfies the encoder contract (module + metadata + encode)."""

    metadata = getattr(model, "metadata", None)
    missing = [what for ok, what in (
        (isinstance(model, torch.nn.Module), "is not a torch.nn.Module"),
        (isinstance(metadata, EncoderMetadata), "has no EncoderMetadata"),
        (callable(getattr(model, "encode", None)), "has no encode()"),
    ) if not ok]
    if missing:
        raise TypeError(f"{type(model).__name__} is not an encoder: it " + " and ".join(missing))
    return metadata


def _check_route(metadata: EncoderMetadata, route: Route | str) -> Route:
    chosen = Route(route)
    if chosen in metadata.routes:
        return chosen
    offered = sorted(r.value for r in metadata.routes)
    raise ValueError(f"route {chosen.value!r} is not offered by {metadata.model_id} (routes: {offered})")


def _contract(metadata: EncoderMetadata, result: Any, layout: tuple[str, ...]) -> torch.Tensor:
    """Check an encoder output against ``layout`` (axis names, last = dimension) and cast it."""

    where = f"{metadata.model_id} output"
    if not torch.is_tensor(result):
        raise TypeError(f"{where} is a {type(result).__name__}, not a tensor")
    if not result.is_floating_point():
        raise TypeError(f"{where} has integer dtype {result.dtype}")
    if result.ndim != len(layout):
        raise ValueError(f"{where} has {result.ndim} axes; expected [{', '.join(layout)}]")
    if layout[0] == "layer" and result.shape[0] < 2:
        raise ValueError(f"{where} holds {result.shape[0]} layer(s); layerwise outputs need at least an "
                         "earlier and the final layer")
    width = result.shape[-1]
    if width != metadata.output_dimension:
        raise ValueError(f"{where} is {width} wide but the metadata declares {metadata.output_dimension}")
    return result.to(active_policy().accumulation_dtype)


def encode(model: Encoder, inputs: Any, *, route: Route | str = Route.GENERIC,
           generator: Any = None) -> torch.Tensor:
    """Encode one batch as ``[batch, dimension]`` in the accumulation dtype."""

    metadata = _metadata(model)
    chosen = _check_route(metadata, route)
    return _contract(metadata, model.encode(inputs, route=chosen, generator=generator), ("batch", "dimension"))


def encode_layers(model: LayerwiseEncoder, inputs: Any, *, route: Route | str = Route.GENERIC,
                  generator: Any = None) -> torch.Tensor:
    """Encode every available depth as ``[layer, batch, dimension]``."""

    metadata = _metadata(model)
    chosen = _check_route(metadata, route)
    layerwise = getattr(model, "encode_layers", None)
    if not callable(layerwise):
        raise TypeError(f"{metadata.model_id} has no encode_layers()")
    return _contract(metadata, layerwise(inputs, route=chosen, generator=generator),
                     ("layer", "batch", "dimension"))


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
