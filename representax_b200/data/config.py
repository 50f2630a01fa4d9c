"""Data-source and distribution configuration.

Parity: ``DataSourceConfig`` and ``DataDistributionConfig`` of
src/representax/data/distribution.py:518-600 (field names and validation kept
identical so job files round-trip).
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from urllib.parse import urlparse

from pydantic import model_validator

from representax_b200._config import FrozenConfig


def _check_mapper(mapper: str) -> None:
    module, sep, attr = mapper.rpartition(":") if ":" in mapper else mapper.rpartition(".")
    if not module or not attr:
        raise ValueError(f"mapper {mapper!r} must be a dotted 'module.attribute' reference")


class DataSourceConfig(FrozenConfig):
    uri: str
    mapper: str
    revision: str | None = None
    split: str | None = None
    subset: str | None = None
    name: str | None = None

    @model_validator(mode="after")
    def _validate(self):
        if not self.uri:
            raise ValueError("source uri must be non-empty")
        _check_mapper(self.mapper)
        return self

    @property
    def scheme(self) -> str:
        return urlparse(self.uri).scheme or "file"


class DataDistributionConfig(FrozenConfig):
    sources: tuple[DataSourceConfig, ...]
    weights: tuple[float, ...]
    seed: int = 0
    shuffle: bool = True

    @model_validator(mode="before")
    @classmethod
    def _default_weights(cls, value: object) -> object:
        if isinstance(value, Mapping) and "weights" not in value:
            sources = value.get("sources")
            if isinstance(sources, Sequence):
                return {**value, "weights": [1.0] * len(sources)}
        return value

    @model_validator(mode="after")
    def _validate(self):
        if not self.sources:
            raise ValueError("a distribution must contain at least one source")
        if len(self.sources) != len(self.weights):
            raise ValueError("weights must match sources")
        if any(not math.isfinite(w) or w <= 0 for w in self.weights):
            raise ValueError("sampling weights must be finite and positive")
        if self.seed < 0:
            raise ValueError("seed must be non-negative")
        names = [s.name for s in self.sources if s.name is not None]
        if len(names) != len(set(names)):
            raise ValueError("named sources must be unique")
        return self

    @property
    def normalized_weights(self) -> tuple[float, ...]:
        total = sum(self.weights)
        return tuple(w / total for w in self.weights)


__all__ = ["DataDistributionConfig", "DataSourceConfig"]
