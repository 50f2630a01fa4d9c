"""Data sources, deterministic mixtures and the host loader."""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from typing import Any

from .config import DataDistributionConfig, DataSourceConfig
from .loader import BatchTelemetry, DataIterator, DataLoader, build_data_loader, identity


def _mapper_id(mapper: str | Callable) -> str:
    if isinstance(mapper, str):
        return mapper
    return f"{mapper.__module__}.{mapper.__qualname__}"


def source(uri: str, *, map: str | Callable, revision: str | None = None, split: str | None = None,
           subset: str | None = None, name: str | None = None) -> DataSourceConfig:
    """Declare one data source without reading it (src/representax/data/distribution.py:594)."""

    return DataSourceConfig(uri=uri, mapper=_mapper_id(map), revision=revision, split=split, subset=subset,
                            name=name)


def mix(*sources: DataSourceConfig | Mapping[str, Any], weights: Sequence[float] | None = None, seed: int = 0,
        shuffle: bool = True) -> DataDistributionConfig:
    """Declare a sampling policy; one source is the ordinary dataset case."""

    resolved = tuple(s if isinstance(s, DataSourceConfig) else DataSourceConfig.model_validate(s) for s in sources)
    return DataDistributionConfig(sources=resolved, weights=tuple(weights) if weights else tuple(1.0 for _ in resolved),
                                  seed=seed, shuffle=shuffle)


__all__ = ["BatchTelemetry", "DataDistributionConfig", "DataIterator", "DataLoader", "DataSourceConfig",
           "build_data_loader", "identity", "mix", "source"]
