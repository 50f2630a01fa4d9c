"""Helpers shared by the task batch containers."""

from __future__ import annotations

from typing import Any

import torch


def as_tensor(value: Any, dtype: torch.dtype | None = None) -> torch.Tensor:
    tensor = value if isinstance(value, torch.Tensor) else torch.as_tensor(value)
    return tensor if dtype is None else tensor.to(dtype)


def leading_rows(payload: Any) -> int:
    """Row count of a model-native payload (a tensor, dataclass or mapping)."""

    size = getattr(payload, "batch_size", None)
    if isinstance(size, int):
        return size
    tensors = list(iter_tensors(payload))
    if not tensors:
        raise ValueError("payload must contain tensors")
    rows = tensors[0].shape[0]
    if any(t.ndim == 0 or t.shape[0] != rows for t in tensors):
        raise ValueError("payloads must be row-major")
    return rows


def iter_tensors(payload: Any):
    if isinstance(payload, torch.Tensor):
        yield payload
    elif isinstance(payload, dict):
        for value in payload.values():
            yield from iter_tensors(value)
    elif isinstance(payload, (list, tuple)):
        for value in payload:
            yield from iter_tensors(value)
    elif hasattr(payload, "__dataclass_fields__"):
        for name in payload.__dataclass_fields__:
            value = getattr(payload, name)
            if name.startswith("_"):
                continue
            yield from iter_tensors(value)


def map_tensors(payload: Any, fn) -> Any:
    """Apply ``fn`` to every tensor of a payload, keeping its structure."""

    import dataclasses

    if isinstance(payload, torch.Tensor):
        return fn(payload)
    if isinstance(payload, dict):
        return {k: map_tensors(v, fn) for k, v in payload.items()}
    if isinstance(payload, tuple):
        return tuple(map_tensors(v, fn) for v in payload)
    if isinstance(payload, list):
        return [map_tensors(v, fn) for v in payload]
    if dataclasses.is_dataclass(payload) and not isinstance(payload, type):
        if hasattr(payload, "map_tensors"):
            return payload.map_tensors(fn)
        changes = {
            f.name: map_tensors(getattr(payload, f.name), fn)
            for f in dataclasses.fields(payload)
            if f.init
        }
        return dataclasses.replace(payload, **changes)
    return payload


def to_device(payload: Any, device: torch.device, non_blocking: bool = True) -> Any:
    return map_tensors(payload, lambda t: t.to(device, non_blocking=non_blocking))


def slice_rows(payload: Any, start: int, stop: int) -> Any:
    """Rows [start, stop) of a model-native payload."""

    import dataclasses

    if hasattr(payload, "rows") and callable(payload.rows):
        return payload.rows(start, stop)
    if isinstance(payload, torch.Tensor):
        return payload[start:stop]
    if isinstance(payload, dict):
        return {k: slice_rows(v, start, stop) for k, v in payload.items()}
    if isinstance(payload, tuple):
        return tuple(slice_rows(v, start, stop) for v in payload)
    if isinstance(payload, list):
        return [slice_rows(v, start, stop) for v in payload]
    if dataclasses.is_dataclass(payload) and not isinstance(payload, type):
        changes = {f.name: slice_rows(getattr(payload, f.name), start, stop)
                   for f in dataclasses.fields(payload) if f.init}
        return dataclasses.replace(payload, **changes)
    return payload
