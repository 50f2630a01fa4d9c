"""Hugging Face checkpoint I/O (config.json + sharded safetensors).

Parity: ``resolve_hf_checkpoint``, ``load_hf_config`` and the
sharded-index-aware ``load_safetensor_subset`` of
src/representax/integrations/huggingface.py:24-171 (local directories only:
this environment has no network).
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterable, Mapping
from pathlib import Path

import torch
from safetensors import safe_open
from safetensors.torch import save_file


def resolve_hf_checkpoint(path: str | os.PathLike) -> Path:
    p = Path(path)
    if not p.is_dir():
        raise FileNotFoundError(f"checkpoint directory {p} does not exist (remote hubs are not reachable)")
    return p


def load_hf_config(path: str | os.PathLike) -> dict:
    p = resolve_hf_checkpoint(path)
    with open(p / "config.json") as handle:
        return json.load(handle)


def _weight_files(p: Path) -> list[Path]:
    index = p / "model.safetensors.index.json"
    if index.exists():
        with open(index) as handle:
            data = json.load(handle)
        return sorted({p / f for f in data["weight_map"].values()})
    single = p / "model.safetensors"
    if single.exists():
        return [single]
    files = sorted(p.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors weights under {p}")
    return files


def load_safetensor_subset(path: str | os.PathLike, names: Iterable[str], *,
                           prefixes: tuple[str, ...] = ("",)) -> dict[str, torch.Tensor]:
    """Load only ``names`` (trying each prefix) from the checkpoint's shards."""

    p = resolve_hf_checkpoint(path)
    wanted = set(names)
    out: dict[str, torch.Tensor] = {}
    for file in _weight_files(p):
        with safe_open(str(file), framework="pt") as handle:
            keys = set(handle.keys())
            for name in wanted - set(out):
                for prefix in prefixes:
                    if prefix + name in keys:
                        out[name] = handle.get_tensor(prefix + name)
                        break
    return out


def save_safetensors(tensors: Mapping[str, torch.Tensor], path: str | os.PathLike,
                     metadata: Mapping[str, str] | None = None) -> None:
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(path),
              metadata=dict(metadata or {"format": "pt"}))


__all__ = ["load_hf_config", "load_safetensor_subset", "resolve_hf_checkpoint", "save_safetensors"]
