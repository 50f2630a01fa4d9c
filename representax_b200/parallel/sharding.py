"""Sharding plans: which state is replicated, which is sharded, and over which ranks.

Parity: ``fsdp_partition_spec``, ``parameter_specs_from_rules`` and
``ShardingPlan.{ddp,fsdp,custom}`` of src/representax/train/sharding.py:46-440
(P1-P4). The reference states a partition spec per parameter and lets XLA
insert the collectives. Here a plan is resolved into this framework's
execution on one NVSwitch box:

  ddp     replicated parameters and optimizer state; one gradient all-reduce
          (NCCL) per step, then the fused AdamW kernel on every rank;
  zero    replicated bf16/fp32 parameters, AdamW moments sharded by
          contiguous ranges of the flat buffer; the gradient reduce-scatter,
          the clipped AdamW update and the parameter all-gather run as peer
          memory kernels (``TrainStep._sharded_update``);
  fsdp    the reference's per-parameter specs (largest divisible dimension of
          every parameter with at least ``minimum_parameter_elements``
          elements) are computed and recorded for checkpoints and planning;
          execution uses the ``zero`` layout, because one B200 holds the full
          bf16 weights of every model family here (180 GB HBM), so sharding
          parameters would only add gathers;
  custom  ordered regex rules over parameter names choose shard / replicate.

A spec is a tuple with one entry per dimension: ``None`` (replicated) or a
mesh axis name.
"""

from __future__ import annotations

import re
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any, Literal

import torch

Spec = tuple[str | None, ...]
REPLICATED: Spec = ()


def fsdp_partition_spec(shape: Sequence[int], *, axis_name: str, axis_size: int,
                        minimum_elements: int = 1024) -> Spec:
    """Shard the largest dimension divisible by ``axis_size`` of a substantial matrix.

    Vectors, scalars and parameters below ``minimum_elements`` stay
    replicated (a norm scale shared along the batch axis would otherwise
    carry two unrelated uses of one mesh axis)."""

    shape = tuple(int(s) for s in shape)
    numel = 1
    for s in shape:
        numel *= s
    if axis_size <= 1 or len(shape) < 2 or numel < minimum_elements:
        return REPLICATED
    candidates = [d for d, s in enumerate(shape) if s % axis_size == 0]
    if not candidates:
        return REPLICATED
    chosen = max(candidates, key=lambda d: shape[d])
    return tuple(axis_name if d == chosen else None for d in range(len(shape)))


def parameter_specs_from_rules(named_shapes: Mapping[str, Sequence[int]], rules: Sequence[tuple[str, Spec]],
                               default: Spec = REPLICATED) -> dict[str, Spec]:
    """First matching regular expression (searched in the parameter name) wins."""

    compiled = [(re.compile(pattern), tuple(spec)) for pattern, spec in rules]
    out = {}
    for name in named_shapes:
        out[name] = next((spec for pattern, spec in compiled if pattern.search(name)), tuple(default))
    return out


@dataclass(frozen=True)
class ShardingPlan:
    kind: Literal["ddp", "zero", "fsdp", "custom"]
    world_size: int
    data_axis: str = "data"
    parameter_axis: str = "data"
    parameter_specs: Mapping[str, Spec] = field(default_factory=dict)

    @classmethod
    def ddp(cls, world_size: int, *, data_axis: str = "data") -> "ShardingPlan":
        return cls("ddp", world_size, data_axis, data_axis)

    @classmethod
    def zero(cls, world_size: int, *, data_axis: str = "data") -> "ShardingPlan":
        return cls("zero", world_size, data_axis, data_axis)

    @classmethod
    def fsdp(cls, model: torch.nn.Module, world_size: int, *, data_axis: str = "data",
             parameter_axis: str | None = None, minimum_parameter_elements: int = 2 ** 18) -> "ShardingPlan":
        axis = parameter_axis or data_axis
        specs = {n: fsdp_partition_spec(tuple(p.shape), axis_name=axis, axis_size=world_size,
                                        minimum_elements=minimum_parameter_elements)
                 for n, p in model.named_parameters() if p.requires_grad}
        return cls("fsdp", world_size, data_axis, axis, specs)

    @classmethod
    def custom(cls, model: torch.nn.Module, world_size: int, rules: Sequence[tuple[str, Spec]], *,
               data_axis: str = "data", default: Spec = REPLICATED) -> "ShardingPlan":
        shapes = {n: tuple(p.shape) for n, p in model.named_parameters() if p.requires_grad}
        specs = parameter_specs_from_rules(shapes, rules, default)
        for name, spec in specs.items():
            if spec and len(spec) != len(shapes[name]):
                raise ValueError(f"spec {spec} of {name} does not match its rank {len(shapes[name])}")
            for d, axis in enumerate(spec):
                if axis is not None and shapes[name][d] % world_size:
                    raise ValueError(f"{name} dimension {d} ({shapes[name][d]}) is not divisible by {world_size}")
        return cls("custom", world_size, data_axis, data_axis, specs)

    @property
    def sharded_optimizer(self) -> bool:
        """Whether execution uses the peer-memory reduce-scatter / AdamW / all-gather step."""

        return self.kind != "ddp" and self.world_size > 1

    @property
    def shards_parameters(self) -> bool:
        """Whether execution shards the parameters themselves (FSDP layout).

        FSDP always does; custom rules do when any rule shards a parameter.
        Execution shards the flat parameter vector in equal per-rank segments
        (``representax_b200.parallel.fsdp``), so the specs decide whether the
        layout is sharded, not which axis a tensor is cut along.
        """

        if self.world_size <= 1:
            return False
        return self.kind == "fsdp" or (self.kind == "custom" and self.has_sharded_parameters)

    @property
    def has_sharded_parameters(self) -> bool:
        return any(any(a is not None for a in spec) for spec in self.parameter_specs.values())

    def sharded_fraction(self, model: torch.nn.Module) -> float:
        """Fraction of trainable elements the parameter specs would shard."""

        total = sharded = 0
        for n, p in model.named_parameters():
            if not p.requires_grad:
                continue
            total += p.numel()
            if any(a is not None for a in self.parameter_specs.get(n, ())):
                sharded += p.numel()
        return sharded / max(total, 1)

    def describe(self) -> dict[str, Any]:
        return {"kind": self.kind, "world_size": self.world_size, "data_axis": self.data_axis,
                "parameter_axis": self.parameter_axis, "sharded_optimizer": self.sharded_optimizer,
                "shards_parameters": self.shards_parameters,
                "sharded_parameter_specs": sum(1 for s in self.parameter_specs.values() if any(s))}


def plan_from_config(sharding: Any, model: torch.nn.Module, world_size: int) -> ShardingPlan:
    """Resolve a job's ``training.sharding`` (DDPConfig / FSDPConfig / CustomShardingConfig)."""

    kind = getattr(sharding, "kind", None) or type(sharding).__name__.lower().replace("config", "")
    if kind in ("ddp",):
        return ShardingPlan.ddp(world_size)
    if kind in ("fsdp",):
        return ShardingPlan.fsdp(model, world_size,
                                 minimum_parameter_elements=getattr(sharding, "minimum_parameter_elements", 2 ** 18))
    if kind in ("custom", "customsharding"):
        rules = [(r.pattern, tuple(r.axes)) for r in getattr(sharding, "parameter_rules", ())]
        default = tuple(getattr(sharding, "default_parameter_axes", ()))
        return ShardingPlan.custom(model, world_size, rules, default=default)
    if kind == "zero":
        return ShardingPlan.zero(world_size)
    raise ValueError(f"unknown sharding kind {kind!r}")


__all__ = ["REPLICATED", "ShardingPlan", "Spec", "fsdp_partition_spec", "parameter_specs_from_rules",
           "plan_from_config"]
