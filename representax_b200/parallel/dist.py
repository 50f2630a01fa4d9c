"""Process-group plumbing: one process per GPU, ``torch.distributed`` on NCCL
(``gloo`` for CPU tests), plus differentiable row gathers used by
global-negative objectives.

Parity: the reference's multi-controller data parallelism
(src/representax/train/sharding.py:383-405,
src/representax/tasks/retrieval/batch.py:97-248) and its SPMD all-gather of
candidate embeddings (src/representax/tasks/retrieval/mnr.py:140-148).
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class DistContext:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    group: object | None = None

    @property
    def enabled(self) -> bool:
        return self.world_size > 1


LOCAL = DistContext()


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> DistContext:
    """Initialise the default group from torchrun's environment (RANK, WORLD_SIZE, ...)."""

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return LOCAL
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(**kwargs)
    return DistContext(rank=rank, world_size=world, local_rank=local_rank, group=None)


class _GatherRows(torch.autograd.Function):
    """All-gather rows; every rank then evaluates the same global objective, so
    the backward pass keeps only this rank's slice (no reduction)."""

    @staticmethod
    def forward(ctx, x, world, rank):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        ctx.rank = rank
        ctx.rows = x.shape[0]
        return torch.cat(parts)

    @staticmethod
    def backward(ctx, g):
        return g[ctx.rank * ctx.rows:(ctx.rank + 1) * ctx.rows], None, None


def gather_rows(x: torch.Tensor, ctx: DistContext) -> torch.Tensor:
    if not ctx.enabled:
        return x
    if x.requires_grad:
        return _GatherRows.apply(x, ctx.world_size, ctx.rank)
    parts = [torch.empty_like(x) for _ in range(ctx.world_size)]
    dist.all_gather(parts, x.contiguous())
    return torch.cat(parts)


def all_reduce_sum_(t: torch.Tensor, ctx: DistContext) -> torch.Tensor:
    if ctx.enabled:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t


def barrier(ctx: DistContext) -> None:
    if ctx.enabled:
        dist.barrier()


class StoreBarrier:
    """Host barrier over the rendezvous key-value store, usable from any thread.

    Collectives of a process group must be issued in the same order by every
    rank from one thread; background work (checkpoint writers) instead meets
    here: each ``wait(name)`` increments a counter under a key unique to that
    name and call count and polls it until all ``world_size`` ranks arrived.
    A rank that never arrives makes the others raise :class:`TimeoutError`
    after ``timeout_s`` (the process keeps running; the caller decides).
    """

    def __init__(self, store, rank: int, world_size: int, *, prefix: str = "rx-barrier",
                 timeout_s: float = 300.0, poll_s: float = 0.005) -> None:
        self.store, self.rank, self.world_size = store, rank, world_size
        self.prefix, self.timeout_s, self.poll_s = prefix, timeout_s, poll_s
        self._calls: dict[str, int] = {}

    @classmethod
    def from_default_group(cls, ctx: DistContext, **kwargs) -> "StoreBarrier | None":
        if not ctx.enabled:
            return None
        from torch.distributed import distributed_c10d

        return cls(distributed_c10d._get_default_store(), ctx.rank, ctx.world_size, **kwargs)

    def wait(self, name: str) -> None:
        import time

        generation = self._calls.get(name, 0)
        self._calls[name] = generation + 1
        key = f"{self.prefix}/{name}/{generation}"
        arrived = self.store.add(key, 1)
        deadline = time.monotonic() + self.timeout_s
        while arrived < self.world_size:
            if time.monotonic() > deadline:
                raise TimeoutError(f"barrier {name!r}: {arrived} of {self.world_size} ranks arrived within "
                                   f"{self.timeout_s:.0f}s (rank {self.rank} waiting)")
            time.sleep(self.poll_s)
            arrived = self.store.add(key, 0)


__all__ = ["DistContext", "LOCAL", "StoreBarrier", "all_reduce_sum_", "barrier", "gather_rows", "init_from_env"]
