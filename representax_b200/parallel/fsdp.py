"""FSDP on one NVSwitch box: parameters sharded over ranks, gathered at use.

Layout (``FlatParameterStore(..., fsdp=True)``): the flat parameter buffer is
cut into ``world`` equal contiguous segments; rank r owns segment r of

* the fp32 master weights and both AdamW moments (local memory),
* the bf16 compute weights (``owner``: an IPC buffer every peer can read),

while the fp32 gradient accumulator stays full-size (GradCache accumulates
every chunk's weight gradient locally, like FSDP's ``no_sync``) and is
reduce-scattered once per step into the owner's shard by peer loads.

Use: every rank keeps a local bf16 ``cache`` of the full compute weights,
valid for one parameter version (one optimizer step):

* the first forward GEMM that consumes a weight in a version runs the
  tcgen05 GEMM with the gather fused in (``gemm_gather``: its epilogue warps
  copy the weight's rows from the owning ranks into the cache over NVLink,
  the producer starts each tile as soon as its rows are in place);
* every other parameter (embeddings, biases, norms) is brought in by one
  ``gather_ranges`` launch at its first use in the version;
* later uses in the same step (GradCache replays, backward products) read
  the cache, so each weight crosses NVLink once per step.

After the sharded AdamW updates the owners' shards the version advances and
every cache entry becomes stale. ``reshard="use"`` would drop the cache after
each use; it is not offered because on a 180 GB GPU the cache (2 bytes per
parameter) costs less than re-gathering every GradCache chunk.

Parity: the reference's FSDP (src/representax/train/sharding.py:46-75,
441-492) shards each parameter's largest divisible axis and lets XLA gather at
use (src/representax/models/components.py:86); here the flat segments replace
per-tensor partition specs and the gather is a fused peer-memory kernel.
"""

from __future__ import annotations

import torch

from representax_b200.ops._ext import ext

# data_ptr of a cache view handed out for a fused gather -> (state, slot index)
_PENDING: dict[int, tuple["FSDPState", int]] = {}


def _align8(n: int) -> int:
    return (n + 7) // 8 * 8


class FSDPState:
    def __init__(self, store) -> None:
        self.store = store
        self.version = 0
        self.gathered = [0] * len(store.slots)  # version each slot's cache entry is valid for
        self.gemm_slots: set[int] = set()  # slots whose first use is a fused-gather GEMM
        self._small_version = -1
        self._ranges_key: frozenset | None = None
        self._ranges: torch.Tensor | None = None
        self.ready = torch.zeros(8192, dtype=torch.int32, device=store.device)
        self.stats = {"fused_gathers": 0, "range_gathers": 0}

    # ------------------------------------------------------------ versions
    def advance(self) -> None:
        """The owners' shards changed (optimizer step, checkpoint load)."""

        self.version += 1
        for ptr in [p for p, (s, _) in _PENDING.items() if s is self]:
            del _PENDING[ptr]

    @property
    def owner_ptrs(self) -> list[int]:
        return self.store.peer_buffer("owner").peer_ptrs

    # ------------------------------------------------------------ gathers
    def _gather_small(self) -> None:
        """Every slot not served by a fused GEMM, in one launch (once per version)."""

        if self._small_version == self.version:
            return
        key = frozenset(self.gemm_slots)
        if key != self._ranges_key:
            spans = []
            for i, slot in enumerate(self.store.slots):
                if i in key:
                    continue
                lo, hi = slot.offset, _align8(slot.offset + slot.numel)
                if spans and spans[-1][1] >= lo - 64:  # merge neighbours (slots are 64-element aligned)
                    spans[-1][1] = max(spans[-1][1], hi)
                else:
                    spans.append([lo, hi])
            self._ranges = torch.tensor(spans or [[0, 0]], dtype=torch.int64, device=self.store.device)
            self._ranges_key = key
        ext().gather_ranges(self.owner_ptrs, self.store.shard_numel, self._ranges, self.store.compute)
        for i in range(len(self.store.slots)):
            if i not in key:
                self.gathered[i] = self.version
        self._small_version = self.version
        self.stats["range_gathers"] += 1

    def _gather_slot(self, i: int) -> None:
        slot = self.store.slots[i]
        span = torch.tensor([[slot.offset, _align8(slot.offset + slot.numel)]], dtype=torch.int64,
                            device=self.store.device)
        ext().gather_ranges(self.owner_ptrs, self.store.shard_numel, span, self.store.compute)
        self.gathered[i] = self.version
        self.stats["range_gathers"] += 1

    def view(self, param: torch.Tensor, *, fused: bool) -> torch.Tensor:
        """The cache view of a parameter, valid for this version (or pending a fused gather)."""

        i = param.fsdp_slot
        view = param.compute
        if fused:
            # remembered even when already gathered: from the next version on, the
            # range gather leaves this weight to its GEMM
            self.gemm_slots.add(i)
        if self.gathered[i] == self.version:
            return view
        if fused:
            _PENDING[view.data_ptr()] = (self, i)
            return view
        if i in self.gemm_slots:
            self._gather_slot(i)
        else:
            self._gather_small()
            if self.gathered[i] != self.version:
                self._gather_slot(i)
        return view

    def gemm_gather_args(self, i: int):
        slot = self.store.slots[i]
        self.gathered[i] = self.version
        self.stats["fused_gathers"] += 1
        return self.owner_ptrs, self.store.shard_numel, slot.offset, self.ready


def take_pending(weight: torch.Tensor):
    """If ``weight`` is a cache view waiting for its fused gather, claim it: (state, slot) or None."""

    if not _PENDING:
        return None
    return _PENDING.pop(weight.data_ptr(), None)


def materialize_pending(weight: torch.Tensor) -> None:
    """A pending cache view reached a consumer that cannot gather: copy it in now."""

    hit = take_pending(weight)
    if hit is not None:
        state, i = hit
        state._gather_slot(i)


__all__ = ["FSDPState", "materialize_pending", "take_pending"]
