"""Flat parameter store: every trainable parameter is a view into one buffer.

One contiguous fp32 buffer each holds the master parameters, their gradient
accumulator and the two AdamW moments; a bf16 buffer holds the compute copy.
The optimizer step, gradient-norm, finite check, clipping and compute-copy
refresh then run as a handful of kernels over the whole model, and gradient
collectives operate on one (bucketable) buffer.

Every parameter starts at a 64-element boundary so views stay 256-byte
aligned for TMA and vector loads. Frozen parameters (``requires_grad=False``)
are stored separately and receive no gradient or moment storage.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

ALIGN = 64


@dataclass
class Slot:
    name: str
    offset: int
    numel: int
    shape: tuple[int, ...]


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class FlatParameterStore:
    """``peer_group`` (CUDA, world > 1) selects the sharded-optimizer layout:
    master, gradient and compute buffers live in peer (IPC) memory so one
    kernel can reduce every rank's gradient for this rank's shard and
    another can write the updated parameters into every rank; the AdamW
    moments hold only this rank's shard ``[shard_offset, shard_offset +
    shard_numel)``."""

    def __init__(self, model: nn.Module, *, device: torch.device, compute_dtype: torch.dtype = torch.float32,
                 optimizer_state: bool = True, peer_group=None, fsdp: bool = False) -> None:
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.slots: list[Slot] = []
        params = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        offset = 0
        for name, p in params:
            self.slots.append(Slot(name, offset, p.numel(), tuple(p.shape)))
            offset = _align(offset + p.numel())
        self.mixed = compute_dtype != torch.float32
        self.group = peer_group
        world = 1 if peer_group is None else peer_group.world
        self.numel = max(_align(-(-offset // world)) * world, ALIGN * world)
        shard = self.numel // world
        rank = 0 if peer_group is None else peer_group.rank
        self.shard_offset, self.shard_numel = rank * shard, shard
        self.fsdp = None
        if fsdp:
            if peer_group is None or not self.mixed:
                raise ValueError("FSDP needs a peer group (CUDA, world > 1) and a bf16 compute copy")
            self._init_fsdp(model, params, peer_group, optimizer_state)
            return
        if peer_group is None:
            self.master = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
            self.compute = torch.zeros(self.numel, dtype=compute_dtype, device=self.device) if self.mixed else None
            moments = self.numel
        else:
            self._peer = {"master": peer_group.buffer(self.numel, torch.float32),
                          "grad": peer_group.buffer(self.numel, torch.float32)}
            if self.mixed:
                self._peer["compute"] = peer_group.buffer(self.numel, compute_dtype)
            for key, buf in self._peer.items():
                buf.tensor.zero_()
            self.master, self.grad = self._peer["master"].tensor, self._peer["grad"].tensor
            self.compute = self._peer["compute"].tensor if self.mixed else None
            moments = shard
        self.exp_avg = torch.zeros(moments, dtype=torch.float32, device=self.device) if optimizer_state else None
        self.exp_avg_sq = torch.zeros(moments, dtype=torch.float32, device=self.device) if optimizer_state else None
        self.params: dict[str, nn.Parameter] = {}
        modules = dict(model.named_modules())
        for slot, (name, p) in zip(self.slots, params):
            view = self.master[slot.offset:slot.offset + slot.numel].view(slot.shape)
            view.copy_(p.detach().to(self.device, torch.float32))
            new = nn.Parameter(view, requires_grad=True)
            new.main_grad = self.grad[slot.offset:slot.offset + slot.numel].view(slot.shape)
            if self.mixed:
                new.compute = self.compute[slot.offset:slot.offset + slot.numel].view(slot.shape)
            owner_name, _, attr = name.rpartition(".")
            owner = modules[owner_name] if owner_name else model
            setattr(owner, attr, new)
            self.params[name] = new
        # Frozen parameters and buffers just move to the device.
        for name, p in model.named_parameters():
            if not p.requires_grad and p.device != self.device:
                owner_name, _, attr = name.rpartition(".")
                owner = modules[owner_name] if owner_name else model
                setattr(owner, attr, nn.Parameter(p.detach().to(self.device), requires_grad=False))
        for name, b in list(model.named_buffers()):
            owner_name, _, attr = name.rpartition(".")
            owner = modules[owner_name] if owner_name else model
            owner._buffers[attr] = b.to(self.device)
        self.refresh_compute()

    def _init_fsdp(self, model: nn.Module, params, group, optimizer_state: bool) -> None:
        """Sharded layout: own segment of master / moments / bf16 owner copy; full grad and bf16 cache."""

        from representax_b200.parallel.fsdp import FSDPState

        lo, n = self.shard_offset, self.shard_numel
        full = torch.zeros(self.numel, dtype=torch.float32, device=self.device)  # init only
        for slot, (_, p) in zip(self.slots, params):
            full[slot.offset:slot.offset + slot.numel].copy_(p.detach().reshape(-1).to(self.device, torch.float32))
        self._peer = {"grad": group.buffer(self.numel, torch.float32),
                      "owner": group.buffer(n, self.compute_dtype)}
        self._peer["grad"].tensor.zero_()
        self.grad = self._peer["grad"].tensor
        self.master = full[lo:lo + n].clone()  # this rank's fp32 master segment
        self.owner = self._peer["owner"].tensor  # this rank's bf16 compute segment (peers read it)
        self.compute = full.to(self.compute_dtype)  # local cache of every rank's segment
        del full
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=self.device) if optimizer_state else None
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=self.device) if optimizer_state else None
        self.master_ptrs = torch.tensor([self.master.data_ptr()], dtype=torch.int64, device=self.device)
        self.owner_ptrs = torch.tensor([self.owner.data_ptr()], dtype=torch.int64, device=self.device)
        state = FSDPState(self)
        self.fsdp = state
        self.params: dict[str, nn.Parameter] = {}
        modules = dict(model.named_modules())
        for i, (slot, (name, _)) in enumerate(zip(self.slots, params)):
            cache = self.compute[slot.offset:slot.offset + slot.numel].view(slot.shape)
            new = nn.Parameter(cache, requires_grad=True)
            new.main_grad = self.grad[slot.offset:slot.offset + slot.numel].view(slot.shape)
            new.compute = cache
            new.fsdp_state = state
            new.fsdp_slot = i
            owner_name, _, attr = name.rpartition(".")
            setattr(modules[owner_name] if owner_name else model, attr, new)
            self.params[name] = new
        for name, p in model.named_parameters():  # frozen parameters stay whole on every rank
            if not p.requires_grad and p.device != self.device:
                owner_name, _, attr = name.rpartition(".")
                setattr(modules[owner_name] if owner_name else model, attr,
                        nn.Parameter(p.detach().to(self.device), requires_grad=False))
        for name, b in list(model.named_buffers()):
            owner_name, _, attr = name.rpartition(".")
            (modules[owner_name] if owner_name else model)._buffers[attr] = b.to(self.device)
        self.refresh_compute()

    def peer_buffer(self, which: str):
        return self._peer[which]

    def gather_master(self) -> torch.Tensor:
        """FSDP: the full fp32 master vector (an all-gather of every rank's segment; collective)."""

        import torch.distributed as dist

        full = torch.empty(self.numel, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, self.master.contiguous())
        return full

    def unshard(self) -> None:
        """FSDP, after training: give every parameter its full fp32 master value (collective)."""

        if self.fsdp is None:
            return
        full = self.gather_master()
        with torch.no_grad():
            for slot, p in zip(self.slots, self.params.values()):
                p.data = full[slot.offset:slot.offset + slot.numel].view(slot.shape)
                p.fsdp_state = None
                p.compute = p.data.to(self.compute_dtype)

    # ------------------------------------------------------------------
    def refresh_compute(self) -> None:
        if self.fsdp is not None:  # owner copy from the master segment; every cache entry is stale
            if self.device.type == "cuda":
                from representax_b200.ops._ext import ext

                ext().cast_bf16(self.master, self.owner)
            else:
                self.owner.copy_(self.master.to(self.compute_dtype))
            self.fsdp.advance()
            return
        if not self.mixed:
            return
        if self.device.type == "cuda":
            from representax_b200.ops._ext import ext

            ext().cast_bf16(self.master, self.compute)
        else:
            self.compute.copy_(self.master.to(self.compute_dtype))

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p in self.params.values():
            p.grad = None

    def collect_autograd_grads(self) -> None:
        """Fold gradients that autograd left in ``.grad`` into the flat accumulator."""

        for p in self.params.values():
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(torch.float32))
                p.grad = None

    @property
    def sharded(self) -> bool:
        return self.group is not None

    def peer_pointers(self, which: str) -> torch.Tensor:
        return self._peer[which].ptrs

    def full_moments(self, ctx) -> tuple[torch.Tensor, torch.Tensor]:
        """AdamW moments over the whole flat buffer (all-gathered when sharded)."""

        if not self.sharded:
            return self.exp_avg, self.exp_avg_sq
        import torch.distributed as dist

        out = []
        for m in (self.exp_avg, self.exp_avg_sq):
            full = torch.empty(self.numel, dtype=m.dtype, device=m.device)
            dist.all_gather_into_tensor(full, m.contiguous())
            out.append(full)
        return out[0], out[1]

    def named_views(self, which: str = "master"):
        if self.fsdp is not None and which != "grad":
            raise ValueError(f"FSDP keeps only this rank's segment of {which!r}; use gather_master() or the shard")
        buf = {"master": self.master, "grad": self.grad, "exp_avg": self.exp_avg,
               "exp_avg_sq": self.exp_avg_sq}[which]
        for slot in self.slots:
            yield slot.name, buf[slot.offset:slot.offset + slot.numel].view(slot.shape)

    def state_dict(self) -> dict[str, torch.Tensor]:
        out = {"master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}
        return {k: v for k, v in out.items() if v is not None}

    def load_state_dict(self, state: dict[str, torch.Tensor]) -> None:
        for key, value in state.items():
            getattr(self, key).copy_(value.to(self.device))
        self.refresh_compute()


__all__ = ["FlatParameterStore", "Slot"]
