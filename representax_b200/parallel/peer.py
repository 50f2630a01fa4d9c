"""Peer memory for one process per GPU: IPC buffers every rank can address.

A :class:`PeerGroup` allocates device buffers with ``cudaMalloc``, exchanges
their IPC handles over the process group once, and opens every peer's
buffer, so kernels load and store other ranks' memory directly over
NVLink / NVSwitch. ``barrier()`` is a device-side barrier on a small signal
pad (monotonic epochs, bounded waits reported through the status word); it
orders the peer loads and stores of fused kernels without a host round trip.

Lifetime: buffers live until :meth:`PeerGroup.close` (called at interpreter
exit); peer mappings are closed before the owning allocations are freed.
"""

from __future__ import annotations

import atexit

import torch
import torch.distributed as dist

from representax_b200.ops._ext import check_status, ext, status

from .dist import DistContext

_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.int32: 2}


class PeerBuffer:
    """One symmetric allocation: a local tensor view plus every rank's address."""

    def __init__(self, group: "PeerGroup", numel: int, dtype: torch.dtype) -> None:
        self.group = group
        self.numel = numel
        self.dtype = dtype
        itemsize = torch.tensor([], dtype=dtype).element_size()
        nbytes = max(256, (numel * itemsize + 255) // 256 * 256)
        C = ext()
        dev = group.device.index
        self.local_ptr = C.ipc_malloc(nbytes, dev)
        handle = C.ipc_handle(self.local_ptr, dev)
        handles = [None] * group.world
        dist.all_gather_object(handles, handle.tolist())
        self.peer_ptrs: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == group.rank:
                self.peer_ptrs.append(self.local_ptr)
            else:
                ptr = C.ipc_open(torch.tensor(h, dtype=torch.uint8), dev)
                self.peer_ptrs.append(ptr)
                self._opened.append(ptr)
        self.ptrs = torch.tensor(self.peer_ptrs, dtype=torch.int64, device=group.device)
        self.tensor = C.wrap_device_pointer(self.local_ptr, numel, _DTYPE_CODE[dtype], dev)

    def close(self) -> None:
        C = ext()
        dev = self.group.device.index
        for ptr in self._opened:
            C.ipc_close(ptr, dev)
        self._opened = []
        if self.local_ptr:
            C.ipc_free(self.local_ptr, dev)
            self.local_ptr = 0


class PeerGroup:
    def __init__(self, ctx: DistContext, device: torch.device) -> None:
        if not ctx.enabled:
            raise ValueError("a peer group needs more than one rank")
        self.ctx = ctx
        self.rank = ctx.rank
        self.world = ctx.world_size
        self.device = torch.device(device)
        self.epoch = 0
        self._buffers: list[PeerBuffer] = []
        self._cache: dict[tuple, PeerBuffer] = {}
        self.pads = self.buffer(self.world, torch.int32)
        dist.barrier()
        atexit.register(self.close)

    def buffer(self, numel: int, dtype: torch.dtype = torch.float32) -> PeerBuffer:
        buf = PeerBuffer(self, numel, dtype)
        self._buffers.append(buf)
        return buf

    def cached(self, key: tuple, numel: int, dtype: torch.dtype = torch.float32) -> PeerBuffer:
        buf = self._cache.get(key)
        if buf is None:
            buf = self.buffer(numel, dtype)
            self._cache[key] = buf
        return buf

    def barrier(self) -> None:
        """Every rank's prior work on its stream (including peer stores) is visible to all."""

        self.epoch += 1
        ext().signal_barrier(self.pads.ptrs, self.rank, self.world, self.epoch, status(self.device))

    def check(self) -> None:
        check_status(self.device)

    def close(self) -> None:
        if not self._buffers:
            return
        try:
            torch.cuda.synchronize(self.device)
            if dist.is_initialized():
                dist.barrier()
        except Exception:
            pass
        for buf in reversed(self._buffers):
            try:
                buf.close()
            except Exception:
                pass
        self._buffers = []
        self._cache = {}


_GROUPS: dict[tuple[int, int], PeerGroup] = {}


def peer_group(ctx: DistContext, device: torch.device) -> PeerGroup:
    key = (ctx.world_size, torch.device(device).index)
    group = _GROUPS.get(key)
    if group is None:
        group = PeerGroup(ctx, device)
        _GROUPS[key] = group
    return group


def close_peer_groups() -> None:
    for group in list(_GROUPS.values()):
        group.close()
    _GROUPS.clear()


__all__ = ["PeerBuffer", "PeerGroup", "close_peer_groups", "peer_group"]
