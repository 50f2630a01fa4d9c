"""Token batches shared by the text encoders, and host-side sequence packing.

A ``TokenBatch`` carries the padded ``[batch, sequence]`` arrays that users and
checkpoints know, plus (after :meth:`TokenBatch.pack`, done on the host before
the batch is copied to the device) a packed description of only the valid
tokens. The native kernels consume the packed form, so padding costs no
compute; ``cu_host`` stays on the host so row slicing never synchronises.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class PackedTokens:
    input_ids: torch.Tensor            # [T] int32
    position_ids: torch.Tensor         # [T] int32
    token_type_ids: torch.Tensor | None  # [T] int32
    cu_seqlens: torch.Tensor           # [B + 1] int32 (moves with the batch)
    cu_host: torch.Tensor              # [B + 1] int64, always on the host
    max_len: int

    @property
    def total(self) -> int:
        return int(self.cu_host[-1])

    def map_tensors(self, fn) -> "PackedTokens":
        return PackedTokens(
            input_ids=fn(self.input_ids),
            position_ids=fn(self.position_ids),
            token_type_ids=None if self.token_type_ids is None else fn(self.token_type_ids),
            cu_seqlens=fn(self.cu_seqlens),
            cu_host=self.cu_host,
            max_len=self.max_len,
        )

    def rows(self, start: int, stop: int) -> "PackedTokens":
        t0, t1 = int(self.cu_host[start]), int(self.cu_host[stop])
        cu_host = self.cu_host[start:stop + 1] - t0
        lengths = cu_host[1:] - cu_host[:-1]
        return PackedTokens(
            input_ids=self.input_ids[t0:t1],
            position_ids=self.position_ids[t0:t1],
            token_type_ids=None if self.token_type_ids is None else self.token_type_ids[t0:t1],
            cu_seqlens=(self.cu_seqlens[start:stop + 1] - t0).to(torch.int32),
            cu_host=cu_host,
            max_len=int(lengths.max()) if lengths.numel() else 0,
        )

    def pin_memory(self) -> "PackedTokens":
        return PackedTokens(
            input_ids=self.input_ids.pin_memory(),
            position_ids=self.position_ids.pin_memory(),
            token_type_ids=None if self.token_type_ids is None else self.token_type_ids.pin_memory(),
            cu_seqlens=self.cu_seqlens.pin_memory(),
            cu_host=self.cu_host,
            max_len=self.max_len,
        )

    def nbytes(self) -> int:
        total = self.input_ids.nbytes + self.position_ids.nbytes + self.cu_seqlens.nbytes
        if self.token_type_ids is not None:
            total += self.token_type_ids.nbytes
        return total


def pack_tokens(input_ids: torch.Tensor, attention_mask: torch.Tensor,
                token_type_ids: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None) -> PackedTokens:
    """Pack the valid tokens of a padded host batch, row-major.

    Positions default to the column index (the Hugging Face convention for
    absolute position embeddings); explicit ``position_ids`` are honoured.
    """

    ids = np.asarray(input_ids.detach().cpu())
    mask = np.asarray(attention_mask.detach().cpu()).astype(bool)
    b, s = mask.shape
    rows, cols = np.nonzero(mask)
    lengths = mask.sum(1).astype(np.int64)
    cu = np.zeros(b + 1, dtype=np.int64)
    np.cumsum(lengths, out=cu[1:])
    packed_ids = ids[rows, cols].astype(np.int32)
    if position_ids is None:
        pos = cols.astype(np.int32)
    else:
        p = np.asarray(position_ids.detach().cpu())
        p = np.broadcast_to(p, (b, s))
        pos = p[rows, cols].astype(np.int32)
    types = None
    if token_type_ids is not None:
        types = torch.from_numpy(np.asarray(token_type_ids.detach().cpu())[rows, cols].astype(np.int32))
    return PackedTokens(
        input_ids=torch.from_numpy(np.ascontiguousarray(packed_ids)),
        position_ids=torch.from_numpy(np.ascontiguousarray(pos)),
        token_type_ids=types,
        cu_seqlens=torch.from_numpy(cu.astype(np.int32)),
        cu_host=torch.from_numpy(cu),
        max_len=int(lengths.max()) if b else 0,
    )


@dataclass
class TokenBatch:
    """Token ids (or input embeddings) and masks accepted by the text encoders."""

    attention_mask: torch.Tensor
    input_ids: torch.Tensor | None = None
    inputs_embeds: torch.Tensor | None = None
    token_type_ids: torch.Tensor | None = None
    position_ids: torch.Tensor | None = None
    packed: PackedTokens | None = field(default=None)

    def __post_init__(self) -> None:
        if (self.input_ids is None) == (self.inputs_embeds is None):
            raise ValueError("specify exactly one of input_ids or inputs_embeds")
        if self.attention_mask.ndim != 2:
            raise ValueError("attention_mask must have shape [batch, sequence]")
        if self.input_ids is not None:
            if self.input_ids.shape != self.attention_mask.shape:
                raise ValueError("input_ids and attention_mask must align")
            if self.input_ids.is_floating_point():
                raise TypeError("input_ids must have an integer dtype")
        else:
            if self.inputs_embeds.ndim != 3 or self.inputs_embeds.shape[:2] != self.attention_mask.shape:
                raise ValueError("inputs_embeds must have shape [batch, sequence, hidden] aligned with the mask")
        if self.token_type_ids is not None and self.token_type_ids.shape != self.attention_mask.shape:
            raise ValueError("token_type_ids and attention_mask must align")
        if self.position_ids is not None:
            if self.position_ids.ndim != 2 or self.position_ids.shape[0] not in {1, self.attention_mask.shape[0]}:
                raise ValueError("position_ids must have shape [batch or 1, sequence]")

    @property
    def batch_size(self) -> int:
        return self.attention_mask.shape[0]

    @classmethod
    def from_arrays(cls, *, input_ids, attention_mask, token_type_ids=None, position_ids=None) -> "TokenBatch":
        """Build from numpy arrays or tensors (ids as int64, mask as int64)."""

        def tensor(value):
            if value is None:
                return None
            return torch.as_tensor(value).to(torch.int64)

        return cls(input_ids=tensor(input_ids), attention_mask=tensor(attention_mask),
                   token_type_ids=tensor(token_type_ids), position_ids=tensor(position_ids))

    def pack(self) -> "TokenBatch":
        """Attach the packed form (host tensors only; call before moving to the device)."""

        if self.input_ids is None:
            return self
        if self.attention_mask.is_cuda:
            raise ValueError("pack() runs on host batches; pack before moving to the device")
        packed = pack_tokens(self.input_ids, self.attention_mask, self.token_type_ids, self.position_ids)
        return dataclasses.replace(self, packed=packed)

    def map_tensors(self, fn) -> "TokenBatch":
        def opt(t):
            return None if t is None else fn(t)

        return TokenBatch(
            attention_mask=fn(self.attention_mask),
            input_ids=opt(self.input_ids),
            inputs_embeds=opt(self.inputs_embeds),
            token_type_ids=opt(self.token_type_ids),
            position_ids=opt(self.position_ids),
            packed=None if self.packed is None else self.packed.map_tensors(fn),
        )

    def rows(self, start: int, stop: int) -> "TokenBatch":
        def opt(t):
            if t is None:
                return None
            return t if t.shape[0] == 1 and self.batch_size != 1 else t[start:stop]

        return TokenBatch(
            attention_mask=self.attention_mask[start:stop],
            input_ids=opt(self.input_ids),
            inputs_embeds=opt(self.inputs_embeds),
            token_type_ids=opt(self.token_type_ids),
            position_ids=opt(self.position_ids),
            packed=None if self.packed is None else self.packed.rows(start, stop),
        )




def packed_segments(batch: "TokenBatch", device: torch.device | str | None = None):
    """(PackedTokens on ``device``, Segments) for a token batch.

    Batches packed on the host by the loader carry ``packed`` already; a
    batch without it is packed here (one device-to-host copy of the mask).
    Positions are the column index of each token.
    """

    from representax_b200.ops.nn import Segments

    device = torch.device(device) if device is not None else batch.attention_mask.device
    pk = batch.packed
    if pk is None:
        ids = batch.input_ids if batch.input_ids is not None else torch.zeros_like(batch.attention_mask)
        pk = pack_tokens(ids, batch.attention_mask, batch.token_type_ids, batch.position_ids)
    if pk.input_ids.device != device:
        pk = pk.map_tensors(lambda t: t.to(device, non_blocking=True))
    seg = Segments([int(v) for v in pk.cu_host.tolist()], pk.cu_seqlens.to(device=device, dtype=torch.int32))
    return pk, seg


__all__ = ["PackedTokens", "TokenBatch", "pack_tokens", "packed_segments"]
