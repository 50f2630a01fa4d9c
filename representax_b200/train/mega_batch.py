"""Mega-batch hardest-negative mining execution.

Parity: ``MegaBatchMining`` of src/representax/train/mega_batch.py:27-146:
anchors and positives of the whole (mega) batch are encoded without autograd
in chunks, each anchor's hardest in-batch positive of another row is mined
(row-chunked argmax of cosine, self excluded), and then anchors, positives
and the mined negative payloads are re-encoded differentiably in chunks for
the margin loss.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from representax_b200.core import LossOutput, Route, encode
from representax_b200.parallel.dist import LOCAL
from representax_b200.tasks._batch import leading_rows, slice_rows
from representax_b200.tasks.objectives import hardest_negative_indices, mega_batch_margin_loss


def _gather_rows(payload, index: torch.Tensor):
    """Rows of a payload in the given order (host index)."""

    from representax_b200.models.text_batch import TokenBatch

    idx = index.cpu()
    if isinstance(payload, torch.Tensor):
        return payload[idx.to(payload.device)]
    if isinstance(payload, TokenBatch):
        picked = TokenBatch(attention_mask=payload.attention_mask[idx.to(payload.attention_mask.device)],
                            input_ids=None if payload.input_ids is None else
                            payload.input_ids[idx.to(payload.input_ids.device)],
                            token_type_ids=None if payload.token_type_ids is None else
                            payload.token_type_ids[idx.to(payload.token_type_ids.device)])
        if payload.packed is not None:
            host = picked.map_tensors(lambda t: t.cpu()).pack()
            return host.map_tensors(lambda t: t.to(payload.attention_mask.device))
        return picked
    raise TypeError("mega-batch mining needs tensor or TokenBatch payloads")


@dataclass(frozen=True)
class MegaBatchMining:
    micro_batch_size: int
    loss_row_chunk_size: int | None = None

    def validate(self, task) -> None:
        from representax_b200.tasks.objectives import MegaBatchMarginTask

        if not isinstance(task, MegaBatchMarginTask):
            raise TypeError("mega-batch mining requires the mega_batch_margin loss")

    def run(self, task, model, batch, *, streams, ctx=LOCAL) -> LossOutput:
        rows = leading_rows(batch.anchor)
        chunk = self.micro_batch_size
        with torch.no_grad():
            a = torch.cat([encode(model, slice_rows(batch.anchor, s, min(rows, s + chunk)), route=Route.QUERY)
                           for s in range(0, rows, chunk)])
            p = torch.cat([encode(model, slice_rows(batch.positive, s, min(rows, s + chunk)), route=Route.DOCUMENT)
                           for s in range(0, rows, chunk)])
        valid = getattr(batch, "valid", None)
        negatives = hardest_negative_indices(a, p, valid, chunk=self.loss_row_chunk_size or chunk)
        negative_payload = _gather_rows(batch.positive, negatives)
        total = torch.zeros((), device=a.device)
        # every chunk's share of the masked mean over the whole mega batch
        count = rows if valid is None else max(int(valid.bool().sum()), 1)
        for s in range(0, rows, chunk):
            e = min(rows, s + chunk)
            ea = encode(model, slice_rows(batch.anchor, s, e), route=Route.QUERY)
            ep = encode(model, slice_rows(batch.positive, s, e), route=Route.DOCUMENT)
            en = encode(model, slice_rows(negative_payload, s, e), route=Route.DOCUMENT)
            v = None if valid is None else valid[s:e]
            n_rows = (e - s) if v is None else int(v.bool().sum())
            part = mega_batch_margin_loss(ea, ep, en, task.positive_margin, task.negative_margin, v) * (n_rows / count)
            part.backward()
            total = total + part.detach()
        return LossOutput(loss=total, metrics={})


__all__ = ["MegaBatchMining"]
