"""Loss executions: how a task's loss and its parameter gradients are computed.

Parity: ``Direct`` (src/representax/train/execution.py:15-58), ``GradCache``
(src/representax/train/grad_cache.py:110-315) and ``MegaBatchMining``
(src/representax/train/mega_batch.py). An execution's ``run`` leaves the
gradient of the (global) loss in the model's gradient accumulators and
returns the detached loss output.

GradCache runs in three stages: every chunk of queries and documents is
encoded without autograd state; the objective and its gradient with respect
to the representations are computed once over the whole batch (with
cross-rank negatives when distributed); then each chunk is re-encoded with
autograd and back-propagated with its slice of the representation gradient.
Replay draws the same random streams as the first pass, so the update equals
the direct one.

Optionally (``retain_bytes``, off by default so GradCache keeps its memory
bound), the first pass keeps the autograd graph of as many chunks as fit in
that many bytes (``"auto"``: the free HBM minus a reserve for replaying the
others): those chunks are back-propagated straight from their first-pass
graph instead of being re-encoded. The gradient is the same; only the
recomputation is skipped.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from representax_b200.core import LossOutput, Route, encode, evaluate_loss
from representax_b200.parallel.dist import LOCAL, DistContext, gather_rows
from representax_b200.tasks._batch import leading_rows, slice_rows

from .rng import StreamFactory


def _detach(out: LossOutput) -> LossOutput:
    return LossOutput(loss=out.loss.detach(), metrics={k: v.detach() for k, v in out.metrics.items()})


def _global_batch(batch, queries, documents, ctx: DistContext, *, fused: bool = False, symmetric: bool = False):
    """Gather representations and the positive relation across ranks.

    A rank-local batch whose mask spans only its own documents is placed at
    its rank's column block; a process-local batch already spans all ranks'
    documents (rank-major). Every rank then evaluates the same global
    objective.
    """

    from representax_b200.tasks.retrieval.batch import RetrievalBatch

    if not ctx.enabled:
        return queries, documents, batch
    if fused and queries.is_cuda:
        from representax_b200.parallel.fused_mnr import ShardedRetrievalBatch

        return queries, documents, ShardedRetrievalBatch.from_local(batch, ctx, symmetric=symmetric)
    local_d = documents.shape[0]
    global_d = local_d * ctx.world_size
    mask = batch.positive_mask
    weights = batch.weights()
    if mask.shape[1] == local_d:
        wide = torch.zeros(mask.shape[0], global_d, dtype=weights.dtype, device=weights.device)
        wide[:, ctx.rank * local_d:(ctx.rank + 1) * local_d] = weights
        weights = wide
    elif mask.shape[1] != global_d:
        raise ValueError("positive_mask columns must cover the local or the global documents")
    q_all = gather_rows(queries, ctx)
    d_all = gather_rows(documents, ctx)
    w_all = gather_rows(weights.contiguous(), ctx)
    qv = gather_rows(batch.query_valid.to(torch.uint8), ctx).bool()
    dv = gather_rows(batch.document_valid.to(torch.uint8), ctx).bool()
    global_batch = RetrievalBatch(query=q_all, document=d_all, positive_mask=w_all > 0,
                                  positive_weights=w_all, query_valid=qv, document_valid=dv)
    return q_all, d_all, global_batch


def _fusion(task, enabled: bool) -> dict:
    """Use the fused cross-rank MNR kernels for MNR (and Matryoshka-wrapped MNR)."""

    from representax_b200.tasks.modifiers import MatryoshkaTask
    from representax_b200.tasks.retrieval import MNRTask

    base = task.task if isinstance(task, MatryoshkaTask) else task
    if enabled and isinstance(base, MNRTask) and base.negative_scope == "global":
        return {"fused": True, "symmetric": base.symmetric}
    return {"fused": False}


@dataclass(frozen=True)
class Direct:
    """Plain full-batch differentiation."""

    fused: bool = True

    def validate(self, task: Any) -> None:
        return None

    def run(self, task, model, batch, *, streams: StreamFactory, ctx: DistContext = LOCAL) -> LossOutput:
        base = getattr(task, "task", task)
        if ctx.enabled and hasattr(base, "loss_from_representations") and hasattr(batch, "positive_mask"):
            gen = streams("direct")
            queries, documents = base.representations(model, batch, generator=gen, encode_fn=encode)
            q_all, d_all, gbatch = _global_batch(batch, queries, documents, ctx, **_fusion(task, self.fused))
            out = task.loss_from_representations((q_all, d_all), gbatch)
        else:
            out = evaluate_loss(task, model, batch, generator=streams("direct"))
        out.loss.backward()
        return _detach(out)


class RetainBudget:
    """Decides which first-pass chunk graphs stay resident (CUDA only).

    A chunk is kept while the memory already held by kept graphs plus the
    largest graph seen so far fits in the budget; the remaining chunks run
    without autograd state and are replayed later. Run the process with
    ``PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True``: with most of HBM
    held by retained graphs, the default allocator fragments and the
    replays slow down.
    """

    RESERVE = 12 * 2 ** 30

    def __init__(self, limit: int | str | None, device: torch.device | None) -> None:
        if limit is not None and limit != "auto" and not (isinstance(limit, int) and limit >= 0):
            raise ValueError(f"retain_bytes is a byte count >= 0, 'auto' or None, not {limit!r}")
        limit = None if limit == "auto" else (limit or 0)
        self.enabled = device is not None and device.type == "cuda" and limit != 0
        self.device = device
        if self.enabled and limit is None:
            free, _ = torch.cuda.mem_get_info(device)
            # blocks cached by the allocator but not in use are available too
            free += torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
            limit = max(0, free - self.RESERVE)
        self.limit = limit or 0
        self.used = 0
        self.largest = 0

    def admit(self) -> bool:
        return self.enabled and self.used + 2 * self.largest <= self.limit

    def record(self, before: int) -> None:
        size = max(0, torch.cuda.memory_allocated(self.device) - before)
        self.used += size
        self.largest = max(self.largest, size)


def _model_device(model) -> torch.device | None:
    for p in model.parameters():
        return p.device
    return None


def _encode_chunks(model, payload, route: Route, chunk: int, streams: StreamFactory, role: str,
                   budget: RetainBudget | None = None):
    """Encode every chunk; returns (detached reps, rows, {start: (stop, graph reps)})."""

    rows = leading_rows(payload)
    outs, kept = [], {}
    for i, start in enumerate(range(0, rows, chunk)):
        stop = min(rows, start + chunk)
        part = slice_rows(payload, start, stop)
        if budget is not None and budget.admit():
            before = torch.cuda.memory_allocated(budget.device)
            with torch.enable_grad():
                reps = encode(model, part, route=route, generator=streams(role, i))
            budget.record(before)
            kept[start] = (stop, reps)
            outs.append(reps.detach())
        else:
            with torch.no_grad():
                outs.append(encode(model, part, route=route, generator=streams(role, i)))
    return torch.cat(outs), rows, kept


def _replay_chunks(model, payload, route: Route, chunk: int, grads: torch.Tensor, streams: StreamFactory,
                   role: str, kept: dict | None = None) -> None:
    rows = leading_rows(payload)
    kept = kept or {}
    done = set(kept)
    # Retained graphs first: their memory is released before any replay runs.
    for start in sorted(kept):
        stop, reps = kept.pop(start)
        reps.backward(grads[start:stop])
        del reps
    for i, start in enumerate(range(0, rows, chunk)):
        if start in done:
            continue
        stop = min(rows, start + chunk)
        part = slice_rows(payload, start, stop)
        with torch.enable_grad():
            reps = encode(model, part, route=route, generator=streams(role, i))
            reps.backward(grads[start:stop])


@dataclass(frozen=True)
class GradCache:
    """Exact cached differentiation bounded by chunk size."""

    query_chunk_size: int
    document_chunk_size: int | None = None
    loss_row_chunk_size: int | None = None
    fused: bool = True
    # Bytes of first-pass chunk graphs that may stay resident: 0/None = replay
    # every chunk (the GradCache memory bound), "auto" = free HBM minus a reserve.
    retain_bytes: int | str | None = 0
    stats: dict = field(default_factory=dict, compare=False, repr=False)

    def __post_init__(self) -> None:
        if self.query_chunk_size <= 0:
            raise ValueError("query_chunk_size must be positive")
        if self.document_chunk_size is not None and self.document_chunk_size <= 0:
            raise ValueError("document_chunk_size must be positive when set")
        if self.loss_row_chunk_size is not None and self.loss_row_chunk_size <= 0:
            raise ValueError("loss_row_chunk_size must be positive when set")

    @property
    def resolved_document_chunk_size(self) -> int:
        return self.document_chunk_size or self.query_chunk_size

    @property
    def resolved_loss_row_chunk_size(self) -> int:
        return self.loss_row_chunk_size or self.query_chunk_size

    def validate(self, task: Any) -> None:
        from representax_b200.tasks.guided import GISTTask
        from representax_b200.tasks.modifiers import MatryoshkaTask
        from representax_b200.tasks.retrieval import MNRTask

        base = task.task if isinstance(task, MatryoshkaTask) else task
        if not isinstance(base, (MNRTask, GISTTask)):
            raise TypeError("GradCache requires MNRTask, GISTTask, or their Matryoshka modifier")

    def run(self, task, model, batch, *, streams: StreamFactory, ctx: DistContext = LOCAL) -> LossOutput:
        from representax_b200.tasks.guided import GISTBatch, GISTTask
        from representax_b200.tasks.modifiers import MatryoshkaTask

        base = task.task if isinstance(task, MatryoshkaTask) else task
        if isinstance(base, GISTTask) and isinstance(batch, GISTBatch):
            return self._run_gist(task, base, model, batch, streams=streams, ctx=ctx)
        qc, dc = self.query_chunk_size, self.resolved_document_chunk_size
        budget = RetainBudget(self.retain_bytes, _model_device(model))
        queries, _, kept_q = _encode_chunks(model, batch.query, Route.QUERY, qc, streams, "query", budget)
        documents, _, kept_d = _encode_chunks(model, batch.document, Route.DOCUMENT, dc, streams, "document",
                                              budget)
        queries.requires_grad_(True)
        documents.requires_grad_(True)
        n_chunks = -(-queries.shape[0] // qc) + -(-documents.shape[0] // dc)
        self.stats.update(retained_chunks=len(kept_q) + len(kept_d), chunks=n_chunks,
                          retained_bytes=budget.used)
        q_all, d_all, gbatch = _global_batch(batch, queries, documents, ctx, **_fusion(task, self.fused))
        with torch.enable_grad():
            out = task.loss_from_representations((q_all, d_all), gbatch,
                                                 row_chunk_size=self.resolved_loss_row_chunk_size)
            out.loss.backward()
        _replay_chunks(model, batch.query, Route.QUERY, qc, queries.grad, streams, "query", kept_q)
        _replay_chunks(model, batch.document, Route.DOCUMENT, dc, documents.grad, streams, "document", kept_d)
        return _detach(out)

    def _run_gist(self, task, base, model, batch, *, streams, ctx):
        if ctx.enabled:
            raise NotImplementedError("distributed cached GIST is not implemented yet")
        roles = base.cached_roles(batch)
        reps = {}
        for name, (payload, route) in roles.items():
            chunk = self.query_chunk_size if route == Route.QUERY else self.resolved_document_chunk_size
            value, _, _ = _encode_chunks(model, payload, route, chunk, streams, name)
            reps[name] = value.requires_grad_(True)
        with torch.enable_grad():
            out = task.loss_from_representations(base.assemble(reps), batch,
                                                 row_chunk_size=self.resolved_loss_row_chunk_size)
            out.loss.backward()
        for name, (payload, route) in roles.items():
            chunk = self.query_chunk_size if route == Route.QUERY else self.resolved_document_chunk_size
            if reps[name].grad is not None:
                _replay_chunks(model, payload, route, chunk, reps[name].grad, streams, name)
        return _detach(out)


__all__ = ["Direct", "GradCache", "RetainBudget"]
