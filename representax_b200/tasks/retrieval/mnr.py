"""Multiple-negatives ranking task.

Parity: ``MNRTask`` and ``mnr_loss_terms`` of
src/representax/tasks/retrieval/mnr.py:26-480. Row tiling
(``row_chunk_size``) is accepted for API compatibility; the native path keeps
the full score matrix (4096 x 4096 fp32 is 64 MB on a 180 GB device) and the
CPU path evaluates it directly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Literal, NamedTuple

import torch

from representax_b200.core import EncodeFunction, LossOutput, Route, encode
from representax_b200.ops.mnr import mnr_loss, mnr_terms_reference

from .batch import RetrievalBatch


class MNRLossTerms(NamedTuple):
    loss: torch.Tensor
    forward_loss: torch.Tensor
    reverse_loss: torch.Tensor
    row_losses: torch.Tensor
    reverse_row_losses: torch.Tensor
    cosine_similarity: torch.Tensor
    scaled_logits: torch.Tensor


def _canonical(query_embeddings, document_embeddings, positive_mask, positive_weights, query_valid,
               document_valid, scale):
    q = torch.as_tensor(query_embeddings)
    d = torch.as_tensor(document_embeddings)
    mask = torch.as_tensor(positive_mask)
    if q.ndim != 2 or d.ndim != 2:
        raise ValueError("query and document embeddings must be matrices")
    if q.shape[1] != d.shape[1]:
        raise ValueError("query and document embedding dimensions must match")
    if mask.shape != (q.shape[0], d.shape[0]):
        raise ValueError("positive_mask shape must match the embedding rows")
    if mask.dtype != torch.bool:
        raise TypeError("positive_mask must be boolean")
    if isinstance(scale, bool) or not isinstance(scale, (int, float)):
        raise TypeError("scale must be a real number")
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("scale must be finite and positive")
    qv = torch.ones(q.shape[0], dtype=torch.bool, device=q.device) if query_valid is None else query_valid.to(torch.bool)
    dv = torch.ones(d.shape[0], dtype=torch.bool, device=q.device) if document_valid is None else document_valid.to(torch.bool)
    if qv.shape != (q.shape[0],):
        raise ValueError("query_valid shape must match query rows")
    if dv.shape != (d.shape[0],):
        raise ValueError("document_valid shape must match document rows")
    w = mask.to(torch.float32) if positive_weights is None else positive_weights.to(torch.float32)
    if w.shape != mask.shape:
        raise ValueError("positive_weights must match positive_mask")
    w = torch.where(mask, w, torch.zeros((), device=w.device))
    return q, d, w, qv, dv


def mnr_loss_terms(query_embeddings, document_embeddings, positive_mask, *, positive_weights=None,
                   query_valid=None, document_valid=None, scale: float = 20.0,
                   symmetric: bool = False) -> MNRLossTerms:
    """Auditable MNR intermediates (reference formulation, any device)."""

    q, d, w, qv, dv = _canonical(query_embeddings, document_embeddings, positive_mask,
                                 positive_weights, query_valid, document_valid, scale)
    loss, fwd, rev, row_f, row_r, cosine, logits = mnr_terms_reference(q, d, w, qv, dv, scale, symmetric)
    return MNRLossTerms(loss, fwd, rev, row_f, row_r, cosine, logits)


@dataclass(frozen=True)
class MNRTask:
    """Direct or symmetric multiple-negatives ranking task."""

    scale: float = 20.0
    symmetric: bool = False
    negative_scope: Literal["local", "global"] = "global"

    def __post_init__(self) -> None:
        if not math.isfinite(self.scale) or self.scale <= 0:
            raise ValueError("scale must be finite and positive")
        if self.negative_scope not in {"local", "global"}:
            raise ValueError("negative_scope must be 'local' or 'global'")

    def loss(self, model: Any, batch: RetrievalBatch, *, generator: Any = None) -> LossOutput:
        reps = self.representations(model, batch, generator=generator, encode_fn=encode)
        return self.loss_from_representations(reps, batch)

    def representations(self, model: Any, batch: RetrievalBatch, *, generator: Any = None,
                        encode_fn: EncodeFunction = encode):
        queries = encode_fn(model, batch.query, route=Route.QUERY, generator=generator)
        documents = encode_fn(model, batch.document, route=Route.DOCUMENT, generator=generator)
        return queries, documents

    def loss_from_representations(self, representations, batch: RetrievalBatch, *,
                                  row_chunk_size: int | None = None) -> LossOutput:
        queries, documents = representations
        return self.loss_from_embeddings(queries, documents, batch, row_chunk_size=row_chunk_size)

    def loss_from_embeddings(self, query_embeddings, document_embeddings, batch: RetrievalBatch, *,
                             row_chunk_size: int | None = None) -> LossOutput:
        if row_chunk_size is not None and row_chunk_size <= 0:
            raise ValueError("row_chunk_size must be positive when set")
        from representax_b200.parallel.fused_mnr import ShardedRetrievalBatch, sharded_mnr_loss

        if isinstance(batch, ShardedRetrievalBatch):
            loss, forward, reverse = sharded_mnr_loss(query_embeddings, document_embeddings, batch,
                                                      scale=self.scale, symmetric=self.symmetric)
            return LossOutput(loss=loss, metrics={"forward_loss": forward, "reverse_loss": reverse})
        q, d, w, qv, dv = _canonical(query_embeddings, document_embeddings, batch.positive_mask,
                                     batch.positive_weights, batch.query_valid,
                                     batch.document_valid, self.scale)
        loss, forward, reverse = mnr_loss(q, d, w, qv, dv, scale=self.scale, symmetric=self.symmetric)
        return LossOutput(loss=loss, metrics={"forward_loss": forward.detach(), "reverse_loss": reverse.detach()})


__all__ = ["MNRLossTerms", "MNRTask", "mnr_loss_terms"]
