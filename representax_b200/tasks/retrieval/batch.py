"""Retrieval batches with an explicit positive relation.

Parity: ``RetrievalCollator``, ``RetrievalBatch`` and
``ProcessLocalRetrievalBatch`` of src/representax/tasks/retrieval/batch.py:22-248.
"""

from __future__ import annotations

import dataclasses
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import torch

from representax_b200.core import Route
from representax_b200.tasks._batch import leading_rows, map_tensors


@dataclass
class RetrievalBatch:
    """Model-native query/document payloads and a dense positive relation."""

    query: Any
    document: Any
    positive_mask: torch.Tensor
    positive_weights: torch.Tensor | None = None
    query_valid: torch.Tensor | None = None
    document_valid: torch.Tensor | None = None

    def __post_init__(self) -> None:
        mask = self.positive_mask
        if mask.ndim != 2 or mask.dtype != torch.bool:
            raise TypeError("positive_mask must be a boolean matrix")
        q, d = mask.shape
        if self.positive_weights is not None:
            if self.positive_weights.shape != mask.shape:
                raise ValueError("positive_weights must match positive_mask")
            if not self.positive_weights.is_floating_point():
                raise TypeError("positive_weights must be floating point")
        if self.query_valid is None:
            self.query_valid = torch.ones(q, dtype=torch.bool, device=mask.device)
        if self.document_valid is None:
            self.document_valid = torch.ones(d, dtype=torch.bool, device=mask.device)
        if self.query_valid.shape != (q,) or self.query_valid.dtype != torch.bool:
            raise ValueError("query_valid must be a boolean vector matching the query dimension")
        if self.document_valid.shape != (d,) or self.document_valid.dtype != torch.bool:
            raise ValueError("document_valid must be a boolean vector matching the document dimension")
        if leading_rows(self.query) != q:
            raise ValueError("query payloads must be row-major")
        if leading_rows(self.document) != d:
            raise ValueError("document payloads must be row-major")

    def weights(self) -> torch.Tensor:
        """Dense fp32 positive weights (zero where the mask is false)."""

        mask = self.positive_mask
        if self.positive_weights is None:
            return mask.to(torch.float32)
        return torch.where(mask, self.positive_weights.to(torch.float32), torch.zeros((), device=mask.device))

    def rows(self, start: int, stop: int) -> "RetrievalBatch":
        """Rows [start, stop) of both columns, with the relation restricted to them."""

        from representax_b200.tasks._batch import slice_rows

        return RetrievalBatch(
            query=slice_rows(self.query, start, stop),
            document=slice_rows(self.document, start, stop),
            positive_mask=self.positive_mask[start:stop, start:stop],
            positive_weights=None if self.positive_weights is None else self.positive_weights[start:stop, start:stop],
            query_valid=self.query_valid[start:stop],
            document_valid=self.document_valid[start:stop],
        )

    @property
    def batch_size(self) -> int:
        return int(self.positive_mask.shape[0])

    def map_tensors(self, fn) -> "RetrievalBatch":
        return RetrievalBatch(
            query=map_tensors(self.query, fn),
            document=map_tensors(self.document, fn),
            positive_mask=fn(self.positive_mask),
            positive_weights=None if self.positive_weights is None else fn(self.positive_weights),
            query_valid=fn(self.query_valid),
            document_valid=fn(self.document_valid),
        )


def retrieval_batch(*, query: Any, document: Any, positive_mask, positive_weights=None,
                    query_valid=None, document_valid=None) -> RetrievalBatch:
    return RetrievalBatch(
        query=query,
        document=document,
        positive_mask=torch.as_tensor(positive_mask, dtype=torch.bool),
        positive_weights=None if positive_weights is None else torch.as_tensor(positive_weights, dtype=torch.float32),
        query_valid=None if query_valid is None else torch.as_tensor(query_valid, dtype=torch.bool),
        document_valid=None if document_valid is None else torch.as_tensor(document_valid, dtype=torch.bool),
    )


@dataclass
class ProcessLocalRetrievalBatch:
    """Rank-local query/document rows whose positive relation spans all ranks' documents.

    ``positive_mask`` is [local_query, global_document]; documents are owned
    rank-major (rank r holds rows [r * local, (r + 1) * local)).
    """

    query: Any
    document: Any
    positive_mask: torch.Tensor
    positive_weights: torch.Tensor | None = None
    query_valid: torch.Tensor | None = None
    document_valid: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if self.positive_mask.ndim != 2 or self.positive_mask.dtype != torch.bool:
            raise TypeError("positive_mask must be a boolean matrix")
        lq = self.positive_mask.shape[0]
        if self.query_valid is None:
            self.query_valid = torch.ones(lq, dtype=torch.bool)
        if self.document_valid is None:
            self.document_valid = torch.ones(leading_rows(self.document), dtype=torch.bool)

    def weights(self) -> torch.Tensor:
        mask = self.positive_mask
        if self.positive_weights is None:
            return mask.to(torch.float32)
        return torch.where(mask, self.positive_weights.to(torch.float32), torch.zeros((), device=mask.device))

    def map_tensors(self, fn) -> "ProcessLocalRetrievalBatch":
        return dataclasses.replace(
            self,
            query=map_tensors(self.query, fn),
            document=map_tensors(self.document, fn),
            positive_mask=fn(self.positive_mask),
            positive_weights=None if self.positive_weights is None else fn(self.positive_weights),
            query_valid=fn(self.query_valid),
            document_valid=fn(self.document_valid),
        )


class RetrievalCollator:
    """Build aligned query/document batches with one model processor."""

    def __init__(self, *, processor: Any, query_field: str = "query", document_field: str = "positive") -> None:
        self.processor = processor
        self.query_field = query_field
        self.document_field = document_field

    def data_contract(self) -> Mapping[str, Any]:
        return {
            "schema_version": "representax-retrieval-collator-v1",
            "processor": self.processor.data_contract(),
            "query_field": self.query_field,
            "document_field": self.document_field,
        }

    def __call__(self, examples: Sequence[Mapping[str, Any]]) -> RetrievalBatch:
        try:
            queries = tuple(str(e[self.query_field]) for e in examples)
            documents = tuple(str(e[self.document_field]) for e in examples)
        except KeyError as error:
            raise KeyError(f"retrieval record is missing field {error.args[0]!r}") from error
        size = len(examples)
        return retrieval_batch(
            query=self.processor(queries, route=Route.QUERY),
            document=self.processor(documents, route=Route.DOCUMENT),
            positive_mask=torch.eye(size, dtype=torch.bool),
        )


__all__ = ["ProcessLocalRetrievalBatch", "RetrievalBatch", "RetrievalCollator", "retrieval_batch"]
