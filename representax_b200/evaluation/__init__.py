"""Evaluators: the training objective, embedding similarity, information retrieval.

Parity: ``Evaluator`` / ``LossEvaluator`` (src/representax/evaluation/protocol.py,
loss.py), ``embedding_similarity_metrics`` (similarity.py: Pearson and
Spearman, average ranks for ties, for cosine / dot / euclidean / manhattan
scores, Sentence Transformers 5.6 semantics) and
``information_retrieval_metrics`` (retrieval.py: binary-relevance
accuracy / precision / recall / MRR / nDCG / MAP at k).
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol

import numpy as np
import torch

SIMILARITY_FUNCTIONS = ("cosine", "dot", "euclidean", "manhattan")


class Evaluator(Protocol):
    name: str

    def initialize(self) -> Any: ...

    def evaluate_batch(self, model: Any, batch: Any) -> Any: ...

    def accumulate(self, state: Any, values: Any) -> Any: ...

    def finalize(self, state: Any) -> dict[str, float]: ...


@dataclass
class LossEvaluator:
    """Mean task loss over validation batches, weighted by active rows when known."""

    task: Any
    name: str = "loss"

    def initialize(self):
        return {"sum": 0.0, "count": 0.0}

    def evaluate_batch(self, model, batch):
        with torch.no_grad():
            out = self.task.loss(model, batch)
        return float(out.loss), 1.0

    def accumulate(self, state, values):
        loss, weight = values
        state["sum"] += loss * weight
        state["count"] += weight
        return state

    def finalize(self, state):
        return {"loss": state["sum"] / max(state["count"], 1e-12)}


def pearson(left, right) -> float:
    a = np.asarray(left, np.float64) - np.mean(left)
    b = np.asarray(right, np.float64) - np.mean(right)
    d = np.linalg.norm(a) * np.linalg.norm(b)
    return float(np.dot(a, b) / d) if d else float("nan")


def rankdata(values) -> np.ndarray:
    values = np.asarray(values)
    order = np.argsort(values, kind="mergesort")
    s = values[order]
    ranks = np.empty(len(values), dtype=np.float64)
    i = 0
    while i < len(values):
        j = i + 1
        while j < len(values) and s[j] == s[i]:
            j += 1
        ranks[order[i:j]] = (i + j - 1) / 2.0 + 1.0
        i = j
    return ranks


def spearman(left, right) -> float:
    return pearson(rankdata(left), rankdata(right))


def pairwise_scores(left, right, function: str) -> np.ndarray:
    left, right = np.asarray(left, np.float64), np.asarray(right, np.float64)
    if function == "cosine":
        d = np.linalg.norm(left, axis=1) * np.linalg.norm(right, axis=1)
        return np.sum(left * right, axis=1) / np.maximum(d, 1e-12)
    if function == "dot":
        return np.sum(left * right, axis=1)
    if function == "euclidean":
        return -np.linalg.norm(left - right, axis=1)
    if function == "manhattan":
        return -np.sum(np.abs(left - right), axis=1)
    raise ValueError(f"unsupported similarity function {function!r}")


def embedding_similarity_metrics(left, right, labels, *, similarity_functions: Sequence[str] = SIMILARITY_FUNCTIONS
                                 ) -> dict[str, float]:
    left, right, labels = np.asarray(left), np.asarray(right), np.asarray(labels)
    if left.ndim != 2 or right.shape != left.shape:
        raise ValueError("paired embeddings must share shape [pair, representation]")
    if labels.shape != (left.shape[0],):
        raise ValueError("labels must have one scalar per embedding pair")
    if left.shape[0] < 2:
        raise ValueError("embedding similarity requires at least two valid pairs")
    if not (np.isfinite(left).all() and np.isfinite(right).all() and np.isfinite(labels).all()):
        raise ValueError("embedding similarity inputs must be finite")
    out = {}
    for f in similarity_functions:
        s = pairwise_scores(left, right, f)
        out[f"pearson_{f}"] = pearson(labels, s)
        out[f"spearman_{f}"] = spearman(labels, s)
    return out


def _dcg(relevance: Sequence[int], k: int) -> float:
    return float(sum(v / np.log2(i + 2) for i, v in enumerate(relevance[:k])))


def information_retrieval_metrics(ranked_document_ids, query_ids, relevant_documents: Mapping[int, Any], *,
                                  accuracy_at_k=(1, 3, 5, 10), precision_recall_at_k=(1, 3, 5, 10),
                                  mrr_at_k=(10,), ndcg_at_k=(10,), map_at_k=(100,)) -> dict[str, float]:
    ranked = np.asarray(ranked_document_ids)
    queries = np.asarray(query_ids)
    if ranked.ndim != 2:
        raise ValueError("ranked document IDs must have shape [query, rank]")
    if queries.shape != (ranked.shape[0],) or not len(queries):
        raise ValueError("query IDs must match ranked result rows")
    totals: dict[str, float] = {}
    for k in accuracy_at_k:
        totals[f"accuracy@{k}"] = 0.0
    for k in precision_recall_at_k:
        totals[f"precision@{k}"] = 0.0
        totals[f"recall@{k}"] = 0.0
    for k in mrr_at_k:
        totals[f"mrr@{k}"] = 0.0
    for k in ndcg_at_k:
        totals[f"ndcg@{k}"] = 0.0
    for k in map_at_k:
        totals[f"map@{k}"] = 0.0
    for qid, row in zip(queries.tolist(), ranked):
        relevant = frozenset(int(x) for x in relevant_documents.get(int(qid), ()))
        if not relevant:
            raise ValueError(f"query {qid!r} has no relevant documents")
        row = [int(x) for x in row]
        if len(set(row)) != len(row):
            raise ValueError(f"query {qid!r} has duplicate ranked documents")
        hits = [d in relevant for d in row]
        for k in accuracy_at_k:
            totals[f"accuracy@{k}"] += float(any(hits[:k]))
        for k in precision_recall_at_k:
            c = sum(hits[:k])
            totals[f"precision@{k}"] += c / k
            totals[f"recall@{k}"] += c / len(relevant)
        for k in mrr_at_k:
            totals[f"mrr@{k}"] += next((1.0 / r for r, h in enumerate(hits[:k], start=1) if h), 0.0)
        for k in ndcg_at_k:
            totals[f"ndcg@{k}"] += _dcg(hits, k) / _dcg([1] * len(relevant), k)
        for k in map_at_k:
            correct, score = 0, 0.0
            for r, h in enumerate(hits[:k], start=1):
                if h:
                    correct += 1
                    score += correct / r
            totals[f"map@{k}"] += score / min(k, len(relevant))
    n = len(queries)
    return {k: v / n for k, v in totals.items()}


@dataclass
class EmbeddingSimilarityEvaluator:
    """Pairs with scalar labels: batches expose ``left``, ``right``, ``labels``."""

    name: str = "similarity"
    similarity_functions: tuple[str, ...] = SIMILARITY_FUNCTIONS
    main_similarity: str | None = None
    left_route: str = "generic"
    right_route: str = "generic"

    def initialize(self):
        return {"left": [], "right": [], "labels": []}

    def evaluate_batch(self, model, batch):
        from representax_b200.core import encode

        with torch.no_grad():
            left = encode(model, batch.left, route=self.left_route).cpu().numpy()
            right = encode(model, batch.right, route=self.right_route).cpu().numpy()
        return left, right, np.asarray(torch.as_tensor(batch.labels).cpu(), dtype=np.float64)

    def accumulate(self, state, values):
        for key, value in zip(("left", "right", "labels"), values):
            state[key].append(value)
        return state

    def finalize(self, state):
        metrics = embedding_similarity_metrics(np.concatenate(state["left"]), np.concatenate(state["right"]),
                                               np.concatenate(state["labels"]),
                                               similarity_functions=self.similarity_functions)
        if self.main_similarity is not None:
            metrics["spearman"] = metrics[f"spearman_{self.main_similarity}"]
        return metrics


@dataclass
class InformationRetrievalEvaluator:
    """Rank a corpus for each query (batches expose ``query``, ``document``, ``positive_mask``)."""

    name: str = "retrieval"
    k_values: tuple[int, ...] = (1, 3, 5, 10)
    similarity: str = "cosine"

    def initialize(self):
        return {"q": [], "d": [], "mask": []}

    def evaluate_batch(self, model, batch):
        from representax_b200.core import Route, encode

        with torch.no_grad():
            q = encode(model, batch.query, route=Route.QUERY).cpu()
            d = encode(model, batch.document, route=Route.DOCUMENT).cpu()
        return q, d, batch.positive_mask.cpu()

    def accumulate(self, state, values):
        for key, value in zip(("q", "d", "mask"), values):
            state[key].append(value)
        return state

    def finalize(self, state):
        q = torch.cat(state["q"]).double()
        d = torch.cat(state["d"]).double()
        if self.similarity == "cosine":
            q = torch.nn.functional.normalize(q, dim=-1)
            d = torch.nn.functional.normalize(d, dim=-1)
        scores = q @ d.T
        # Block-diagonal relevance: batch b's mask relates its queries to its documents.
        relevant: dict[int, set[int]] = {}
        qoff = doff = 0
        for m in state["mask"]:
            rows, cols = torch.nonzero(m, as_tuple=True)
            for r, c in zip(rows.tolist(), cols.tolist()):
                relevant.setdefault(qoff + r, set()).add(doff + c)
            qoff += m.shape[0]
            doff += m.shape[1]
        kmax = min(max(max(self.k_values), 100), d.shape[0])
        ranked = torch.topk(scores, kmax, dim=1).indices.numpy()
        qids = np.array(sorted(relevant))
        ks = [k for k in self.k_values if k <= kmax]
        return information_retrieval_metrics(ranked[qids], qids, relevant, accuracy_at_k=ks,
                                             precision_recall_at_k=ks, mrr_at_k=(min(10, kmax),),
                                             ndcg_at_k=(min(10, kmax),), map_at_k=(kmax,))


__all__ = ["EmbeddingSimilarityEvaluator", "Evaluator", "InformationRetrievalEvaluator", "LossEvaluator",
           "SIMILARITY_FUNCTIONS", "embedding_similarity_metrics", "information_retrieval_metrics", "pearson",
           "rankdata", "spearman"]
