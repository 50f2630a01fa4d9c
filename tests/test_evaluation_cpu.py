"""Evaluator metrics against known answers and scipy (E1-E3).

Parity: src/representax/evaluation/similarity.py:43-245 (Pearson / Spearman
with average ranks for ties, Sentence Transformers semantics) and
evaluation/retrieval.py:77-396 (binary-relevance accuracy, precision, recall,
MRR, nDCG and MAP at k).
"""

import math
from dataclasses import dataclass

import numpy as np
import pytest
import torch
from scipy import stats

from representax_b200.evaluation import (
    EmbeddingSimilarityEvaluator,
    InformationRetrievalEvaluator,
    LossEvaluator,
    embedding_similarity_metrics,
    information_retrieval_metrics,
    pearson,
    rankdata,
    spearman,
)


def test_rank_correlations_match_scipy_with_ties():
    rng = np.random.default_rng(0)
    a = rng.integers(0, 5, size=40).astype(float)  # many ties
    b = a * 0.5 + rng.normal(size=40)
    assert np.allclose(rankdata(a), stats.rankdata(a))
    assert math.isclose(pearson(a, b), stats.pearsonr(a, b)[0], rel_tol=1e-12)
    assert math.isclose(spearman(a, b), stats.spearmanr(a, b)[0], rel_tol=1e-12)


def test_similarity_metrics_per_function():
    rng = np.random.default_rng(1)
    left, right = rng.normal(size=(12, 6)), rng.normal(size=(12, 6))
    labels = rng.uniform(size=12)
    out = embedding_similarity_metrics(left, right, labels)
    cos = np.array([l @ r / np.linalg.norm(l) / np.linalg.norm(r) for l, r in zip(left, right)])
    dot = np.array([l @ r for l, r in zip(left, right)])
    euc = -np.array([np.linalg.norm(l - r) for l, r in zip(left, right)])
    man = -np.array([np.abs(l - r).sum() for l, r in zip(left, right)])
    for name, scores in (("cosine", cos), ("dot", dot), ("euclidean", euc), ("manhattan", man)):
        assert math.isclose(out[f"pearson_{name}"], stats.pearsonr(labels, scores)[0], rel_tol=1e-10)
        assert math.isclose(out[f"spearman_{name}"], stats.spearmanr(labels, scores)[0], rel_tol=1e-10)
    with pytest.raises(ValueError):
        embedding_similarity_metrics(left[:1], right[:1], labels[:1])


def test_retrieval_metrics_known_answers():
    # query 0: relevant {10, 12}; ranking 11, 10, 13, 12 -> hits at ranks 2 and 4
    # query 1: relevant {20};     ranking 20, 21, 22, 23 -> hit at rank 1
    ranked = np.array([[11, 10, 13, 12], [20, 21, 22, 23]])
    out = information_retrieval_metrics(ranked, [0, 1], {0: [10, 12], 1: [20]}, accuracy_at_k=(1, 3),
                                        precision_recall_at_k=(1, 3), mrr_at_k=(4,), ndcg_at_k=(4,),
                                        map_at_k=(4,))
    assert out["accuracy@1"] == pytest.approx(0.5)
    assert out["accuracy@3"] == pytest.approx(1.0)
    assert out["precision@1"] == pytest.approx(0.5)
    assert out["precision@3"] == pytest.approx((1 / 3 + 1 / 3) / 2)
    assert out["recall@3"] == pytest.approx((1 / 2 + 1) / 2)
    assert out["mrr@4"] == pytest.approx((1 / 2 + 1) / 2)
    dcg0 = 1 / math.log2(3) + 1 / math.log2(5)
    idcg0 = 1 + 1 / math.log2(3)
    assert out["ndcg@4"] == pytest.approx((dcg0 / idcg0 + 1.0) / 2)
    ap0 = (1 / 2 + 2 / 4) / 2
    assert out["map@4"] == pytest.approx((ap0 + 1.0) / 2)
    with pytest.raises(ValueError, match="duplicate"):
        information_retrieval_metrics(np.array([[1, 1]]), [0], {0: [1]}, accuracy_at_k=(1,))


@dataclass
class _Pairs:
    left: torch.Tensor
    right: torch.Tensor
    labels: torch.Tensor


@dataclass
class _Retrieval:
    query: torch.Tensor
    document: torch.Tensor
    positive_mask: torch.Tensor


class _Table(torch.nn.Module):
    """Encoder whose inputs are row indices into a fixed embedding table."""

    def __init__(self, table):
        super().__init__()
        from representax_b200.core import EncoderMetadata

        self.table = torch.nn.Parameter(table, requires_grad=False)
        self.metadata = EncoderMetadata(model_id="table", revision="1", output_dimension=table.shape[1])

    def encode(self, idx, *, route, generator=None):
        return self.table[idx]


def test_evaluators_end_to_end():
    rng = np.random.default_rng(2)
    table = torch.tensor(rng.normal(size=(20, 5)), dtype=torch.float32)
    model = _Table(table)
    sim = EmbeddingSimilarityEvaluator(main_similarity="cosine")
    state = sim.initialize()
    labels = torch.tensor(rng.uniform(size=10))
    for half in (slice(0, 5), slice(5, 10)):
        batch = _Pairs(torch.arange(0, 10)[half], torch.arange(10, 20)[half], labels[half])
        state = sim.accumulate(state, sim.evaluate_batch(model, batch))
    metrics = sim.finalize(state)
    direct = embedding_similarity_metrics(table[:10].numpy(), table[10:].numpy(), labels.numpy())
    assert metrics["spearman"] == pytest.approx(direct["spearman_cosine"])

    ir = InformationRetrievalEvaluator(k_values=(1, 3))
    state = ir.initialize()
    # two batches of (3 queries, 4 documents); query i of a batch is relevant to document i
    for off in (0, 10):
        batch = _Retrieval(torch.arange(off, off + 3), torch.arange(off + 3, off + 7),
                           torch.eye(3, 4, dtype=torch.bool))
        state = ir.accumulate(state, ir.evaluate_batch(model, batch))
    got = ir.finalize(state)
    q = torch.nn.functional.normalize(torch.cat([table[0:3], table[10:13]]).double(), dim=1)
    d = torch.nn.functional.normalize(torch.cat([table[3:7], table[13:17]]).double(), dim=1)
    ranked = torch.argsort(q @ d.T, dim=1, descending=True).numpy()
    relevant = {0: [0], 1: [1], 2: [2], 3: [4], 4: [5], 5: [6]}
    want = information_retrieval_metrics(ranked, list(range(6)), relevant, accuracy_at_k=(1, 3),
                                         precision_recall_at_k=(1, 3), mrr_at_k=(8,), ndcg_at_k=(8,), map_at_k=(8,))
    for key in ("accuracy@1", "accuracy@3", "recall@3", "mrr@8", "ndcg@8", "map@8"):
        assert got[key] == pytest.approx(want[key]), key


def test_loss_evaluator_weighted_mean():
    from representax_b200.core import LossOutput

    class _Task:
        def loss(self, model, batch):
            return LossOutput(loss=torch.tensor(float(batch)), metrics={})

    ev = LossEvaluator(_Task())
    state = ev.initialize()
    for value in (1.0, 2.0, 6.0):
        state = ev.accumulate(state, ev.evaluate_batch(None, value))
    assert ev.finalize(state)["loss"] == pytest.approx(3.0)
