"""Objective formulas on CPU against direct restatements."""

import math

import pytest
import torch

from representax_b200.tasks import BUILTIN_LOSSES, BUILTIN_LOSS_MODIFIERS, BUILTIN_TASKS
from representax_b200.tasks import objectives as O


def test_registry_counts_match_reference():
    assert len(BUILTIN_TASKS.definitions) == 14
    assert len(BUILTIN_LOSSES.definitions) == 18
    assert set(BUILTIN_LOSS_MODIFIERS.definitions) == {"matryoshka", "adaptive_layer", "matryoshka_2d"}


def test_cosent_matches_formula():
    torch.manual_seed(0)
    u, v = torch.randn(6, 8), torch.randn(6, 8)
    y = torch.tensor([0.1, 0.9, 0.5, 0.3, 0.7, 0.2])
    s = torch.nn.functional.cosine_similarity(u, v) * 20
    terms = [0.0] + [float(s[i] - s[j]) for i in range(6) for j in range(6) if y[i] < y[j]]
    expected = math.log(sum(math.exp(t) for t in terms))
    assert abs(float(O.pair_ranking_loss(u, v, y)) - expected) < 1e-4


def test_batch_hard_triplet():
    torch.manual_seed(1)
    x = torch.randn(8, 4)
    labels = torch.tensor([0, 0, 1, 1, 2, 2, 0, 1])
    d = torch.cdist(x, x)
    rows = []
    for i in range(8):
        pos = [d[i, j] for j in range(8) if j != i and labels[j] == labels[i]]
        neg = [d[i, j] for j in range(8) if labels[j] != labels[i]]
        rows.append(max(0.0, float(max(pos) - min(neg) + 5.0)))
    got = float(O.batch_hard_triplet_loss(x, labels, metric="euclidean", margin=5.0))
    assert abs(got - sum(rows) / len(rows)) < 1e-4


def test_semi_hard_and_all_run_and_are_finite():
    torch.manual_seed(2)
    x = torch.randn(10, 5, requires_grad=True)
    labels = torch.tensor([0, 0, 1, 1, 2, 2, 0, 1, 2, 3])
    for fn in (O.batch_all_triplet_loss, O.batch_semi_hard_triplet_loss, O.batch_hard_soft_margin_triplet_loss):
        loss = fn(x, labels)
        loss.backward()
        assert torch.isfinite(loss) and torch.isfinite(x.grad).all()


def test_gor_and_distillation():
    torch.manual_seed(3)
    a, n = torch.randn(16, 8), torch.randn(16, 8)
    an, nn_ = torch.nn.functional.normalize(a, dim=1), torch.nn.functional.normalize(n, dim=1)
    dots = (an * nn_).sum(1)
    expected = dots.mean() ** 2 + torch.relu((dots ** 2).mean() - 1 / 8)
    assert torch.allclose(O.global_orthogonal_regularization(a, n), expected, atol=1e-6)
    s, t = torch.randn(5, 3), torch.randn(5, 3)
    kl = O.distribution_kl_loss(s, t)
    ref = torch.nn.functional.kl_div(torch.log_softmax(s, -1), torch.log_softmax(t, -1), log_target=True,
                                     reduction="batchmean")
    assert torch.allclose(kl, ref, atol=1e-6)


@pytest.mark.parametrize("kind", sorted(BUILTIN_LOSSES.definitions))
def test_every_loss_config_parses(kind):
    definition = BUILTIN_LOSSES.definition(kind)
    config = definition.config_type()
    assert BUILTIN_LOSSES.parse(config.model_dump()) == config


def test_task_family_import_paths():
    """Each objective family is importable from its own subpackage, as in the reference layout."""

    import importlib

    expected = {
        "pairwise": ["CoSENTTask", "AnglETask", "ContrastiveTask", "CosineRegressionTask", "PairwiseBatch"],
        "triplet": ["BatchTripletTask", "ExplicitTripletTask", "LabeledExamplesBatch"],
        "distillation": ["EmbeddingDistillationTask", "MarginDistillationTask", "DistributionDistillationTask"],
        "classification": ["SoftmaxClassificationTask", "PairClassificationBatch"],
        "contrastive_tension": ["ContrastiveTensionTask", "ContrastiveTensionInBatchTask"],
        "mega_batch": ["MegaBatchMarginTask", "MegaBatch"],
        "reconstruction": ["DenoisingAutoEncoderTask", "DenoisingBatch"],
        "regularization": ["GlobalOrthogonalRegularizationTask", "RegularizationBatch"],
    }
    for family, names in expected.items():
        module = importlib.import_module(f"representax_b200.tasks.{family}")
        for name in names:
            assert name in module.__all__ and getattr(module, name) is not None, (family, name)
