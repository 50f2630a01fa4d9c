"""Compound models and the executions that use them (M3, T4, K7, K8, K10).

Parity: models/composition.py:90-249 (EncoderPair, PairClassifier, the TSDAE
decoder), train/mega_batch.py:27-146 (mining execution) and the task
families built on them in the reference.
"""

from dataclasses import dataclass

import torch

from representax_b200.core import EncoderMetadata, LossOutput
from representax_b200.precision import FP32_POLICY, precision_context
from representax_b200.tasks import objectives as O


class _Table(torch.nn.Module):
    """Encoder: integer row ids -> rows of a trainable table."""

    def __init__(self, rows, dim, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.table = torch.nn.Parameter(torch.randn(rows, dim, generator=g))
        self.metadata = EncoderMetadata(model_id=f"table{seed}", revision="1", output_dimension=dim)

    def encode(self, idx, *, route=None, generator=None):
        return self.table[idx]


def test_mega_batch_mining_gradient_equals_direct_margin_loss():
    from representax_b200.train.mega_batch import MegaBatchMining

    model = _Table(16, 6, seed=0)
    batch = O.MegaBatch(anchor=torch.arange(0, 8), positive=torch.arange(8, 16))
    task = O.MegaBatchMarginTask()
    with precision_context(FP32_POLICY):
        out = MegaBatchMining(micro_batch_size=3).run(task, model, batch, streams=None)
    mined = model.table.grad.clone()
    model.table.grad = None
    a, p = model.table[:8], model.table[8:]
    with torch.no_grad():
        cos = torch.nn.functional.normalize(a, dim=1) @ torch.nn.functional.normalize(p, dim=1).T
        cos.fill_diagonal_(float("-inf"))
        hardest = cos.argmax(1)
    direct = O.mega_batch_margin_loss(a, p, p[hardest])
    direct.backward()
    assert torch.allclose(out.loss, direct.detach(), atol=1e-6)
    assert torch.allclose(mined, model.table.grad, atol=1e-6)


def test_mega_batch_mining_honours_valid_rows():
    """Padding rows are neither mined as negatives nor counted in the margin mean."""

    from representax_b200.train.mega_batch import MegaBatchMining

    model = _Table(16, 6, seed=3)
    valid = torch.tensor([True, True, False, True, True, True, False, True])
    batch = O.MegaBatch(anchor=torch.arange(0, 8), positive=torch.arange(8, 16), valid=valid)
    task = O.MegaBatchMarginTask(positive_margin=0.9, negative_margin=-0.5)
    with precision_context(FP32_POLICY):
        out = MegaBatchMining(micro_batch_size=3).run(task, model, batch, streams=None)
        via_task = task.loss_from_representations((model.table[:8], model.table[8:]), batch).loss
    mined = model.table.grad.clone()
    model.table.grad = None
    a, p = model.table[:8].double(), model.table[8:].double()
    with torch.no_grad():
        cos = torch.nn.functional.normalize(a, dim=1) @ torch.nn.functional.normalize(p, dim=1).T
        cos.fill_diagonal_(float("-inf"))
        cos[:, ~valid] = float("-inf")
        hardest = cos.argmax(1)
    assert not valid[hardest].logical_not().any()
    cp = torch.nn.functional.cosine_similarity(a, p, dim=1)
    cn = torch.nn.functional.cosine_similarity(a, p[hardest], dim=1)
    rows = torch.relu(0.9 - cp) + torch.relu(cn + 0.5)
    direct = (rows * valid).sum() / valid.sum()
    direct.backward()
    assert abs(float(out.loss) - float(direct)) < 1e-6
    assert abs(float(via_task) - float(direct)) < 1e-6
    assert torch.allclose(mined.double(), model.table.grad.double(), atol=1e-6)


def test_hardest_candidates_masks_and_offsets():
    from representax_b200.ops.mnr import hardest_candidates

    g = torch.Generator().manual_seed(5)
    a, c = torch.randn(10, 5, generator=g), torch.randn(14, 5, generator=g)
    valid = torch.rand(14, generator=g) > 0.3
    got = hardest_candidates(a, c, valid, exclude_offset=4)
    cos = torch.nn.functional.normalize(a.double(), dim=1) @ torch.nn.functional.normalize(c.double(), dim=1).T
    cos[:, ~valid] = float("-inf")
    cos[torch.arange(10), torch.arange(10) + 4] = float("-inf")
    assert torch.equal(got, cos.argmax(1))
    assert torch.equal(hardest_candidates(a, c, exclude_offset=None), (a @ c.T / c.norm(dim=1)).argmax(1))


def test_pair_classifier_softmax_task():
    from representax_b200.models.composition import PairClassifier

    model = PairClassifier(_Table(10, 4, seed=1), num_labels=3, concatenation=("u", "v", "abs_diff", "mul"))
    assert model.classifier_weight.shape == (3, 16)
    batch = O.PairClassificationBatch(left=torch.arange(0, 5), right=torch.arange(5, 10),
                                      labels=torch.tensor([0, 1, 2, 1, 0]), valid=None)
    task = O.SoftmaxClassificationTask(concatenation=("u", "v", "abs_diff", "mul"))
    with precision_context(FP32_POLICY):
        out = task.loss(model, batch)
    u, v = model.encoder.table[:5], model.encoder.table[5:]
    feats = torch.cat([u, v, (u - v).abs(), u * v], 1)
    logits = feats @ model.classifier_weight.T + model.classifier_bias
    want = torch.nn.functional.cross_entropy(logits, batch.labels)
    assert torch.allclose(out.loss, want, atol=1e-6)
    assert 0.0 <= float(out.metrics["accuracy"]) <= 1.0
    out.loss.backward()
    assert model.classifier_weight.grad is not None and model.encoder.table.grad is not None


def test_contrastive_tension_uses_both_towers():
    from representax_b200.models.composition import EncoderPair

    pair = EncoderPair(_Table(6, 4, seed=2), _Table(6, 4, seed=3))
    aligned = O.ContrastiveTensionBatch(left=torch.arange(0, 3), right=torch.arange(3, 6),
                                        labels=torch.tensor([1.0, 0.0, 0.0]))
    with precision_context(FP32_POLICY):
        out = O.ContrastiveTensionTask().loss(pair, aligned)
        want = O.contrastive_tension_loss(pair.first.table[:3], pair.second.table[3:], aligned.labels)
        assert torch.allclose(out.loss, want)
        out.loss.backward()
        assert pair.first.table.grad is not None and pair.second.table.grad is not None
        examples = O.ContrastiveTensionExamples(examples=torch.arange(0, 6))
        inb = O.ContrastiveTensionInBatchTask(scale=10.0).loss(pair, examples)
        assert torch.allclose(inb.loss, O.contrastive_tension_in_batch_loss(pair.first.table, pair.second.table,
                                                                            10.0))


def test_tsdae_reconstruction_cross_entropy():
    from representax_b200.models.composition import DenoisingAutoEncoder, TokenReconstructionDecoder

    torch.manual_seed(4)
    vocab, dim = 30, 8
    model = DenoisingAutoEncoder(_Table(4, dim, seed=5), TokenReconstructionDecoder(vocab, dim, heads=2))
    targets = torch.randint(0, vocab, (4, 6))
    mask = torch.ones(4, 6, dtype=torch.int32)
    mask[1, 4:] = 0
    batch = O.DenoisingBatch(noisy=torch.arange(4), target_ids=targets, target_mask=mask)
    with precision_context(FP32_POLICY):
        out = O.DenoisingAutoEncoderTask().loss(model, batch)
    logits = model.decoder(model.encoder.table, targets)
    total, count = 0.0, 0
    for b in range(4):
        for t in range(1, 6):
            if mask[b, t]:
                total += torch.nn.functional.cross_entropy(logits[b, t - 1][None], targets[b, t][None])
                count += 1
    assert torch.allclose(out.loss, total / count, atol=1e-5)
    # causal: the logits at position t do not depend on targets after t
    changed = targets.clone()
    changed[:, 5] = (changed[:, 5] + 1) % vocab
    again = model.decoder(model.encoder.table, changed)
    assert torch.allclose(again[:, :5], logits[:, :5], atol=1e-5)
