"""Pairwise, triplet, distillation, classification, contrastive-tension,
regularization, reconstruction and mega-batch objectives.

Parity (formulas, defaults, masking):
  src/representax/tasks/pairwise/losses.py:82-275   cosine regression, (online) contrastive, CoSENT, AnglE
  src/representax/tasks/triplet/losses.py:88-326    explicit triplet, batch all / hard / semi-hard / soft margin
  src/representax/tasks/distillation/losses.py      embedding MSE / L2 / cosine, MarginMSE, distribution KL
  src/representax/tasks/classification/losses.py    SoftmaxLoss on (u, v, |u - v|[, u * v])
  src/representax/tasks/contrastive_tension/        aligned-pair BCE, in-batch cross-entropy
  src/representax/tasks/regularization/losses.py    global orthogonal regularization
  src/representax/tasks/reconstruction/losses.py    TSDAE token reconstruction cross-entropy
  src/representax/tasks/mega_batch/losses.py        hardest-negative margin

Each task follows the representation seam: ``representations`` encodes the
batch columns, ``loss_from_representations`` evaluates the objective, so
modifiers (Matryoshka, adaptive layers) compose with every one of them. The
objectives run on representations ([batch, dim], at most a few thousand rows)
with PyTorch ops on whichever device the representations live.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Literal

import torch
import torch.nn.functional as F
from pydantic import Field

from representax_b200._config import FinitePositiveFloat
from representax_b200.core import LossOutput, Route, encode

from .config import LossConfig, TaskConfig


def _valid(n: int, valid, device) -> torch.Tensor:
    return torch.ones(n, dtype=torch.bool, device=device) if valid is None else valid.to(device).bool()


def _masked_mean(values: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    m = mask.to(values.dtype)
    return (values * m).sum() / torch.clamp(m.sum(), min=1.0)


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float32)


# =============================================================== pairwise
def pairwise_cosine_similarity(left, right):
    left, right = _f32(left), _f32(right)
    ln = torch.clamp(left.norm(dim=1), min=1e-8)
    rn = torch.clamp(right.norm(dim=1), min=1e-8)
    return (left * right).sum(1) / (ln * rn)


def pairwise_angle_similarity(left, right):
    left, right = _f32(left), _f32(right)
    if left.shape[1] % 2:
        left, right = F.pad(left, (0, 1)), F.pad(right, (0, 1))
    a, b = left.chunk(2, dim=1)
    c, d = right.chunk(2, dim=1)
    denom = (c ** 2 + d ** 2).sum(1, keepdim=True)
    real = (a * c + b * d) / denom
    imag = (b * c - a * d) / denom
    ratio = (a ** 2 + b ** 2).sum(1, keepdim=True).sqrt() / (c ** 2 + d ** 2).sum(1, keepdim=True).sqrt()
    return torch.cat((real / ratio, imag / ratio), 1).sum(1).abs()


def pairwise_distance(left, right, metric: str):
    if metric == "cosine":
        return 1.0 - pairwise_cosine_similarity(left, right)
    diff = _f32(left) - _f32(right) + 1e-6
    if metric == "euclidean":
        return diff.norm(p=2, dim=1)
    if metric == "manhattan":
        return diff.norm(p=1, dim=1)
    raise ValueError(f"unsupported pair distance {metric!r}")


def cosine_regression_loss(left, right, labels, valid=None):
    s = pairwise_cosine_similarity(left, right)
    return _masked_mean((s - _f32(labels)) ** 2, _valid(s.shape[0], valid, s.device))


def contrastive_loss(left, right, labels, valid=None, metric="cosine", margin=0.5):
    d = pairwise_distance(left, right, metric)
    y = _f32(labels)
    rows = 0.5 * (y * d ** 2 + (1 - y) * F.relu(margin - d) ** 2)
    return _masked_mean(rows, _valid(d.shape[0], valid, d.device))


def online_contrastive_loss(left, right, labels, valid=None, metric="cosine", margin=0.5):
    d = pairwise_distance(left, right, metric)
    y = _f32(labels)
    v = _valid(d.shape[0], valid, d.device)
    pos, neg = v & (y == 1.0), v & (y == 0.0)
    npos, nneg = pos.sum(), neg.sum()
    inf = torch.tensor(float("inf"), device=d.device)
    pos_max = torch.where(pos, d, -inf).max()
    neg_min = torch.where(neg, d, inf).min()
    pos_mean = torch.where(pos, d, torch.zeros_like(d)).sum() / torch.clamp(npos, min=1)
    neg_mean = torch.where(neg, d, torch.zeros_like(d)).sum() / torch.clamp(nneg, min=1)
    neg_cut = torch.where(npos > 1, pos_max, neg_mean)
    pos_cut = torch.where(nneg > 1, neg_min, pos_mean)
    sel_neg = neg & (d < neg_cut)
    sel_pos = pos & (d > pos_cut)
    rows = torch.where(sel_pos, d ** 2, torch.where(sel_neg, F.relu(margin - d) ** 2, torch.zeros_like(d)))
    return rows.sum()


def pair_ranking_loss(left, right, labels, valid=None, scale=20.0, similarity="cosine"):
    s = pairwise_cosine_similarity(left, right) if similarity == "cosine" else pairwise_angle_similarity(left, right)
    y = _f32(labels)
    v = _valid(s.shape[0], valid, s.device)
    scaled = s * scale
    diff = scaled[:, None] - scaled[None, :]
    ordered = (y[:, None] < y[None, :]) & v[:, None] & v[None, :]
    cand = torch.where(ordered, diff, torch.full_like(diff, float("-inf"))).reshape(-1)
    return torch.logsumexp(torch.cat((torch.zeros(1, device=s.device), cand)), 0)


# =============================================================== triplet
def aligned_triplet_distance(left, right, metric: str):
    left, right = _f32(left), _f32(right)
    if metric == "cosine":
        return 1 - (left * right).sum(1) / (torch.clamp(left.norm(dim=1), min=1e-12)
                                            * torch.clamp(right.norm(dim=1), min=1e-12))
    diff = left - right
    if metric == "euclidean":
        return diff.pow(2).sum(1).sqrt()
    if metric == "manhattan":
        return diff.abs().sum(1)
    raise ValueError(f"unsupported explicit triplet distance {metric!r}")


def pairwise_triplet_distances(x, metric: str):
    x = _f32(x)
    if metric == "cosine":
        n = x / torch.clamp(x.norm(dim=1, keepdim=True), min=1e-12)
        return 1 - n @ n.T
    prod = x @ x.T
    sq = torch.diagonal(prod)
    squared = torch.clamp(sq[None, :] - 2 * prod + sq[:, None], min=0.0)
    if metric == "squared_euclidean":
        return squared
    if metric == "euclidean":
        zero = squared == 0
        return (~zero).float() * torch.sqrt(squared + zero.float() * 1e-16)
    raise ValueError(f"unsupported batch triplet distance {metric!r}")


def explicit_triplet_loss(a, p, n, valid=None, metric="euclidean", margin=5.0):
    dp = aligned_triplet_distance(a, p, metric)
    dn = aligned_triplet_distance(a, n, metric)
    return _masked_mean(F.relu(dp - dn + margin), _valid(dp.shape[0], valid, dp.device))


def triplet_masks(labels, valid=None):
    labels = torch.as_tensor(labels)
    v = _valid(labels.shape[0], valid, labels.device)
    same = labels[:, None] == labels[None, :]
    distinct = ~torch.eye(labels.shape[0], dtype=torch.bool, device=labels.device)
    both = v[:, None] & v[None, :]
    positive = both & distinct & same
    negative = both & ~same
    return positive, negative, positive[:, :, None] & negative[:, None, :]


def batch_all_triplet_loss(x, labels, valid=None, metric="euclidean", margin=5.0):
    d = pairwise_triplet_distances(x, metric)
    _, _, trip = triplet_masks(labels.to(d.device), valid)
    losses = F.relu(d[:, :, None] - d[:, None, :] + margin)
    return _masked_mean(losses, trip & (losses > 1e-16))


def _hard(d, positive, negative):
    inf = torch.tensor(float("inf"), device=d.device)
    hp = torch.where(positive, d, -inf).max(1).values
    hn = torch.where(negative, d, inf).min(1).values
    eligible = positive.any(1) & negative.any(1)
    return hp, hn, eligible


def batch_hard_triplet_loss(x, labels, valid=None, metric="euclidean", margin=5.0):
    d = pairwise_triplet_distances(x, metric)
    positive, negative, _ = triplet_masks(labels.to(d.device), valid)
    hp, hn, eligible = _hard(d, positive, negative)
    rows = torch.where(eligible, F.relu(hp - hn + margin), torch.zeros_like(hp))
    return _masked_mean(rows, eligible)


def batch_hard_soft_margin_triplet_loss(x, labels, valid=None, metric="euclidean"):
    d = pairwise_triplet_distances(x, metric)
    positive, negative, _ = triplet_masks(labels.to(d.device), valid)
    hp, hn, eligible = _hard(d, positive, negative)
    rows = torch.where(eligible, torch.log1p(torch.exp(hp - hn)), torch.zeros_like(hp))
    return _masked_mean(rows, eligible)


def batch_semi_hard_triplet_loss(x, labels, valid=None, metric="euclidean", margin=5.0):
    d = pairwise_triplet_distances(x, metric)
    n = d.shape[0]
    positive, negative, _ = triplet_masks(labels.to(d.device), valid)
    inf = torch.tensor(float("inf"), device=d.device)
    dap = d[:, :, None]
    dan = d[:, None, :].expand(n, n, n)
    neg = negative[:, None, :].expand(n, n, n)
    outside = neg & (dan > dap)
    semi = torch.where(outside, dan, inf).min(2).values
    inside = torch.where(neg, dan, -inf).max(2).values
    chosen = torch.where(outside.any(2), semi, inside)
    losses = F.relu(d - chosen + margin)
    return _masked_mean(losses, positive & negative.any(1)[:, None])


# =============================================================== distillation
def embedding_distillation_loss(student, teacher, valid=None, metric="mse"):
    s, t = _f32(student), _f32(teacher)
    v = _valid(s.shape[0], valid, s.device)
    if metric == "mse":
        rows = ((s - t) ** 2).mean(1)
    elif metric == "l2":
        rows = (s - t).norm(dim=1)
    elif metric == "cosine":
        rows = 1 - F.cosine_similarity(s, t, dim=1, eps=1e-8)
    else:
        raise ValueError(f"unsupported embedding distillation metric {metric!r}")
    return _masked_mean(rows, v)


def margin_mse_loss(q, p, n, teacher_margin, valid=None, similarity="dot"):
    q, p, n = _f32(q), _f32(p), _f32(n)
    if similarity == "cosine":
        q, p, n = (F.normalize(t, dim=1) for t in (q, p, n))
    margin = (q * p).sum(1) - (q * n).sum(1)
    return _masked_mean((margin - _f32(teacher_margin)) ** 2, _valid(q.shape[0], valid, q.device))


def distribution_kl_loss(student_scores, teacher_scores, valid=None, temperature=1.0):
    s = torch.log_softmax(_f32(student_scores) / temperature, -1)
    t = torch.log_softmax(_f32(teacher_scores) / temperature, -1)
    rows = (t.exp() * (t - s)).sum(-1) * temperature ** 2
    return _masked_mean(rows, _valid(s.shape[0], valid, s.device))


# =============================================================== other
def softmax_classification_loss(u, v, labels, weight, bias, *, concatenation=("u", "v", "abs_diff"), valid=None):
    u, v = _f32(u), _f32(v)
    parts = {"u": u, "v": v, "abs_diff": (u - v).abs(), "mul": u * v}
    features = torch.cat([parts[k] for k in concatenation], 1)
    logits = F.linear(features, weight.float(), None if bias is None else bias.float())
    rows = F.cross_entropy(logits, labels.long().to(logits.device), reduction="none")
    return _masked_mean(rows, _valid(u.shape[0], valid, u.device)), logits


def global_orthogonal_regularization(anchor, negative, *, mean_weight=1.0, second_moment_weight=1.0):
    a, n = F.normalize(_f32(anchor), dim=1), F.normalize(_f32(negative), dim=1)
    dots = (a * n).sum(1)
    m1 = dots.mean()
    m2 = (dots ** 2).mean()
    return mean_weight * m1 ** 2 + second_moment_weight * F.relu(m2 - 1.0 / a.shape[1])


def contrastive_tension_loss(u, v, labels):
    logits = (_f32(u) * _f32(v)).sum(1)
    return F.binary_cross_entropy_with_logits(logits, _f32(labels))


def contrastive_tension_in_batch_loss(u, v, scale=20.0):
    cos = F.normalize(_f32(u), dim=1) @ F.normalize(_f32(v), dim=1).T * scale
    target = torch.arange(cos.shape[0], device=cos.device)
    return (F.cross_entropy(cos, target) + F.cross_entropy(cos.T, target)) / 2


def mega_batch_margin_loss(anchor, positive, negative, positive_margin=0.8, negative_margin=0.3, valid=None):
    cp = F.cosine_similarity(_f32(anchor), _f32(positive), dim=1)
    cn = F.cosine_similarity(_f32(anchor), _f32(negative), dim=1)
    rows = F.relu(positive_margin - cp) + F.relu(cn - negative_margin)
    return _masked_mean(rows, _valid(rows.shape[0], valid, rows.device))


def hardest_negative_indices(anchor, candidates, valid=None, chunk: int = 1024) -> torch.Tensor:
    """Each anchor's most similar candidate other than its own pair, among valid candidates.

    The fused tcgen05 mining kernel on CUDA (``ops.mnr.hardest_candidates``);
    ``chunk`` bounds the rows scored at once on the CPU path only."""

    from representax_b200.ops.mnr import hardest_candidates

    del chunk
    return hardest_candidates(anchor, candidates, valid, exclude_offset=0)


# =============================================================== batches
@dataclass
class PairwiseBatch:
    left: Any
    right: Any
    labels: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class ExplicitTripletBatch:
    anchor: Any
    positive: Any
    negative: Any
    valid: torch.Tensor | None = None


@dataclass
class LabeledExamplesBatch:
    examples: Any
    labels: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class EmbeddingDistillationBatch:
    inputs: Any
    teacher: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class MarginDistillationBatch:
    query: Any
    positive: Any
    negative: Any
    teacher_margin: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class DistributionDistillationBatch:
    query: Any
    candidates: tuple
    teacher_scores: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class PairClassificationBatch:
    left: Any
    right: Any
    labels: torch.Tensor
    valid: torch.Tensor | None = None


@dataclass
class ContrastiveTensionBatch:
    left: Any
    right: Any
    labels: torch.Tensor


@dataclass
class ContrastiveTensionExamples:
    examples: Any


@dataclass
class RegularizationBatch:
    anchor: Any
    negative: Any


@dataclass
class DenoisingBatch:
    noisy: Any
    target_ids: torch.Tensor
    target_mask: torch.Tensor


@dataclass
class MegaBatch:
    anchor: Any
    positive: Any
    valid: torch.Tensor | None = None  # rows that take part (padding rows do not)


# =============================================================== tasks
class _RepresentationTask:
    """Shared ``loss`` for tasks following the representation seam."""

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        return self.loss_from_representations(self.representations(model, batch, generator=generator), batch)


@dataclass(frozen=True)
class CosineRegressionTask(_RepresentationTask):
    left_route: Route = Route.GENERIC
    right_route: Route = Route.GENERIC

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return (encode_fn(model, batch.left, route=self.left_route, generator=generator),
                encode_fn(model, batch.right, route=self.right_route, generator=generator))

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=cosine_regression_loss(reps[0], reps[1], batch.labels, batch.valid))

    def accumulation_weight(self, part, whole):
        return float(part.labels.shape[0]) / float(whole.labels.shape[0])


@dataclass(frozen=True)
class ContrastiveTask(CosineRegressionTask):
    distance: str = "cosine"
    margin: float = 0.5
    online: bool = False

    def loss_from_representations(self, reps, batch):
        fn = online_contrastive_loss if self.online else contrastive_loss
        return LossOutput(loss=fn(reps[0], reps[1], batch.labels, batch.valid, self.distance, self.margin))


@dataclass(frozen=True)
class CoSENTTask(CosineRegressionTask):
    scale: float = 20.0

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=pair_ranking_loss(reps[0], reps[1], batch.labels, batch.valid, self.scale, "cosine"))


@dataclass(frozen=True)
class AnglETask(CosineRegressionTask):
    scale: float = 20.0

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=pair_ranking_loss(reps[0], reps[1], batch.labels, batch.valid, self.scale, "angle"))


@dataclass(frozen=True)
class ExplicitTripletTask(_RepresentationTask):
    distance: str = "euclidean"
    margin: float = 5.0
    anchor_route: Route = Route.QUERY
    positive_route: Route = Route.DOCUMENT
    negative_route: Route = Route.DOCUMENT

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return (encode_fn(model, batch.anchor, route=self.anchor_route, generator=generator),
                encode_fn(model, batch.positive, route=self.positive_route, generator=generator),
                encode_fn(model, batch.negative, route=self.negative_route, generator=generator))

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=explicit_triplet_loss(*reps, batch.valid, self.distance, self.margin))


@dataclass(frozen=True)
class BatchTripletTask(_RepresentationTask):
    strategy: Literal["all", "hard", "semi_hard", "hard_soft_margin"] = "all"
    distance: str = "euclidean"
    margin: float = 5.0
    route: Route = Route.GENERIC

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return encode_fn(model, batch.examples, route=self.route, generator=generator)

    def loss_from_representations(self, reps, batch):
        if self.strategy == "all":
            loss = batch_all_triplet_loss(reps, batch.labels, batch.valid, self.distance, self.margin)
        elif self.strategy == "hard":
            loss = batch_hard_triplet_loss(reps, batch.labels, batch.valid, self.distance, self.margin)
        elif self.strategy == "semi_hard":
            loss = batch_semi_hard_triplet_loss(reps, batch.labels, batch.valid, self.distance, self.margin)
        else:
            loss = batch_hard_soft_margin_triplet_loss(reps, batch.labels, batch.valid, self.distance)
        return LossOutput(loss=loss)


@dataclass(frozen=True)
class EmbeddingDistillationTask(_RepresentationTask):
    metric: str = "mse"
    route: Route = Route.GENERIC

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return encode_fn(model, batch.inputs, route=self.route, generator=generator)

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=embedding_distillation_loss(reps, batch.teacher, batch.valid, self.metric))


@dataclass(frozen=True)
class MarginDistillationTask(_RepresentationTask):
    similarity: str = "dot"

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return (encode_fn(model, batch.query, route=Route.QUERY, generator=generator),
                encode_fn(model, batch.positive, route=Route.DOCUMENT, generator=generator),
                encode_fn(model, batch.negative, route=Route.DOCUMENT, generator=generator))

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=margin_mse_loss(*reps, batch.teacher_margin, batch.valid, self.similarity))


@dataclass(frozen=True)
class DistributionDistillationTask(_RepresentationTask):
    temperature: float = 1.0
    similarity: str = "dot"

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        q = encode_fn(model, batch.query, route=Route.QUERY, generator=generator)
        cands = tuple(encode_fn(model, c, route=Route.DOCUMENT, generator=generator) for c in batch.candidates)
        return (q, *cands)

    def loss_from_representations(self, reps, batch):
        q, *cands = reps
        if self.similarity == "cosine":
            q = F.normalize(_f32(q), dim=1)
            cands = [F.normalize(_f32(c), dim=1) for c in cands]
        scores = torch.stack([(_f32(q) * _f32(c)).sum(1) for c in cands], 1)
        return LossOutput(loss=distribution_kl_loss(scores, batch.teacher_scores, batch.valid, self.temperature))


@dataclass(frozen=True)
class GORTask(_RepresentationTask):
    mean_weight: float = 1.0
    second_moment_weight: float = 1.0

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return (encode_fn(model, batch.anchor, route=Route.QUERY, generator=generator),
                encode_fn(model, batch.negative, route=Route.DOCUMENT, generator=generator))

    def loss_from_representations(self, reps, batch):
        return LossOutput(loss=global_orthogonal_regularization(*reps, mean_weight=self.mean_weight,
                                                                second_moment_weight=self.second_moment_weight))


@dataclass(frozen=True)
class MegaBatchMarginTask(_RepresentationTask):
    positive_margin: float = 0.8
    negative_margin: float = 0.3

    def representations(self, model, batch, *, generator=None, encode_fn=encode):
        return (encode_fn(model, batch.anchor, route=Route.QUERY, generator=generator),
                encode_fn(model, batch.positive, route=Route.DOCUMENT, generator=generator))

    def loss_from_representations(self, reps, batch):
        a, p = reps
        valid = getattr(batch, "valid", None)
        idx = hardest_negative_indices(a, p, valid)
        return LossOutput(loss=mega_batch_margin_loss(a, p, p[idx.to(p.device)], self.positive_margin,
                                                      self.negative_margin, valid))


@dataclass(frozen=True)
class SoftmaxClassificationTask:
    """Needs a ``PairClassifier`` model (encoder + linear head)."""

    concatenation: tuple[str, ...] = ("u", "v", "abs_diff")

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        u = encode(model.encoder, batch.left, route=Route.GENERIC, generator=generator)
        v = encode(model.encoder, batch.right, route=Route.GENERIC, generator=generator)
        loss, logits = softmax_classification_loss(u, v, batch.labels, model.classifier_weight,
                                                    model.classifier_bias, concatenation=self.concatenation,
                                                    valid=batch.valid)
        acc = (logits.argmax(1) == batch.labels.to(logits.device)).float().mean()
        return LossOutput(loss=loss, metrics={"accuracy": acc.detach()})


@dataclass(frozen=True)
class ContrastiveTensionTask:
    """Aligned-pair BCE over an ``EncoderPair`` (two towers)."""

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        u = encode(model.first, batch.left, generator=generator)
        v = encode(model.second, batch.right, generator=generator)
        return LossOutput(loss=contrastive_tension_loss(u, v, batch.labels))


@dataclass(frozen=True)
class ContrastiveTensionInBatchTask:
    scale: float = 20.0

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        u = encode(model.first, batch.examples, generator=generator)
        v = encode(model.second, batch.examples, generator=generator)
        return LossOutput(loss=contrastive_tension_in_batch_loss(u, v, self.scale))


@dataclass(frozen=True)
class DenoisingAutoEncoderTask:
    """TSDAE: a decoder reconstructs the clean tokens from the noisy sentence's embedding."""

    def loss(self, model, batch, *, generator=None) -> LossOutput:
        emb = encode(model.encoder, batch.noisy, generator=generator)
        logits = model.decoder(emb, batch.target_ids)
        mask = batch.target_mask.bool()
        targets = batch.target_ids[:, 1:]
        rows = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), targets.reshape(-1).long(),
                               reduction="none")
        return LossOutput(loss=_masked_mean(rows, mask[:, 1:].reshape(-1)))


# =============================================================== configs
class PairwiseConfig(TaskConfig):
    kind: Literal["pairwise"] = "pairwise"
    left_route: Route = Route.GENERIC
    right_route: Route = Route.GENERIC


class CosineRegressionConfig(LossConfig):
    kind: Literal["cosine_regression"] = "cosine_regression"


class ContrastiveConfig(LossConfig):
    kind: Literal["contrastive"] = "contrastive"
    distance: Literal["cosine", "euclidean", "manhattan"] = "cosine"
    margin: FinitePositiveFloat = 0.5
    mining: Literal["none", "online"] = "none"


class CoSENTConfig(LossConfig):
    kind: Literal["cosent"] = "cosent"
    scale: FinitePositiveFloat = 20.0


class AngleConfig(LossConfig):
    kind: Literal["angle"] = "angle"
    scale: FinitePositiveFloat = 20.0


class ExplicitTripletConfig(TaskConfig):
    kind: Literal["explicit_triplet"] = "explicit_triplet"
    anchor_route: Route = Route.QUERY
    positive_route: Route = Route.DOCUMENT
    negative_route: Route = Route.DOCUMENT


class ExplicitTripletLossConfig(LossConfig):
    kind: Literal["triplet"] = "triplet"
    distance: Literal["cosine", "euclidean", "manhattan"] = "euclidean"
    margin: FinitePositiveFloat = 5.0


class LabeledExamplesConfig(TaskConfig):
    kind: Literal["labeled_examples"] = "labeled_examples"
    route: Route = Route.GENERIC


class BatchTripletLossConfig(LossConfig):
    kind: Literal["batch_triplet"] = "batch_triplet"
    strategy: Literal["all", "hard", "semi_hard"] = "all"
    distance: Literal["cosine", "euclidean", "squared_euclidean"] = "euclidean"
    margin: FinitePositiveFloat = 5.0


class BatchHardSoftMarginLossConfig(LossConfig):
    kind: Literal["batch_hard_soft_margin"] = "batch_hard_soft_margin"
    distance: Literal["cosine", "euclidean", "squared_euclidean"] = "euclidean"


class EmbeddingDistillationConfig(TaskConfig):
    kind: Literal["embedding_distillation"] = "embedding_distillation"


class EmbeddingDistillationLossConfig(LossConfig):
    kind: Literal["embedding_distillation"] = "embedding_distillation"
    metric: Literal["mse", "l2", "cosine"] = "mse"


class MarginDistillationConfig(TaskConfig):
    kind: Literal["margin_distillation"] = "margin_distillation"


class MarginMSELossConfig(LossConfig):
    kind: Literal["margin_mse"] = "margin_mse"
    similarity: Literal["dot", "cosine"] = "dot"


class DistributionDistillationConfig(TaskConfig):
    kind: Literal["distribution_distillation"] = "distribution_distillation"


class DistributionKLLossConfig(LossConfig):
    kind: Literal["distribution_kl"] = "distribution_kl"
    temperature: FinitePositiveFloat = 1.0
    similarity: Literal["dot", "cosine"] = "dot"


class PairClassificationConfig(TaskConfig):
    kind: Literal["pair_classification"] = "pair_classification"


class SoftmaxClassificationConfig(LossConfig):
    kind: Literal["softmax_classification"] = "softmax_classification"
    concatenation: tuple[Literal["u", "v", "abs_diff", "mul"], ...] = ("u", "v", "abs_diff")


class ContrastiveTensionPairsConfig(TaskConfig):
    kind: Literal["contrastive_tension_pairs"] = "contrastive_tension_pairs"


class ContrastiveTensionConfig(LossConfig):
    kind: Literal["contrastive_tension"] = "contrastive_tension"


class ContrastiveTensionExamplesConfig(TaskConfig):
    kind: Literal["contrastive_tension_examples"] = "contrastive_tension_examples"


class ContrastiveTensionInBatchConfig(LossConfig):
    kind: Literal["contrastive_tension_in_batch"] = "contrastive_tension_in_batch"
    scale: FinitePositiveFloat = 20.0


class RegularizationConfig(TaskConfig):
    kind: Literal["representation_regularization"] = "representation_regularization"


class GORConfig(LossConfig):
    kind: Literal["global_orthogonal_regularization"] = "global_orthogonal_regularization"
    mean_weight: float = Field(default=1.0, ge=0)
    second_moment_weight: float = Field(default=1.0, ge=0)


class DenoisingConfig(TaskConfig):
    kind: Literal["denoising_reconstruction"] = "denoising_reconstruction"


class DenoisingAutoEncoderConfig(LossConfig):
    kind: Literal["denoising_autoencoder"] = "denoising_autoencoder"


class MegaBatchConfig(TaskConfig):
    kind: Literal["mega_batch"] = "mega_batch"


class MegaBatchMarginConfig(LossConfig):
    kind: Literal["mega_batch_margin"] = "mega_batch_margin"
    positive_margin: float = 0.8
    negative_margin: float = 0.3


__all__ = [name for name in dir() if not name.startswith("_")]
