"""GISTEmbed guided in-batch negatives.

Parity: ``GISTBatch``, ``gist_loss_terms`` and ``GISTTask`` of
src/representax/tasks/guided/{batch,losses,task}.py: candidates the offline
guide model scores above the positive (minus an absolute or relative margin)
are masked out of the softmax, optionally with anchor-anchor and
positive-positive blocks, at a fixed temperature.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Literal, NamedTuple

import torch
from pydantic import Field

from representax_b200._config import FinitePositiveFloat
from representax_b200.core import LossOutput, Route, encode
from representax_b200.tasks._batch import leading_rows
from representax_b200.tasks.config import LossConfig, TaskConfig


class GuidedRetrievalConfig(TaskConfig):
    kind: Literal["guided_retrieval"] = "guided_retrieval"


class GISTConfig(LossConfig):
    kind: Literal["gist"] = "gist"
    temperature: FinitePositiveFloat = 0.01
    margin_strategy: Literal["absolute", "relative"] = "absolute"
    margin: float = Field(default=0.0, ge=0)
    contrast_anchors: bool = True
    contrast_positives: bool = True


@dataclass
class GISTBatch:
    anchor: Any
    positive: Any
    guide_anchor: torch.Tensor
    guide_positive: torch.Tensor
    negatives: tuple = ()
    guide_negatives: tuple = ()
    valid: torch.Tensor | None = None

    def __post_init__(self) -> None:
        rows = self.guide_anchor.shape[0]
        if self.valid is None:
            self.valid = torch.ones(rows, dtype=torch.bool, device=self.guide_anchor.device)
        guides = (self.guide_anchor, self.guide_positive, *self.guide_negatives)
        if any(g.ndim != 2 or not g.is_floating_point() or g.shape[0] != rows for g in guides):
            raise TypeError("GIST guide embeddings have to be float matrices with one row per batch row")
        if len(self.negatives) != len(self.guide_negatives):
            raise ValueError(f"{len(self.negatives)} negative columns but {len(self.guide_negatives)} guide columns for them")
        for payload in (self.anchor, self.positive, *self.negatives):
            if leading_rows(payload) != rows:
                raise ValueError("GIST payloads must contain one row per batch row")


def gist_batch(*, anchor, positive, guide_anchor, guide_positive, negatives=(), guide_negatives=(),
               valid=None) -> GISTBatch:
    return GISTBatch(anchor=anchor, positive=positive, guide_anchor=torch.as_tensor(guide_anchor).float(),
                     guide_positive=torch.as_tensor(guide_positive).float(), negatives=tuple(negatives),
                     guide_negatives=tuple(torch.as_tensor(g).float() for g in guide_negatives), valid=valid)


class GISTLossTerms(NamedTuple):
    loss: torch.Tensor
    row_losses: torch.Tensor
    masked_candidates: torch.Tensor


def _check_gist_options(temperature: float, margin_strategy: str, margin: float) -> None:
    wrong = []
    if not (math.isfinite(temperature) and temperature > 0):
        wrong.append(f"temperature {temperature} (needs a finite value > 0)")
    if margin_strategy not in ("absolute", "relative"):
        wrong.append(f"margin_strategy {margin_strategy!r} (absolute or relative)")
    if not (math.isfinite(margin) and margin >= 0):
        wrong.append(f"margin {margin} (needs a finite value >= 0)")
    if wrong:
        raise ValueError("GIST: bad " + "; ".join(wrong))


def _n(x):
    x = x.float()
    return x / torch.clamp(torch.linalg.vector_norm(x, dim=-1, keepdim=True), min=1e-12)


def gist_loss_terms(embeddings, guide_embeddings, *, valid=None, temperature=0.01, margin_strategy="absolute",
                    margin=0.0, contrast_anchors=True, contrast_positives=True, row_chunk_size=None) -> GISTLossTerms:
    if not 2 <= len(embeddings) == len(guide_embeddings):
        raise ValueError(f"GIST takes >= 2 embedding columns (anchor, positive, ...) with one guide column each; "
                         f"got {len(embeddings)} and {len(guide_embeddings)}")
    _check_gist_options(temperature, margin_strategy, 0.0)
    emb = [_n(e) for e in embeddings]
    guide = [_n(g) for g in guide_embeddings]
    b = emb[0].shape[0]
    device = emb[0].device
    valid = torch.ones(b, dtype=torch.bool, device=device) if valid is None else valid.to(device).bool()
    anchor, positive, *negs = emb
    g_anchor, g_positive, *g_negs = guide
    pos_score = (g_anchor * g_positive).sum(-1, keepdim=True)
    threshold = pos_score - margin if margin_strategy == "absolute" else pos_score - pos_score.abs() * margin
    idx = torch.arange(b, device=device)

    def block(rows, cands, grows, gcands, protect):
        scores = rows @ cands.T
        gscores = grows @ gcands.T
        masked = gscores > threshold
        if protect:
            masked = masked & ~(idx[None, :] == idx[:, None])
        masked = masked | ~valid[None, :]
        return scores.masked_fill(masked, float("-inf")), masked.sum()

    blocks, count = [], torch.zeros((), dtype=torch.long, device=device)
    for rows, cands, grows, gcands, protect in (
        [(anchor, positive, g_anchor, g_positive, True)]
        + ([(anchor, anchor, g_anchor, g_anchor, False)] if contrast_anchors else [])
        + ([(positive, positive, g_positive, g_positive, False)] if contrast_positives else [])
        + [(anchor, n, g_anchor, gn, False) for n, gn in zip(negs, g_negs)]
    ):
        blk, c = block(rows, cands, grows, gcands, protect)
        blocks.append(blk)
        count = count + c
    logits = torch.cat(blocks, 1) / temperature
    logits = torch.where(valid[:, None], logits, torch.zeros((), device=device))
    row_losses = -torch.log_softmax(logits, 1)[idx, idx]
    row_losses = torch.where(valid, row_losses, torch.zeros((), device=device))
    loss = row_losses.sum() / torch.clamp(valid.sum(), min=1).float()
    return GISTLossTerms(loss, row_losses, count)


@dataclass(frozen=True)
class GISTTask:
    temperature: float = 0.01
    margin_strategy: Literal["absolute", "relative"] = "absolute"
    margin: float = 0.0
    contrast_anchors: bool = True
    contrast_positives: bool = True

    def __post_init__(self) -> None:
        _check_gist_options(self.temperature, self.margin_strategy, self.margin)

    def representations(self, model, batch: GISTBatch, *, generator=None, encode_fn=encode):
        anchor = encode_fn(model, batch.anchor, route=Route.QUERY, generator=generator)
        positive = encode_fn(model, batch.positive, route=Route.DOCUMENT, generator=generator)
        negatives = tuple(encode_fn(model, n, route=Route.DOCUMENT, generator=generator) for n in batch.negatives)
        return (anchor, positive, *negatives)

    def cached_roles(self, batch: GISTBatch):
        roles = {"anchor": (batch.anchor, Route.QUERY), "positive": (batch.positive, Route.DOCUMENT)}
        for i, n in enumerate(batch.negatives):
            roles[f"negative{i}"] = (n, Route.DOCUMENT)
        return roles

    def assemble(self, reps: dict):
        negs = [reps[k] for k in sorted(k for k in reps if k.startswith("negative"))]
        return (reps["anchor"], reps["positive"], *negs)

    def loss_from_representations(self, representations, batch: GISTBatch, *, row_chunk_size=None) -> LossOutput:
        terms = gist_loss_terms(representations, (batch.guide_anchor, batch.guide_positive, *batch.guide_negatives),
                                valid=batch.valid, temperature=self.temperature,
                                margin_strategy=self.margin_strategy, margin=self.margin,
                                contrast_anchors=self.contrast_anchors, contrast_positives=self.contrast_positives,
                                row_chunk_size=row_chunk_size)
        return LossOutput(loss=terms.loss, metrics={"masked_candidates": terms.masked_candidates.float(),
                                                    "valid_examples": batch.valid.sum().float()})

    def loss(self, model, batch: GISTBatch, *, generator=None) -> LossOutput:
        return self.loss_from_representations(self.representations(model, batch, generator=generator), batch)


__all__ = ["GISTBatch", "GISTConfig", "GISTLossTerms", "GISTTask", "GuidedRetrievalConfig", "gist_batch",
           "gist_loss_terms"]
