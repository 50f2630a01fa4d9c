"""Evaluation runner (src/representax/train/evaluation.py:24-153).

Builds the configured evaluators, streams the validation batches through
them under the training precision policy and returns ``{metric: value}``
(the loop publishes them in the ``valid/`` namespace).
"""

from __future__ import annotations

from typing import Any

import torch

from representax_b200.evaluation import EmbeddingSimilarityEvaluator, InformationRetrievalEvaluator, LossEvaluator
from representax_b200.precision import precision_context
from representax_b200.tasks._batch import to_device


def build_evaluator(config: Any, task: Any):
    if config.kind == "loss":
        return LossEvaluator(task=task, name=config.name)
    if config.kind == "embedding_similarity":
        return EmbeddingSimilarityEvaluator(name=config.name, similarity_functions=config.similarity_functions,
                                            main_similarity=config.main_similarity,
                                            left_route=config.left_route, right_route=config.right_route)
    if config.kind == "information_retrieval":
        return InformationRetrievalEvaluator(name=config.name, k_values=config.k_values,
                                             similarity=config.similarity)
    raise ValueError(f"unknown evaluator kind {config.kind!r}")


class EvaluationRunner:
    def __init__(self, config: Any, *, model, task, precision, device, resolvers=None, mappers=None) -> None:
        self.config = config
        self.model = model
        self.task = task
        self.precision = precision
        self.device = device
        self.resolvers = resolvers
        self.mappers = mappers
        self.evaluators = [build_evaluator(c, task) for c in config.evaluators]

    def batches(self):
        from .job import build_batches

        count = self.config.max_batches
        return build_batches(self.config.data, batch_size=self.config.batch_size,
                             processor=getattr(self.model, "processor", None), resolvers=self.resolvers,
                             mappers=self.mappers, num_batches=count)

    def __call__(self, iteration: int) -> dict[str, float]:
        loader = self.batches()
        states = [e.initialize() for e in self.evaluators]
        limit = self.config.max_batches or loader.epoch_batches
        loader.num_batches = limit
        iterator = iter(loader)
        try:
            with precision_context(self.precision):
                for i, batch in enumerate(iterator):
                    batch = to_device(batch, self.device)
                    for j, e in enumerate(self.evaluators):
                        states[j] = e.accumulate(states[j], e.evaluate_batch(self.model, batch))
        finally:
            iterator.close()
        out: dict[str, float] = {}
        for e, s in zip(self.evaluators, states):
            for k, v in e.finalize(s).items():
                out[k if e.name == "loss" and k == "loss" else f"{e.name}/{k}"] = v
        return out


def evaluate(model, evaluators, batches, *, precision=None, device="cpu") -> dict[str, float]:
    """Offline evaluation of an already-built model over an iterable of batches."""

    states = [e.initialize() for e in evaluators]
    ctx = precision_context(precision) if precision is not None else torch.no_grad()
    with ctx:
        for batch in batches:
            batch = to_device(batch, torch.device(device))
            for j, e in enumerate(evaluators):
                states[j] = e.accumulate(states[j], e.evaluate_batch(model, batch))
    out = {}
    for e, s in zip(evaluators, states):
        out.update({f"{e.name}/{k}": v for k, v in e.finalize(s).items()})
    return out


__all__ = ["EvaluationRunner", "build_evaluator", "evaluate"]
