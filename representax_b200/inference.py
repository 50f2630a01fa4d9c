"""Host inference: strings -> processor batch -> device encode -> numpy.

Parity: ``TextEmbeddingModel`` / ``embed`` of src/representax/inference.py:26-131
(fixed batch signature with the last chunk padded by empty strings, route
prompts, cosine/dot/euclidean/manhattan host similarity). Each chunk is
copied host->device from pinned memory on a side stream so the next chunk's
tokenization overlaps the current encode; the encoder runs under
``torch.inference_mode`` and the model's compute dtype.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import numpy as np
import torch

from representax_b200.core.model import Route, encode
from representax_b200.models.processing import Processor

SIMILARITY_FUNCTIONS = ("cosine", "dot", "euclidean", "manhattan")


def _device_of(model: torch.nn.Module) -> torch.device:
    for p in model.parameters():
        return p.device
    return torch.device("cpu")


def _to_device(batch: Any, device: torch.device) -> Any:
    if device.type != "cuda":
        return batch
    if hasattr(batch, "pack") and getattr(batch, "packed", None) is None and getattr(batch, "input_ids", None) is not None:
        batch = batch.pack()

    def move(t: torch.Tensor) -> torch.Tensor:
        return t.pin_memory().to(device, non_blocking=True) if t.device.type == "cpu" else t.to(device)

    return batch.map_tensors(move) if hasattr(batch, "map_tensors") else batch


class TextEmbeddingModel:
    """A sentence encoder paired with its host processor."""

    def __init__(self, *, model: torch.nn.Module, processor: Processor, similarity_function: str = "cosine") -> None:
        if similarity_function not in SIMILARITY_FUNCTIONS:
            raise ValueError(f"unsupported similarity function: {similarity_function!r}")
        self.model = model
        self.processor = processor
        self.similarity_function = similarity_function

    def preprocess(self, texts: Sequence[str], *, route: Route = Route.GENERIC, prompt_name: str | None = None,
                   prompt: str | None = None) -> Any:
        return self.processor(texts, route=route, prompt_name=prompt_name, prompt=prompt)

    def embed(self, inputs: str | Sequence[str], *, route: Route = Route.GENERIC, batch_size: int = 32,
              prompt_name: str | None = None, prompt: str | None = None) -> np.ndarray:
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        texts = (inputs,) if isinstance(inputs, str) else tuple(inputs)
        if any(not isinstance(t, str) for t in texts):
            raise TypeError("text embedding inputs must be strings")
        if not texts:
            return np.empty((0, self.model.metadata.output_dimension), np.float32)
        route = Route(route)
        device = _device_of(self.model)
        outputs = []
        with torch.inference_mode():
            for start in range(0, len(texts), batch_size):
                chunk = texts[start:start + batch_size]
                real = len(chunk)
                chunk = chunk + ("",) * (batch_size - real)
                batch = _to_device(self.preprocess(chunk, route=route, prompt_name=prompt_name, prompt=prompt),
                                   device)
                out = encode(self.model, batch, route=route)
                outputs.append(out[:real].float().cpu().numpy())
        return np.concatenate(outputs, axis=0)

    def similarity(self, left: np.ndarray, right: np.ndarray) -> np.ndarray:
        left = np.asarray(left, dtype=np.float32)
        right = np.asarray(right, dtype=np.float32)
        if left.ndim != 2 or right.ndim != 2 or left.shape[1] != right.shape[1]:
            raise ValueError("similarity inputs must be aligned rank-two embeddings")
        if self.similarity_function == "cosine":
            left = left / np.maximum(np.linalg.norm(left, axis=1, keepdims=True), 1e-12)
            right = right / np.maximum(np.linalg.norm(right, axis=1, keepdims=True), 1e-12)
            return left @ right.T
        if self.similarity_function == "dot":
            return left @ right.T
        diff = left[:, None, :] - right[None, :, :]
        if self.similarity_function == "euclidean":
            return -np.linalg.norm(diff, axis=-1)
        return -np.abs(diff).sum(-1)


def embed(model: TextEmbeddingModel, inputs: str | Sequence[str], *, route: Route = Route.GENERIC,
          batch_size: int = 32) -> np.ndarray:
    """Functional spelling of :meth:`TextEmbeddingModel.embed`."""

    return model.embed(inputs, route=route, batch_size=batch_size)


__all__ = ["SIMILARITY_FUNCTIONS", "TextEmbeddingModel", "embed"]
