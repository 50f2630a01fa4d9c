"""Compound models used by objectives that need more than one encoder.

Parity: ``EncoderPair``, ``PairClassifier``, ``ReconstructionDecoder``,
``TokenReconstructionDecoder`` and ``DenoisingAutoEncoder`` of
src/representax/models/composition.py:90-249.
"""

from __future__ import annotations

import math

import torch
from torch import nn


class EncoderPair(nn.Module):
    """Two towers (contrastive tension trains a copy of the encoder against itself)."""

    def __init__(self, first: nn.Module, second: nn.Module, *, log_scale: float | None = None) -> None:
        super().__init__()
        self.first = first
        self.second = second
        self.log_scale = None if log_scale is None else nn.Parameter(torch.tensor(float(log_scale)))
        self.metadata = first.metadata


class PairClassifier(nn.Module):
    """Encoder plus a linear head over (u, v, |u - v| [, u * v]) features (SoftmaxLoss)."""

    def __init__(self, encoder: nn.Module, num_labels: int, *, concatenation=("u", "v", "abs_diff"),
                 seed: int = 0) -> None:
        super().__init__()
        dim = encoder.metadata.output_dimension * len(concatenation)
        g = torch.Generator().manual_seed(seed)
        bound = 1 / math.sqrt(dim)
        self.encoder = encoder
        self.classifier_weight = nn.Parameter((torch.rand(num_labels, dim, generator=g) * 2 - 1) * bound)
        self.classifier_bias = nn.Parameter((torch.rand(num_labels, generator=g) * 2 - 1) * bound)
        self.metadata = encoder.metadata

    def encode(self, inputs, **kwargs):
        return self.encoder.encode(inputs, **kwargs)


class TokenReconstructionDecoder(nn.Module):
    """A small causal decoder conditioned on the sentence embedding (TSDAE).

    The embedding is the first key/value position of every decoder layer;
    logits are tied to a learned output projection over the vocabulary.
    """

    def __init__(self, vocab_size: int, hidden_size: int, *, layers: int = 1, heads: int = 4,
                 max_positions: int = 512, seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.embed = nn.Parameter(torch.randn(vocab_size, hidden_size, generator=g) * 0.02)
        self.position = nn.Parameter(torch.randn(max_positions, hidden_size, generator=g) * 0.02)
        layer = nn.TransformerDecoderLayer(hidden_size, heads, 4 * hidden_size, dropout=0.0, batch_first=True)
        self.decoder = nn.TransformerDecoder(layer, layers)
        self.output = nn.Linear(hidden_size, vocab_size)

    def forward(self, sentence_embedding: torch.Tensor, target_ids: torch.Tensor) -> torch.Tensor:
        s = target_ids.shape[1]
        x = self.embed[target_ids.long()] + self.position[:s]
        memory = sentence_embedding[:, None, :].to(x.dtype)
        causal = torch.triu(torch.full((s, s), float("-inf"), device=x.device), diagonal=1)
        return self.output(self.decoder(x, memory, tgt_mask=causal))


class DenoisingAutoEncoder(nn.Module):
    def __init__(self, encoder: nn.Module, decoder: nn.Module) -> None:
        super().__init__()
        self.encoder = encoder
        self.decoder = decoder
        self.metadata = encoder.metadata

    def encode(self, inputs, **kwargs):
        return self.encoder.encode(inputs, **kwargs)


__all__ = ["DenoisingAutoEncoder", "EncoderPair", "PairClassifier", "TokenReconstructionDecoder"]
