"""A shared linear projection encoder for numeric features (tests, recipes).

Parity: ``DenseEncoder`` of src/representax/models/dense.py:18-71.
"""

from __future__ import annotations

import torch
from torch import nn

from representax_b200.core import BUILTIN_MODALITIES, EncoderMetadata, Route


class DenseEncoder(nn.Module):
    def __init__(self, input_dimension: int, output_dimension: int, *, seed: int = 0, normalize: bool = True) -> None:
        super().__init__()
        if input_dimension <= 0 or output_dimension <= 0:
            raise ValueError("input and output dimensions must be positive")
        g = torch.Generator().manual_seed(seed)
        bound = 1.0 / input_dimension ** 0.5
        self.weight = nn.Parameter((torch.rand(output_dimension, input_dimension, generator=g) * 2 - 1) * bound)
        self.bias = nn.Parameter((torch.rand(output_dimension, generator=g) * 2 - 1) * bound)
        self.metadata = EncoderMetadata(model_id="representax/dense", revision="1", output_dimension=output_dimension,
                                        routes=frozenset(Route), modalities=BUILTIN_MODALITIES)
        self.normalize = normalize

    def encode(self, inputs, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        values = torch.as_tensor(inputs)
        if values.ndim != 2:
            raise ValueError("DenseEncoder inputs must have shape [batch, features]")
        out = torch.nn.functional.linear(values.to(self.weight.dtype), self.weight, self.bias).float()
        if not self.normalize:
            return out
        return out / torch.clamp(torch.linalg.vector_norm(out, dim=-1, keepdim=True), min=1e-12)


__all__ = ["DenseEncoder"]
