"""Pinned loaders for the upstream checkpoints the reference names.

Parity: src/representax/integrations/jina.py:33-70 and
src/representax/integrations/modernvbert.py:33-68 (I4). This framework
runs offline: the loaders take a local snapshot directory of the pinned
repository and revision.
"""

from __future__ import annotations

import os

import torch

from representax_b200.models.jina_v5 import JINA_V5_MODEL_ID, load_jina_v5_small_text_encoder
from representax_b200.models.modernvbert import MODERNVBERT_MODEL_ID, ModernVBERTCheckpointAdapter


def load_modernvbert_text_encoder(path: str | os.PathLike, *, compute_dtype: torch.dtype = torch.float32, **kwargs):
    """The ModernVBERT text tower alone (ModernBERT encoder, mean pool + L2)."""

    return ModernVBERTCheckpointAdapter.load(path, text_only=True, compute_dtype=compute_dtype, **kwargs)


def load_modernvbert(path: str | os.PathLike, *, compute_dtype: torch.dtype = torch.float32, **kwargs):
    return ModernVBERTCheckpointAdapter.load(path, compute_dtype=compute_dtype, **kwargs)


__all__ = ["JINA_V5_MODEL_ID", "MODERNVBERT_MODEL_ID", "load_jina_v5_small_text_encoder", "load_modernvbert",
           "load_modernvbert_text_encoder"]
