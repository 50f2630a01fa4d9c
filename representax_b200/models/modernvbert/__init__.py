"""ModernVBERT (ModernBERT text + SigLIP vision) retriever and its text tower."""

from .checkpoint import ModernVBERTCheckpointAdapter
from .config import MODERNVBERT_MODEL_ID, ModernVBERTConfig, ModernVBERTTextConfig, SigLIPVisionConfig
from .model import (
    ModernBertTextTower,
    ModernVBERTBatch,
    ModernVBERTEncoder,
    ModernVBERTTextEncoder,
    SigLIPVisionTower,
    merge_image_features,
    patchify,
    pixel_shuffle,
)


def build_modernvbert(*, seed: int = 0, compute_dtype: str = "float32", text_only: bool = False, **config):
    """Dotted-target factory: ``ModernVBERTConfig`` fields (``text``/``vision`` mappings)."""

    import torch

    dtype = getattr(torch, compute_dtype)
    if text_only:
        return ModernVBERTTextEncoder(ModernVBERTTextConfig(**config), seed=seed, compute_dtype=dtype)
    return ModernVBERTEncoder(ModernVBERTConfig(**config), seed=seed, compute_dtype=dtype)


__all__ = ["MODERNVBERT_MODEL_ID", "ModernBertTextTower", "ModernVBERTBatch", "ModernVBERTCheckpointAdapter",
           "ModernVBERTConfig", "ModernVBERTEncoder", "ModernVBERTTextConfig", "ModernVBERTTextEncoder",
           "SigLIPVisionConfig", "SigLIPVisionTower", "build_modernvbert", "merge_image_features", "patchify",
           "pixel_shuffle"]
