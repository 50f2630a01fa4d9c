"""Hugging Face / Sentence-Transformers integration, family catalog, pinned loaders."""

from .families import (
    MODEL_FAMILIES,
    FamilySupport,
    ModelFamily,
    get_hugging_face_architecture,
    get_model_family,
    get_model_type_family,
    resolve_native_loader,
)
from .huggingface import load_hf_config, load_safetensor_subset, resolve_hf_checkpoint, save_safetensors

__all__ = ["FamilySupport", "MODEL_FAMILIES", "ModelFamily", "get_hugging_face_architecture", "get_model_family",
           "get_model_type_family", "load_hf_config", "load_safetensor_subset", "resolve_hf_checkpoint",
           "resolve_native_loader", "save_safetensors"]
