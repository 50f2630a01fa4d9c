"""Semantic model families and the Transformers architecture catalog.

Parity: src/representax/integrations/families.py, architectures.py and the
generated tables they read (I3). The family rows below state, for each
native implementation, the upstream ``model_type`` values it owns, its
modalities, components, input / output contracts, adapters and the
acceptance gates this repository checks (tests named per family). The
architecture catalog is derived from the installed Transformers auto
mappings at import time (no generated source file); its identity is the
library version plus a sha256 of the table.
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Mapping
from dataclasses import dataclass
from enum import StrEnum
from functools import lru_cache
from types import MappingProxyType

from representax_b200.core.model import Modality


class FamilySupport(StrEnum):
    CATALOGUED = "catalogued"
    NATIVE = "native"
    VERIFIED = "verified"


class AcceptanceGate(StrEnum):
    CONFIG_MAPPING = "config_mapping"
    CHECKPOINT_ROUNDTRIP = "checkpoint_roundtrip"
    FORWARD = "forward"
    INPUT_GRADIENT = "input_gradient"
    PARAMETER_GRADIENT = "parameter_gradient"
    OPTIMIZER_UPDATE = "optimizer_update"
    EXPORT_RELOAD = "export_reload"
    PERFORMANCE = "performance"


class CheckpointLayout(StrEnum):
    HUGGING_FACE_SAFETENSORS = "huggingface_safetensors"


@dataclass(frozen=True)
class ModelInputContract:
    name: str
    fields: tuple[str, ...]


@dataclass(frozen=True)
class ModelFamily:
    name: str
    model_types: tuple[str, ...]
    modalities: tuple[Modality, ...]
    components: tuple[str, ...]
    input_contracts: tuple[ModelInputContract, ...]
    output_contracts: tuple[str, ...]
    config_adapter: str
    checkpoint_adapter: str
    implementation_module: str
    acceptance_gates: frozenset[AcceptanceGate]
    support: FamilySupport
    checkpoint_layout: CheckpointLayout = CheckpointLayout.HUGGING_FACE_SAFETENSORS
    native_kernels: tuple[str, ...] = ()


_G = AcceptanceGate
_TEXT = ModelInputContract("text", ("input_ids", "attention_mask"))
_ALL_GATES = frozenset(_G)
_FORWARD_GATES = frozenset({_G.CONFIG_MAPPING, _G.CHECKPOINT_ROUNDTRIP, _G.FORWARD, _G.INPUT_GRADIENT,
                            _G.PARAMETER_GRADIENT})

_FAMILIES = (
    ModelFamily("bert", ("bert",), (Modality.TEXT,),
                ("token_embedding", "absolute_position_embedding", "token_type_embedding", "multi_head_attention",
                 "post_norm_residual", "dense_mlp", "pooler", "mean_pooling", "l2_normalization"),
                (_TEXT,), ("last_hidden_state", "pooler_output", "mean_pooled_l2_normalized_representation"),
                "representax_b200.models.bert.BertConfig.from_hf_config",
                "representax_b200.models.bert.BertCheckpointAdapter", "representax_b200.models.bert", _ALL_GATES,
                FamilySupport.VERIFIED,
                native_kernels=("gemm_tcgen05", "embed_layernorm", "attention_packed", "layernorm_fused_bias",
                                "pool_l2")),
    ModelFamily("mpnet", ("mpnet",), (Modality.TEXT,),
                ("token_embedding", "absolute_position_embedding", "relative_position_bias", "post_norm_residual",
                 "dense_mlp", "mean_pooling", "l2_normalization"),
                (_TEXT,), ("last_hidden_state", "mean_pooled_l2_normalized_representation"),
                "representax_b200.models.mpnet.MPNetConfig.from_hf_config",
                "representax_b200.models.mpnet.MPNetCheckpointAdapter", "representax_b200.models.mpnet",
                _FORWARD_GATES, FamilySupport.NATIVE),
    ModelFamily("modernvbert", ("modernvbert", "modernbert"), (Modality.TEXT, Modality.IMAGE),
                ("token_embedding", "rotary_position_embedding", "sliding_window_attention", "geglu_mlp",
                 "siglip_vision_tower", "pixel_shuffle_connector", "mean_pooling", "l2_normalization"),
                (_TEXT, ModelInputContract("text_image", ("input_ids", "attention_mask", "pixel_values"))),
                ("last_hidden_state", "mean_pooled_l2_normalized_representation"),
                "representax_b200.models.modernvbert.ModernVBERTConfig.from_hf_config",
                "representax_b200.models.modernvbert.ModernVBERTCheckpointAdapter",
                "representax_b200.models.modernvbert", _FORWARD_GATES, FamilySupport.VERIFIED,
                native_kernels=("gemm_tcgen05", "rope", "attention_packed_window", "gated_activation", "layernorm")),
    ModelFamily("jina_v5", ("qwen3", "qwen3_vl_text"), (Modality.TEXT,),
                ("token_embedding", "causal_grouped_query_attention", "rotary_position_embedding",
                 "query_key_rms_normalization", "swiglu_mlp", "last_token_pooling", "matryoshka_truncation",
                 "l2_normalization"),
                (_TEXT,), ("last_hidden_state", "last_token_l2_normalized_representation"),
                "representax_b200.models.qwen3.Qwen3TextConfig.from_hf_config",
                "representax_b200.models.jina_v5.JinaV5CheckpointAdapter", "representax_b200.models.jina_v5",
                _FORWARD_GATES, FamilySupport.VERIFIED,
                native_kernels=("gemm_tcgen05", "qk_rmsnorm_rope", "attention_packed_causal_gqa", "gated_activation",
                                "rmsnorm")),
    ModelFamily("qwen3_vl", ("qwen3_vl",), (Modality.TEXT, Modality.IMAGE),
                ("vision_patch_transformer", "vision_2d_rope", "interpolated_position_embedding", "patch_merger",
                 "deepstack", "interleaved_mrope", "causal_grouped_query_attention", "last_token_pooling",
                 "binary_rerank_head"),
                (_TEXT, ModelInputContract("text_image", ("input_ids", "attention_mask", "pixel_values",
                                                          "image_grid_thw"))),
                ("last_token_l2_normalized_representation", "relevance_score"),
                "representax_b200.models.qwen3_vl.Qwen3VLConfig.from_hf_config",
                "representax_b200.models.qwen3_vl.Qwen3VLCheckpointAdapter", "representax_b200.models.qwen3_vl",
                _FORWARD_GATES, FamilySupport.VERIFIED),
    ModelFamily("qwen2_5_omni", ("qwen2_5_omni", "qwen2_5_omni_thinker"),
                (Modality.TEXT, Modality.IMAGE, Modality.AUDIO, Modality.VIDEO),
                ("windowed_vision_transformer", "audio_conv_transformer", "sectioned_mrope", "swiglu_mlp",
                 "last_token_pooling", "l2_normalization"),
                (_TEXT, ModelInputContract("omni", ("input_ids", "attention_mask", "pixel_values", "image_grid_thw",
                                                    "input_features", "feature_lens"))),
                ("last_token_l2_normalized_representation",),
                "representax_b200.models.qwen2_5_omni.Qwen2_5OmniConfig.from_hf_config",
                "representax_b200.models.qwen2_5_omni.Qwen2_5OmniCheckpointAdapter",
                "representax_b200.models.qwen2_5_omni", _FORWARD_GATES, FamilySupport.VERIFIED),
    ModelFamily("clip", ("clip",), (Modality.TEXT, Modality.IMAGE),
                ("causal_text_transformer", "vision_patch_transformer", "text_projection", "vision_projection",
                 "additive_late_fusion", "optional_l2_normalization"),
                (_TEXT, ModelInputContract("image", ("pixel_values",)),
                 ModelInputContract("text_image", ("input_ids", "attention_mask", "pixel_values"))),
                ("projected_representation", "optionally_l2_normalized_representation"),
                "representax_b200.models.clip.CLIPConfig.from_hf_config",
                "representax_b200.models.clip.CLIPCheckpointAdapter", "representax_b200.models.clip",
                _FORWARD_GATES, FamilySupport.VERIFIED),
)

MODEL_FAMILIES: Mapping[str, ModelFamily] = MappingProxyType({f.name: f for f in _FAMILIES})
MODEL_TYPE_TO_FAMILY: Mapping[str, ModelFamily] = MappingProxyType(
    {t: f for f in _FAMILIES for t in f.model_types})


def get_model_family(name: str) -> ModelFamily:
    try:
        return MODEL_FAMILIES[name]
    except KeyError as error:
        raise KeyError(f"unknown model family {name!r}") from error


def get_model_type_family(model_type: str) -> ModelFamily | None:
    return MODEL_TYPE_TO_FAMILY.get(model_type)


# ---------------------------------------------------------- architectures
class ArchitectureSupport(StrEnum):
    CATALOGUED = "catalogued"
    NATIVE = "native"
    VERIFIED = "verified"


@dataclass(frozen=True)
class HuggingFaceArchitecture:
    model_type: str
    config_class: str
    auto_model_classes: tuple[str, ...]
    support: ArchitectureSupport
    family: str | None

    @property
    def has_auto_model(self) -> bool:
        return bool(self.auto_model_classes)


@lru_cache(maxsize=1)
def _catalog() -> tuple[str, str, Mapping[str, HuggingFaceArchitecture]]:
    import transformers
    from transformers.models.auto.configuration_auto import CONFIG_MAPPING_NAMES
    from transformers.models.auto.modeling_auto import MODEL_MAPPING_NAMES

    rows = {}
    for model_type, config_class in sorted(CONFIG_MAPPING_NAMES.items()):
        auto = MODEL_MAPPING_NAMES.get(model_type, ())
        auto = (auto,) if isinstance(auto, str) else tuple(auto)
        family = get_model_type_family(model_type)
        rows[model_type] = HuggingFaceArchitecture(
            model_type, config_class, auto,
            ArchitectureSupport.CATALOGUED if family is None else ArchitectureSupport(family.support.value),
            None if family is None else family.name)
    digest = hashlib.sha256(json.dumps([[a.model_type, a.config_class, list(a.auto_model_classes)]
                                        for a in rows.values()]).encode()).hexdigest()
    return transformers.__version__, digest, MappingProxyType(rows)


def hugging_face_architectures() -> Mapping[str, HuggingFaceArchitecture]:
    return _catalog()[2]


def catalog_identity() -> tuple[str, str]:
    """(Transformers version, sha256 of the architecture table)."""

    version, digest, _ = _catalog()
    return version, digest


def get_hugging_face_architecture(model_type: str) -> HuggingFaceArchitecture:
    table = hugging_face_architectures()
    if model_type not in table:
        raise KeyError(f"{model_type!r} is not registered by Transformers {catalog_identity()[0]}")
    return table[model_type]


def resolve_native_loader(model_type: str):
    """The checkpoint adapter class of the native family owning ``model_type``."""

    import importlib

    family = get_model_type_family(model_type)
    if family is None:
        raise ValueError(f"Transformers architecture {model_type!r} is catalogued but has no native family")
    module, _, name = family.checkpoint_adapter.rpartition(".")
    return getattr(importlib.import_module(module), name)


__all__ = ["AcceptanceGate", "ArchitectureSupport", "CheckpointLayout", "FamilySupport", "HuggingFaceArchitecture",
           "MODEL_FAMILIES", "MODEL_TYPE_TO_FAMILY", "ModelFamily", "ModelInputContract", "catalog_identity",
           "get_hugging_face_architecture", "get_model_family", "get_model_type_family", "hugging_face_architectures",
           "resolve_native_loader"]
