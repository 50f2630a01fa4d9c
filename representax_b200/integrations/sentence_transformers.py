"""Sentence-Transformers artifact loader (no checkpoint Python is executed).

Parity: src/representax/integrations/sentence_transformers.py:96-954 —
``modules.json`` parsing, role classification of the module graph (dense
embedding, direct embedding, generative / feature reranker, legacy CLIP,
Router-routed encoder), Router structure parsing with ``(task, modality)``
selectors, Pooling/Dense/Normalize loading with the same trusted activation
allow-list, prompt / similarity / truncation metadata, and
``load_sentence_transformer`` returning a ``TextEmbeddingModel``. Only
local directories resolve (this framework runs offline).
"""

from __future__ import annotations

import json
from ast import literal_eval
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from enum import StrEnum
from pathlib import Path
from types import MappingProxyType
from typing import Any

import torch

from representax_b200.core.model import EncoderMetadata, Modality, Route
from representax_b200.models.sentence import (
    POOLING_MODES,
    SentenceBatch,
    SentenceDense,
    SentenceEncoder,
    SentenceNormalize,
    SentencePooling,
)

from .huggingface import load_hf_config, load_safetensor_subset, resolve_hf_checkpoint

SENTENCE_TRANSFORMERS_ORACLE_VERSION = "5.6.1"

_LEGACY_POOLING_KEYS = (
    ("pooling_mode_cls_token", "cls"),
    ("pooling_mode_max_tokens", "max"),
    ("pooling_mode_mean_tokens", "mean"),
    ("pooling_mode_mean_sqrt_len_tokens", "mean_sqrt_len_tokens"),
    ("pooling_mode_weightedmean_tokens", "weightedmean"),
    ("pooling_mode_lasttoken", "lasttoken"),
)

# Trusted activation spellings only; anything else is rejected, never imported.
_DENSE_ACTIVATIONS = MappingProxyType({
    f"torch.nn.{short}": name
    for short, name in (("Identity", "identity"), ("Tanh", "tanh"), ("ReLU", "relu"), ("GELU", "gelu"),
                        ("SiLU", "silu"))
} | {
    "torch.nn.modules.linear.Identity": "identity",
    "torch.nn.modules.activation.Tanh": "tanh",
    "torch.nn.modules.activation.ReLU": "relu",
    "torch.nn.modules.activation.GELU": "gelu",
    "torch.nn.modules.activation.SiLU": "silu",
})


class SentenceTransformerModuleRole(StrEnum):
    TRANSFORMER = "transformer"
    POOLING = "pooling"
    DENSE = "dense"
    NORMALIZE = "normalize"
    LOGIT_SCORE = "logit_score"
    LEGACY_CLIP = "legacy_clip"
    ROUTER = "router"
    CUSTOM = "custom"


class SentenceTransformerGraphKind(StrEnum):
    DENSE_EMBEDDING = "dense_embedding"
    DIRECT_EMBEDDING = "direct_embedding"
    GENERATIVE_RERANKER = "generative_reranker"
    FEATURE_RERANKER = "feature_reranker"
    LEGACY_CLIP = "legacy_clip"
    ROUTED_ENCODER = "routed_encoder"


_ROLES = MappingProxyType({
    "Transformer": SentenceTransformerModuleRole.TRANSFORMER,
    "Pooling": SentenceTransformerModuleRole.POOLING,
    "Dense": SentenceTransformerModuleRole.DENSE,
    "Normalize": SentenceTransformerModuleRole.NORMALIZE,
    "LogitScore": SentenceTransformerModuleRole.LOGIT_SCORE,
    "CLIPModel": SentenceTransformerModuleRole.LEGACY_CLIP,
    "Router": SentenceTransformerModuleRole.ROUTER,
})


@dataclass(frozen=True)
class SentenceTransformerModuleSpec:
    index: int
    name: str
    path: str
    type: str

    @property
    def kind(self) -> str:
        return self.type.rsplit(".", 1)[-1]

    @property
    def role(self) -> SentenceTransformerModuleRole:
        if not self.type.startswith("sentence_transformers."):
            return SentenceTransformerModuleRole.CUSTOM
        return _ROLES.get(self.kind, SentenceTransformerModuleRole.CUSTOM)


@dataclass(frozen=True)
class SentenceTransformerInputSpec:
    name: str
    modalities: tuple[Modality, ...]
    method: str
    output_name: str
    format: str | None = None


@dataclass(frozen=True)
class SentenceTransformerRouteMapping:
    task: str | None
    modalities: tuple[Modality, ...]
    route: str


@dataclass(frozen=True)
class SentenceTransformerRouteSpec:
    name: str
    modules: tuple[SentenceTransformerModuleSpec, ...]


@dataclass(frozen=True)
class SentenceTransformerGraphSpec:
    kind: SentenceTransformerGraphKind
    model_type: str
    transformer_task: str | None
    module_output_name: str | None
    modules: tuple[SentenceTransformerModuleSpec, ...]
    inputs: tuple[SentenceTransformerInputSpec, ...]
    routes: tuple[SentenceTransformerRouteSpec, ...] = ()
    route_mappings: tuple[SentenceTransformerRouteMapping, ...] = ()
    default_route: str | None = None
    allow_empty_key: bool | None = None

    @property
    def modalities(self) -> frozenset[Modality]:
        return frozenset(m for spec in (*self.inputs, *self.route_mappings) for m in spec.modalities)


@dataclass(frozen=True)
class LoadedSentenceTransformer:
    encoder: SentenceEncoder
    checkpoint: Path
    processor_path: Path
    max_sequence_length: int
    do_lower_case: bool
    prompts: Mapping[str, str]
    default_prompt_name: str | None
    similarity_function: str


def _json(path: Path, *, required: bool = True) -> dict[str, Any]:
    if not path.is_file():
        if required:
            raise FileNotFoundError(f"Sentence Transformers metadata not found: {path}")
        return {}
    with open(path) as handle:
        value = json.load(handle)
    if not isinstance(value, dict):
        raise TypeError(f"{path} must contain a JSON object")
    return value


def _module_directory(root: Path, relative: str) -> Path:
    base = root.resolve()
    directory = (base / relative).resolve()
    if directory != base and base not in directory.parents:
        raise ValueError(f"module path escapes checkpoint root: {relative!r}")
    if not directory.is_dir():
        raise FileNotFoundError(f"Sentence Transformers module directory not found: {directory}")
    return directory


def load_sentence_transformer_modules(checkpoint: str | Path) -> tuple[SentenceTransformerModuleSpec, ...]:
    root = Path(checkpoint)
    path = root / "modules.json"
    if not path.is_file():
        raise FileNotFoundError(f"Sentence Transformers modules not found: {path}")
    with open(path) as handle:
        raw = json.load(handle)
    if not isinstance(raw, list):
        raise TypeError("modules.json must contain a JSON array")
    specs = []
    for entry in raw:
        if not isinstance(entry, dict):
            raise TypeError("each modules.json entry must be an object")
        try:
            specs.append(SentenceTransformerModuleSpec(int(entry["idx"]), str(entry["name"]), str(entry["path"]),
                                                       str(entry["type"])))
        except KeyError as error:
            raise ValueError(f"modules.json entry is missing {error.args[0]!r}") from error
    specs.sort(key=lambda s: s.index)
    if [s.index for s in specs] != list(range(len(specs))):
        raise ValueError("modules.json indices must be unique and contiguous")
    if len({s.name for s in specs}) != len(specs):
        raise ValueError("modules.json names must be unique")
    if not specs:
        raise ValueError("modules.json must contain at least one module")
    return tuple(specs)


def _atomic_modalities(name: str) -> tuple[Modality, ...]:
    """``"text+image"`` -> (text, image); ``"message"`` is a container, not a modality."""

    if name == "message":
        return ()
    parts = tuple(p.strip() for p in name.split("+") if p.strip())
    if not parts:
        raise ValueError("modality names must be non-empty")
    return tuple(Modality(p) for p in parts)


def _input_specs(config: Mapping[str, Any], *, legacy_clip: bool) -> tuple[SentenceTransformerInputSpec, ...]:
    raw = config.get("modality_config")
    default_out = str(config.get("module_output_name", "token_embeddings"))
    if raw is None:
        names = ("text", "image") if legacy_clip else ("text",)
        return tuple(SentenceTransformerInputSpec(n, (Modality(n),), "forward", default_out) for n in names)
    if not isinstance(raw, dict):
        raise TypeError("modality_config must be a JSON object")
    out = []
    for name, spec in raw.items():
        if not isinstance(spec, dict):
            raise TypeError(f"modality_config[{name!r}] must be a JSON object")
        out.append(SentenceTransformerInputSpec(
            str(name), _atomic_modalities(str(name)), str(spec.get("method", "forward")),
            str(spec.get("method_output_name", spec.get("output_name", default_out))),
            None if spec.get("format") is None else str(spec["format"])))
    if not out:
        raise ValueError("modality_config must contain at least one input form")
    return tuple(out)


def _classify(modules, *, model_type: str, module_output_name: str | None) -> SentenceTransformerGraphKind:
    R = SentenceTransformerModuleRole
    first, *suffix = [m.role for m in modules]
    post = {R.POOLING, R.DENSE, R.NORMALIZE}
    if first is R.ROUTER:
        if any(r not in post for r in suffix):
            raise ValueError(f"unsupported or executable routed graph roles: {[first, *suffix]}")
        return SentenceTransformerGraphKind.ROUTED_ENCODER
    if first is R.LEGACY_CLIP:
        if any(r is not R.NORMALIZE for r in suffix):
            raise ValueError(f"unsupported or executable legacy CLIP graph roles: {[first, *suffix]}")
        return SentenceTransformerGraphKind.LEGACY_CLIP
    if first not in {R.TRANSFORMER, R.CUSTOM}:
        raise ValueError(f"unsupported or executable Sentence Transformers graph roles: {[first, *suffix]}")
    if suffix == [R.LOGIT_SCORE]:
        return SentenceTransformerGraphKind.GENERATIVE_RERANKER
    if R.POOLING in suffix:
        if suffix[0] is not R.POOLING or any(r not in {R.DENSE, R.NORMALIZE} for r in suffix[1:]):
            raise ValueError(f"unsupported or executable pooled graph roles: {[first, *suffix]}")
        if model_type == "CrossEncoder":
            return SentenceTransformerGraphKind.FEATURE_RERANKER
        if model_type != "SentenceTransformer":
            raise ValueError(f"unsupported pooled model type: {model_type!r}")
        return SentenceTransformerGraphKind.DENSE_EMBEDDING
    if module_output_name == "sentence_embedding" and all(r in {R.DENSE, R.NORMALIZE} for r in suffix):
        return SentenceTransformerGraphKind.DIRECT_EMBEDDING
    raise ValueError(f"unsupported or executable Sentence Transformers graph roles: {[first, *suffix]}")


def _router_mapping(key: str, route: str, *, route_names: frozenset[str]) -> SentenceTransformerRouteMapping:
    try:
        selector = literal_eval(key)
    except (ValueError, SyntaxError) as error:
        raise ValueError(f"invalid Router selector: {key!r}") from error
    if not isinstance(selector, tuple) or len(selector) != 2:
        raise ValueError(f"Router selector must be a (task, modality) pair: {key!r}")
    task, modality = selector
    if task is not None and not isinstance(task, str):
        raise TypeError("Router task selectors must be strings or null")
    if modality is None:
        modalities: tuple[Modality, ...] = ()
    elif isinstance(modality, str):
        modalities = _atomic_modalities(modality)
    elif isinstance(modality, tuple) and all(isinstance(v, str) for v in modality):
        modalities = tuple(Modality(v) for v in modality)
    else:
        raise TypeError("Router modality selectors must be strings, tuples, or null")
    if route not in route_names:
        raise ValueError(f"Router selector targets unknown route {route!r}")
    return SentenceTransformerRouteMapping(task, modalities, route)


def _router_spec(root: Path, module: SentenceTransformerModuleSpec):
    directory = _module_directory(root, module.path)
    config = _json(directory / "router_config.json")
    types, structure, params = config.get("types"), config.get("structure"), config.get("parameters", {})
    if not isinstance(types, dict) or not isinstance(structure, dict):
        raise TypeError("Router config requires types and structure objects")
    if not isinstance(params, dict):
        raise TypeError("Router parameters must be a JSON object")
    routes, used = [], set()
    R = SentenceTransformerModuleRole
    for name, ids in structure.items():
        name = str(name)
        if not isinstance(ids, list) or not ids:
            raise ValueError(f"Router route {name!r} must contain modules")
        mods = []
        for i, module_id in enumerate(map(str, ids)):
            if module_id not in types:
                raise ValueError(f"Router route {name!r} references unknown module {module_id!r}")
            used.add(module_id)
            path = _module_directory(directory, module_id).relative_to(root.resolve())
            mods.append(SentenceTransformerModuleSpec(i, module_id, str(path), str(types[module_id])))
        if mods[0].role not in {R.TRANSFORMER, R.CUSTOM, R.LEGACY_CLIP}:
            raise ValueError(f"Router route {name!r} lacks an input module")
        routes.append(SentenceTransformerRouteSpec(name, tuple(mods)))
    unused = set(map(str, types)) - used
    if unused:
        raise ValueError(f"Router config contains unused modules: {sorted(unused)}")
    names = frozenset(r.name for r in routes)
    default = params.get("default_route")
    if default is not None and str(default) not in names:
        raise ValueError(f"Router default route {default!r} is unknown")
    raw_maps = params.get("route_mappings", {})
    if not isinstance(raw_maps, dict):
        raise TypeError("Router route_mappings must be a JSON object")
    maps = tuple(_router_mapping(str(k), str(v), route_names=names) for k, v in raw_maps.items())
    allow_empty = params.get("allow_empty_key", True)
    if not isinstance(allow_empty, bool):
        raise TypeError("Router allow_empty_key must be a boolean")
    return tuple(routes), maps, None if default is None else str(default), allow_empty


def load_sentence_transformer_graph(checkpoint: str | Path) -> SentenceTransformerGraphSpec:
    """Inspect a local Sentence-Transformers graph without executing it."""

    root = Path(checkpoint)
    modules = load_sentence_transformer_modules(root)
    model_type = str(_json(root / "config_sentence_transformers.json", required=False)
                     .get("model_type", "SentenceTransformer"))
    tconf = _json(_module_directory(root, modules[0].path) / "sentence_bert_config.json", required=False)
    out_name = tconf.get("module_output_name")
    out_name = None if out_name is None else str(out_name)
    kind = _classify(modules, model_type=model_type, module_output_name=out_name)
    routes, maps, default, allow_empty = (), (), None, None
    if kind is SentenceTransformerGraphKind.ROUTED_ENCODER:
        routes, maps, default, allow_empty = _router_spec(root, modules[0])
        inputs = ()
    else:
        inputs = _input_specs(tconf, legacy_clip=kind is SentenceTransformerGraphKind.LEGACY_CLIP)
    task = tconf.get("transformer_task")
    return SentenceTransformerGraphSpec(kind, model_type, None if task is None else str(task), out_name, modules,
                                        inputs, routes, maps, default, allow_empty)


def _pooling_modes(config: Mapping[str, Any]) -> tuple[str, ...]:
    configured = config.get("pooling_mode")
    if configured is None:
        modes = tuple(mode for key, mode in _LEGACY_POOLING_KEYS if bool(config.get(key, False)))
        return modes or ("mean",)
    modes = (configured,) if isinstance(configured, str) else tuple(map(str, configured))
    bad = tuple(m for m in modes if m not in POOLING_MODES)
    if bad:
        raise ValueError(f"unsupported pooling modes: {bad}")
    return modes


def _load_pooling(directory: Path, *, input_dimension: int) -> SentencePooling:
    config = _json(directory / "config.json")
    dim = int(config.get("embedding_dimension", config.get("word_embedding_dimension", 0)))
    if dim != input_dimension:
        raise ValueError(f"pooling input dimension does not match the token backbone: {dim} != {input_dimension}")
    return SentencePooling(input_dimension, _pooling_modes(config), bool(config.get("include_prompt", True)))


def _dense_activation(config: Mapping[str, Any]) -> str:
    configured = config.get("activation_function", "torch.nn.modules.activation.Tanh")
    if configured is None:
        return "identity"
    try:
        return _DENSE_ACTIVATIONS[str(configured)]
    except KeyError as error:
        raise ValueError(f"untrusted or unsupported Sentence Transformers Dense activation: {configured!r}") from error


def _load_dense(directory: Path, *, input_dimension: int) -> SentenceDense:
    config = _json(directory / "config.json")
    fan_in, fan_out = int(config["in_features"]), int(config["out_features"])
    if fan_in != input_dimension:
        raise ValueError(f"Dense input dimension does not match the preceding module: {fan_in} != {input_dimension}")
    if fan_out <= 0:
        raise ValueError("Dense output dimension must be positive")
    in_name = str(config.get("module_input_name", "sentence_embedding"))
    if in_name != "sentence_embedding" or str(config.get("module_output_name", in_name)) != "sentence_embedding":
        raise ValueError("named Dense feature routing is not supported")
    has_bias = bool(config.get("bias", True))
    names = {"linear.weight"} | ({"linear.bias"} if has_bias else set())
    state = load_safetensor_subset(directory, names)
    weight = state["linear.weight"]
    if tuple(weight.shape) != (fan_out, fan_in):
        raise ValueError(f"Dense weight has shape {tuple(weight.shape)}; expected {(fan_out, fan_in)}")
    bias = state.get("linear.bias")
    if bias is not None and tuple(bias.shape) != (fan_out,):
        raise ValueError(f"Dense bias has shape {tuple(bias.shape)}; expected {(fan_out,)}")
    return SentenceDense(weight, bias, _dense_activation(config))


def _text_backbone(checkpoint: Path, *, compute_dtype: torch.dtype, model_id: str):
    model_type = str(load_hf_config(checkpoint).get("model_type", ""))
    if model_type == "bert":
        from representax_b200.models.bert import BertCheckpointAdapter

        return BertCheckpointAdapter.load(checkpoint, model_id=model_id, compute_dtype=compute_dtype)
    if model_type == "mpnet":
        from representax_b200.models.mpnet import MPNetCheckpointAdapter

        return MPNetCheckpointAdapter.load(checkpoint, model_id=model_id, compute_dtype=compute_dtype)
    raise ValueError(f"Sentence Transformers backbone {model_type!r} is catalogued but not native")


def _model_metadata(checkpoint: Path):
    config = _json(checkpoint / "config_sentence_transformers.json", required=False)
    model_type = str(config.get("model_type", "SentenceTransformer"))
    if model_type != "SentenceTransformer":
        raise ValueError(f"expected a dense SentenceTransformer artifact; found {model_type!r}")
    prompts = config.get("prompts", {})
    if not isinstance(prompts, dict):
        raise TypeError("Sentence Transformers prompts must be an object")
    prompts = MappingProxyType({str(k): str(v) for k, v in prompts.items()})
    default = config.get("default_prompt_name")
    if default is not None:
        default = str(default)
        if default not in prompts:
            raise ValueError("default_prompt_name does not name a saved prompt")
    similarity = str(config.get("similarity_fn_name") or "cosine")
    if similarity not in ("cosine", "dot", "euclidean", "manhattan"):
        raise ValueError(f"unsupported similarity function: {similarity!r}")
    truncate = config.get("truncate_dim")
    return prompts, default, similarity, None if truncate is None else int(truncate)


def load_sentence_transformer_artifact(model_name_or_path: str | Path, *,
                                       compute_dtype: torch.dtype = torch.float32,
                                       **_: Any) -> LoadedSentenceTransformer:
    """Load a standard dense Sentence-Transformers directory into native modules."""

    root = resolve_hf_checkpoint(model_name_or_path)
    graph = load_sentence_transformer_graph(root)
    if graph.kind is not SentenceTransformerGraphKind.DENSE_EMBEDDING:
        raise ValueError(f"Sentence Transformers graph is {graph.kind.value!r}; "
                         "the native dense loader requires 'dense_embedding'")
    first = graph.modules[0]
    if first.role is not SentenceTransformerModuleRole.TRANSFORMER:
        raise ValueError(f"input module {first.type!r} is catalogued but not a registered native backbone")
    tdir = _module_directory(root, first.path)
    hf_config = load_hf_config(tdir)
    backbone = _text_backbone(tdir, compute_dtype=compute_dtype, model_id=root.name)
    width = int(backbone.metadata.output_dimension)
    pooling, post, current = None, [], width
    R = SentenceTransformerModuleRole
    for module in graph.modules[1:]:
        if module.role is R.POOLING:
            if pooling is not None or post:
                raise ValueError("Pooling must occur exactly once before dense modules")
            pooling = _load_pooling(_module_directory(root, module.path), input_dimension=width)
            current = pooling.output_dimension
        elif module.role is R.DENSE:
            if pooling is None:
                raise ValueError("Dense cannot precede Pooling")
            dense = _load_dense(_module_directory(root, module.path), input_dimension=current)
            post.append(dense)
            current = dense.output_dimension
        elif module.role is R.NORMALIZE:
            if pooling is None:
                raise ValueError("Normalize cannot precede Pooling")
            post.append(SentenceNormalize())
        else:
            raise ValueError(f"unsupported or executable Sentence Transformers module: {module.type!r}")
    if pooling is None:
        raise ValueError("dense sentence models require exactly one Pooling module")
    prompts, default, similarity, truncate = _model_metadata(root)
    if truncate is not None and not 0 < truncate <= current:
        raise ValueError("truncate_dim must index the final embedding dimension")
    encoder = SentenceEncoder(backbone, pooling, post, EncoderMetadata(
        model_id=root.name, revision="local", output_dimension=truncate or current, routes=frozenset(Route),
        modalities=graph.modalities or frozenset({Modality.TEXT})), truncate)
    sconf = _json(tdir / "sentence_bert_config.json", required=False)
    maximum = int(sconf.get("max_seq_length", hf_config.get("max_position_embeddings", 0)))
    if maximum <= 0:
        raise ValueError("unable to determine a positive maximum sequence length")
    return LoadedSentenceTransformer(encoder, root, tdir, maximum, bool(sconf.get("do_lower_case", False)), prompts,
                                     default, similarity)


def load_sentence_transformer(model_name_or_path: str | Path, *, compute_dtype: torch.dtype = torch.float32,
                              processor: Any | None = None, sequence_length_buckets: Sequence[int] | None = None,
                              device: str | torch.device | None = None, **options: Any):
    """Load a dense Sentence-Transformers directory plus its host tokenizer."""

    from representax_b200.inference import TextEmbeddingModel
    from representax_b200.models.processing import make_text_processor

    loaded = load_sentence_transformer_artifact(model_name_or_path, compute_dtype=compute_dtype, **options)
    if processor is None:
        from transformers import AutoTokenizer

        kwargs: dict[str, Any] = {"local_files_only": True}
        if loaded.do_lower_case:
            kwargs["do_lower_case"] = True
        processor = AutoTokenizer.from_pretrained(str(loaded.processor_path), **kwargs)
    native = make_text_processor(
        tokenizer=processor, batch_builder=type(loaded.encoder.backbone).make_batch,
        max_sequence_length=loaded.max_sequence_length, sequence_length_buckets=sequence_length_buckets,
        prompts=loaded.prompts, default_prompt_name=loaded.default_prompt_name,
        include_prompt=loaded.encoder.pooling.include_prompt, pooling_batch_builder=SentenceBatch)
    model = loaded.encoder
    if device is not None:
        model = model.to(device)
    return TextEmbeddingModel(model=model, processor=native, similarity_function=loaded.similarity_function)


__all__ = ["LoadedSentenceTransformer", "SENTENCE_TRANSFORMERS_ORACLE_VERSION", "SentenceTransformerGraphKind",
           "SentenceTransformerGraphSpec", "SentenceTransformerInputSpec", "SentenceTransformerModuleRole",
           "SentenceTransformerModuleSpec", "SentenceTransformerRouteMapping", "SentenceTransformerRouteSpec",
           "load_sentence_transformer", "load_sentence_transformer_artifact", "load_sentence_transformer_graph",
           "load_sentence_transformer_modules"]
