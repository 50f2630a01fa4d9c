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

import ast
import importlib
import json
import re
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


def _read_object(path: Path, *, optional: bool = False) -> dict[str, Any]:
    """Parse a JSON file that has to hold an object; ``{}`` for an absent optional file."""

    if not path.is_file():
        if optional:
            return {}
        raise FileNotFoundError(f"no {path.name} at {path.parent} (not a Sentence Transformers directory?)")
    parsed = json.loads(path.read_text())
    if isinstance(parsed, dict):
        return parsed
    raise TypeError(f"{path} holds a JSON {type(parsed).__name__}; an object was expected")


def _inside(root: Path, relative: str) -> Path:
    """``root / relative`` as an existing directory that stays under ``root``."""

    anchor = root.resolve()
    target = anchor.joinpath(relative).resolve()
    if not target.is_relative_to(anchor):
        raise ValueError(f"module path {relative!r} points outside {anchor}")
    if not target.is_dir():
        raise FileNotFoundError(f"module directory {target} does not exist")
    return target


def load_sentence_transformer_modules(checkpoint: str | Path) -> tuple[SentenceTransformerModuleSpec, ...]:
    """The ordered module list of ``modules.json``."""

    listing = Path(checkpoint) / "modules.json"
    if not listing.is_file():
        raise FileNotFoundError(f"no modules.json in {listing.parent}")
    entries = json.loads(listing.read_text())
    if not isinstance(entries, list):
        raise TypeError(f"modules.json holds a JSON {type(entries).__name__}; a list of modules was expected")
    specs: list[SentenceTransformerModuleSpec] = []
    for position, entry in enumerate(entries):
        if not isinstance(entry, dict):
            raise TypeError(f"modules.json entry {position} is not an object")
        absent = [key for key in ("idx", "name", "path", "type") if key not in entry]
        if absent:
            raise ValueError(f"modules.json entry {position} has no {', '.join(absent)}")
        specs.append(SentenceTransformerModuleSpec(int(entry["idx"]), str(entry["name"]), str(entry["path"]),
                                                   str(entry["type"])))
    if not specs:
        raise ValueError("modules.json lists no module")
    specs.sort(key=lambda spec: spec.index)
    order = [spec.index for spec in specs]
    if order != list(range(len(specs))):
        raise ValueError(f"modules.json indices {order} are not 0..{len(specs) - 1}")
    names = [spec.name for spec in specs]
    if len(set(names)) < len(names):
        raise ValueError(f"modules.json repeats a module name: {names}")
    return tuple(specs)


def _atomic_modalities(name: str) -> tuple[Modality, ...]:
    """``"text+image"`` -> (text, image); ``"message"`` is a container, not a modality."""

    if name == "message":
        return ()
    pieces = [piece.strip() for piece in name.split("+")]
    if not any(pieces):
        raise ValueError(f"input form {name!r} names no modality")
    return tuple(Modality(piece) for piece in pieces if piece)


def _input_specs(config: Mapping[str, Any], *, legacy_clip: bool) -> tuple[SentenceTransformerInputSpec, ...]:
    """Input forms of the first module (``modality_config``), or its implicit text/image forms."""

    fallback_output = str(config.get("module_output_name", "token_embeddings"))
    declared = config.get("modality_config")
    if declared is None:
        implicit = ("text", "image") if legacy_clip else ("text",)
        return tuple(SentenceTransformerInputSpec(form, (Modality(form),), "forward", fallback_output)
                     for form in implicit)
    if not isinstance(declared, dict) or not declared:
        raise TypeError("modality_config has to be a non-empty object of input forms")
    forms = []
    for form, options in declared.items():
        if not isinstance(options, dict):
            raise TypeError(f"options of input form {form!r} are not an object")
        output = options.get("method_output_name", options.get("output_name", fallback_output))
        wire = options.get("format")
        forms.append(SentenceTransformerInputSpec(str(form), _atomic_modalities(str(form)),
                                                  str(options.get("method", "forward")), str(output),
                                                  None if wire is None else str(wire)))
    return tuple(forms)


# Graph classification: the module roles are spelled as one letter each and the
# resulting word is matched against the shapes each graph kind may take.
_ROLE_LETTER = {
    SentenceTransformerModuleRole.TRANSFORMER: "T", SentenceTransformerModuleRole.CUSTOM: "C",
    SentenceTransformerModuleRole.POOLING: "P", SentenceTransformerModuleRole.DENSE: "D",
    SentenceTransformerModuleRole.NORMALIZE: "N", SentenceTransformerModuleRole.LOGIT_SCORE: "L",
    SentenceTransformerModuleRole.LEGACY_CLIP: "X", SentenceTransformerModuleRole.ROUTER: "R",
}
_GRAPH_SHAPES = (
    (re.compile(r"R[PDN]*"), "routed"),
    (re.compile(r"XN*"), "clip"),
    (re.compile(r"[TC]L"), "logit"),
    (re.compile(r"[TC]P[DN]*"), "pooled"),
    (re.compile(r"[TC][DN]*"), "direct"),
)


def _classify(modules, *, model_type: str, module_output_name: str | None) -> SentenceTransformerGraphKind:
    word = "".join(_ROLE_LETTER[m.role] for m in modules)
    shape = next((name for pattern, name in _GRAPH_SHAPES if pattern.fullmatch(word)), None)
    K = SentenceTransformerGraphKind
    if shape == "routed":
        return K.ROUTED_ENCODER
    if shape == "clip":
        return K.LEGACY_CLIP
    if shape == "logit":
        return K.GENERATIVE_RERANKER
    if shape == "pooled":
        by_type = {"CrossEncoder": K.FEATURE_RERANKER, "SentenceTransformer": K.DENSE_EMBEDDING}
        if model_type not in by_type:
            raise ValueError(f"a pooled module graph of model type {model_type!r} is not supported")
        return by_type[model_type]
    if shape == "direct" and module_output_name == "sentence_embedding":
        return K.DIRECT_EMBEDDING
    roles = [m.role.value for m in modules]
    raise ValueError(f"module graph {roles} is not one of the supported (non-executable) layouts")


def _selector_value(node: ast.AST, key: str):
    """A ``None`` / string / tuple-of-strings literal from a Router selector."""

    if isinstance(node, ast.Constant) and (node.value is None or isinstance(node.value, str)):
        return node.value
    if isinstance(node, ast.Tuple) and all(isinstance(e, ast.Constant) and isinstance(e.value, str)
                                           for e in node.elts):
        return tuple(e.value for e in node.elts)
    raise TypeError(f"Router selector {key!r}: each part has to be null, a string or a tuple of strings")


def _router_mapping(key: str, route: str, *, route_names: frozenset[str]) -> SentenceTransformerRouteMapping:
    """Parse one ``route_mappings`` key, the Python literal ``"(task, modality)"``."""

    try:
        tree = ast.parse(key.strip(), mode="eval").body
    except SyntaxError as error:
        raise ValueError(f"Router selector {key!r} is not a Python literal") from error
    if not isinstance(tree, ast.Tuple) or len(tree.elts) != 2:
        raise ValueError(f"Router selector {key!r} is not a (task, modality) pair")
    task = _selector_value(tree.elts[0], key)
    modality = _selector_value(tree.elts[1], key)
    if isinstance(task, tuple):
        raise TypeError(f"Router selector {key!r}: the task part is a single name or null")
    if modality is None:
        modalities: tuple[Modality, ...] = ()
    elif isinstance(modality, str):
        modalities = _atomic_modalities(modality)
    else:
        modalities = tuple(Modality(name) for name in modality)
    if route not in route_names:
        raise ValueError(f"Router selector {key!r} sends inputs to route {route!r}, which is not defined")
    return SentenceTransformerRouteMapping(task, modalities, route)


_ROUTE_INPUT_ROLES = frozenset({SentenceTransformerModuleRole.TRANSFORMER, SentenceTransformerModuleRole.CUSTOM,
                                SentenceTransformerModuleRole.LEGACY_CLIP})


def _router_spec(root: Path, module: SentenceTransformerModuleSpec):
    """Routes, selector mappings, default route and empty-key policy of a Router module."""

    here = _inside(root, module.path)
    config = _read_object(here / "router_config.json")
    types, structure = config.get("types"), config.get("structure")
    options = config.get("parameters", {})
    if not (isinstance(types, dict) and isinstance(structure, dict) and isinstance(options, dict)):
        raise TypeError("router_config.json needs object-valued 'types' and 'structure' (and 'parameters')")
    anchor = root.resolve()
    routes: list[SentenceTransformerRouteSpec] = []
    referenced: set[str] = set()
    for route, members in structure.items():
        if not isinstance(members, list) or not members:
            raise ValueError(f"Router route {route!r} has no module list")
        unknown = [str(m) for m in members if str(m) not in types]
        if unknown:
            raise ValueError(f"Router route {route!r} uses undeclared module(s) {unknown}")
        chain = tuple(
            SentenceTransformerModuleSpec(position, str(member),
                                          str(_inside(here, str(member)).relative_to(anchor)), str(types[str(member)]))
            for position, member in enumerate(members))
        if chain[0].role not in _ROUTE_INPUT_ROLES:
            raise ValueError(f"Router route {route!r} starts with {chain[0].type!r}, not an input module")
        referenced.update(spec.name for spec in chain)
        routes.append(SentenceTransformerRouteSpec(str(route), chain))
    orphans = sorted(set(map(str, types)) - referenced)
    if orphans:
        raise ValueError(f"Router declares module(s) {orphans} that no route uses")
    names = frozenset(r.name for r in routes)
    default = options.get("default_route")
    default = None if default is None else str(default)
    if default is not None and default not in names:
        raise ValueError(f"Router default_route {default!r} is not one of {sorted(names)}")
    selectors = options.get("route_mappings", {})
    if not isinstance(selectors, dict):
        raise TypeError("Router route_mappings has to be an object of selector -> route")
    mappings = tuple(_router_mapping(str(k), str(v), route_names=names) for k, v in selectors.items())
    allow_empty = options.get("allow_empty_key", True)
    if type(allow_empty) is not bool:
        raise TypeError(f"Router allow_empty_key is {allow_empty!r}; true or false expected")
    return tuple(routes), mappings, default, allow_empty


def load_sentence_transformer_graph(checkpoint: str | Path) -> SentenceTransformerGraphSpec:
    """Inspect a local Sentence-Transformers graph without executing it."""

    root = Path(checkpoint)
    modules = load_sentence_transformer_modules(root)
    model_type = str(_read_object(root / "config_sentence_transformers.json", optional=True)
                     .get("model_type", "SentenceTransformer"))
    first = _read_object(_inside(root, modules[0].path) / "sentence_bert_config.json", optional=True)
    output_name = None if first.get("module_output_name") is None else str(first["module_output_name"])
    kind = _classify(modules, model_type=model_type, module_output_name=output_name)
    task = None if first.get("transformer_task") is None else str(first["transformer_task"])
    if kind is SentenceTransformerGraphKind.ROUTED_ENCODER:
        routes, mappings, default, allow_empty = _router_spec(root, modules[0])
        return SentenceTransformerGraphSpec(kind, model_type, task, output_name, modules, (), routes, mappings,
                                            default, allow_empty)
    inputs = _input_specs(first, legacy_clip=kind is SentenceTransformerGraphKind.LEGACY_CLIP)
    return SentenceTransformerGraphSpec(kind, model_type, task, output_name, modules, inputs)


def _pooling_modes(config: Mapping[str, Any]) -> tuple[str, ...]:
    chosen = config.get("pooling_mode")
    if chosen is None:  # older artifacts: one boolean flag per mode
        flagged = tuple(mode for flag, mode in _LEGACY_POOLING_KEYS if config.get(flag))
        return flagged if flagged else ("mean",)
    modes = (chosen,) if isinstance(chosen, str) else tuple(str(m) for m in chosen)
    unknown = [m for m in modes if m not in POOLING_MODES]
    if unknown:
        raise ValueError(f"pooling mode(s) {unknown} are not among {sorted(POOLING_MODES)}")
    return modes


def _load_pooling(directory: Path, *, input_dimension: int) -> SentencePooling:
    config = _read_object(directory / "config.json")
    width = int(config.get("embedding_dimension", config.get("word_embedding_dimension", 0)))
    if width != input_dimension:
        raise ValueError(f"Pooling expects {width}-wide token vectors but the backbone emits {input_dimension}")
    return SentencePooling(input_dimension, _pooling_modes(config), bool(config.get("include_prompt", True)))


def _dense_activation(config: Mapping[str, Any]) -> str:
    spelled = config.get("activation_function", "torch.nn.modules.activation.Tanh")
    if spelled is None:
        return "identity"
    name = _DENSE_ACTIVATIONS.get(str(spelled))
    if name is None:
        raise ValueError(f"Dense activation {spelled!r} is not on the trusted list {sorted(_DENSE_ACTIVATIONS)}")
    return name


def _load_dense(directory: Path, *, input_dimension: int) -> SentenceDense:
    config = _read_object(directory / "config.json")
    fan_in, fan_out = int(config["in_features"]), int(config["out_features"])
    if fan_in != input_dimension or fan_out < 1:
        raise ValueError(f"Dense maps {fan_in} -> {fan_out} features but receives {input_dimension}")
    routed_in = str(config.get("module_input_name", "sentence_embedding"))
    routed_out = str(config.get("module_output_name", routed_in))
    if {routed_in, routed_out} != {"sentence_embedding"}:
        raise ValueError(f"Dense reads {routed_in!r} and writes {routed_out!r}; only the sentence embedding "
                         "is supported")
    wanted = ["linear.weight"] + (["linear.bias"] if config.get("bias", True) else [])
    tensors = load_safetensor_subset(directory, set(wanted))
    weight, bias = tensors["linear.weight"], tensors.get("linear.bias")
    shapes_ok = tuple(weight.shape) == (fan_out, fan_in) and (bias is None or tuple(bias.shape) == (fan_out,))
    if not shapes_ok:
        got = {k: tuple(v.shape) for k, v in tensors.items()}
        raise ValueError(f"Dense tensors {got} do not fit {fan_in} -> {fan_out}")
    return SentenceDense(weight, bias, _dense_activation(config))


_NATIVE_BACKBONES = {
    "bert": ("representax_b200.models.bert", "BertCheckpointAdapter"),
    "mpnet": ("representax_b200.models.mpnet", "MPNetCheckpointAdapter"),
}


def _text_backbone(checkpoint: Path, *, compute_dtype: torch.dtype, model_id: str):
    model_type = str(load_hf_config(checkpoint).get("model_type", ""))
    if model_type not in _NATIVE_BACKBONES:
        raise ValueError(f"backbone model_type {model_type!r} has no native text encoder here "
                         f"(native: {sorted(_NATIVE_BACKBONES)})")
    module_name, adapter = _NATIVE_BACKBONES[model_type]
    adapter_cls = getattr(importlib.import_module(module_name), adapter)
    return adapter_cls.load(checkpoint, model_id=model_id, compute_dtype=compute_dtype)


_SIMILARITIES = ("cosine", "dot", "euclidean", "manhattan")


def _model_metadata(checkpoint: Path):
    """(prompts, default prompt name, similarity function, truncate_dim) of the artifact."""

    config = _read_object(checkpoint / "config_sentence_transformers.json", optional=True)
    if config.get("model_type", "SentenceTransformer") != "SentenceTransformer":
        raise ValueError(f"artifact model_type is {config['model_type']!r}; the dense loader reads "
                         "'SentenceTransformer' artifacts")
    saved = config.get("prompts", {})
    if not isinstance(saved, dict):
        raise TypeError("'prompts' in config_sentence_transformers.json is not an object")
    prompts = MappingProxyType({str(name): str(text) for name, text in saved.items()})
    default = None if config.get("default_prompt_name") is None else str(config["default_prompt_name"])
    if default is not None and default not in prompts:
        raise ValueError(f"default_prompt_name {default!r} is none of the saved prompts {sorted(prompts)}")
    similarity = str(config.get("similarity_fn_name") or "cosine")
    if similarity not in _SIMILARITIES:
        raise ValueError(f"similarity_fn_name {similarity!r} is not one of {_SIMILARITIES}")
    truncate = config.get("truncate_dim")
    return prompts, default, similarity, None if truncate is None else int(truncate)


def _post_modules(root: Path, graph: SentenceTransformerGraphSpec, width: int):
    """Load Pooling and the Dense / Normalize chain after it; returns (pooling, chain, out width)."""

    R = SentenceTransformerModuleRole
    pooling, chain = None, []
    for module in graph.modules[1:]:
        where = _inside(root, module.path)
        if module.role is R.POOLING:
            if pooling is not None:
                raise ValueError("the module graph pools twice")
            pooling = _load_pooling(where, input_dimension=width)
            width = pooling.output_dimension
            continue
        if pooling is None:
            raise ValueError(f"{module.type!r} comes before Pooling; it needs a pooled sentence vector")
        if module.role is R.DENSE:
            dense = _load_dense(where, input_dimension=width)
            chain.append(dense)
            width = dense.output_dimension
        elif module.role is R.NORMALIZE:
            chain.append(SentenceNormalize())
        else:
            raise ValueError(f"module {module.type!r} after Pooling is not supported")
    if pooling is None:
        raise ValueError("the module graph has no Pooling module")
    return pooling, chain, width


def load_sentence_transformer_artifact(model_name_or_path: str | Path, *,
                                       compute_dtype: torch.dtype = torch.float32,
                                       **_: Any) -> LoadedSentenceTransformer:
    """Load a standard dense Sentence-Transformers directory into native modules."""

    root = resolve_hf_checkpoint(model_name_or_path)
    graph = load_sentence_transformer_graph(root)
    if graph.kind is not SentenceTransformerGraphKind.DENSE_EMBEDDING:
        raise ValueError(f"this loader builds dense embedding models; the artifact is a {graph.kind.value}")
    first = graph.modules[0]
    if first.role is not SentenceTransformerModuleRole.TRANSFORMER:
        raise ValueError(f"input module {first.type!r} is not a transformers backbone")
    backbone_dir = _inside(root, first.path)
    hf_config = load_hf_config(backbone_dir)
    backbone = _text_backbone(backbone_dir, compute_dtype=compute_dtype, model_id=root.name)
    pooling, chain, width = _post_modules(root, graph, int(backbone.metadata.output_dimension))
    prompts, default, similarity, truncate = _model_metadata(root)
    if truncate is not None and not 1 <= truncate <= width:
        raise ValueError(f"truncate_dim {truncate} is outside 1..{width}")
    encoder = SentenceEncoder(backbone, pooling, chain, EncoderMetadata(
        model_id=root.name, revision="local", output_dimension=truncate or width, routes=frozenset(Route),
        modalities=graph.modalities or frozenset({Modality.TEXT})), truncate)
    backbone_options = _read_object(backbone_dir / "sentence_bert_config.json", optional=True)
    longest = int(backbone_options.get("max_seq_length", hf_config.get("max_position_embeddings", 0)))
    if longest < 1:
        raise ValueError("neither max_seq_length nor max_position_embeddings gives a sequence length")
    return LoadedSentenceTransformer(encoder, root, backbone_dir, longest,
                                     bool(backbone_options.get("do_lower_case", False)), prompts, default, similarity)


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
