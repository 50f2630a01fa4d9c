"""Host processors: raw artifacts -> one model-native fixed-shape batch.

Parity: src/representax/models/processing.py:21-561 —
``select_static_shape_bucket`` (the unique dimension-wise minimal admitted
shape, rejecting incomparable candidates), ``Processor(process, contract)``
with a JSON ``data_contract()`` fingerprint, and the media/image/audio/video/
text processor builders (route-dependent prompts, length buckets, prompt
exclusion from pooling). The contract schema strings are kept so that data
contract fingerprints in resumed runs compare equal.

On this framework the batch builders receive numpy arrays and build torch
batches (``TokenBatch`` for text); fixed shapes matter less here than under a
tracing compiler, but the buckets still bound the number of distinct CUDA
graph shapes a serving loop captures.
"""

from __future__ import annotations

import hashlib
import inspect
import json
import operator
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from types import MappingProxyType
from typing import Any

import numpy as np

from representax_b200.core.model import Modality, Route
from representax_b200.data.artifact import Artifact


def _shape(value: Sequence[int], *, name: str) -> tuple[int, ...]:
    dims = []
    for d in value:
        if isinstance(d, bool):
            raise ValueError(f"{name} must contain positive integer dimensions")
        try:
            d = operator.index(d)
        except TypeError as error:
            raise ValueError(f"{name} must contain positive integer dimensions") from error
        if d <= 0:
            raise ValueError(f"{name} must contain positive integer dimensions")
        dims.append(d)
    if not dims:
        raise ValueError(f"{name} must contain positive integer dimensions")
    return tuple(dims)


def select_static_shape_bucket(required_shape: Sequence[int],
                               admitted_shapes: Sequence[Sequence[int]]) -> tuple[int, ...]:
    """The unique smallest admitted shape that contains ``required_shape``.

    Order is dimension-wise; when several minimal candidates are incomparable
    (e.g. more frames vs. higher resolution) the choice is model policy, so
    this raises instead of guessing.
    """

    required = _shape(required_shape, name="required_shape")
    buckets = tuple(dict.fromkeys(_shape(s, name="static shape buckets") for s in admitted_shapes))
    if not buckets:
        raise ValueError("at least one static shape bucket is required")
    if any(len(b) != len(required) for b in buckets):
        raise ValueError("static shape buckets must match required_shape rank")
    fits = [b for b in buckets if all(r <= a for r, a in zip(required, b))]
    if not fits:
        raise ValueError(f"required shape {required!r} exceeds admitted buckets {buckets!r}")
    minimal = [b for b in fits if not any(o != b and all(x <= y for x, y in zip(o, b)) for o in fits)]
    if len(minimal) != 1:
        raise ValueError(f"required shape {required!r} has incomparable admitted buckets {tuple(minimal)!r}; "
                         "the model processor must choose explicitly")
    return minimal[0]


@dataclass(frozen=True)
class Processor:
    """A host processor bound to a model artifact (no parameters inside)."""

    process: Callable[..., Any] = field(repr=False)
    contract: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not callable(self.process):
            raise TypeError("processor process must be callable")
        contract = dict(self.contract)
        try:
            json.dumps(contract, sort_keys=True)
        except (TypeError, ValueError) as error:
            raise TypeError("processor contract must be JSON serializable") from error
        object.__setattr__(self, "contract", MappingProxyType(contract))

    def data_contract(self) -> dict[str, Any]:
        return dict(self.contract)

    def fingerprint(self) -> str:
        return hashlib.sha256(json.dumps(self.data_contract(), sort_keys=True).encode()).hexdigest()

    def __call__(self, artifacts: Sequence[Any], *, route: Route | str = Route.GENERIC, seed: int | None = None,
                 **options: Any) -> Any:
        return self.process(artifacts, route=Route(route), seed=seed, **options)


def _callable_contract(value: Callable[..., Any]) -> dict[str, str]:
    module = getattr(value, "__module__", type(value).__module__)
    qual = getattr(value, "__qualname__", type(value).__qualname__)
    identity = f"{module}.{qual}"
    target = value if inspect.isfunction(value) or inspect.isclass(value) or inspect.ismethod(value) else type(value)
    try:
        path = inspect.getsourcefile(target)
    except TypeError:
        path = None
    if path is not None and Path(path).is_file():
        return {"callable": identity, "module_file_sha256": hashlib.sha256(Path(path).read_bytes()).hexdigest()}
    try:
        source = inspect.getsource(target).encode()
    except (OSError, TypeError):
        return {"callable": identity}
    return {"callable": identity, "callable_source_sha256": hashlib.sha256(source).hexdigest()}


def _as_artifact(value: Any, modality: Modality) -> Artifact:
    if isinstance(value, Artifact):
        if value.modality != modality:
            raise TypeError(f"{modality} processors cannot consume {value.modality} artifacts")
        return value
    return Artifact.inline(modality, value)


def make_media_processor(*, modality: Modality | str, admitted_shapes: Sequence[Sequence[int]],
                         probe: Callable[..., Sequence[int]], prepare: Callable[..., Mapping[str, Any]],
                         batch_builder: Callable[..., Any], configuration: Mapping[str, Any]) -> Processor:
    """Media processor: probe -> one batch-wide bucket -> prepare rows -> stack -> build.

    ``probe(artifact, route=)`` returns the shape the artifact needs without
    decoding it; ``prepare(artifact, bucket=, route=, rng=)`` returns a
    mapping of arrays for exactly that bucket; the stacked arrays go to
    ``batch_builder(**arrays)``. Per-row RNGs derive from ``seed`` with
    ``numpy.random.SeedSequence.spawn`` so augmentation replays exactly.
    """

    modality = Modality(modality)
    if not (callable(probe) and callable(prepare) and callable(batch_builder)):
        raise TypeError("media probe, prepare and batch_builder must be callable")
    config = dict(configuration)
    try:
        json.dumps(config, sort_keys=True)
    except (TypeError, ValueError) as error:
        raise TypeError("media processor configuration must be JSON serializable") from error
    shapes = tuple(dict.fromkeys(_shape(s, name="admitted media shapes") for s in admitted_shapes))
    if not shapes:
        raise ValueError("at least one admitted media shape is required")
    rank = len(shapes[0])
    if any(len(s) != rank for s in shapes):
        raise ValueError("admitted media shapes must have one consistent rank")

    def process(artifacts: Sequence[Any], *, route: Route, seed: int | None) -> Any:
        if not artifacts:
            raise ValueError("media processor batches must be non-empty")
        items = [_as_artifact(a, modality) for a in artifacts]
        needs = [_shape(probe(a, route=route), name=f"{modality} shape requirement") for a in items]
        if any(len(n) != rank for n in needs):
            raise ValueError(f"{modality} shape requirements must have rank {rank}")
        bucket = select_static_shape_bucket(tuple(max(v) for v in zip(*needs)), shapes)
        seeds = [None] * len(items) if seed is None else np.random.SeedSequence(seed).spawn(len(items))
        rows = []
        for item, s in zip(items, seeds):
            prepared = prepare(item, bucket=bucket, route=route, rng=None if s is None else np.random.default_rng(s))
            if not isinstance(prepared, Mapping) or not prepared:
                raise TypeError("media prepare must return a non-empty mapping")
            rows.append({k: np.asarray(v) for k, v in prepared.items()})
        names = tuple(rows[0])
        if any(tuple(r) != names for r in rows[1:]):
            raise ValueError("media prepare fields must be identical for every row")
        arrays = {}
        for name in names:
            if len({r[name].shape for r in rows}) != 1:
                raise ValueError(f"prepared media field {name!r} has unstable shapes for bucket {bucket!r}")
            arrays[name] = np.stack([r[name] for r in rows])
        return batch_builder(**arrays)

    return Processor(process=process, contract={
        "schema_version": "representax-media-processor-v1",
        "modality": modality.value,
        "admitted_shapes": [list(s) for s in shapes],
        "probe": _callable_contract(probe),
        "prepare": _callable_contract(prepare),
        "batch_builder": _callable_contract(batch_builder),
        "configuration": config,
    })


def _media_with_rank(modality: Modality, rank: int, what: str):
    def build(*, admitted_shapes, probe, prepare, batch_builder, configuration) -> Processor:
        if any(len(tuple(s)) != rank for s in admitted_shapes):
            raise ValueError(f"{modality} admitted shapes must be {what}")
        return make_media_processor(modality=modality, admitted_shapes=admitted_shapes, probe=probe,
                                    prepare=prepare, batch_builder=batch_builder, configuration=configuration)

    build.__name__ = f"make_{modality.value}_processor"
    build.__doc__ = f"Build a {modality.value} processor whose shapes mean {what}."
    return build


make_image_processor = _media_with_rank(Modality.IMAGE, 2, "(height, width)")
make_audio_processor = _media_with_rank(Modality.AUDIO, 1, "(samples,)")
make_video_processor = _media_with_rank(Modality.VIDEO, 3, "(frames, height, width)")


def make_text_processor(*, tokenizer: Any, batch_builder: Callable[..., Any], max_sequence_length: int | None = None,
                        sequence_length_buckets: Sequence[int] | None = None, prompts: Mapping[str, str] | None = None,
                        default_prompt_name: str | None = None, include_prompt: bool = True,
                        pooling_batch_builder: Callable[[Any, Any], Any] | None = None) -> Processor:
    """Tokenize (with a route prompt), pad to a length bucket, build the batch.

    Route prompts: an explicit ``prompt`` or ``prompt_name`` wins; otherwise
    QUERY uses "query", DOCUMENT the first of "document"/"passage"/"corpus",
    GENERIC the default prompt. With ``include_prompt=False`` the prompt
    tokens are masked out of pooling through ``pooling_batch_builder``.
    """

    if sequence_length_buckets is None:
        if max_sequence_length is None:
            raise ValueError("max_sequence_length or sequence_length_buckets is required")
        sequence_length_buckets = (max_sequence_length,)
    lengths = tuple(sequence_length_buckets)
    if not lengths or any(not isinstance(n, int) or isinstance(n, bool) or n <= 0 for n in lengths):
        raise ValueError("sequence_length_buckets must be positive integers")
    lengths = tuple(sorted(set(lengths)))
    if max_sequence_length is not None and lengths[-1] > max_sequence_length:
        raise ValueError("sequence length buckets cannot exceed max_sequence_length")
    prompt_values = dict(prompts or {})
    if default_prompt_name is not None and default_prompt_name not in prompt_values:
        raise ValueError("default_prompt_name does not name a configured prompt")
    if not include_prompt and pooling_batch_builder is None:
        raise ValueError("prompt exclusion requires pooling_batch_builder")
    maximum = lengths[-1]

    def route_prompt(route: Route, prompt_name: str | None, prompt: str | None) -> str:
        if prompt_name is not None and prompt is not None:
            raise ValueError("specify prompt_name or prompt, not both")
        if prompt is not None:
            return prompt
        if prompt_name is not None:
            if prompt_name not in prompt_values:
                raise KeyError(f"unknown prompt {prompt_name!r}")
            return prompt_values[prompt_name]
        if route is Route.QUERY:
            names = ("query",)
        elif route is Route.DOCUMENT:
            names = ("document", "passage", "corpus")
        else:
            names = () if default_prompt_name is None else (default_prompt_name,)
        return next((prompt_values[n] for n in names if n in prompt_values), "")

    def pad_id() -> int:
        value = getattr(tokenizer, "pad_token_id", None)
        if value is None:
            value = getattr(tokenizer, "pad_id", 0)
        if value is None:
            raise ValueError("text tokenizer must define a pad token")
        return int(value)

    def tokenize(texts: Sequence[str]) -> dict[str, np.ndarray]:
        if not texts:
            raise ValueError("processor batches must be non-empty")
        encoded = tokenizer(list(texts), padding=True, truncation=True, max_length=maximum, return_tensors="np")
        if not isinstance(encoded, Mapping):
            encoded = dict(encoded)
        arrays = {k: np.asarray(v) for k, v in encoded.items()}
        if "input_ids" not in arrays:
            raise KeyError("tokenizer output is missing 'input_ids'")
        ids = arrays["input_ids"]
        if ids.ndim != 2 or ids.shape[0] != len(texts):
            raise ValueError("tokenizer input_ids must have shape [batch, sequence]")
        bucket = select_static_shape_bucket((ids.shape[1],), tuple((n,) for n in lengths))[0]
        out = {}
        for name, value in arrays.items():
            if value.ndim != 2 or value.shape[0] != len(texts):
                out[name] = value
                continue
            if value.shape[1] != ids.shape[1]:
                raise ValueError(f"tokenizer field {name!r} has a different sequence length")
            fill = pad_id() if name == "input_ids" else 0
            out[name] = np.pad(value, ((0, 0), (0, bucket - value.shape[1])), constant_values=fill)
        return out

    def prompt_length(prefix: str) -> int:
        if not prefix:
            return 0
        ids = np.asarray(tokenizer([prefix], padding=True, truncation=True, max_length=maximum,
                                   return_tensors="np")["input_ids"])
        n = int(ids.shape[-1])
        special = frozenset(getattr(tokenizer, "all_special_ids", ()))
        if n and int(ids[0, -1]) in special:
            n -= 1
        return n

    def process(artifacts: Sequence[str | Artifact], *, route: Route, seed: int | None,
                prompt_name: str | None = None, prompt: str | None = None) -> Any:
        del seed
        texts = []
        for a in artifacts:
            if isinstance(a, Artifact):
                if a.modality != Modality.TEXT or not isinstance(a.data, str):
                    raise TypeError("text processors require inline text artifacts")
                texts.append(a.data)
            elif isinstance(a, str):
                texts.append(a)
            else:
                raise TypeError("text processors require strings or artifacts")
        prefix = route_prompt(route, prompt_name, prompt)
        enc = tokenize([prefix + t for t in texts])
        if "attention_mask" not in enc:
            raise KeyError("tokenizer output is missing required field 'attention_mask'")
        inputs = batch_builder(input_ids=enc["input_ids"], attention_mask=enc["attention_mask"],
                               token_type_ids=enc.get("token_type_ids"))
        if include_prompt or not prefix:
            return inputs
        mask = np.array(enc["attention_mask"], copy=True)
        first = np.argmax(mask, axis=1)
        positions = np.arange(mask.shape[1])[None, :]
        mask[positions < (first + prompt_length(prefix))[:, None]] = 0
        return pooling_batch_builder(inputs, mask)

    kind = type(tokenizer)
    return Processor(process=process, contract={
        "schema_version": "representax-text-processor-v1",
        "tokenizer_type": f"{kind.__module__}.{kind.__qualname__}",
        "batch_builder": _callable_contract(batch_builder),
        "max_sequence_length": maximum,
        "sequence_length_buckets": list(lengths),
        "prompts": prompt_values,
        "default_prompt_name": default_prompt_name,
        "include_prompt": include_prompt,
    })


__all__ = ["Processor", "make_audio_processor", "make_image_processor", "make_media_processor",
           "make_text_processor", "make_video_processor", "select_static_shape_bucket"]
