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


def _dims(value: Sequence[int], *, what: str) -> tuple[int, ...]:
    """A non-empty tuple of positive Python ints (bools and floats rejected)."""

    def whole(d: Any) -> int | None:
        if isinstance(d, bool):
            return None
        try:
            return operator.index(d)
        except TypeError:
            return None

    dims = tuple(whole(d) for d in value)
    if not dims or any(d is None or d < 1 for d in dims):
        raise ValueError(f"{what} {tuple(value)!r}: dimensions have to be whole numbers >= 1")
    return dims  # type: ignore[return-value]


def _covers(bigger: tuple[int, ...], smaller: tuple[int, ...]) -> bool:
    return all(b >= s for b, s in zip(bigger, smaller))


def select_static_shape_bucket(required_shape: Sequence[int],
                               admitted_shapes: Sequence[Sequence[int]]) -> tuple[int, ...]:
    """The unique smallest admitted shape that contains ``required_shape``.

    Order is dimension-wise; when several minimal candidates are incomparable
    (e.g. more frames vs. higher resolution) the choice is model policy, so
    this raises instead of guessing.
    """

    need = _dims(required_shape, what="required shape")
    menu = list(dict.fromkeys(_dims(s, what="admitted shape") for s in admitted_shapes))
    if not menu or {len(s) for s in menu} != {len(need)}:
        raise ValueError(f"admitted shapes {menu} have to be a non-empty list of rank-{len(need)} shapes")
    covering = [s for s in menu if _covers(s, need)]
    if not covering:
        raise ValueError(f"required shape {need} exceeds every admitted shape {menu}")
    # a covering shape is minimal when no other covering shape fits inside it
    minimal = [s for s in covering if not any(o != s and _covers(s, o) for o in covering)]
    if len(minimal) > 1:
        raise ValueError(f"required shape {need} fits incomparable minimal shapes {minimal}; the model's "
                         "processor has to pick one itself")
    return minimal[0]


def _frozen_json(values: Mapping[str, Any], *, what: str) -> MappingProxyType:
    """A read-only copy of ``values`` after checking it serialises to JSON."""

    copy = dict(values)
    try:
        json.dumps(copy, sort_keys=True)
    except (TypeError, ValueError) as error:
        raise TypeError(f"{what} has to be JSON data: {error}") from error
    return MappingProxyType(copy)


@dataclass(frozen=True)
class Processor:
    """A host processor bound to a model artifact (no parameters inside)."""

    process: Callable[..., Any] = field(repr=False)
    contract: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not callable(self.process):
            raise TypeError(f"Processor.process is a {type(self.process).__name__}, not a function")
        object.__setattr__(self, "contract", _frozen_json(self.contract, what="Processor.contract"))

    def data_contract(self) -> dict[str, Any]:
        return dict(self.contract)

    def fingerprint(self) -> str:
        return hashlib.sha256(json.dumps(self.data_contract(), sort_keys=True).encode()).hexdigest()

    def __call__(self, artifacts: Sequence[Any], *, route: Route | str = Route.GENERIC, seed: int | None = None,
                 **options: Any) -> Any:
        return self.process(artifacts, route=Route(route), seed=seed, **options)


def _callable_contract(value: Callable[..., Any]) -> dict[str, str]:
    """Identity of a callable plus a digest of the code that defines it.

    The digest covers the whole defining module file when there is one (so a
    change anywhere in it changes the data contract), else the callable's own
    source, else nothing beyond the dotted name.
    """

    owner = value if (inspect.isfunction(value) or inspect.isclass(value) or inspect.ismethod(value)) \
        else type(value)
    name = f"{getattr(value, '__module__', owner.__module__)}.{getattr(value, '__qualname__', owner.__qualname__)}"
    record = {"callable": name}
    try:
        source_file = inspect.getsourcefile(owner)
    except TypeError:
        source_file = None
    if source_file and Path(source_file).is_file():
        record["module_file_sha256"] = hashlib.sha256(Path(source_file).read_bytes()).hexdigest()
        return record
    try:
        record["callable_source_sha256"] = hashlib.sha256(inspect.getsource(owner).encode()).hexdigest()
    except (OSError, TypeError):
        pass
    return record


def _as_artifact(value: Any, modality: Modality) -> Artifact:
    if not isinstance(value, Artifact):
        return Artifact.inline(modality, value)
    if value.modality == modality:
        return value
    raise TypeError(f"a {modality} processor was given a {value.modality} artifact")


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
    not_callable = [n for n, f in (("probe", probe), ("prepare", prepare), ("batch_builder", batch_builder))
                    if not callable(f)]
    if not_callable:
        raise TypeError(f"media processor: {', '.join(not_callable)} not callable")
    config = dict(_frozen_json(configuration, what="media processor configuration"))
    shapes = tuple(dict.fromkeys(_dims(s, what="admitted media shape") for s in admitted_shapes))
    ranks = {len(s) for s in shapes}
    if len(ranks) != 1:
        raise ValueError(f"admitted media shapes {list(shapes)} need one common, non-zero rank")
    rank = ranks.pop()

    def process(artifacts: Sequence[Any], *, route: Route, seed: int | None) -> Any:
        if len(artifacts) == 0:
            raise ValueError("a media batch needs at least one artifact")
        items = [_as_artifact(a, modality) for a in artifacts]
        needs = [_dims(probe(a, route=route), what=f"{modality} probe result") for a in items]
        if {len(n) for n in needs} != {rank}:
            raise ValueError(f"{modality} probe results have to be rank {rank}, got {needs}")
        bucket = select_static_shape_bucket(tuple(max(v) for v in zip(*needs)), shapes)
        seeds = [None] * len(items) if seed is None else np.random.SeedSequence(seed).spawn(len(items))
        rows = []
        for item, s in zip(items, seeds):
            prepared = prepare(item, bucket=bucket, route=route, rng=None if s is None else np.random.default_rng(s))
            if not (isinstance(prepared, Mapping) and prepared):
                raise TypeError(f"prepare() returned {type(prepared).__name__}; a non-empty dict of arrays "
                                "was expected")
            rows.append({k: np.asarray(v) for k, v in prepared.items()})
        names = tuple(rows[0])
        odd = [i for i, r in enumerate(rows) if tuple(r) != names]
        if odd:
            raise ValueError(f"prepare() returned other fields for rows {odd} than {list(names)}")
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
        wrong = [tuple(s) for s in admitted_shapes if len(tuple(s)) != rank]
        if wrong:
            raise ValueError(f"{modality} shapes are {what}; got {wrong}")
        return make_media_processor(modality=modality, admitted_shapes=admitted_shapes, probe=probe,
                                    prepare=prepare, batch_builder=batch_builder, configuration=configuration)

    build.__name__ = f"make_{modality.value}_processor"
    build.__doc__ = f"Build a {modality.value} processor whose shapes mean {what}."
    return build


make_image_processor = _media_with_rank(Modality.IMAGE, 2, "(height, width)")
make_audio_processor = _media_with_rank(Modality.AUDIO, 1, "(samples,)")
make_video_processor = _media_with_rank(Modality.VIDEO, 3, "(frames, height, width)")


_ROUTE_PROMPTS = {Route.QUERY: ("query",), Route.DOCUMENT: ("document", "passage", "corpus")}


def _length_buckets(longest: int | None, buckets: Sequence[int] | None) -> tuple[int, ...]:
    """Sorted distinct padding lengths; a single bucket of ``longest`` when none are given."""

    if buckets is None:
        if longest is None:
            raise ValueError("give max_sequence_length, sequence_length_buckets or both")
        buckets = (longest,)
    picked = tuple(buckets)
    if not picked or not all(type(n) is int and n > 0 for n in picked):
        raise ValueError(f"sequence_length_buckets {picked!r}: lengths have to be ints >= 1")
    ordered = tuple(sorted(set(picked)))
    if longest is not None and ordered[-1] > longest:
        raise ValueError(f"bucket {ordered[-1]} is longer than max_sequence_length {longest}")
    return ordered


def _text_of(item: Any) -> str:
    if isinstance(item, str):
        return item
    if isinstance(item, Artifact) and item.modality == Modality.TEXT and isinstance(item.data, str):
        return item.data
    raise TypeError(f"text processor input {item!r} is neither a string nor an inline text artifact")


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

    lengths = _length_buckets(max_sequence_length, sequence_length_buckets)
    prompt_values = dict(prompts or {})
    if default_prompt_name is not None and default_prompt_name not in prompt_values:
        raise ValueError(f"default prompt {default_prompt_name!r} is none of {sorted(prompt_values)}")
    if not include_prompt and pooling_batch_builder is None:
        raise ValueError("include_prompt=False masks prompt tokens through pooling_batch_builder; pass one")
    maximum = lengths[-1]

    def route_prompt(route: Route, prompt_name: str | None, prompt: str | None) -> str:
        if prompt is not None:
            if prompt_name is not None:
                raise ValueError("pass a prompt text or a prompt name, not both")
            return prompt
        if prompt_name is not None:
            if prompt_name not in prompt_values:
                raise KeyError(f"no prompt named {prompt_name!r} (have {sorted(prompt_values)})")
            return prompt_values[prompt_name]
        candidates = _ROUTE_PROMPTS.get(route, ())
        if route is Route.GENERIC and default_prompt_name is not None:
            candidates = (default_prompt_name,)
        return next((prompt_values[n] for n in candidates if n in prompt_values), "")

    def pad_id() -> int:
        value = getattr(tokenizer, "pad_token_id", None)
        if value is None:
            value = getattr(tokenizer, "pad_id", 0)
        if value is None:
            raise ValueError(f"{type(tokenizer).__name__} has no pad token; set pad_token_id")
        return int(value)

    def tokenize(texts: Sequence[str]) -> dict[str, np.ndarray]:
        if len(texts) == 0:
            raise ValueError("a text batch needs at least one text")
        encoded = tokenizer(list(texts), padding=True, truncation=True, max_length=maximum, return_tensors="np")
        if not isinstance(encoded, Mapping):
            encoded = dict(encoded)
        arrays = {k: np.asarray(v) for k, v in encoded.items()}
        if "input_ids" not in arrays:
            raise KeyError("tokenizer output is missing 'input_ids'")
        ids = arrays["input_ids"]
        if ids.shape[:1] != (len(texts),) or ids.ndim != 2:
            raise ValueError(f"tokenizer returned input_ids of shape {ids.shape} for {len(texts)} texts")
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
        texts = [_text_of(a) for a in artifacts]
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
