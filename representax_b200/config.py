"""Serializable user-facing configuration for reproducible training.

Parity: every class of src/representax/config.py:46-773 with the same field
names, defaults and roles (``Scientific`` / ``Execution``) and the same
accept/reject decisions, so a job file written for the reference validates
here unchanged. The checks are stated as (rule, complaint) pairs; one
``ValueError`` lists every broken rule of an object. Execution-only
fields specific to this framework (tensor-parallel degree, fused-kernel
toggles) live in ``B200ExecutionConfig`` under ``TrainingConfig.b200`` and
carry the ``Execution`` role, leaving the scientific fingerprint unchanged.
"""

from __future__ import annotations

import math
import re
from collections.abc import Mapping
from typing import Annotated, Literal

from pydantic import (
    Discriminator,
    Field,
    NonNegativeInt,
    PositiveFloat,
    PositiveInt,
    SerializeAsAny,
    Tag,
    ValidationInfo,
    field_validator,
    model_validator,
)
from typing_extensions import TypeAliasType

from ._config import Execution, FrozenConfig, NonEmptyString, ParameterRole, Scientific, project_parameters
from .core import Route
from .data.config import DataDistributionConfig
from .tasks.config import LossConfig, LossModifierConfig, TaskConfig

RematerializationPolicy = Literal["none", "selective", "full"]
PrecisionDType = Literal["float32", "bfloat16"]
MatrixDType = Literal["float32", "bfloat16", "float8_e4m3fn"]
MetricMode = Literal["min", "max"]
ExportSelection = Literal["final", "best"]
JsonScalar = str | int | float | bool | None
JsonValue = TypeAliasType("JsonValue", JsonScalar | list["JsonValue"] | dict[str, "JsonValue"])


# --- validation helpers -----------------------------------------------------------------
# Every validator below states its rules as (holds, complaint) pairs and hands them to
# ``_check``, which reports all broken rules of one object in a single ValueError.

def _check(*rules: tuple[bool, str]) -> None:
    broken = [complaint for holds, complaint in rules if not holds]
    if broken:
        raise ValueError("; ".join(broken))


def _repeated(values) -> list:
    """Values that occur more than once, in first-seen order."""

    seen: set = set()
    twice: list = []
    for value in values:
        if value in seen and value not in twice:
            twice.append(value)
        seen.add(value)
    return twice


def _regex_problem(pattern: str) -> str | None:
    try:
        re.compile(pattern)
    except re.error as error:
        return str(error)
    return None


def _axis_names(entries) -> list[str]:
    """Mesh-axis names named by a sequence of partition entries (None = replicated)."""

    names: list[str] = []
    for entry in entries:
        if entry is None:
            continue
        names.extend(entry if isinstance(entry, tuple) else (entry,))
    return names


def _context_registry(info: ValidationInfo, key: str, fallback, expected: type):
    """A registry passed through pydantic's validation context, else the built-in one."""

    supplied = (info.context or {}).get(key)
    if supplied is None:
        return fallback
    if not isinstance(supplied, expected):
        raise TypeError(f"validation context entry {key!r} is a {type(supplied).__name__}, "
                        f"expected {expected.__name__}")
    return supplied


class ComponentConfig(FrozenConfig):
    target: NonEmptyString
    parameters: dict[str, JsonValue] = Field(default_factory=dict)


class ModelConfig(ComponentConfig):
    """Model definition consumed by a model builder (dotted target)."""


class OptimizationConfig(FrozenConfig):
    optimizer: ComponentConfig
    schedule: ComponentConfig | None = None
    schedule_parameter: NonEmptyString = "learning_rate"
    max_gradient_norm: Scientific[PositiveFloat | None] = 1.0


class DataConfig(FrozenConfig):
    distribution: Scientific[DataDistributionConfig]
    collate: Scientific[ComponentConfig | None] = None
    drop_remainder: Scientific[bool] = True
    num_threads: Execution[NonNegativeInt] = 16
    prefetch_buffer_size: Execution[NonNegativeInt] = 16
    host_memory_budget_bytes: Execution[PositiveInt | None] = None
    data_wait_heartbeat_seconds: Execution[PositiveFloat | None] = None
    data_wait_timeout_seconds: Execution[PositiveFloat | None] = None

    @model_validator(mode="before")
    @classmethod
    def _accept_bare_distribution(cls, value: object) -> object:
        # ``DataConfig(distribution)`` shorthand: a distribution (object or mapping with
        # ``sources``) given where the data config is expected.
        bare = isinstance(value, DataDistributionConfig) or (
            isinstance(value, Mapping) and "sources" in value and "distribution" not in value)
        return {"distribution": value} if bare else value

    @model_validator(mode="after")
    def _heartbeat_before_deadline(self):
        beat, deadline = self.data_wait_heartbeat_seconds, self.data_wait_timeout_seconds
        _check((beat is None or deadline is None or beat < deadline,
                f"the data-wait heartbeat ({beat} s) has to fire before the data-wait timeout ({deadline} s)"))
        return self


Similarity = Literal["cosine", "dot", "euclidean", "manhattan"]


class EvaluatorConfig(FrozenConfig):
    kind: Literal["loss"] = "loss"
    name: NonEmptyString = "loss"


class EmbeddingSimilarityEvaluatorConfig(EvaluatorConfig):
    kind: Literal["embedding_similarity"] = "embedding_similarity"  # type: ignore[assignment]
    name: NonEmptyString = "similarity"
    similarity_functions: tuple[Similarity, ...] = ("cosine", "dot", "euclidean", "manhattan")
    main_similarity: Similarity | None = None
    left_route: Route = Route.GENERIC
    right_route: Route = Route.GENERIC

    @model_validator(mode="after")
    def _functions_cover_main(self):
        functions = self.similarity_functions
        _check((len(functions) > 0, "similarity_functions is empty"),
               (not _repeated(functions), f"similarity_functions lists {_repeated(functions)} more than once"),
               (self.main_similarity is None or self.main_similarity in functions,
                f"main_similarity {self.main_similarity!r} is not among similarity_functions {list(functions)}"))
        return self


class InformationRetrievalEvaluatorConfig(EvaluatorConfig):
    kind: Literal["information_retrieval"] = "information_retrieval"  # type: ignore[assignment]
    name: NonEmptyString = "retrieval"
    k_values: tuple[PositiveInt, ...] = (1, 3, 5, 10)
    similarity: Literal["cosine", "dot"] = "cosine"


def _evaluator_kind(value: object) -> str:
    """Discriminator of the evaluator union; a mapping without ``kind`` is a loss evaluator."""

    if isinstance(value, Mapping):
        return str(value.get("kind", "loss"))
    return str(getattr(value, "kind", "loss"))


AnyEvaluatorConfig = Annotated[
    Annotated[EvaluatorConfig, Tag("loss")]
    | Annotated[EmbeddingSimilarityEvaluatorConfig, Tag("embedding_similarity")]
    | Annotated[InformationRetrievalEvaluatorConfig, Tag("information_retrieval")],
    Discriminator(_evaluator_kind),
]


class EvaluationConfig(FrozenConfig):
    data: DataConfig
    batch_size: Scientific[PositiveInt]
    evaluators: Scientific[tuple[AnyEvaluatorConfig, ...]] = (EvaluatorConfig(),)
    every_steps: PositiveInt | None = None
    on_start: bool = False
    on_end: bool = True
    max_batches: Scientific[PositiveInt | None] = None
    primary_metric: Scientific[NonEmptyString] = "valid/loss"
    primary_metric_mode: Scientific[MetricMode] = "min"
    save_best: bool = True
    keep_best: PositiveInt = 1

    @model_validator(mode="after")
    def _consistent_selection(self):
        names = [e.name for e in self.evaluators]
        scheduled = self.on_start or self.on_end or self.every_steps is not None
        _check((len(names) > 0, "evaluation needs an evaluator"),
               (not _repeated(names), f"evaluator name(s) {_repeated(names)} used twice; metrics would collide"),
               (self.primary_metric.startswith("valid/"),
                f"primary_metric {self.primary_metric!r} is not a validation metric (prefix 'valid/')"),
               (scheduled or not self.save_best,
                "save_best is set but evaluation never runs (no on_start, on_end or every_steps)"))
        return self


class HuggingFaceExportConfig(FrozenConfig):
    source_checkpoint: NonEmptyString
    adapter: ComponentConfig
    verify_reload: bool = True


class ExportConfig(FrozenConfig):
    enabled: bool = True
    selection: ExportSelection = "final"
    directory_name: NonEmptyString = "final-model"
    huggingface: HuggingFaceExportConfig | None = None

    @field_validator("directory_name")
    @classmethod
    def _single_component(cls, value: str) -> str:
        _check((value not in (".", "..") and not any(sep in value for sep in "/\\"),
                f"export directory_name {value!r} has to be a plain directory name inside the run directory"))
        return value


class MeshConfig(FrozenConfig):
    axis_shapes: tuple[PositiveInt, ...] = (1,)
    axis_names: tuple[NonEmptyString, ...] = ("data",)

    @model_validator(mode="after")
    def _names_match_shapes(self):
        names, shapes = self.axis_names, self.axis_shapes
        _check((len(names) > 0, "the mesh has no axes"),
               (len(names) == len(shapes), f"{len(names)} mesh axis names for {len(shapes)} axis sizes"),
               (not _repeated(names), f"mesh axis name(s) {_repeated(names)} repeat"))
        return self

    @property
    def axes(self) -> dict[str, int]:
        """Axis name -> size."""

        return dict(zip(self.axis_names, self.axis_shapes))

    @property
    def device_count(self) -> int:
        return math.prod(self.axes.values())

    def axis_size(self, name: str) -> int:
        size = self.axes.get(name)
        if size is None:
            raise KeyError(f"no mesh axis named {name!r} (axes: {list(self.axis_names)})")
        return size


PartitionAxis = NonEmptyString | tuple[NonEmptyString, ...] | None


class PartitionRuleConfig(FrozenConfig):
    pattern: NonEmptyString
    axes: tuple[PartitionAxis, ...] = ()

    @model_validator(mode="after")
    def _compiles_and_axes_distinct(self):
        problem = _regex_problem(self.pattern)
        grouped_empty = any(isinstance(a, tuple) and not a for a in self.axes)
        used = _axis_names(self.axes)
        _check((problem is None, f"partition-rule pattern {self.pattern!r} does not compile ({problem})"),
               (not grouped_empty, "an axis group of a partition rule is the empty tuple"),
               (not _repeated(used), f"partition rule shards over mesh axis {_repeated(used)} more than once"))
        return self


class DDPConfig(FrozenConfig):
    kind: Literal["ddp"] = "ddp"
    axis: NonEmptyString = "data"


class FSDPConfig(FrozenConfig):
    kind: Literal["fsdp"] = "fsdp"
    data_axis: NonEmptyString = "data"
    parameter_axis: NonEmptyString | None = None
    minimum_parameter_elements: PositiveInt = 2 ** 18

    @property
    def resolved_parameter_axis(self) -> str:
        return self.parameter_axis or self.data_axis


class CustomShardingConfig(FrozenConfig):
    kind: Literal["custom"] = "custom"
    data_axis: NonEmptyString | None = None
    parameter_axes: tuple[NonEmptyString, ...]
    parameter_rules: tuple[PartitionRuleConfig, ...]
    default_parameter_axes: tuple[PartitionAxis, ...] = ()

    @model_validator(mode="after")
    def _rules_within_axes(self):
        axes = self.parameter_axes
        named = set(_axis_names(self.default_parameter_axes))
        for rule in self.parameter_rules:
            named.update(_axis_names(rule.axes))
        stray = sorted(named - set(axes))
        _check((len(axes) > 0, "custom sharding names no parameter axis"),
               (not _repeated(axes), f"parameter axis {_repeated(axes)} listed twice"),
               (len(self.parameter_rules) > 0, "custom sharding has no parameter rule"),
               (not stray, f"partition rules shard over {stray}, which parameter_axes does not declare"))
        return self

    @property
    def referenced_axes(self) -> set[str]:
        return set(self.parameter_axes) | ({self.data_axis} if self.data_axis else set())


class TensorParallelConfig(FrozenConfig):
    """Megatron-style tensor parallelism inside a model axis (new capability)."""

    kind: Literal["tensor_parallel"] = "tensor_parallel"
    data_axis: NonEmptyString = "data"
    model_axis: NonEmptyString = "model"
    fsdp_over_data: bool = True


ShardingConfig = Annotated[DDPConfig | FSDPConfig | CustomShardingConfig | TensorParallelConfig,
                           Field(discriminator="kind")]


def _sharding_axes(sharding) -> set[str]:
    if isinstance(sharding, DDPConfig):
        return {sharding.axis}
    if isinstance(sharding, FSDPConfig):
        return {sharding.data_axis, sharding.resolved_parameter_axis}
    if isinstance(sharding, TensorParallelConfig):
        return {sharding.data_axis, sharding.model_axis}
    return sharding.referenced_axes


class BatchConfig(FrozenConfig):
    micro_batch_size: PositiveInt
    gradient_accumulation_steps: PositiveInt = 1


class GradCacheConfig(FrozenConfig):
    micro_batch_size: PositiveInt = Field(description="Examples encoded by each replayed forward pass.")
    query_micro_batch_size: PositiveInt | None = None
    document_micro_batch_size: PositiveInt | None = None
    loss_row_chunk_size: PositiveInt | None = None

    @property
    def resolved_query_micro_batch_size(self) -> int:
        return self.query_micro_batch_size or self.micro_batch_size

    @property
    def resolved_document_micro_batch_size(self) -> int:
        return self.document_micro_batch_size or self.micro_batch_size

    @property
    def resolved_loss_row_chunk_size(self) -> int:
        return self.loss_row_chunk_size or self.micro_batch_size


class MegaBatchMiningConfig(FrozenConfig):
    micro_batch_size: PositiveInt
    loss_row_chunk_size: PositiveInt | None = None

    @property
    def resolved_loss_row_chunk_size(self) -> int:
        return self.loss_row_chunk_size or self.micro_batch_size


class PrecisionConfig(FrozenConfig):
    parameter_dtype: Literal["float32"] = "float32"
    compute_dtype: PrecisionDType = "float32"
    activation_dtype: PrecisionDType = "float32"
    matrix_dtype: MatrixDType | None = None
    accumulation_dtype: Literal["float32"] = "float32"
    loss_dtype: Literal["float32"] = "float32"
    # float8 matrices: one scale per tensor (the reference's recipe) or one
    # power-of-two scale per 32-value block (MXFP8)
    fp8_scaling: Literal["tensor", "block"] = "tensor"

    @classmethod
    def bfloat16_mixed(cls) -> "PrecisionConfig":
        return cls(compute_dtype="bfloat16", activation_dtype="bfloat16")

    @classmethod
    def float8_mixed(cls) -> "PrecisionConfig":
        return cls(compute_dtype="bfloat16", activation_dtype="bfloat16", matrix_dtype="float8_e4m3fn")

    @property
    def resolved_matrix_dtype(self) -> MatrixDType:
        return self.matrix_dtype or self.compute_dtype

    @property
    def communication_dtype(self) -> PrecisionDType:
        return self.compute_dtype


class QuantizedLoRAConfig(FrozenConfig):
    bits: Literal[4] = 4
    rank: PositiveInt
    alpha: PositiveFloat
    target_pattern: NonEmptyString = ".*"
    initialization_scale: PositiveFloat | None = None

    @field_validator("target_pattern")
    @classmethod
    def _pattern_compiles(cls, pattern: str) -> str:
        problem = _regex_problem(pattern)
        _check((problem is None, f"adapter target_pattern {pattern!r} does not compile ({problem})"))
        return pattern


class B200ExecutionConfig(FrozenConfig):
    """Execution knobs of this framework (none changes what is learned)."""

    fused_mnr_collectives: bool = True
    overlap_gradient_reduction: bool = True
    gradient_bucket_bytes: PositiveInt = 64 * 2 ** 20
    cuda_graphs: bool = False
    deterministic: bool = True
    # GradCache: device bytes that first-pass chunk graphs may keep so their
    # replay forward is skipped (exact same gradient). None (the default) and 0
    # both mean: replay every chunk, the memory bound GradCache is chosen for;
    # "auto" keeps as many as the free HBM allows.
    grad_cache_retain_bytes: NonNegativeInt | Literal["auto"] | None = None


class TrainingConfig(FrozenConfig):
    global_batch_size: Scientific[PositiveInt]
    max_steps: Scientific[PositiveInt]
    seed: Scientific[NonNegativeInt]
    mesh: Execution[MeshConfig] = MeshConfig()
    sharding: Execution[ShardingConfig] = DDPConfig()
    batch: Execution[BatchConfig]
    grad_cache: Execution[GradCacheConfig | None] = None
    mega_batch_mining: Execution[MegaBatchMiningConfig | None] = None
    adapter: Scientific[QuantizedLoRAConfig | None] = None
    precision: Execution[PrecisionConfig] = PrecisionConfig()
    activation_rematerialization: Execution[RematerializationPolicy] = "full"
    donate_buffers: Execution[bool] = True
    b200: Execution[B200ExecutionConfig] = B200ExecutionConfig()

    @model_validator(mode="after")
    def _one_execution_and_known_axes(self):
        missing = sorted(_sharding_axes(self.sharding) - set(self.mesh.axis_names))
        _check((self.grad_cache is None or self.mega_batch_mining is None,
                "grad_cache and mega_batch_mining are alternative loss executions; set at most one"),
               (not missing, f"the sharding plan uses mesh axes {missing} that the mesh does not define"))
        return self


class LoggingConfig(FrozenConfig):
    console_every: PositiveInt = 1
    reporter_queue_size: PositiveInt = 16


class CheckpointConfig(FrozenConfig):
    every: PositiveInt
    keep: PositiveInt = 3
    additional_iterations: tuple[PositiveInt, ...] = ()
    save_final: bool = True
    asynchronous: bool = True

    @model_validator(mode="after")
    def _distinct_extra_iterations(self):
        twice = _repeated(self.additional_iterations)
        _check((not twice, f"additional checkpoint iteration(s) {twice} listed twice"))
        return self

    def should_save(self, iteration: int, *, final: bool) -> bool:
        return iteration % self.every == 0 or iteration in self.additional_iterations or (final and self.save_final)


_EXCLUSIVE_MODIFIERS = frozenset({"matryoshka", "adaptive_layer", "matryoshka_2d"})


class JobConfig(FrozenConfig):
    """Fully serializable configuration of one reproducible training job."""

    name: NonEmptyString
    model: Scientific[ModelConfig]
    task: Scientific[SerializeAsAny[TaskConfig]]
    loss: Scientific[SerializeAsAny[LossConfig]]
    loss_modifiers: Scientific[tuple[SerializeAsAny[LossModifierConfig], ...]] = ()
    optimization: Scientific[OptimizationConfig]
    data: DataConfig
    training: TrainingConfig
    checkpointing: CheckpointConfig | None = None
    logging: LoggingConfig = LoggingConfig()
    evaluation: EvaluationConfig | None = None
    export: ExportConfig = ExportConfig()

    # Task, loss and modifier configs are open families: each registry parses its own
    # kinds. A caller may validate against its own registries through the validation
    # context (keys task_registry / loss_registry / modifier_registry).

    @field_validator("task", mode="before")
    @classmethod
    def _parse_task(cls, value: object, info: ValidationInfo) -> TaskConfig:
        from .tasks.registry import BUILTIN_TASKS, TaskRegistry

        return _context_registry(info, "task_registry", BUILTIN_TASKS, TaskRegistry).parse(value)

    @field_validator("loss", mode="before")
    @classmethod
    def _parse_loss(cls, value: object, info: ValidationInfo) -> LossConfig:
        from .tasks.registry import BUILTIN_LOSSES, LossRegistry

        return _context_registry(info, "loss_registry", BUILTIN_LOSSES, LossRegistry).parse(value)

    @field_validator("loss_modifiers", mode="before")
    @classmethod
    def _parse_modifiers(cls, value: object, info: ValidationInfo):
        from .tasks.registry import BUILTIN_LOSS_MODIFIERS, LossModifierRegistry

        registry = _context_registry(info, "modifier_registry", BUILTIN_LOSS_MODIFIERS, LossModifierRegistry)
        if isinstance(value, (str, bytes, Mapping)) or not isinstance(value, (list, tuple)):
            raise TypeError(f"loss_modifiers takes a sequence of modifier configs, got {type(value).__name__}")
        parsed = tuple(registry.parse(item) for item in value)
        kinds = [m.kind for m in parsed]
        _check((not _repeated(kinds), f"loss modifier(s) {_repeated(kinds)} applied twice"),
               (len(kinds) < 2 or not _EXCLUSIVE_MODIFIERS.intersection(kinds),
                f"modifiers {kinds} cannot be stacked: matryoshka, adaptive_layer and matryoshka_2d each "
                "rewrite the representation; matryoshka_2d is the combined dimension x layer objective"))
        return parsed

    @model_validator(mode="after")
    def _loss_supports_plan(self, info: ValidationInfo):
        from .tasks.registry import BUILTIN_LOSS_MODIFIERS, BUILTIN_LOSSES, LossModifierRegistry, LossRegistry

        losses = _context_registry(info, "loss_registry", BUILTIN_LOSSES, LossRegistry)
        modifiers = _context_registry(info, "modifier_registry", BUILTIN_LOSS_MODIFIERS, LossModifierRegistry)
        loss = losses.definition(self.loss.kind)
        strategy = self.training_strategy
        accumulating = self.training.batch.gradient_accumulation_steps > 1
        rules = [
            (self.task.kind in loss.task_kinds,
             f"loss {self.loss.kind!r} is defined for tasks {sorted(loss.task_kinds)}, not {self.task.kind!r}"),
            (strategy in loss.training_strategies,
             f"loss {self.loss.kind!r} cannot run under the {strategy!r} execution"),
            (not accumulating or strategy == "direct",
             f"gradient_accumulation_steps > 1 needs direct execution; {strategy!r} already splits the "
             "logical batch into its own chunks"),
            (not accumulating or loss.microbatch_accumulation,
             f"loss {self.loss.kind!r} couples examples across the batch, so microbatch accumulation would "
             "change its value"),
        ]
        for modifier in self.loss_modifiers:
            spec = modifiers.definition(modifier.kind)
            rules.append((strategy in spec.training_strategies,
                          f"modifier {modifier.kind!r} cannot run under the {strategy!r} execution"))
            rules.append((not accumulating or spec.microbatch_accumulation,
                          f"modifier {modifier.kind!r} is not exact under microbatch accumulation"))
        _check(*rules)
        return self

    @model_validator(mode="after")
    def _schedules_fit(self):
        extra = () if self.checkpointing is None else self.checkpointing.additional_iterations
        late = sorted(i for i in extra if i > self.training.max_steps)
        selects_best = self.evaluation is not None and self.evaluation.save_best
        _check((not late, f"checkpoint iteration(s) {late} come after the last step {self.training.max_steps}"),
               (not selects_best or self.checkpointing is not None,
                "evaluation.save_best keeps the best checkpoint, so checkpointing must be configured"),
               (not (self.export.enabled and self.export.selection == "best") or selects_best,
                "export.selection='best' needs evaluation with save_best"))
        return self

    @property
    def training_strategy(self) -> str:
        if self.training.grad_cache is not None:
            return "grad_cache"
        if self.training.mega_batch_mining is not None:
            return "mega_batch_mining"
        return "direct"

    def parameters(self, role: ParameterRole) -> dict[str, object]:
        return project_parameters(self, role)


__all__ = [
    "AnyEvaluatorConfig", "B200ExecutionConfig", "BatchConfig", "CheckpointConfig", "ComponentConfig",
    "CustomShardingConfig", "DDPConfig", "DataConfig", "EmbeddingSimilarityEvaluatorConfig", "EvaluationConfig",
    "EvaluatorConfig", "ExportConfig", "FSDPConfig", "GradCacheConfig", "HuggingFaceExportConfig",
    "InformationRetrievalEvaluatorConfig", "JobConfig", "LoggingConfig", "MegaBatchMiningConfig", "MeshConfig",
    "ModelConfig", "OptimizationConfig", "ParameterRole", "PartitionAxis", "PartitionRuleConfig", "PrecisionConfig",
    "QuantizedLoRAConfig", "RematerializationPolicy", "ShardingConfig", "TensorParallelConfig", "TrainingConfig",
]
