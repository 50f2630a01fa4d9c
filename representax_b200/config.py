"""Serializable user-facing configuration for reproducible training.

Parity: every class of src/representax/config.py:46-773 with the same field
names, defaults, roles (``Scientific`` / ``Execution``) and validation, so a
job file written for the reference validates here unchanged. Execution-only
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
    Field,
    NonNegativeInt,
    PositiveFloat,
    PositiveInt,
    SerializeAsAny,
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
    def wrap_distribution(cls, value: object) -> object:
        if isinstance(value, DataDistributionConfig):
            return {"distribution": value}
        if isinstance(value, Mapping) and "distribution" not in value and "sources" in value:
            return {"distribution": value}
        return value

    @model_validator(mode="after")
    def validate_data_wait_thresholds(self):
        if (self.data_wait_heartbeat_seconds is not None and self.data_wait_timeout_seconds is not None
                and self.data_wait_heartbeat_seconds >= self.data_wait_timeout_seconds):
            raise ValueError("data_wait_heartbeat_seconds must be below data_wait_timeout_seconds")
        return self


class EvaluatorConfig(FrozenConfig):
    kind: Literal["loss"] = "loss"
    name: NonEmptyString = "loss"


class EmbeddingSimilarityEvaluatorConfig(EvaluatorConfig):
    kind: Literal["embedding_similarity"] = "embedding_similarity"  # type: ignore[assignment]
    name: NonEmptyString = "similarity"
    similarity_functions: tuple[Literal["cosine", "dot", "euclidean", "manhattan"], ...] = (
        "cosine", "dot", "euclidean", "manhattan")
    main_similarity: Literal["cosine", "dot", "euclidean", "manhattan"] | None = None
    left_route: Route = Route.GENERIC
    right_route: Route = Route.GENERIC

    @model_validator(mode="after")
    def validate_similarity(self):
        if not self.similarity_functions:
            raise ValueError("at least one similarity function is required")
        if len(set(self.similarity_functions)) != len(self.similarity_functions):
            raise ValueError("similarity functions must be unique")
        if self.main_similarity is not None and self.main_similarity not in self.similarity_functions:
            raise ValueError("main_similarity must be one of similarity_functions")
        return self


class InformationRetrievalEvaluatorConfig(EvaluatorConfig):
    kind: Literal["information_retrieval"] = "information_retrieval"  # type: ignore[assignment]
    name: NonEmptyString = "retrieval"
    k_values: tuple[PositiveInt, ...] = (1, 3, 5, 10)
    similarity: Literal["cosine", "dot"] = "cosine"


_EVALUATORS = {
    "loss": EvaluatorConfig,
    "embedding_similarity": EmbeddingSimilarityEvaluatorConfig,
    "information_retrieval": InformationRetrievalEvaluatorConfig,
}


class EvaluationConfig(FrozenConfig):
    data: DataConfig
    batch_size: Scientific[PositiveInt]
    evaluators: Scientific[tuple[SerializeAsAny[EvaluatorConfig], ...]] = (EvaluatorConfig(),)
    every_steps: PositiveInt | None = None
    on_start: bool = False
    on_end: bool = True
    max_batches: Scientific[PositiveInt | None] = None
    primary_metric: Scientific[NonEmptyString] = "valid/loss"
    primary_metric_mode: Scientific[MetricMode] = "min"
    save_best: bool = True
    keep_best: PositiveInt = 1

    @field_validator("evaluators", mode="before")
    @classmethod
    def validate_evaluators(cls, value: object) -> object:
        if not isinstance(value, (list, tuple)):
            raise TypeError("evaluators must be a list or tuple")
        parsed = []
        for evaluator in value:
            if isinstance(evaluator, EvaluatorConfig):
                parsed.append(evaluator)
                continue
            if not isinstance(evaluator, Mapping):
                raise TypeError("each evaluator must be a config or mapping")
            kind = evaluator.get("kind", "loss")
            if kind not in _EVALUATORS:
                raise ValueError(f"unknown evaluator kind {kind!r}")
            parsed.append(_EVALUATORS[kind].model_validate(evaluator))
        return tuple(parsed)

    @model_validator(mode="after")
    def validate_evaluation(self):
        names = tuple(e.name for e in self.evaluators)
        if not names:
            raise ValueError("evaluation requires at least one evaluator")
        if len(set(names)) != len(names):
            raise ValueError("evaluator names must be unique")
        if not self.primary_metric.startswith("valid/"):
            raise ValueError("primary_metric must use the valid/ namespace")
        if self.save_best and not (self.on_start or self.on_end or self.every_steps is not None):
            raise ValueError("best-model selection requires an evaluation cadence")
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
    def validate_directory_name(cls, value: str) -> str:
        if value in {".", ".."} or "/" in value or "\\" in value:
            raise ValueError("export directory_name must be one path component")
        return value


class MeshConfig(FrozenConfig):
    axis_shapes: tuple[PositiveInt, ...] = (1,)
    axis_names: tuple[NonEmptyString, ...] = ("data",)

    @model_validator(mode="after")
    def validate_axes(self):
        if len(self.axis_shapes) != len(self.axis_names):
            raise ValueError("mesh axis_shapes and axis_names must have equal length")
        if not self.axis_names:
            raise ValueError("a mesh must contain at least one logical axis")
        if len(set(self.axis_names)) != len(self.axis_names):
            raise ValueError("mesh axis names must be unique")
        return self

    @property
    def device_count(self) -> int:
        return math.prod(self.axis_shapes)

    def axis_size(self, name: str) -> int:
        try:
            return self.axis_shapes[self.axis_names.index(name)]
        except ValueError as error:
            raise KeyError(f"mesh axis {name!r} is not defined") from error


PartitionAxis = NonEmptyString | tuple[NonEmptyString, ...] | None


class PartitionRuleConfig(FrozenConfig):
    pattern: NonEmptyString
    axes: tuple[PartitionAxis, ...] = ()

    @field_validator("pattern")
    @classmethod
    def validate_pattern(cls, value: str) -> str:
        try:
            re.compile(value)
        except re.error as error:
            raise ValueError(f"invalid partition-rule regular expression: {error}") from error
        return value

    @field_validator("axes")
    @classmethod
    def validate_partition_axes(cls, value):
        names: list[str] = []
        for axis in value:
            if isinstance(axis, tuple) and not axis:
                raise ValueError("a grouped partition axis cannot be empty")
            if axis is None:
                continue
            names.extend(axis if isinstance(axis, tuple) else (axis,))
        if len(set(names)) != len(names):
            raise ValueError("a partition rule cannot reuse one mesh axis")
        return value


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
    def validate_custom_sharding(self):
        if not self.parameter_axes:
            raise ValueError("custom sharding requires at least one parameter axis")
        if len(set(self.parameter_axes)) != len(self.parameter_axes):
            raise ValueError("custom parameter axes must be unique")
        if not self.parameter_rules:
            raise ValueError("custom sharding requires at least one parameter rule")
        return self


class TensorParallelConfig(FrozenConfig):
    """Megatron-style tensor parallelism inside a model axis (new capability)."""

    kind: Literal["tensor_parallel"] = "tensor_parallel"
    data_axis: NonEmptyString = "data"
    model_axis: NonEmptyString = "model"
    fsdp_over_data: bool = True


ShardingConfig = Annotated[DDPConfig | FSDPConfig | CustomShardingConfig | TensorParallelConfig,
                           Field(discriminator="kind")]


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
    def validate_target_pattern(cls, pattern: str) -> str:
        try:
            re.compile(pattern)
        except re.error as error:
            raise ValueError(f"invalid adapter target_pattern: {error}") from error
        return pattern


class B200ExecutionConfig(FrozenConfig):
    """Execution knobs of this framework (none changes what is learned)."""

    fused_mnr_collectives: bool = True
    overlap_gradient_reduction: bool = True
    gradient_bucket_bytes: PositiveInt = 64 * 2 ** 20
    cuda_graphs: bool = False
    deterministic: bool = True
    # GradCache: device bytes that first-pass chunk graphs may keep so their
    # replay forward is skipped (exact same gradient). None = size from free
    # HBM at run time; 0 = always replay.
    grad_cache_retain_bytes: NonNegativeInt | None = None


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
    def validate_loss_execution(self):
        if self.grad_cache is not None and self.mega_batch_mining is not None:
            raise ValueError("configure only one specialized loss execution")
        return self

    @model_validator(mode="after")
    def validate_sharding_axes(self):
        mesh_axes = set(self.mesh.axis_names)
        s = self.sharding
        if isinstance(s, DDPConfig):
            referenced = {s.axis}
        elif isinstance(s, FSDPConfig):
            referenced = {s.data_axis, s.resolved_parameter_axis}
        elif isinstance(s, TensorParallelConfig):
            referenced = {s.data_axis, s.model_axis}
        else:
            referenced = set(s.parameter_axes)
            if s.data_axis is not None:
                referenced.add(s.data_axis)
            rule_axes = {n for r in s.parameter_rules for a in r.axes if a is not None
                         for n in (a if isinstance(a, tuple) else (a,))}
            default_axes = {n for a in s.default_parameter_axes if a is not None
                            for n in (a if isinstance(a, tuple) else (a,))}
            unsupported = (rule_axes | default_axes) - set(s.parameter_axes)
            if unsupported:
                raise ValueError(f"partition rules use axes absent from parameter_axes: {sorted(unsupported)}")
        unknown = referenced - mesh_axes
        if unknown:
            raise ValueError(f"sharding axes are absent from the mesh: {sorted(unknown)}")
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
    def validate_iterations(self):
        if len(set(self.additional_iterations)) != len(self.additional_iterations):
            raise ValueError("additional checkpoint iterations must be unique")
        return self

    def should_save(self, iteration: int, *, final: bool) -> bool:
        return iteration % self.every == 0 or iteration in self.additional_iterations or (final and self.save_final)


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

    @field_validator("task", mode="before")
    @classmethod
    def validate_registered_task(cls, value: object, info: ValidationInfo) -> TaskConfig:
        from .tasks.registry import BUILTIN_TASKS, TaskRegistry

        registry = None if info.context is None else info.context.get("task_registry")
        registry = BUILTIN_TASKS if registry is None else registry
        if not isinstance(registry, TaskRegistry):
            raise TypeError("task_registry validation context must be a TaskRegistry")
        return registry.parse(value)

    @field_validator("loss", mode="before")
    @classmethod
    def validate_registered_loss(cls, value: object, info: ValidationInfo) -> LossConfig:
        from .tasks.registry import BUILTIN_LOSSES, LossRegistry

        registry = None if info.context is None else info.context.get("loss_registry")
        registry = BUILTIN_LOSSES if registry is None else registry
        if not isinstance(registry, LossRegistry):
            raise TypeError("loss_registry validation context must be a LossRegistry")
        return registry.parse(value)

    @field_validator("loss_modifiers", mode="before")
    @classmethod
    def validate_registered_loss_modifiers(cls, value: object, info: ValidationInfo):
        from .tasks.registry import BUILTIN_LOSS_MODIFIERS, LossModifierRegistry

        registry = None if info.context is None else info.context.get("modifier_registry")
        registry = BUILTIN_LOSS_MODIFIERS if registry is None else registry
        if not isinstance(registry, LossModifierRegistry):
            raise TypeError("modifier_registry validation context must be a LossModifierRegistry")
        if not isinstance(value, (list, tuple)):
            raise TypeError("loss_modifiers must be a list or tuple")
        parsed = tuple(registry.parse(m) for m in value)
        kinds = tuple(m.kind for m in parsed)
        if len(set(kinds)) != len(kinds):
            raise ValueError("loss modifier kinds must be unique")
        if len(parsed) > 1 and any(k in {"matryoshka", "adaptive_layer", "matryoshka_2d"} for k in kinds):
            raise ValueError("dimension/layer modifiers are mutually exclusive; use matryoshka_2d for their "
                             "joint objective")
        return parsed

    @model_validator(mode="after")
    def validate_loss_capabilities(self, info: ValidationInfo):
        from .tasks.registry import BUILTIN_LOSS_MODIFIERS, BUILTIN_LOSSES

        losses = (info.context or {}).get("loss_registry") or BUILTIN_LOSSES
        definition = losses.definition(self.loss.kind)
        if self.task.kind not in definition.task_kinds:
            raise ValueError(f"loss {self.loss.kind!r} does not support task {self.task.kind!r}")
        strategy = self.training_strategy
        if strategy not in definition.training_strategies:
            raise ValueError(f"loss {self.loss.kind!r} does not support training strategy {strategy!r}")
        steps = self.training.batch.gradient_accumulation_steps
        if steps > 1:
            if strategy != "direct":
                raise ValueError("gradient accumulation composes only with direct execution; GradCache and "
                                 "mega-batch execution already own their logical batch decomposition")
            if not definition.microbatch_accumulation:
                raise ValueError(f"loss {self.loss.kind!r} does not decompose exactly across "
                                 "gradient-accumulation microbatches")
        modifiers = (info.context or {}).get("modifier_registry") or BUILTIN_LOSS_MODIFIERS
        for modifier in self.loss_modifiers:
            md = modifiers.definition(modifier.kind)
            if strategy not in md.training_strategies:
                raise ValueError(f"loss modifier {modifier.kind!r} does not support training strategy "
                                 f"{strategy!r}")
            if steps > 1 and not md.microbatch_accumulation:
                raise ValueError(f"loss modifier {modifier.kind!r} does not decompose exactly across "
                                 "gradient-accumulation microbatches")
        return self

    @model_validator(mode="after")
    def validate_checkpoint_schedule(self):
        if self.checkpointing is not None and any(
                i > self.training.max_steps for i in self.checkpointing.additional_iterations):
            raise ValueError("additional checkpoint iterations cannot exceed training.max_steps")
        if self.evaluation is not None and self.evaluation.save_best and self.checkpointing is None:
            raise ValueError("best-model selection requires checkpointing")
        if (self.export.enabled and self.export.selection == "best"
                and (self.evaluation is None or not self.evaluation.save_best)):
            raise ValueError("best-model export requires evaluation.save_best")
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
    "B200ExecutionConfig", "BatchConfig", "CheckpointConfig", "ComponentConfig", "CustomShardingConfig", "DDPConfig",
    "DataConfig", "EmbeddingSimilarityEvaluatorConfig", "EvaluationConfig", "EvaluatorConfig", "ExportConfig",
    "FSDPConfig", "GradCacheConfig", "HuggingFaceExportConfig", "InformationRetrievalEvaluatorConfig", "JobConfig",
    "LoggingConfig", "MegaBatchMiningConfig", "MeshConfig", "ModelConfig", "OptimizationConfig", "ParameterRole",
    "PartitionAxis", "PartitionRuleConfig", "PrecisionConfig", "QuantizedLoRAConfig", "RematerializationPolicy",
    "ShardingConfig", "TensorParallelConfig", "TrainingConfig",
]
