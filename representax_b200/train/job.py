"""Configured training jobs: from a ``JobConfig`` to a trained, exported model.

Parity: ``resolve_target``, ``build_component``, ``load_model``,
``prepare_model``, ``build_collate``, ``build_batches``,
``build_job_runtime`` and ``run_job`` of src/representax/train/job.py:43-410.
Dotted targets written for the reference (``representax.…``, ``optax.…``)
resolve to their counterparts here, so job files port unchanged.
"""

from __future__ import annotations

import inspect
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from functools import partial
from importlib import import_module
from pathlib import Path
from typing import Any

import torch

from representax_b200.config import JobConfig
from representax_b200.parallel.dist import LOCAL, DistContext, StoreBarrier
from representax_b200.precision import resolve_precision_policy

from .checkpoint import CheckpointManager, scientific_fingerprint
from .execution import Direct, GradCache
from .logging import RunLogger
from .loop import TrainingResult, run_training
from .optimizer import build_optimizer
from .step import TrainStep, init_train_state

_ALIASES = {"representax.": "representax_b200."}


def resolve_target(target: str) -> Callable[..., Any]:
    """Resolve one trusted dotted Python target from a serialized recipe."""

    for old, new in _ALIASES.items():
        if target.startswith(old) and not target.startswith(new):
            target = new + target[len(old):]
    module_name, sep, attribute_path = target.partition(":")
    if not sep:
        module_name, sep, attribute_path = target.rpartition(".")
    if not sep or not module_name or not attribute_path:
        raise ValueError(f"component target must be a dotted import path: {target!r}")
    # Walk back until an importable module is found (supports Class.method targets).
    parts = (module_name + "." + attribute_path).split(".")
    for cut in range(len(parts) - 1, 0, -1):
        try:
            value: Any = import_module(".".join(parts[:cut]))
        except ModuleNotFoundError:
            continue
        try:
            for attribute in parts[cut:]:
                value = getattr(value, attribute)
        except AttributeError:
            continue
        if not callable(value):
            raise TypeError(f"component target {target!r} is not callable")
        return value
    raise ImportError(f"could not resolve component target {target!r}")


def build_component(config: Any) -> Any:
    return resolve_target(config.target)(**config.parameters)


def load_model(job_or_config: Any, *, seed: int | None = None) -> torch.nn.Module:
    """Instantiate the configured model (and attach its processor when one is returned)."""

    config = job_or_config.model if isinstance(job_or_config, JobConfig) else job_or_config
    if seed is None and isinstance(job_or_config, JobConfig):
        seed = job_or_config.training.seed
    factory = resolve_target(config.target)
    params = dict(config.parameters)
    sig = inspect.signature(factory)
    if "seed" in sig.parameters and "seed" not in params and seed is not None:
        params["seed"] = seed
    result = factory(**params)
    processor = None
    if isinstance(result, tuple) and len(result) == 2:
        result, processor = result
    if not isinstance(result, torch.nn.Module):
        raise TypeError(f"model target {config.target!r} must return a torch.nn.Module")
    result.processor = processor
    return result


def prepare_model(model: torch.nn.Module, job: JobConfig | None = None, *, adapter: Any = None,
                  seed: int = 0) -> torch.nn.Module:
    """Apply the job's INT4 + LoRA adapter recipe (freezing the base) when configured."""

    adapter = adapter if adapter is not None else (job.training.adapter if job is not None else None)
    if adapter is None:
        return model
    from representax_b200.models.adapters import apply_quantized_lora

    return apply_quantized_lora(model, rank=adapter.rank, alpha=adapter.alpha, seed=seed,
                                target_pattern=adapter.target_pattern,
                                initialization_scale=adapter.initialization_scale)


def build_collate(config: Any, *, processor: Any = None) -> Callable | None:
    if config.collate is None:
        return None
    collate = resolve_target(config.collate.target)
    params = dict(config.collate.parameters)
    try:
        accepts_processor = "processor" in inspect.signature(collate).parameters
    except (TypeError, ValueError):
        accepts_processor = False
    if processor is not None and accepts_processor and "processor" not in params:
        params["processor"] = processor
    if inspect.isclass(collate):
        return collate(**params)
    return partial(collate, **params) if params else collate


def build_batches(config: Any, *, batch_size: int, processor: Any = None, resolvers=None, mappers=None,
                  shard: tuple[int, int] = (0, 1), num_batches: int | None = None):
    from representax_b200.data import build_data_loader

    return build_data_loader(config.distribution, batch_size=batch_size,
                             collate=build_collate(config, processor=processor),
                             drop_remainder=config.drop_remainder, num_threads=max(1, config.num_threads),
                             prefetch=max(1, config.prefetch_buffer_size), num_batches=num_batches, shard=shard,
                             host_memory_budget_bytes=config.host_memory_budget_bytes, resolvers=resolvers,
                             mappers=mappers)


def build_execution(training: Any):
    if training.grad_cache is not None:
        g = training.grad_cache
        return GradCache(query_chunk_size=g.resolved_query_micro_batch_size,
                         document_chunk_size=g.resolved_document_micro_batch_size,
                         loss_row_chunk_size=g.resolved_loss_row_chunk_size,
                         fused=training.b200.fused_mnr_collectives,
                         retain_bytes=training.b200.grad_cache_retain_bytes)
    if training.mega_batch_mining is not None:
        from .mega_batch import MegaBatchMining

        m = training.mega_batch_mining
        return MegaBatchMining(micro_batch_size=m.micro_batch_size, loss_row_chunk_size=m.resolved_loss_row_chunk_size)
    return Direct()


@dataclass
class JobRuntime:
    state: Any
    step: TrainStep
    batches: Any
    model: torch.nn.Module
    task: Any
    device: torch.device
    evaluate: Callable[[int], dict[str, float]] | None = None


def build_job_runtime(job: JobConfig, *, device: torch.device | str | None = None, resolvers=None, mappers=None,
                      dist: DistContext = LOCAL) -> JobRuntime:
    from representax_b200.tasks.registry import build_task

    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    torch.manual_seed(job.training.seed)
    if job.training.b200.deterministic:
        # Bitwise-reproducible PyTorch ops (the CPU reference path). The native
        # kernels reduce some gradients with atomics and are reproducible only
        # to rounding.
        torch.use_deterministic_algorithms(True, warn_only=True)
    model = load_model(job)
    model = prepare_model(model, job, seed=job.training.seed)
    task = build_task(job.task, job.loss, job.loss_modifiers)
    precision = resolve_precision_policy(job.training.precision)
    if hasattr(model, "compute_dtype"):
        model.compute_dtype = precision.compute_dtype
    from representax_b200.parallel.sharding import plan_from_config

    plan = plan_from_config(job.training.sharding, model, dist.world_size)
    cuda = torch.device(device).type == "cuda"
    state = init_train_state(model, device=device, precision=precision, dist=dist,
                             sharded_optimizer=plan.sharded_optimizer,
                             fsdp=plan.shards_parameters and cuda and precision.compute_dtype != torch.float32)
    optimizer = build_optimizer(job.optimization)
    execution = build_execution(job.training)
    if job.training.global_batch_size % dist.world_size:
        raise ValueError("global batch size must divide evenly over data-parallel ranks")
    step = TrainStep(state, task, optimizer=optimizer, precision=precision, execution=execution,
                     max_gradient_norm=job.optimization.max_gradient_norm, seed=job.training.seed,
                     accumulation_steps=job.training.batch.gradient_accumulation_steps, dist=dist)
    batches = build_batches(job.data, batch_size=job.training.global_batch_size,
                            processor=getattr(model, "processor", None), resolvers=resolvers, mappers=mappers,
                            shard=(dist.rank, dist.world_size))
    evaluate = None
    if job.evaluation is not None:
        from .evaluation import EvaluationRunner

        runner = EvaluationRunner(job.evaluation, model=model, task=task, precision=precision, device=device,
                                  resolvers=resolvers, mappers=mappers)
        evaluate = runner
    return JobRuntime(state=state, step=step, batches=batches, model=model, task=task, device=device,
                      evaluate=evaluate)


def run_job(job: JobConfig, run_directory: str | Path, *, resume: bool = False, resolvers=None, mappers=None,
            device: torch.device | str | None = None, dist: DistContext = LOCAL, console: bool = False):
    """Train one configured job and publish its inference bundle."""

    from representax_b200.export import export_inference_bundle

    run_directory = Path(run_directory)
    runtime = build_job_runtime(job, device=device, resolvers=resolvers, mappers=mappers, dist=dist)
    iterator = iter(runtime.batches)
    sci = scientific_fingerprint(job)
    data_fp = runtime.batches.data_fingerprint
    manifest = {"name": job.name, "config": job.model_dump(mode="json"), "scientific_fingerprint": sci,
                "scientific": job.parameters("scientific"), "execution": job.parameters("execution"),
                "data_contract": runtime.batches.data_contract, "data_fingerprint": data_fp}
    checkpoints = None
    resume_cursor = None
    initial_step = 0
    if job.checkpointing is not None:
        checkpoints = CheckpointManager(run_directory / "checkpoints", keep=job.checkpointing.keep,
                                        asynchronous=job.checkpointing.asynchronous, scientific=sci, data=data_fp,
                                        rank=dist.rank, world_size=dist.world_size,
                                        metric_mode=job.evaluation.primary_metric_mode if job.evaluation else "min",
                                        barrier=StoreBarrier.from_default_group(dist))
        if resume:
            record = checkpoints.latest()
            if record is not None:
                _, progress = checkpoints.restore(record)
                resume_cursor = progress.get("logging_cursor")
                initial_step = int(progress.get("optimizer_step", 0))
    logger = None
    if dist.rank == 0:
        logger = RunLogger(run_directory, manifest=manifest, resume_cursor=resume_cursor,
                           queue_size=job.logging.reporter_queue_size, initial_optimizer_step=initial_step,
                           console=console)
    try:
        result: TrainingResult = run_training(
            runtime.step, iterator, max_steps=job.training.max_steps, device=runtime.device, logger=logger,
            checkpoints=checkpoints, checkpoint_config=job.checkpointing, evaluate=runtime.evaluate,
            evaluation_config=job.evaluation, resume=resume, seed=job.training.seed,
            heartbeat_seconds=job.data.data_wait_heartbeat_seconds,
            timeout_seconds=job.data.data_wait_timeout_seconds)
        bundle = None
        if job.export.enabled and getattr(runtime.state.store, "fsdp", None) is not None:
            runtime.state.store.unshard()  # collective: every rank takes part
        if job.export.enabled and dist.rank == 0:
            if job.export.selection == "best" and checkpoints is not None and checkpoints.best() is not None:
                from .checkpoint import load_training_tensors

                tensors, _ = checkpoints.restore(checkpoints.best(), device=runtime.device)
                load_training_tensors(runtime.state, tensors)
            bundle = export_inference_bundle(runtime.model, job, run_directory / job.export.directory_name,
                                             iteration=result.completed_iterations)
        if logger is not None:
            logger.close(status="completed", completed_iterations=result.completed_iterations,
                         optimizer_steps=result.optimizer_steps)
        return result, bundle
    except BaseException as error:
        if logger is not None:
            logger.close(status="failed", error=str(error), error_type=type(error).__name__)
        raise


__all__ = ["JobRuntime", "build_batches", "build_collate", "build_component", "build_execution",
           "build_job_runtime", "load_model", "prepare_model", "resolve_target", "run_job"]
