"""Host training loop.

Parity: ``run_training`` and ``DataStarvationError`` of
src/representax/train/loop.py:32-747: data-wait heartbeat and fatal
deadline, per-batch telemetry, host->device placement, per-iteration random
streams, one-step-delayed metric publication (the device keeps running while
the previous step's scalars are read), evaluation and checkpoint cadence with
best-model tracking, exact resume (state, data cursor, logging cursor), and a
failure path that records ``training_failed`` and closes every resource.

The heartbeat is a watchdog thread (no SIGALRM, so the loop also works off
the main thread): while ``next(iterator)`` blocks it emits
``data_wait_heartbeat`` events, and past the deadline it marks the wait as
starved; the loop raises :class:`DataStarvationError` as soon as the batch
arrives or the deadline passes.
"""

from __future__ import annotations

import math
import threading
import time
from collections.abc import Callable, Iterator
from dataclasses import dataclass
from typing import Any

import torch

from representax_b200.tasks._batch import to_device

from .checkpoint import CheckpointManager, load_training_tensors, training_tensors
from .logging import RunLogger


class DataStarvationError(RuntimeError):
    """The data pipeline did not produce a batch within the configured deadline."""


class _DataWatchdog:
    def __init__(self, logger: RunLogger | None, heartbeat: float | None, timeout: float | None) -> None:
        self.logger = logger
        self.heartbeat = heartbeat
        self.timeout = timeout

    def next(self, iterator: Iterator, iteration: int):
        if self.heartbeat is None and self.timeout is None:
            return next(iterator)
        result: dict[str, Any] = {}
        done = threading.Event()

        def fetch():
            try:
                result["batch"] = next(iterator)
            except BaseException as error:
                result["error"] = error
            finally:
                done.set()

        worker = threading.Thread(target=fetch, name="rx-data-wait", daemon=True)
        started = time.perf_counter()
        worker.start()
        beat = self.heartbeat or self.timeout
        while not done.wait(timeout=beat):
            waited = time.perf_counter() - started
            if self.timeout is not None and waited >= self.timeout:
                if self.logger is not None:
                    self.logger.event("data_starvation", iteration=iteration, waited_seconds=waited)
                raise DataStarvationError(f"no batch for iteration {iteration} after {waited:.1f}s")
            if self.logger is not None and self.heartbeat is not None:
                self.logger.event("data_wait_heartbeat", iteration=iteration, waited_seconds=waited)
        if "error" in result:
            raise result["error"]
        return result["batch"]


@dataclass
class TrainingResult:
    completed_iterations: int
    optimizer_steps: int
    best_metric: float | None
    last_metrics: dict[str, Any]


def run_training(step: Callable[[Any, int], Any], iterator: Iterator, *, max_steps: int, device: torch.device,
                 logger: RunLogger | None = None, checkpoints: CheckpointManager | None = None,
                 checkpoint_config: Any = None, evaluate: Callable[[int], dict[str, float]] | None = None,
                 evaluation_config: Any = None, resume: bool = False, heartbeat_seconds: float | None = None,
                 timeout_seconds: float | None = None, seed: int = 0) -> TrainingResult:
    """Drive ``step(batch, iteration)`` for ``max_steps`` iterations."""

    state = getattr(step, "state", None)
    start = 0
    best: float | None = None
    mode = getattr(evaluation_config, "primary_metric_mode", "min")
    primary = getattr(evaluation_config, "primary_metric", "valid/loss")
    if resume and checkpoints is not None:
        record = checkpoints.latest()
        if record is not None:
            tensors, progress = checkpoints.restore(record, device=device)
            load_training_tensors(state, tensors)
            start = int(progress["iteration"])
            if hasattr(iterator, "set_state") and "data_state" in progress:
                iterator.set_state(progress["data_state"])
            best = progress.get("best_metric")
            if logger is not None:
                logger.event("training_resumed", iteration=start)
    watchdog = _DataWatchdog(logger, heartbeat_seconds, timeout_seconds)
    pending = None  # (iteration, metrics) published one step late
    last: dict[str, Any] = {}

    def publish(item):
        nonlocal last
        if item is None or logger is None:
            return
        it, metrics = item
        values = metrics.to_host()
        last = values
        logger.set_optimizer_step(values["optimizer_step"])
        logger.metrics("train", it, {k: v for k, v in values.items() if k != "optimizer_step"},
                       optimizer_step=values["optimizer_step"])
        if not values["finite"]:
            logger.event("nonfinite_update_skipped", iteration=it)

    def save(iteration: int, final: bool, metric: float | None = None, is_best: bool = False):
        if checkpoints is None or checkpoint_config is None:
            return
        if not (checkpoint_config.should_save(iteration, final=final) or is_best):
            return
        cursor = logger.cursor() if logger is not None else {}
        progress = {"iteration": iteration, "optimizer_step": int(state.scalars[2].item()),
                    "data_state": iterator.get_state() if hasattr(iterator, "get_state") else {},
                    "logging_cursor": cursor, "seed": seed, "best_metric": best}
        checkpoints.save(iteration, training_tensors(state), progress, metric=metric, best=is_best)
        if logger is not None:
            logger.event("checkpoint_saved", iteration=iteration)

    try:
        if evaluate is not None and getattr(evaluation_config, "on_start", False) and start == 0:
            values = evaluate(0)
            if logger is not None:
                logger.metrics("valid", 0, values)
        for iteration in range(start, max_steps):
            t0 = time.perf_counter()
            batch = watchdog.next(iterator, iteration)
            telemetry = getattr(iterator, "last_telemetry", None)
            t1 = time.perf_counter()
            placed = to_device(batch, device)
            t2 = time.perf_counter()
            metrics = step(placed, iteration)
            t3 = time.perf_counter()
            publish(pending)
            pending = (iteration, metrics)
            if logger is not None:
                perf = {"data_wait_seconds": t1 - t0, "placement_seconds": t2 - t1, "dispatch_seconds": t3 - t2}
                if telemetry is not None:
                    perf["preprocess_seconds"] = telemetry.preprocess_seconds
                    perf["host_batch_bytes"] = telemetry.host_batch_bytes
                    perf["prefetch_ready_batches"] = telemetry.prefetch_ready_batches
                logger.metrics("perf", iteration, perf)
            done = iteration + 1
            is_eval = evaluate is not None and evaluation_config is not None and (
                (evaluation_config.every_steps and done % evaluation_config.every_steps == 0)
                or (done == max_steps and evaluation_config.on_end))
            metric, is_best = None, False
            if is_eval:
                publish(pending)
                pending = None
                values = evaluate(done)
                if logger is not None:
                    logger.metrics("valid", done, values)
                metric = values.get(primary.split("/", 1)[-1], values.get(primary))
                if metric is not None and math.isfinite(metric):
                    better = best is None or (metric < best if mode == "min" else metric > best)
                    if better and getattr(evaluation_config, "save_best", False):
                        best, is_best = metric, True
            if checkpoints is not None and checkpoint_config is not None and (
                    checkpoint_config.should_save(done, final=done == max_steps) or is_best):
                publish(pending)
                pending = None
                save(done, final=done == max_steps, metric=metric, is_best=is_best)
        publish(pending)
        if checkpoints is not None:
            checkpoints.wait()
        if logger is not None:
            logger.event("training_completed", iterations=max_steps)
        steps = int(state.scalars[2].item()) if state is not None else max_steps
        return TrainingResult(max_steps, steps, best, last)
    except BaseException as error:
        if logger is not None:
            try:
                logger.event("training_failed", error=str(error), error_type=type(error).__name__)
            except Exception:
                pass
        raise
    finally:
        close = getattr(iterator, "close", None)
        if close is not None:
            close()


__all__ = ["DataStarvationError", "TrainingResult", "run_training"]
