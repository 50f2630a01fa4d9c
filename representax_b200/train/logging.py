"""Durable run logging: ``run.json``, ``events.jsonl``, ``metrics.jsonl``.

Parity: ``RunLogger``, ``Reporter`` and ``MetricRecord`` of
src/representax/train/logging.py:54-439 — the same file names and schema
versions (``representax-run-v1`` / ``-event-v1`` / ``-metrics-v1``), an
append-only JSONL source of truth written by one worker thread behind a
bounded queue (device tensors are read on that thread, so the training loop
never blocks on them), reporter fan-out, a ``cursor()`` of byte offsets taken
after draining and fsyncing, and truncation to a checkpoint's cursor on
resume so the logs match the restored state exactly.
"""

from __future__ import annotations

import datetime as _dt
import json
import os
import queue
import threading
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Protocol

import torch

RUN_SCHEMA = "representax-run-v1"
EVENT_SCHEMA = "representax-event-v1"
METRICS_SCHEMA = "representax-metrics-v1"


def _timestamp() -> str:
    return _dt.datetime.now(_dt.timezone.utc).isoformat()


def _json_value(value: Any) -> Any:
    if isinstance(value, torch.Tensor):
        value = value.detach()
        if value.numel() == 1:
            return value.item()
        return value.cpu().tolist()
    if isinstance(value, Mapping):
        return {str(k): _json_value(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_json_value(v) for v in value]
    if isinstance(value, float) and (value != value or value in (float("inf"), float("-inf"))):
        return str(value)
    return value


def _atomic_write_json(path: Path, document: Mapping[str, Any]) -> None:
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "w", encoding="utf-8") as handle:
        json.dump(document, handle, indent=2, sort_keys=True, default=str)
        handle.write("\n")
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, path)


@dataclass(frozen=True)
class MetricRecord:
    """One published metrics row (host values)."""

    namespace: str
    iteration: int
    optimizer_step: int
    values: Mapping[str, Any]
    sequence: int = 0
    time: str = field(default_factory=_timestamp)


class Reporter(Protocol):
    def report(self, record: MetricRecord) -> None: ...

    def close(self) -> None: ...


class _Item:
    __slots__ = ("kind", "payload", "done")

    def __init__(self, kind: str, payload: Any = None) -> None:
        self.kind = kind
        self.payload = payload
        self.done = threading.Event()


class RunLogger:
    def __init__(self, run_directory: str | Path, *, manifest: Mapping[str, Any],
                 reporters: Sequence[Reporter] = (), resume_cursor: Mapping[str, int] | None = None,
                 queue_size: int = 16, initial_optimizer_step: int = 0, console: bool = False) -> None:
        if queue_size <= 0:
            raise ValueError("reporter queue_size must be positive")
        self.run_directory = Path(run_directory).expanduser().resolve()
        self._events_path = self.run_directory / "events.jsonl"
        self._metrics_path = self.run_directory / "metrics.jsonl"
        self._reporters = tuple(reporters)
        self._queue: queue.Queue[_Item] = queue.Queue(maxsize=queue_size)
        self._error: BaseException | None = None
        self._closed = False
        self._console = console
        self._optimizer_step = initial_optimizer_step
        if resume_cursor is None:
            self.run_directory.mkdir(parents=True, exist_ok=False)
            self._events = open(self._events_path, "x", encoding="utf-8", buffering=1)
            self._metrics = open(self._metrics_path, "x", encoding="utf-8", buffering=1)
            self._sequence = 0
            self._manifest = {**_json_value(manifest), "schema_version": RUN_SCHEMA, "kind": "train",
                              "status": "running", "started_at": _timestamp()}
        else:
            self._manifest = self._resume(manifest, resume_cursor)
        _atomic_write_json(self.run_directory / "run.json", self._manifest)
        self._worker = threading.Thread(target=self._run, name="representax-reporter", daemon=True)
        self._worker.start()

    # ------------------------------------------------------------------ resume
    def _resume(self, manifest: Mapping[str, Any], cursor: Mapping[str, int]) -> dict[str, Any]:
        run_path = self.run_directory / "run.json"
        if not run_path.is_file():
            raise FileNotFoundError(f"run manifest is missing: {run_path}")
        previous = json.loads(run_path.read_text())
        if previous.get("schema_version") != RUN_SCHEMA or previous.get("kind") != "train":
            raise ValueError(f"run manifest is incompatible: {run_path}")
        normalized = _json_value(manifest)
        for name in ("scientific", "scientific_fingerprint", "data_contract", "data_fingerprint"):
            if previous.get(name) != normalized.get(name):
                raise ValueError(f"resumed run {name} differs")
        required = {"events_bytes", "metrics_bytes", "optimizer_step", "sequence"}
        if set(cursor) != required:
            raise ValueError(f"logging cursor keys differ; expected={sorted(required)}, actual={sorted(cursor)}")
        pos = {k: int(v) for k, v in cursor.items()}
        if any(v < 0 for v in pos.values()):
            raise ValueError("logging cursor values must be non-negative")
        if pos["optimizer_step"] != self._optimizer_step:
            raise ValueError("logging cursor optimizer_step differs from restored training state")
        self._truncate(self._events_path, pos["events_bytes"])
        self._truncate(self._metrics_path, pos["metrics_bytes"])
        self._events = open(self._events_path, "a", encoding="utf-8", buffering=1)
        self._metrics = open(self._metrics_path, "a", encoding="utf-8", buffering=1)
        self._sequence = pos["sequence"]
        terminal = {"checkpoint", "completed_iterations", "config", "error", "error_type", "execution",
                    "finished_at", "optimizer_steps", "runtime", "scientific"}
        active = {k: v for k, v in previous.items() if k not in terminal}
        return {**active, "config": normalized.get("config"), "execution": normalized.get("execution"),
                "scientific": normalized.get("scientific"), "status": "running", "resumed_at": _timestamp(),
                "resume_count": int(previous.get("resume_count", 0)) + 1}

    @staticmethod
    def _truncate(path: Path, position: int) -> None:
        if not path.is_file():
            raise FileNotFoundError(f"append-only run log is missing: {path}")
        size = path.stat().st_size
        if position > size:
            raise ValueError(f"log cursor {position} is beyond the end of {path} ({size} bytes)")
        with open(path, "r+b") as handle:
            handle.truncate(position)
            handle.flush()
            os.fsync(handle.fileno())

    # ------------------------------------------------------------------ worker
    def _run(self) -> None:
        while True:
            item = self._queue.get()
            try:
                if item.kind == "stop":
                    item.done.set()
                    return
                if self._error is None:
                    self._handle(item)
            except BaseException as error:  # surfaced on the training thread
                self._error = error
            finally:
                item.done.set()

    def _handle(self, item: _Item) -> None:
        if item.kind == "event":
            self._events.write(json.dumps(item.payload, sort_keys=True, default=str) + "\n")
        elif item.kind == "metrics":
            namespace, iteration, step, values = item.payload
            host = _json_value(values)
            self._sequence += 1
            row = {"schema_version": METRICS_SCHEMA, "namespace": namespace, "iteration": iteration,
                   "optimizer_step": _json_value(step), "sequence": self._sequence, "time": _timestamp(),
                   "values": host}
            self._metrics.write(json.dumps(row, sort_keys=True, default=str) + "\n")
            record = MetricRecord(namespace, iteration, int(row["optimizer_step"]), host, self._sequence)
            for reporter in self._reporters:
                reporter.report(record)
            if self._console:
                shown = " ".join(f"{k}={v:.5g}" if isinstance(v, float) else f"{k}={v}" for k, v in host.items())
                print(f"[{namespace}] iter {iteration} step {row['optimizer_step']} {shown}", flush=True)
        elif item.kind == "flush":
            for handle in (self._events, self._metrics):
                handle.flush()
                os.fsync(handle.fileno())

    def _put(self, item: _Item) -> _Item:
        if self._closed:
            raise RuntimeError("run logger is closed")
        self.raise_if_failed()
        self._queue.put(item)
        return item

    def raise_if_failed(self) -> None:
        if self._error is not None:
            raise RuntimeError(f"run logger worker failed: {self._error}") from self._error

    # ------------------------------------------------------------------ API
    def event(self, name: str, **fields: Any) -> None:
        self._put(_Item("event", {"schema_version": EVENT_SCHEMA, "event": name, "time": _timestamp(),
                                  **_json_value(fields)}))

    def metrics(self, namespace: str, iteration: int, values: Mapping[str, Any], *,
                optimizer_step: Any = None) -> None:
        if namespace not in {"train", "valid", "perf"}:
            raise ValueError("metric namespace must be train, valid or perf")
        self._put(_Item("metrics", (namespace, iteration,
                                    self._optimizer_step if optimizer_step is None else optimizer_step,
                                    dict(values))))

    def set_optimizer_step(self, step: int) -> None:
        self._optimizer_step = int(step)

    def cursor(self) -> dict[str, int]:
        """Drain, fsync and return byte offsets that a checkpoint can restore."""

        item = self._put(_Item("flush"))
        item.done.wait()
        self.raise_if_failed()
        return {"events_bytes": self._events_path.stat().st_size,
                "metrics_bytes": self._metrics_path.stat().st_size,
                "optimizer_step": int(self._optimizer_step), "sequence": int(self._sequence)}

    def close(self, *, status: str = "completed", **fields: Any) -> None:
        if self._closed:
            return
        stop = _Item("stop")
        try:
            flush = self._put(_Item("flush"))
            flush.done.wait()
        finally:
            self._closed = True
            self._queue.put(stop)
            self._worker.join()
            self._events.close()
            self._metrics.close()
            for reporter in self._reporters:
                reporter.close()
        self._manifest.update({"status": status, "finished_at": _timestamp(), **_json_value(fields)})
        _atomic_write_json(self.run_directory / "run.json", self._manifest)
        self.raise_if_failed()


__all__ = ["EVENT_SCHEMA", "METRICS_SCHEMA", "MetricRecord", "RUN_SCHEMA", "Reporter", "RunLogger"]
