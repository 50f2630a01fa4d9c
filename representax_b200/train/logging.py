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

import contextlib
import datetime as _dt
import json
import math
import os
import queue
import tempfile
import threading
from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Any, Protocol

import torch

RUN_SCHEMA = "representax-run-v1"
EVENT_SCHEMA = "representax-event-v1"
METRICS_SCHEMA = "representax-metrics-v1"
_NAMESPACES = frozenset({"train", "valid", "perf"})


def _timestamp() -> str:
    return _dt.datetime.now(_dt.timezone.utc).isoformat()


def _json_value(value: Any) -> Any:
    """Host JSON form of a metric value: tensors read out, non-finite floats as strings."""

    if isinstance(value, torch.Tensor):
        host = value.detach().cpu()
        return host.item() if host.numel() == 1 else host.tolist()
    if isinstance(value, Mapping):
        return {str(key): _json_value(item) for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        return list(map(_json_value, value))
    if isinstance(value, float) and not math.isfinite(value):
        return repr(value)  # 'nan', 'inf', '-inf'
    return value


def _atomic_write_json(path: Path, document: Mapping[str, Any]) -> None:
    """Replace ``path`` by a fully written, fsynced JSON file (readers never see half a file)."""

    fd, scratch = tempfile.mkstemp(prefix=f".{path.name}.", dir=path.parent)
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as handle:
            handle.write(json.dumps(document, indent=2, sort_keys=True, default=str) + "\n")
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(scratch, path)
    except BaseException:
        with contextlib.suppress(FileNotFoundError):
            os.unlink(scratch)
        raise


@dataclass(frozen=True)
class LogCursor:
    """Where a checkpoint's view of the run logs ends."""

    events_bytes: int
    metrics_bytes: int
    optimizer_step: int
    sequence: int

    @classmethod
    def parse(cls, values: Mapping[str, int]) -> "LogCursor":
        names = [f.name for f in fields(cls)]
        if sorted(values) != sorted(names):
            raise ValueError(f"log cursor has keys {sorted(values)}; a cursor has exactly {sorted(names)}")
        parsed = cls(**{name: int(values[name]) for name in names})
        negative = [name for name in names if getattr(parsed, name) < 0]
        if negative:
            raise ValueError(f"log cursor fields {negative} are negative")
        return parsed


def _cut_log(path: Path, length: int) -> None:
    """Drop everything after byte ``length`` of an append-only log (resume to a checkpoint)."""

    try:
        size = path.stat().st_size
    except FileNotFoundError:
        raise FileNotFoundError(f"cannot resume: the run log {path} is gone") from None
    if length > size:
        raise ValueError(f"cannot resume: checkpoint expects {length} bytes of {path.name}, the file has {size}")
    with open(path, "r+b") as handle:
        handle.truncate(length)
        os.fsync(handle.fileno())


_RESUME_MUST_MATCH = ("scientific", "scientific_fingerprint", "data_contract", "data_fingerprint")
_DROPPED_ON_RESUME = frozenset({"checkpoint", "completed_iterations", "config", "error", "error_type", "execution",
                                "finished_at", "optimizer_steps", "runtime", "scientific"})


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
        if not queue_size >= 1:
            raise ValueError(f"queue_size {queue_size} leaves no room for a single report")
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
        try:
            previous = json.loads((self.run_directory / "run.json").read_text())
        except FileNotFoundError:
            raise FileNotFoundError(f"cannot resume: {self.run_directory} has no run.json") from None
        if (previous.get("schema_version"), previous.get("kind")) != (RUN_SCHEMA, "train"):
            raise ValueError(f"cannot resume: {self.run_directory}/run.json is not a {RUN_SCHEMA} training run")
        incoming = _json_value(manifest)
        changed = [key for key in _RESUME_MUST_MATCH if previous.get(key) != incoming.get(key)]
        if changed:
            raise ValueError(f"cannot resume: the job changed {changed} since the run started")
        position = LogCursor.parse(cursor)
        if position.optimizer_step != self._optimizer_step:
            raise ValueError(f"cannot resume: logs end at optimizer step {position.optimizer_step} but the "
                             f"restored state is at step {self._optimizer_step}")
        _cut_log(self._events_path, position.events_bytes)
        _cut_log(self._metrics_path, position.metrics_bytes)
        self._events = open(self._events_path, "a", encoding="utf-8", buffering=1)
        self._metrics = open(self._metrics_path, "a", encoding="utf-8", buffering=1)
        self._sequence = position.sequence
        kept = {key: value for key, value in previous.items() if key not in _DROPPED_ON_RESUME}
        kept.update(config=incoming.get("config"), execution=incoming.get("execution"),
                    scientific=incoming.get("scientific"), status="running", resumed_at=_timestamp(),
                    resume_count=int(previous.get("resume_count", 0)) + 1)
        return kept

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
            raise RuntimeError("RunLogger.close() was called; nothing more can be logged")
        self.raise_if_failed()
        self._queue.put(item)
        return item

    def raise_if_failed(self) -> None:
        if self._error is not None:
            raise RuntimeError(f"the log writer thread stopped: {self._error!r}") from self._error

    # ------------------------------------------------------------------ API
    def event(self, name: str, **fields: Any) -> None:
        self._put(_Item("event", {"schema_version": EVENT_SCHEMA, "event": name, "time": _timestamp(),
                                  **_json_value(fields)}))

    def metrics(self, namespace: str, iteration: int, values: Mapping[str, Any], *,
                optimizer_step: Any = None) -> None:
        if namespace not in _NAMESPACES:
            raise ValueError(f"metric namespace {namespace!r} is not one of {sorted(_NAMESPACES)}")
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
        position = LogCursor(events_bytes=self._events_path.stat().st_size,
                             metrics_bytes=self._metrics_path.stat().st_size,
                             optimizer_step=int(self._optimizer_step), sequence=int(self._sequence))
        return asdict(position)

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
