"""Checkpoint manager: atomic, fingerprinted, asynchronous, with retention.

Parity: the marker / pointer protocol of src/representax/train/checkpoint.py
(``checkpoint.json`` manifest with a self-fingerprint, the
``REPRESENTAX_COMPLETE`` marker holding that fingerprint, atomic ``latest`` /
``best`` pointer files, LatestN + BestN retention, at most one save in
flight with backpressure, background failures surfaced on the training
thread, incomplete or foreign checkpoints rejected on restore).

Storage differs by design: instead of Orbax, each checkpoint directory holds
``state.safetensors`` (fp32 master parameters by name, both AdamW moments,
the optimizer scalars) written by a background thread from a pinned host
snapshot taken on a side CUDA stream, plus ``progress.json`` (iteration,
optimizer step, data cursor, logging cursor, rng seed).

With several ranks every rank writes its own ``state.rank{r}.safetensors``
(its optimizer shard plus the parameters it holds) into a staging directory;
ranks meet at host barriers (``StoreBarrier``, safe from the writer thread)
before writing, after writing and after publication. Only rank 0 clears a
stale staging directory (before the first barrier), hashes every shard,
writes ``progress.json`` / ``checkpoint.json`` / the marker and renames the
staging directory into place; nobody removes a directory another rank may
still be writing. Restore checks that the checkpoint was written by the same
number of ranks and reads the calling rank's shard.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import threading
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from safetensors.torch import load_file, save_file

CHECKPOINT_SCHEMA = "representax-b200-checkpoint-v1"
LATEST_SCHEMA = "representax-checkpoint-latest-v1"
BEST_SCHEMA = "representax-checkpoint-best-v1"
PROGRESS_SCHEMA = "representax-training-progress-v1"
COMPLETE_MARKER = "REPRESENTAX_COMPLETE"
CHECKPOINT_MANIFEST = "checkpoint.json"
LATEST_POINTER = "latest"
BEST_POINTER = "best"
STATE_FILE = "state.safetensors"
PROGRESS_FILE = "progress.json"


class IncompleteCheckpointError(RuntimeError):
    """A checkpoint directory is unfinished, corrupt or from another job."""


class CheckpointWriteError(RuntimeError):
    """A background checkpoint write failed."""


def _canonical(value: Any) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), default=str)


def fingerprint(value: Any) -> str:
    return hashlib.sha256(_canonical(value).encode()).hexdigest()


def scientific_fingerprint(job: Any) -> str:
    from representax_b200._config import ParameterRole

    return fingerprint(job.parameters(ParameterRole.SCIENTIFIC))


def _sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


def _atomic_write_text(path: Path, text: str) -> None:
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "w", encoding="utf-8") as handle:
        handle.write(text)
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, path)


def _atomic_write_json(path: Path, document: Mapping[str, Any]) -> None:
    _atomic_write_text(path, json.dumps(document, indent=2, sort_keys=True, default=str) + "\n")


def _fsync_dir(path: Path) -> None:
    fd = os.open(path, os.O_RDONLY | getattr(os, "O_DIRECTORY", 0))
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _manifest_fingerprint(manifest: Mapping[str, Any]) -> str:
    return fingerprint({k: v for k, v in manifest.items() if k != "checkpoint_fingerprint"})


@dataclass(frozen=True)
class CheckpointRecord:
    iteration: int
    path: Path
    checkpoint_fingerprint: str
    scientific_fingerprint: str
    data_fingerprint: str
    metric: float | None = None


def validate_complete_checkpoint(path: str | Path, *, expected_scientific_fingerprint: str | None = None,
                                 expected_data_fingerprint: str | None = None) -> CheckpointRecord:
    directory = Path(path).expanduser().resolve()
    required = [directory / CHECKPOINT_MANIFEST, directory / COMPLETE_MARKER, directory / PROGRESS_FILE]
    missing = [p.name for p in required if not p.is_file()]
    if missing:
        raise IncompleteCheckpointError(f"incomplete checkpoint {directory}; missing {', '.join(missing)}")
    manifest = json.loads((directory / CHECKPOINT_MANIFEST).read_text())
    if manifest.get("schema_version") != CHECKPOINT_SCHEMA:
        raise IncompleteCheckpointError(f"unsupported checkpoint manifest: {directory}")
    fp = manifest.get("checkpoint_fingerprint")
    if not isinstance(fp, str) or fp != _manifest_fingerprint(manifest):
        raise IncompleteCheckpointError(f"checkpoint manifest fingerprint differs: {directory}")
    if (directory / COMPLETE_MARKER).read_text().strip() != fp:
        raise IncompleteCheckpointError(f"checkpoint completion marker differs: {directory}")
    for name, digest in manifest.get("files", {}).items():
        file = directory / name
        if not file.is_file() or _sha256_file(file) != digest:
            raise IncompleteCheckpointError(f"checkpoint file {name} is missing or corrupt: {directory}")
    sci = manifest.get("scientific_fingerprint")
    if expected_scientific_fingerprint is not None and sci != expected_scientific_fingerprint:
        raise IncompleteCheckpointError(f"checkpoint scientific configuration differs: {directory}")
    data = manifest.get("data_fingerprint")
    if expected_data_fingerprint is not None and data != expected_data_fingerprint:
        raise IncompleteCheckpointError(f"checkpoint data contract differs: {directory}")
    iteration = manifest.get("iteration")
    if not isinstance(iteration, int) or iteration < 0:
        raise IncompleteCheckpointError(f"invalid checkpoint iteration: {directory}")
    return CheckpointRecord(iteration, directory, fp, sci, data, manifest.get("metric"))


class CheckpointManager:
    """Saves and restores training state under ``root``.

    ``save`` snapshots device tensors to pinned host memory on a side stream
    and returns; a worker thread writes the files, the manifest, the
    completion marker and the pointers. A second ``save`` waits for the
    first (one in flight). A failed background write raises
    :class:`CheckpointWriteError` on the next ``save``/``wait`` call.
    """

    def __init__(self, root: str | Path, *, keep: int = 3, keep_best: int = 1, asynchronous: bool = True,
                 scientific: str = "", data: str = "", rank: int = 0, world_size: int = 1,
                 metric_mode: str = "min", barrier=None) -> None:
        if world_size > 1 and barrier is None:
            raise ValueError("a multi-rank CheckpointManager needs a host barrier (StoreBarrier)")
        self.root = Path(root)
        self.keep = keep
        self.keep_best = keep_best
        self.asynchronous = asynchronous
        self.scientific = scientific
        self.data = data
        self.rank = rank
        self.world_size = world_size
        self.metric_mode = metric_mode
        self.barrier = barrier
        self._thread: threading.Thread | None = None
        self._error: BaseException | None = None
        self.events: list[dict[str, Any]] = []

    # -------------------------------------------------------------- helpers
    def _dir(self, iteration: int) -> Path:
        return self.root / f"{iteration:010d}"

    def _state_name(self) -> str:
        return STATE_FILE if self.world_size == 1 else f"state.rank{self.rank}.safetensors"

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            error, self._error = self._error, None
            raise CheckpointWriteError(f"background checkpoint write failed: {error}") from error

    # -------------------------------------------------------------- save
    def save(self, iteration: int, tensors: Mapping[str, torch.Tensor], progress: Mapping[str, Any], *,
             metric: float | None = None, best: bool = False, write_hook=None) -> None:
        if self._thread is not None:
            self.events.append({"event": "checkpoint_backpressure", "iteration": iteration})
        self.wait()
        snapshot = _host_snapshot(tensors)
        progress = dict(progress)
        progress.setdefault("schema_version", PROGRESS_SCHEMA)
        progress["iteration"] = iteration

        def work() -> None:
            try:
                if write_hook is not None:
                    write_hook(iteration)
                self._write(iteration, snapshot, progress, metric, best)
            except BaseException as error:  # surfaced on the training thread
                self._error = error

        if self.asynchronous:
            self._thread = threading.Thread(target=work, name=f"checkpoint-{iteration}", daemon=True)
            self._thread.start()
        else:
            work()
            self.wait()

    def _meet(self, name: str, iteration: int) -> None:
        if self.barrier is not None:
            self.barrier.wait(f"checkpoint-{iteration}-{name}")

    def _write(self, iteration: int, snapshot: dict[str, torch.Tensor], progress: dict, metric, best) -> None:
        final = self._dir(iteration)
        staging = self.root / f".{final.name}.staging"
        if self.rank == 0:
            self.root.mkdir(parents=True, exist_ok=True)
            if staging.exists():  # left by an interrupted save; nobody writes it before "begin"
                shutil.rmtree(staging)
            staging.mkdir(parents=True)
        self._meet("begin", iteration)
        save_file(snapshot, str(staging / self._state_name()))
        self._meet("written", iteration)
        if self.rank == 0:
            self._publish(iteration, staging, final, progress, metric, best)
        self._meet("published", iteration)

    def _publish(self, iteration: int, staging: Path, final: Path, progress: dict, metric, best) -> None:
        directory = staging
        shards = sorted(p.name for p in directory.glob("*.safetensors"))
        expected = [STATE_FILE] if self.world_size == 1 else sorted(
            f"state.rank{r}.safetensors" for r in range(self.world_size))
        if shards != expected:
            raise CheckpointWriteError(f"staging {directory} holds {shards}, expected {expected}")
        _atomic_write_json(directory / PROGRESS_FILE, progress)
        files = {p.name: _sha256_file(p) for p in sorted(directory.iterdir())
                 if p.name.endswith(".safetensors") or p.name == PROGRESS_FILE}
        manifest = {
            "schema_version": CHECKPOINT_SCHEMA,
            "iteration": iteration,
            "scientific_fingerprint": self.scientific,
            "data_fingerprint": self.data,
            "files": files,
            "world_size": self.world_size,
            "metric": metric,
        }
        manifest["checkpoint_fingerprint"] = _manifest_fingerprint(manifest)
        _atomic_write_json(directory / CHECKPOINT_MANIFEST, manifest)
        _atomic_write_text(directory / COMPLETE_MARKER, manifest["checkpoint_fingerprint"] + "\n")
        _fsync_dir(directory)
        if final.exists():  # same iteration saved again (e.g. final == periodic)
            shutil.rmtree(final)
        os.replace(directory, final)
        _fsync_dir(self.root)
        _atomic_write_json(self.root / LATEST_POINTER, {"schema_version": LATEST_SCHEMA, "iteration": iteration,
                                                        "path": final.name})
        if best:
            _atomic_write_json(self.root / BEST_POINTER, {"schema_version": BEST_SCHEMA, "iteration": iteration,
                                                          "path": final.name, "metric": metric})
        _fsync_dir(self.root)
        self._retain()

    def _retain(self) -> None:
        complete = []
        if not self.root.is_dir():
            return
        for d in sorted(self.root.iterdir()):
            if d.is_dir() and (d / COMPLETE_MARKER).is_file():
                complete.append(d)
        protected = set(complete[-self.keep:])
        best = self._pointer(BEST_POINTER)
        if best is not None:
            protected.add(best.resolve())
        for d in complete:
            if d.resolve() not in {p.resolve() for p in protected}:
                shutil.rmtree(d, ignore_errors=True)

    # -------------------------------------------------------------- restore
    def _pointer(self, name: str) -> Path | None:
        path = self.root / name
        if not path.is_file():
            return None
        doc = json.loads(path.read_text())
        return self.root / doc["path"]

    def latest(self) -> CheckpointRecord | None:
        directory = self._pointer(LATEST_POINTER)
        if directory is None:
            return None
        return validate_complete_checkpoint(directory, expected_scientific_fingerprint=self.scientific or None,
                                            expected_data_fingerprint=self.data or None)

    def best(self) -> CheckpointRecord | None:
        directory = self._pointer(BEST_POINTER)
        if directory is None:
            return None
        return validate_complete_checkpoint(directory, expected_scientific_fingerprint=self.scientific or None,
                                            expected_data_fingerprint=self.data or None)

    def restore(self, record: CheckpointRecord, device: torch.device | str = "cpu") -> tuple[dict, dict]:
        self.wait()
        written_by = json.loads((record.path / CHECKPOINT_MANIFEST).read_text()).get("world_size", 1)
        if written_by != self.world_size:
            raise IncompleteCheckpointError(f"{record.path} holds {written_by} rank shard(s); this run has "
                                            f"{self.world_size} ranks")
        tensors = load_file(str(record.path / self._state_name()), device=str(device))
        progress = json.loads((record.path / PROGRESS_FILE).read_text())
        return tensors, progress


def _host_snapshot(tensors: Mapping[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Copy device tensors to (pinned) host memory on a side stream."""

    cuda = [t for t in tensors.values() if t.is_cuda]
    out: dict[str, torch.Tensor] = {}
    if cuda:
        device = cuda[0].device
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for name, t in tensors.items():
                if t.is_cuda:
                    host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                    host.copy_(t, non_blocking=True)
                    out[name] = host
                else:
                    out[name] = t.detach().clone()
        stream.synchronize()
    else:
        out = {name: t.detach().clone().contiguous() for name, t in tensors.items()}
    return out


def training_tensors(state) -> dict[str, torch.Tensor]:
    """Named tensors of a train state: master params, AdamW moments, scalars."""

    store = state.store
    out: dict[str, torch.Tensor] = {}
    if getattr(store, "fsdp", None) is not None:
        # FSDP: each rank's file holds its own segment of the master weights and moments
        out["model/master_segment"] = store.master
        if store.exp_avg is not None:
            out["optimizer/exp_avg_shard"] = store.exp_avg
            out["optimizer/exp_avg_sq_shard"] = store.exp_avg_sq
        out["optimizer/shard"] = torch.tensor([store.shard_offset, store.shard_numel, store.group.world])
        out["optimizer/scalars"] = state.scalars
        return {k: v.contiguous() for k, v in out.items()}
    for name, view in store.named_views("master"):
        out[f"model/{name}"] = view
    if store.exp_avg is not None and getattr(store, "sharded", False):
        # sharded optimizer: each rank's file holds its own moment shard
        out["optimizer/exp_avg_shard"] = store.exp_avg
        out["optimizer/exp_avg_sq_shard"] = store.exp_avg_sq
        out["optimizer/shard"] = torch.tensor([store.shard_offset, store.shard_numel, store.group.world])
    elif store.exp_avg is not None:
        for name, view in store.named_views("exp_avg"):
            out[f"optimizer/exp_avg/{name}"] = view
        for name, view in store.named_views("exp_avg_sq"):
            out[f"optimizer/exp_avg_sq/{name}"] = view
    for name, buf in getattr(state, "optimizer_state", {}).items():
        out[f"optimizer/flat/{name}"] = buf
    out["optimizer/scalars"] = state.scalars
    return {k: v.contiguous() for k, v in out.items()}


def load_training_tensors(state, tensors: Mapping[str, torch.Tensor]) -> None:
    store = state.store
    sharded = getattr(store, "sharded", False)
    if getattr(store, "fsdp", None) is not None:
        meta = tensors.get("optimizer/shard")
        if (meta is None or "model/master_segment" not in tensors
                or tuple(int(v) for v in meta) != (store.shard_offset, store.shard_numel, store.group.world)):
            raise IncompleteCheckpointError("checkpoint segments do not match this run's FSDP layout")
        with torch.no_grad():
            store.master.copy_(tensors["model/master_segment"].to(store.device))
            if store.exp_avg is not None:
                store.exp_avg.copy_(tensors["optimizer/exp_avg_shard"].to(store.device))
                store.exp_avg_sq.copy_(tensors["optimizer/exp_avg_sq_shard"].to(store.device))
            state.scalars.copy_(tensors["optimizer/scalars"].to(state.scalars.device))
        store.refresh_compute()
        return
    with torch.no_grad():
        if sharded:
            meta = tensors.get("optimizer/shard")
            if meta is None or tuple(int(v) for v in meta) != (store.shard_offset, store.shard_numel,
                                                                 store.group.world):
                raise IncompleteCheckpointError("checkpoint optimizer shards do not match this run's sharding")
            store.exp_avg.copy_(tensors["optimizer/exp_avg_shard"].to(store.device))
            store.exp_avg_sq.copy_(tensors["optimizer/exp_avg_sq_shard"].to(store.device))
        kinds = (("master", "model/"),) if sharded else (("master", "model/"), ("exp_avg", "optimizer/exp_avg/"),
                                                          ("exp_avg_sq", "optimizer/exp_avg_sq/"))
        for which, prefix in kinds:
            for name, view in store.named_views(which):
                key = prefix + name
                if key not in tensors:
                    raise IncompleteCheckpointError(f"checkpoint lacks {key}")
                view.copy_(tensors[key].to(view.device))
        state.scalars.copy_(tensors["optimizer/scalars"].to(state.scalars.device))
        flat = {k[len("optimizer/flat/"):]: v for k, v in tensors.items() if k.startswith("optimizer/flat/")}
        if flat:
            state.optimizer_state.clear()
            state.optimizer_state.update({k: v.to(store.device).clone() for k, v in flat.items()})
    store.refresh_compute()


__all__ = [
    "BEST_POINTER", "CHECKPOINT_MANIFEST", "COMPLETE_MARKER", "CheckpointManager", "CheckpointRecord",
    "CheckpointWriteError", "IncompleteCheckpointError", "LATEST_POINTER", "fingerprint", "load_training_tensors",
    "scientific_fingerprint", "training_tensors", "validate_complete_checkpoint",
]
