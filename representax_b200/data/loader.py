"""Deterministic host data pipeline with an exact-resume cursor.

Parity: ``build_dataset`` / ``build_data_loader`` / ``DataIterator`` /
``BatchTelemetry`` of src/representax/data/distribution.py:204-813. The
reference composes Grain datasets; here the same contract is met without
Grain:

* the record order is a pure function of (distribution seed, epoch, index):
  each source is permuted per epoch with a seeded generator and sources are
  interleaved by a seeded weighted choice, so every host and every resume
  sees the same stream;
* the iterator state is one integer (batches consumed), so
  ``get_state`` / ``set_state`` resume exactly regardless of worker count or
  prefetch depth;
* mapping and collation run on a thread pool with a bounded prefetch queue;
* each batch carries telemetry (data wait, preprocessing time, host bytes,
  prefetch occupancy) for the ``perf/`` metrics;
* a data contract (distribution, mapper / collate identities, batch size,
  remainder policy) is fingerprinted and checked on resume.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import queue
import threading
import time
from collections.abc import Callable, Iterator, Mapping, Sequence
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from .config import DataDistributionConfig


def resolve_callable(reference: str | Callable) -> Callable:
    if callable(reference):
        return reference
    module, _, attr = reference.rpartition(":") if ":" in reference else reference.rpartition(".")
    return getattr(importlib.import_module(module), attr)


def identity(record: Any) -> Any:
    return record


@dataclass(frozen=True)
class BatchTelemetry:
    data_wait_seconds: float
    preprocess_seconds: float | None
    host_batch_bytes: int
    prefetch_ready_batches: int | None
    prefetch_capacity: int | None


def host_nbytes(batch: Any) -> int:
    """Bytes of the host arrays in a batch (torch tensors and numpy arrays, found
    through dicts, sequences and dataclasses such as packed token batches)."""

    seen: set[int] = set()

    def walk(x: Any) -> int:
        if isinstance(x, torch.Tensor):
            if x.is_cuda:
                raise TypeError("host preprocessing emitted a device tensor; let the training loop place batches")
            return x.numel() * x.element_size()
        if isinstance(x, np.ndarray):
            return int(x.nbytes)
        if isinstance(x, dict):
            return sum(walk(v) for v in x.values())
        if isinstance(x, (list, tuple)):
            return sum(walk(v) for v in x)
        if hasattr(x, "__dataclass_fields__") and id(x) not in seen:
            seen.add(id(x))
            return sum(walk(getattr(x, name)) for name in x.__dataclass_fields__ if not name.startswith("_"))
        return 0

    return walk(batch)


class MixtureSampler:
    """Global record index -> (source, row), deterministic in (seed, epoch)."""

    def __init__(self, sizes: Sequence[int], weights: Sequence[float], seed: int, shuffle: bool) -> None:
        if not sizes or any(s <= 0 for s in sizes):
            raise ValueError("every source must contain at least one record")
        self.sizes = list(sizes)
        w = np.asarray(weights, dtype=np.float64)
        self.weights = w / w.sum()
        self.seed = seed
        self.shuffle = shuffle
        # One epoch = enough draws to exhaust the largest-weight-normalised source once.
        self.epoch_length = int(max(np.ceil(s / p) for s, p in zip(self.sizes, self.weights)))
        self._cache: dict[int, tuple[np.ndarray, list[np.ndarray]]] = {}

    def _epoch(self, epoch: int):
        cached = self._cache.get(epoch)
        if cached is None:
            rng = np.random.default_rng([self.seed, epoch])
            choice = rng.choice(len(self.sizes), size=self.epoch_length, p=self.weights)
            perms = [rng.permutation(s) if self.shuffle else np.arange(s) for s in self.sizes]
            rank = np.empty(self.epoch_length, dtype=np.int64)
            for s in range(len(self.sizes)):
                where = np.nonzero(choice == s)[0]
                rank[where] = np.arange(where.size)
            cached = (choice, perms, rank)
            self._cache = {epoch: cached}
        return cached

    def __getitem__(self, index: int) -> tuple[int, int]:
        epoch, offset = divmod(index, self.epoch_length)
        choice, perms, rank = self._epoch(epoch)
        source = int(choice[offset])
        return source, int(perms[source][int(rank[offset]) % self.sizes[source]])


class DataIterator:
    """Iterator over collated host batches with telemetry and an integer state."""

    def __init__(self, loader: "DataLoader", start_batch: int = 0) -> None:
        self._loader = loader
        self._next_batch = start_batch
        self._consumed = start_batch
        self.last_telemetry: BatchTelemetry | None = None
        self._queue: queue.Queue = queue.Queue(maxsize=max(1, loader.prefetch))
        self._stop = threading.Event()
        self._pool = ThreadPoolExecutor(max_workers=max(1, loader.num_threads), thread_name_prefix="rx-data")
        self._producer = threading.Thread(target=self._produce, name="rx-data-producer", daemon=True)
        self._producer.start()

    def _produce(self) -> None:
        try:
            while not self._stop.is_set():
                index = self._next_batch
                future = self._pool.submit(self._loader.make_batch, index)
                self._next_batch += 1
                while not self._stop.is_set():
                    try:
                        self._queue.put(future, timeout=0.1)
                        break
                    except queue.Full:
                        continue
        except BaseException as error:  # surfaced by __next__
            self._queue.put(error)

    def __iter__(self) -> "DataIterator":
        return self

    def __next__(self) -> Any:
        if self._loader.num_batches is not None and self._consumed >= self._loader.num_batches:
            raise StopIteration
        ready = self._queue.qsize()
        started = time.perf_counter()
        item = self._queue.get()
        if isinstance(item, BaseException):
            raise item
        batch, seconds, nbytes = item.result()
        waited = time.perf_counter() - started
        self._consumed += 1
        self.last_telemetry = BatchTelemetry(waited, seconds, nbytes, ready, self._loader.prefetch)
        return batch

    def get_state(self) -> dict[str, Any]:
        return {"schema_version": "representax-b200-data-state-v1", "batches_consumed": self._consumed}

    def set_state(self, state: Mapping[str, Any]) -> None:
        self.close()
        self.__init__(self._loader, int(state["batches_consumed"]))

    def close(self) -> None:
        self._stop.set()
        try:
            while True:
                self._queue.get_nowait()
        except queue.Empty:
            pass
        self._producer.join(timeout=5)
        self._pool.shutdown(wait=False, cancel_futures=True)


class DataLoader:
    """Batches of collated records drawn from a deterministic mixture."""

    def __init__(self, sources: Sequence[Sequence[Any]], *, weights: Sequence[float], seed: int = 0,
                 shuffle: bool = True, mappers: Sequence[Callable] | None = None,
                 collate: Callable[[list[Any]], Any] | None = None, batch_size: int,
                 drop_remainder: bool = True, num_threads: int = 4, prefetch: int = 4,
                 num_batches: int | None = None, shard: tuple[int, int] = (0, 1),
                 contract: Mapping[str, Any] | None = None, host_memory_budget_bytes: int | None = None,
                 token_length: Callable[[Any], int] | None = None) -> None:
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if num_threads < 0 or prefetch < 0:
            raise ValueError("num_threads and prefetch must be non-negative")
        if host_memory_budget_bytes is not None:
            # the budget covers every model-ready batch the loader can hold at
            # once: the prefetch queue plus the batch being handed out
            if host_memory_budget_bytes <= 0:
                raise ValueError("host_memory_budget_bytes must be positive or None")
            if host_memory_budget_bytes // (max(prefetch, 1) + 1) == 0:
                raise ValueError(f"host_memory_budget_bytes={host_memory_budget_bytes} cannot hold "
                                 f"{max(prefetch, 1) + 1} batch slots")
        self.sources = list(sources)
        self.sampler = MixtureSampler([len(s) for s in self.sources], weights, seed, shuffle)
        self.mappers = list(mappers) if mappers is not None else [identity] * len(self.sources)
        self.collate = collate or (lambda records: records)
        self.batch_size = batch_size
        self.drop_remainder = drop_remainder
        self.num_threads = num_threads
        self.prefetch = prefetch
        self.num_batches = num_batches
        self.shard_index, self.shard_count = shard
        if batch_size % self.shard_count:
            raise ValueError("global batch size must divide evenly over data shards")
        self.host_memory_budget_bytes = host_memory_budget_bytes
        # With several shards and a token_length function, every rank maps the
        # whole global batch and keeps its token-balanced share of the rows
        # (representax_b200.data.balance) instead of a contiguous slice.
        self.token_length = token_length
        self.data_contract = dict(contract or {})
        if token_length is not None and self.shard_count > 1:
            self.data_contract.setdefault("rank_assignment", "token_balanced")
        self.data_contract.setdefault("batch_size", batch_size)
        self.data_contract.setdefault("drop_remainder", drop_remainder)

    @property
    def epoch_batches(self) -> int:
        """Whole batches in one pass over the mixture."""

        full, rest = divmod(self.sampler.epoch_length, self.batch_size)
        return full if (self.drop_remainder or rest == 0) else full + 1

    @property
    def data_fingerprint(self) -> str:
        text = json.dumps(self.data_contract, sort_keys=True, default=str)
        return hashlib.sha256(text.encode()).hexdigest()

    def make_batch(self, index: int):
        started = time.perf_counter()
        local = self.batch_size // self.shard_count
        if self.token_length is not None and self.shard_count > 1:
            from .balance import token_balanced_shards

            start = index * self.batch_size
            everything = []
            for i in range(start, start + self.batch_size):
                source, row = self.sampler[i]
                everything.append(self.mappers[source](self.sources[source][row]))
            mine = token_balanced_shards([self.token_length(r) for r in everything], self.shard_count)
            records = [everything[i] for i in mine[self.shard_index]]
        else:
            base = index * self.batch_size + self.shard_index * local
            records = []
            for i in range(base, base + local):
                source, row = self.sampler[i]
                records.append(self.mappers[source](self.sources[source][row]))
        batch = self.collate(records)
        nbytes = host_nbytes(batch) if not isinstance(batch, list) else 0
        if self.host_memory_budget_bytes is not None:
            slot = self.host_memory_budget_bytes // (max(self.prefetch, 1) + 1)
            if nbytes > slot:
                raise MemoryError(f"host batch uses {nbytes} bytes; per-slot limit is {slot} bytes")
        return batch, time.perf_counter() - started, nbytes

    def __iter__(self) -> Iterator[Any]:
        return DataIterator(self)


def build_data_loader(distribution: DataDistributionConfig, *, batch_size: int, collate=None, batch_fn=None,
                      drop_remainder: bool = True, num_threads: int = 4, prefetch: int | None = None,
                      prefetch_buffer_size: int | None = None, num_batches: int | None = None,
                      shard: tuple[int, int] = (0, 1), host_memory_budget_bytes: int | None = None,
                      resolvers=None, mappers: Mapping[str, Callable] | None = None) -> DataLoader:
    """Build the loader of a distribution (``batch_fn`` / ``prefetch_buffer_size``
    are accepted as the reference's names for ``collate`` / ``prefetch``)."""

    from .resolvers import read_source

    collate = collate if collate is not None else batch_fn
    prefetch = prefetch if prefetch is not None else (prefetch_buffer_size if prefetch_buffer_size is not None else 4)
    sources = [read_source(s, resolvers=resolvers) for s in distribution.sources]
    mapper_table = dict(mappers or {})
    resolved_mappers = [mapper_table.get(s.mapper) or resolve_callable(s.mapper) for s in distribution.sources]
    contract_fn = getattr(collate, "data_contract", None)
    contract = {
        "schema_version": "representax-b200-data-contract-v1",
        "distribution": distribution.model_dump(mode="json"),
        "collate": contract_fn() if callable(contract_fn) else getattr(collate, "__qualname__", repr(collate)),
    }
    return DataLoader(sources, weights=distribution.weights, seed=distribution.seed, shuffle=distribution.shuffle,
                      mappers=resolved_mappers, collate=collate, batch_size=batch_size,
                      drop_remainder=drop_remainder, num_threads=num_threads, prefetch=max(1, prefetch),
                      num_batches=num_batches, shard=shard, contract=contract,
                      host_memory_budget_bytes=host_memory_budget_bytes)


__all__ = ["BatchTelemetry", "DataIterator", "DataLoader", "MixtureSampler", "build_data_loader", "host_nbytes",
           "identity", "resolve_callable"]
