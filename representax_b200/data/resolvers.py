"""Source resolvers: turn a ``DataSourceConfig`` URI into an indexable record list.

Parity: src/representax/data/resolvers.py:75-474 -- local JSONL (line-offset
index), Parquet (row groups read on demand through a small LRU cache), Arrow
IPC and directories of such files; ``hf://namespace/dataset`` sources pinned
to an explicit revision and split; HTTP(S) data files. A resolver registry
lets users add schemes.

Remote sources are materialised once into a local cache directory
(``$REPRESENTAX_CACHE`` or ``~/.cache/representax_b200/data``) and then read
with the local readers: ``hf://`` through ``huggingface_hub`` (the dataset
repository's files for the split, at the pinned revision), HTTP(S) by a
plain GET whose ``ETag`` names the cached copy, so a changed object is never
mixed with an old one.
"""

from __future__ import annotations

import hashlib
import json
import os
import threading
from collections import OrderedDict
from collections.abc import Callable, Mapping, Sequence
from pathlib import Path
from typing import Any
from urllib.parse import unquote, urlparse


class JsonlRecords(Sequence):
    def __init__(self, path: Path) -> None:
        self.path = path
        self._offsets: list[int] = []
        with open(path, "rb") as handle:
            pos = 0
            for line in handle:
                if line.strip():
                    self._offsets.append(pos)
                pos += len(line)

    def __len__(self) -> int:
        return len(self._offsets)

    def __getitem__(self, index: int) -> Any:
        with open(self.path, "rb") as handle:
            handle.seek(self._offsets[index])
            return json.loads(handle.readline())


class TableRecords(Sequence):
    """Row access into a pyarrow table (Parquet or Arrow IPC)."""

    def __init__(self, table) -> None:
        self.table = table
        self.columns = table.column_names

    def __len__(self) -> int:
        return self.table.num_rows

    def __getitem__(self, index: int) -> Mapping[str, Any]:
        row = self.table.slice(index, 1).to_pylist()[0]
        return row


class ParquetRecords(Sequence):
    """Rows of a Parquet file, reading one row group at a time.

    Only the row groups recently touched stay in memory (an LRU of
    ``cache_size`` decoded groups), so a multi-GB file is indexable with a
    small, fixed host footprint; loader threads share the cache under a lock.
    """

    def __init__(self, path: Path, *, cache_size: int = 2) -> None:
        import pyarrow.parquet as pq

        if cache_size < 1:
            raise ValueError(f"row-group cache needs room for at least one group, got {cache_size}")
        self.path = path
        self._file = pq.ParquetFile(path, memory_map=True)
        meta = self._file.metadata
        self._starts = []
        total = 0
        for g in range(meta.num_row_groups):
            self._starts.append(total)
            total += meta.row_group(g).num_rows
        self._rows = total
        self.columns = tuple(self._file.schema_arrow.names)
        self._cache: OrderedDict[int, Any] = OrderedDict()
        self._cache_size = cache_size
        self._lock = threading.Lock()
        self.group_reads = 0

    def __len__(self) -> int:
        return self._rows

    def _group(self, g: int):
        with self._lock:
            table = self._cache.pop(g, None)
            if table is None:
                table = self._file.read_row_group(g)
                self.group_reads += 1
            self._cache[g] = table  # most recent last
            while len(self._cache) > self._cache_size:
                self._cache.popitem(last=False)
            return table

    def __getitem__(self, index: int) -> Mapping[str, Any]:
        import bisect

        if index < 0:
            index += self._rows
        if not 0 <= index < self._rows:
            raise IndexError(f"row {index} of a {self._rows}-row Parquet file")
        g = bisect.bisect_right(self._starts, index) - 1
        table = self._group(g)
        return {name: table.column(i)[index - self._starts[g]].as_py() for i, name in enumerate(self.columns)}


def _read_file(path: Path, split: str | None = None) -> Sequence:
    suffix = path.suffix.lower()
    if suffix in {".jsonl", ".json", ".ndjson"}:
        return JsonlRecords(path)
    if suffix == ".parquet":
        return ParquetRecords(path)
    if suffix in {".arrow", ".feather", ".ipc"}:
        import pyarrow as pa

        with pa.memory_map(str(path)) as source:
            try:
                table = pa.ipc.open_file(source).read_all()
            except pa.ArrowInvalid:
                source.seek(0)
                table = pa.ipc.open_stream(source).read_all()
        return TableRecords(table)
    raise ValueError(f"unsupported data file {path}")


class _Concat(Sequence):
    def __init__(self, parts: list[Sequence]) -> None:
        self.parts = parts
        self.starts = []
        total = 0
        for p in parts:
            self.starts.append(total)
            total += len(p)
        self.total = total

    def __len__(self) -> int:
        return self.total

    def __getitem__(self, index: int) -> Any:
        import bisect

        i = bisect.bisect_right(self.starts, index) - 1
        return self.parts[i][index - self.starts[i]]


_DATA_SUFFIXES = {".jsonl", ".ndjson", ".parquet", ".arrow"}


def _directory(path: Path, split: str | None) -> Sequence:
    """Every data file of a directory tree (of one split when given), in path order."""

    def in_split(p: Path) -> bool:
        if split is None:
            return True
        rel = p.relative_to(path).parts
        return any(part == split or part.startswith(f"{split}-") or part.startswith(f"{split}.")
                   or part.startswith(f"{split}_") for part in rel)

    files = sorted(p for p in path.rglob("*") if p.is_file() and p.suffix.lower() in _DATA_SUFFIXES and in_split(p))
    if not files:
        raise FileNotFoundError(f"no {'/'.join(sorted(_DATA_SUFFIXES))} files for split {split!r} under {path}")
    return _Concat([_read_file(f) for f in files])


def _local(source: Any) -> Sequence:
    uri, split = source.uri, source.split
    parsed = urlparse(uri)
    if parsed.scheme == "file" and parsed.netloc not in ("", "localhost"):
        raise ValueError(f"file:// source {uri!r} names another host")
    path = Path(unquote(parsed.path) if parsed.scheme == "file" else uri).expanduser()
    if path.is_dir():
        return _directory(path, split)
    if not path.exists():
        raise FileNotFoundError(f"data source {path} does not exist")
    return _read_file(path, split)


def cache_root() -> Path:
    root = Path(os.environ.get("REPRESENTAX_CACHE", Path.home() / ".cache" / "representax_b200" / "data"))
    root.mkdir(parents=True, exist_ok=True)
    return root


def huggingface_dataset_id(uri: str) -> str:
    """``hf://namespace/name`` -> ``namespace/name``."""

    parsed = urlparse(uri)
    if parsed.scheme != "hf" or parsed.query or parsed.fragment or parsed.params:
        raise ValueError(f"{uri!r} is not a plain hf://namespace/dataset URI")
    repo = "/".join(part for part in (parsed.netloc, parsed.path.strip("/")) if part)
    if not repo:
        raise ValueError(f"{uri!r} names no dataset repository")
    return unquote(repo)


def _huggingface(source: Any) -> Sequence:
    """A dataset repository on the Hub, pinned to ``revision``, one ``split`` of it.

    The repository's data files for the split (and ``subset`` directory when
    given) are fetched with ``huggingface_hub.snapshot_download`` into the
    cache (a pinned revision is immutable, so a later run reuses them) and
    read with the local readers.
    """

    if not source.revision:
        raise ValueError(f"{source.uri}: hf:// sources need an explicit revision (a commit hash or tag)")
    if not source.split:
        raise ValueError(f"{source.uri}: hf:// sources need an explicit split")
    import huggingface_hub

    repo = huggingface_dataset_id(source.uri)
    prefix = f"{source.subset}/" if source.subset else ""
    patterns = [f"{prefix}**{source.split}*{suffix}" for suffix in sorted(_DATA_SUFFIXES)] + [
        f"{prefix}**{source.split}/**{suffix}" for suffix in sorted(_DATA_SUFFIXES)]
    local = huggingface_hub.snapshot_download(repo_id=repo, repo_type="dataset", revision=source.revision,
                                              allow_patterns=patterns,
                                              cache_dir=str(cache_root() / "huggingface"))
    root = Path(local) / source.subset if source.subset else Path(local)
    return _directory(root, source.split)


def _http(source: Any) -> Sequence:
    """One JSONL / Parquet / Arrow file over HTTP(S), cached under its URL and ETag."""

    import urllib.request

    suffix = Path(urlparse(source.uri).path).suffix.lower()
    if suffix not in _DATA_SUFFIXES:
        raise ValueError(f"{source.uri}: HTTP sources are single {sorted(_DATA_SUFFIXES)} files")
    key = hashlib.sha256(source.uri.encode()).hexdigest()[:32]
    folder = cache_root() / "http" / key
    folder.mkdir(parents=True, exist_ok=True)
    request = urllib.request.Request(source.uri)
    if source.revision:  # a pinned ETag: the server must still hold exactly that object
        request.add_header("If-Match", source.revision)
    with urllib.request.urlopen(request) as response:  # noqa: S310 - explicit user data URI
        etag = (response.headers.get("ETag") or "").strip()
        if source.revision and etag and etag.strip('"') != source.revision.strip('"'):
            raise OSError(f"{source.uri}: server ETag {etag!r} differs from the pinned {source.revision!r}")
        name = hashlib.sha256((etag or "no-etag").encode()).hexdigest()[:16] + suffix
        target = folder / name
        if not (etag and target.is_file()):
            scratch = folder / f".{name}.{os.getpid()}.part"
            with open(scratch, "wb") as handle:
                while chunk := response.read(1 << 22):
                    handle.write(chunk)
            os.replace(scratch, target)
    return _read_file(target, source.split)


BUILTIN_RESOLVERS: dict[str, Callable[..., Sequence]] = {
    "file": _local,
    "": _local,
    "hf": _huggingface,
    "http": _http,
    "https": _http,
}


def read_source(source: Any, resolvers: Mapping[str, Callable[..., Sequence]] | None = None) -> Sequence:
    table = dict(BUILTIN_RESOLVERS)
    table.update(resolvers or {})
    scheme = urlparse(source.uri).scheme
    if scheme not in table:
        raise ValueError(f"no resolver for scheme {scheme!r}")
    return table[scheme](source)


__all__ = ["BUILTIN_RESOLVERS", "JsonlRecords", "ParquetRecords", "TableRecords", "cache_root",
           "huggingface_dataset_id", "read_source"]
