"""Source resolvers: turn a ``DataSourceConfig`` URI into an indexable record list.

Parity: the local resolvers of src/representax/data/resolvers.py:75-322
(JSONL, Parquet, Arrow IPC and directories of such files). Remote schemes
(``hf://``, HTTP ranges) need a network, which this environment does not
have; they raise a clear error naming the scheme. A resolver registry lets
users add schemes.
"""

from __future__ import annotations

import json
from collections.abc import Callable, Mapping, Sequence
from pathlib import Path
from typing import Any
from urllib.parse import urlparse


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


def _read_file(path: Path, split: str | None = None) -> Sequence:
    suffix = path.suffix.lower()
    if suffix in {".jsonl", ".json"}:
        return JsonlRecords(path)
    if suffix == ".parquet":
        import pyarrow.parquet as pq

        return TableRecords(pq.read_table(path))
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


def _local(source: Any) -> Sequence:
    uri, split = source.uri, source.split
    parsed = urlparse(uri)
    path = Path(parsed.path if parsed.scheme == "file" else uri).expanduser()
    if path.is_dir():
        files = sorted(p for p in path.rglob("*") if p.suffix.lower() in {".jsonl", ".parquet", ".arrow"}
                       and (split is None or split in p.name or split in p.parent.name))
        if not files:
            raise FileNotFoundError(f"no data files under {path}")
        return _Concat([_read_file(f) for f in files])
    if not path.exists():
        raise FileNotFoundError(f"data source {path} does not exist")
    return _read_file(path, split)


def _remote(source: Any) -> Sequence:
    raise ConnectionError(f"remote data source {source.uri!r} needs network access, which this environment lacks; "
                          "stage the files locally")


BUILTIN_RESOLVERS: dict[str, Callable[..., Sequence]] = {
    "file": _local,
    "": _local,
    "hf": _remote,
    "http": _remote,
    "https": _remote,
}


def read_source(source: Any, resolvers: Mapping[str, Callable[..., Sequence]] | None = None) -> Sequence:
    table = dict(BUILTIN_RESOLVERS)
    table.update(resolvers or {})
    scheme = urlparse(source.uri).scheme
    if scheme not in table:
        raise ValueError(f"no resolver for scheme {scheme!r}")
    return table[scheme](source)


__all__ = ["BUILTIN_RESOLVERS", "JsonlRecords", "TableRecords", "read_source"]
