"""Dataset resolvers and remote artifact reads, offline (D1, D2).

The network is replaced by fakes: ``huggingface_hub.snapshot_download`` by a
function that lays out a dataset repository on disk, ``urllib.request.urlopen``
by canned responses. Parity model: tests/data/test_resolvers.py of the
reference (HTTP range / ETag handling, hf:// pinning).
"""

import io
import json
from pathlib import Path

import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from representax_b200.data.artifact import Artifact, read_artifact
from representax_b200.data.config import DataSourceConfig
from representax_b200.data.resolvers import ParquetRecords, huggingface_dataset_id, read_source


def _source(uri, **kw):
    return DataSourceConfig(uri=uri, mapper="json.loads", **kw)


def test_parquet_row_groups_are_read_lazily_with_a_bounded_cache(tmp_path):
    path = tmp_path / "rows.parquet"
    pq.write_table(pa.table({"i": list(range(100)), "s": [f"r{i}" for i in range(100)]}), path, row_group_size=10)
    rows = ParquetRecords(path, cache_size=2)
    assert len(rows) == 100 and rows[37] == {"i": 37, "s": "r37"} and rows[-1]["i"] == 99
    assert rows.group_reads == 2
    for i in (30, 31, 95, 39):  # groups 3 and 9 are both cached
        rows[i]
    assert rows.group_reads == 2
    rows[5]  # group 0 is read and evicts the least recently used group (9)
    assert rows.group_reads == 3
    rows[95]
    assert rows.group_reads == 4
    with pytest.raises(IndexError):
        rows[100]


def _fake_hub(tmp_path, calls):
    def snapshot_download(*, repo_id, repo_type, revision, allow_patterns, cache_dir):
        calls.append(dict(repo_id=repo_id, repo_type=repo_type, revision=revision, allow_patterns=allow_patterns))
        root = tmp_path / "hub" / repo_id.replace("/", "--") / revision
        (root / "data").mkdir(parents=True, exist_ok=True)
        pq.write_table(pa.table({"q": ["a", "b", "c"]}), root / "data" / "train-00000-of-00001.parquet")
        (root / "data" / "test-00000-of-00001.jsonl").write_text("\n".join(json.dumps({"q": x}) for x in "xy"))
        return str(root)

    return snapshot_download


def test_hf_source_pins_revision_and_split(tmp_path, monkeypatch):
    import huggingface_hub

    calls = []
    monkeypatch.setattr(huggingface_hub, "snapshot_download", _fake_hub(tmp_path, calls))
    monkeypatch.setenv("REPRESENTAX_CACHE", str(tmp_path / "cache"))
    train = read_source(_source("hf://sentence-transformers/all-nli", revision="abc123", split="train"))
    assert [train[i]["q"] for i in range(len(train))] == ["a", "b", "c"]
    test = read_source(_source("hf://sentence-transformers/all-nli", revision="abc123", split="test"))
    assert [test[i]["q"] for i in range(len(test))] == ["x", "y"]
    assert calls[0]["repo_id"] == "sentence-transformers/all-nli" and calls[0]["repo_type"] == "dataset"
    assert calls[0]["revision"] == "abc123" and any("train" in p for p in calls[0]["allow_patterns"])
    with pytest.raises(ValueError, match="revision"):
        read_source(_source("hf://a/b", split="train"))
    with pytest.raises(ValueError, match="split"):
        read_source(_source("hf://a/b", revision="r"))
    assert huggingface_dataset_id("hf://org/name%20x") == "org/name x"
    with pytest.raises(ValueError):
        huggingface_dataset_id("hf://org/name?x=1")


class _Response(io.BytesIO):
    def __init__(self, body: bytes, headers: dict, status: int = 200):
        super().__init__(body)
        self.headers = headers
        self.status = status

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def test_http_source_caches_by_etag(tmp_path, monkeypatch):
    import urllib.request

    monkeypatch.setenv("REPRESENTAX_CACHE", str(tmp_path / "cache"))
    body = b"\n".join(json.dumps({"k": i}).encode() for i in range(4))
    seen = []

    def urlopen(request):
        seen.append(dict(request.header_items()))
        return _Response(body, {"ETag": '"v1"'})

    monkeypatch.setattr(urllib.request, "urlopen", urlopen)
    rows = read_source(_source("https://example.org/data/pairs.jsonl"))
    assert [rows[i]["k"] for i in range(len(rows))] == [0, 1, 2, 3]
    cached = list((tmp_path / "cache" / "http").rglob("*.jsonl"))
    assert len(cached) == 1
    body = b'{"k": 99}'  # a changed object under the same ETag is not re-read: the cache holds v1
    again = read_source(_source("https://example.org/data/pairs.jsonl", revision='"v1"'))
    assert len(again) == 4 and seen[-1].get("If-match") == '"v1"'
    monkeypatch.setattr(urllib.request, "urlopen", lambda request: _Response(body, {"ETag": '"v2"'}))
    with pytest.raises(OSError, match="ETag"):
        read_source(_source("https://example.org/data/pairs.jsonl", revision='"v1"'))
    with pytest.raises(ValueError, match="single"):
        read_source(_source("https://example.org/data/pairs.csv"))


def test_http_artifact_range_and_etag(monkeypatch):
    import urllib.request

    payload = bytes(range(256)) * 4
    art = Artifact(modality="image", uri="https://example.org/blob.bin", etag='"e1"', byte_range=(10, 20))
    monkeypatch.setattr(urllib.request, "urlopen", lambda r: _Response(
        payload[10:20], {"ETag": '"e1"', "Content-Range": "bytes 10-19/1024"}, status=206))
    assert read_artifact(art) == payload[10:20]
    # a server that ignores Range (200 with the whole object) is refused
    monkeypatch.setattr(urllib.request, "urlopen", lambda r: _Response(payload, {"ETag": '"e1"'}, status=200))
    with pytest.raises(OSError, match="Content-Range"):
        read_artifact(art)
    monkeypatch.setattr(urllib.request, "urlopen", lambda r: _Response(
        payload[10:20], {"ETag": '"other"', "Content-Range": "bytes 10-19/1024"}, status=206))
    with pytest.raises(ValueError, match="ETag"):
        read_artifact(art)
    member = Artifact(modality="image", uri="https://example.org/a.zip", etag='"e1"', archive_member="x.png")
    with pytest.raises(ValueError, match="archive"):
        read_artifact(member)


def test_token_balanced_shards_equalise_work():
    import numpy as np

    from representax_b200.data.balance import token_balanced_shards
    from representax_b200.data.loader import DataLoader

    rng = np.random.default_rng(0)
    lengths = rng.integers(64, 513, size=4096)
    for world in (2, 4, 8):
        shards = token_balanced_shards(lengths, world)
        assert sorted(np.concatenate(shards).tolist()) == list(range(4096))  # a partition
        assert {len(s) for s in shards} == {4096 // world}
        sums = [int(lengths[s].sum()) for s in shards]
        assert max(sums) - min(sums) <= lengths.max()  # within one row's length
    records = [{"n": int(n)} for n in rng.integers(1, 100, size=64)]
    seen = []
    for rank in range(4):
        loader = DataLoader([records], weights=[1.0], seed=0, batch_size=32, shard=(rank, 4), num_threads=1,
                            prefetch=1, token_length=lambda r: r["n"])
        batch, _, _ = loader.make_batch(0)
        seen.extend(r["n"] for r in batch)
        assert len(batch) == 8
        assert loader.data_contract["rank_assignment"] == "token_balanced"
    whole = DataLoader([records], weights=[1.0], seed=0, batch_size=32, num_threads=1, prefetch=1)
    assert sorted(seen) == sorted(r["n"] for r in whole.make_batch(0)[0])  # same global batch


def test_host_memory_budget_bounds_each_prefetch_slot():
    """The budget is split over prefetch + 1 model-ready batch slots (ref data/distribution.py:700-720)."""

    import numpy as np

    from representax_b200.data.loader import DataLoader

    rows = [np.zeros(16, dtype=np.float32) for _ in range(64)]  # 64 bytes a row

    def collate(records):
        return np.stack(records)

    ok = DataLoader([rows], weights=[1.0], batch_size=4, collate=collate, prefetch=3, num_batches=2,
                    host_memory_budget_bytes=4 * 256)  # 256 bytes a slot: one 4-row batch fits
    assert [b.shape for b in ok] == [(4, 16), (4, 16)]
    tight = DataLoader([rows], weights=[1.0], batch_size=8, collate=collate, prefetch=3, num_batches=1,
                       host_memory_budget_bytes=4 * 256)  # 512-byte batches do not
    with pytest.raises(MemoryError, match="per-slot limit"):
        list(tight)
    with pytest.raises(ValueError, match="cannot hold"):
        DataLoader([rows], weights=[1.0], batch_size=4, prefetch=3, host_memory_budget_bytes=3)
    with pytest.raises(ValueError, match="positive"):
        DataLoader([rows], weights=[1.0], batch_size=4, host_memory_budget_bytes=0)
