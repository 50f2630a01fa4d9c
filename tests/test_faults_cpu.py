"""Failure paths, made on the host: stalled data, failing and overlapping
checkpoint writes, damaged checkpoints, a rank that leaves between steps, a
kernel status word reported through the step metrics, and multi-rank
checkpoint save / resume on gloo ranks.

Parity: tests/train/test_loop.py:187-246 (starvation) and
tests/train/test_checkpoint.py:119-364 (write failures, backpressure,
rejection of incomplete or foreign checkpoints) of the reference.
"""

import json
import os
import socket
import threading
import time

import pytest
import torch
import torch.multiprocessing as mp

from representax_b200.train.checkpoint import (
    COMPLETE_MARKER,
    CheckpointManager,
    CheckpointWriteError,
    IncompleteCheckpointError,
    validate_complete_checkpoint,
)


def _tensors(value=1.0):
    return {"model/w": torch.full((4, 3), value), "optimizer/scalars": torch.zeros(8)}


# --------------------------------------------------------------------------- data starvation
class _SlowIterator:
    def __init__(self, delay):
        self.delay = delay

    def __iter__(self):
        return self

    def __next__(self):
        time.sleep(self.delay)
        return {"x": torch.zeros(1)}


def test_stalled_data_source_raises_starvation(tmp_path):
    from representax_b200.train.logging import RunLogger
    from representax_b200.train.loop import DataStarvationError, run_training

    logger = RunLogger(tmp_path / "run", manifest={"name": "starve"})
    calls = []
    started = time.perf_counter()
    with pytest.raises(DataStarvationError):
        run_training(lambda batch, it: calls.append(it), _SlowIterator(5.0), max_steps=3, device=torch.device("cpu"),
                     logger=logger, heartbeat_seconds=0.1, timeout_seconds=0.5)
    elapsed = time.perf_counter() - started
    logger.close(status="failed")
    assert calls == [] and elapsed < 4.0
    events = [json.loads(l)["event"] for l in (tmp_path / "run" / "events.jsonl").read_text().splitlines()]
    assert "data_wait_heartbeat" in events and "data_starvation" in events and "training_failed" in events


def _identity(record):
    return record


def test_heartbeat_must_precede_timeout():
    from representax_b200.config import DataConfig
    from representax_b200.data import mix, source

    with pytest.raises(ValueError, match="heartbeat"):
        DataConfig(distribution=mix(source("memory://x", map=_identity), seed=0), data_wait_heartbeat_seconds=5,
                   data_wait_timeout_seconds=1)


# --------------------------------------------------------------------------- checkpoint writes
def test_background_write_failure_surfaces_on_next_call(tmp_path):
    manager = CheckpointManager(tmp_path / "ck", asynchronous=True)

    def explode(iteration):
        raise OSError(f"disk full at {iteration}")

    manager.save(1, _tensors(), {"optimizer_step": 1}, write_hook=explode)
    with pytest.raises(CheckpointWriteError, match="disk full at 1"):
        manager.wait()
    assert manager.latest() is None
    manager.save(2, _tensors(2.0), {"optimizer_step": 2})  # the manager stays usable
    manager.wait()
    assert manager.latest().iteration == 2


def test_one_save_in_flight_with_backpressure(tmp_path):
    manager = CheckpointManager(tmp_path / "ck", asynchronous=True)
    release = threading.Event()
    entered = threading.Event()

    def hold(iteration):
        entered.set()
        assert release.wait(10)

    manager.save(1, _tensors(), {"optimizer_step": 1}, write_hook=hold)
    assert entered.wait(5)
    threading.Timer(0.3, release.set).start()
    started = time.perf_counter()
    manager.save(2, _tensors(2.0), {"optimizer_step": 2})  # waits for save 1
    assert time.perf_counter() - started >= 0.25
    manager.wait()
    assert [e["event"] for e in manager.events] == ["checkpoint_backpressure"]
    assert manager.latest().iteration == 2


def _saved(tmp_path):
    manager = CheckpointManager(tmp_path / "ck", asynchronous=False, scientific="sci", data="data")
    manager.save(3, _tensors(), {"optimizer_step": 3})
    return manager, manager.latest().path


def test_missing_marker_is_rejected(tmp_path):
    manager, path = _saved(tmp_path)
    (path / COMPLETE_MARKER).unlink()
    with pytest.raises(IncompleteCheckpointError, match=COMPLETE_MARKER):
        manager.latest()


def test_corrupted_manifest_is_rejected(tmp_path):
    manager, path = _saved(tmp_path)
    manifest = json.loads((path / "checkpoint.json").read_text())
    manifest["iteration"] = 4  # content no longer matches its fingerprint
    (path / "checkpoint.json").write_text(json.dumps(manifest))
    with pytest.raises(IncompleteCheckpointError, match="fingerprint"):
        manager.latest()


def test_corrupted_state_file_is_rejected(tmp_path):
    manager, path = _saved(tmp_path)
    with open(path / "state.safetensors", "r+b") as handle:
        handle.seek(-4, os.SEEK_END)
        handle.write(b"\x00\x01\x02\x03")
    with pytest.raises(IncompleteCheckpointError, match="corrupt"):
        manager.latest()


def test_foreign_checkpoint_is_rejected(tmp_path):
    _, path = _saved(tmp_path)
    with pytest.raises(IncompleteCheckpointError, match="scientific"):
        validate_complete_checkpoint(path, expected_scientific_fingerprint="another job")
    with pytest.raises(IncompleteCheckpointError, match="data"):
        validate_complete_checkpoint(path, expected_data_fingerprint="another data contract")


def test_restore_refuses_other_rank_count(tmp_path):
    manager, _ = _saved(tmp_path)
    record = manager.latest()

    class _Never:
        def wait(self, name):
            raise AssertionError("no barrier on restore")

    two = CheckpointManager(tmp_path / "ck", world_size=2, rank=0, barrier=_Never())
    with pytest.raises(IncompleteCheckpointError, match="1 rank"):
        two.restore(record)


# --------------------------------------------------------------------------- device status word
def test_step_metrics_raise_on_device_status():
    from representax_b200.ops._ext import KernelTimeoutError
    from representax_b200.train.state import StepMetrics

    ok = StepMetrics(loss=torch.tensor(1.0), gradient_norm=torch.tensor(0.5), finite=torch.tensor(True),
                     learning_rate=1e-3, optimizer_step=torch.tensor(1.0), device_status=torch.tensor([0]))
    assert ok.to_host()["loss"] == 1.0
    bad = StepMetrics(loss=torch.tensor(1.0), gradient_norm=torch.tensor(0.5), finite=torch.tensor(True),
                      learning_rate=1e-3, optimizer_step=torch.tensor(1.0), device_status=torch.tensor([4]))
    with pytest.raises(KernelTimeoutError, match="peer wait"):
        bad.to_host()


# --------------------------------------------------------------------------- gloo ranks
def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=30):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from representax_b200.parallel.dist import init_from_env

    return init_from_env(backend="gloo", timeout_s=timeout_s)


def _leaving_rank(rank, world, port, out):
    import torch.distributed as dist

    from representax_b200.parallel.dist import StoreBarrier

    ctx = _init(rank, world, port)
    meet = StoreBarrier.from_default_group(ctx, timeout_s=1.5)
    meet.wait("step-1")  # both ranks finish step 1
    if rank == 1:
        return  # leaves between steps: no kernel or collective in flight
    try:
        meet.wait("step-2")
        result = "not detected"
    except TimeoutError as error:
        result = f"detected: {error}"
    with open(out, "w") as handle:
        handle.write(result)
    dist.destroy_process_group()


@pytest.mark.distributed
def test_rank_leaving_between_steps_is_detected(tmp_path):
    out = str(tmp_path / "result.txt")
    mp.start_processes(_leaving_rank, args=(2, _port(), out), nprocs=2, join=True, start_method="spawn")
    text = open(out).read()
    assert text.startswith("detected") and "1 of 2" in text


def _job_rank(rank, world, port, root, mode):
    import torch.distributed as dist

    from tests.test_job_cpu import _job, resolve_memory
    from representax_b200.train.job import run_job

    ctx = _init(rank, world, port)
    torch.use_deterministic_algorithms(True)
    job = _job(max_steps=6, checkpoint_every=3)
    job = job.model_copy(update={
        "export": job.export.model_copy(update={"enabled": False}),
        "training": job.training.model_copy(update={"global_batch_size": 8})})
    run_job(job, root, resolvers={"memory": resolve_memory}, device="cpu", dist=ctx, resume=mode == "resume")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.distributed
def test_two_rank_checkpoint_resume_matches_uninterrupted(tmp_path):
    import shutil

    a, b = tmp_path / "a", tmp_path / "b"
    for root in (a, b):
        mp.start_processes(_job_rank, args=(2, _port(), str(root), "fresh"), nprocs=2, join=True,
                           start_method="spawn")
    ck_b = CheckpointManager(b / "checkpoints")
    record = validate_complete_checkpoint(b / "checkpoints" / f"{6:010d}")
    assert sorted(p.name for p in record.path.glob("*.safetensors")) == [
        "state.rank0.safetensors", "state.rank1.safetensors"]
    # Interrupt after the step-3 checkpoint: drop step 6 and point `latest` back.
    shutil.rmtree(record.path)
    (b / "checkpoints" / "latest").write_text(json.dumps(
        {"schema_version": "representax-checkpoint-latest-v1", "iteration": 3, "path": f"{3:010d}"}))
    mp.start_processes(_job_rank, args=(2, _port(), str(b), "resume"), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        ma = CheckpointManager(a / "checkpoints", rank=rank, world_size=2, barrier=object())
        mb = CheckpointManager(b / "checkpoints", rank=rank, world_size=2, barrier=object())
        ta, _ = ma.restore(ma.latest())
        tb, _ = mb.restore(mb.latest())
        assert set(ta) == set(tb)
        for key in ta:
            assert torch.equal(ta[key], tb[key]), (rank, key)
    assert not list((b / "checkpoints").glob(".*staging"))
    rows = (b / "metrics.jsonl").read_text().count('"namespace": "train"')
    assert rows == 6
