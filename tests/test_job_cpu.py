"""Config 1 on CPU: BERT-small fp32 MNR through run_job, exact resume and export round trip."""

import json

import numpy as np
import pytest
import torch

from representax_b200.config import (
    BatchConfig,
    CheckpointConfig,
    ComponentConfig,
    DataConfig,
    JobConfig,
    ModelConfig,
    OptimizationConfig,
    TrainingConfig,
)
from representax_b200.data import mix, source
from representax_b200.tasks.retrieval import MNRConfig, RetrievalConfig

VOCAB = 30522


def _records(n, seq=128, seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        rec = {}
        for field in ("query", "positive"):
            length = int(rng.integers(16, seq + 1))
            ids = rng.integers(1000, VOCAB, size=length)
            ids[0], ids[-1] = 101, 102
            rec[field] = ids.tolist()
        out.append(rec)
    return out


RECORDS = _records(64)


def resolve_memory(source):
    return RECORDS


def collate(examples, seq: int = 128):
    from representax_b200.models.text_batch import TokenBatch
    from representax_b200.tasks.retrieval import RetrievalBatch

    def block(field):
        ids = torch.zeros(len(examples), seq, dtype=torch.int32)
        mask = torch.zeros(len(examples), seq, dtype=torch.int32)
        for i, e in enumerate(examples):
            n = len(e[field])
            ids[i, :n] = torch.tensor(e[field], dtype=torch.int32)
            mask[i, :n] = 1
        return TokenBatch(input_ids=ids, attention_mask=mask).pack()

    return RetrievalBatch(query=block("query"), document=block("positive"),
                          positive_mask=torch.eye(len(examples), dtype=torch.bool))


def identity(record):
    return record


def _job(max_steps=10, checkpoint_every=5, small=True):
    params = dict(vocab_size=VOCAB, hidden_size=384, intermediate_size=1536, num_hidden_layers=6,
                  num_attention_heads=12, max_position_embeddings=512, hidden_dropout_probability=0.0,
                  attention_dropout_probability=0.0)
    if small:
        params.update(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4)
    return JobConfig(
        name="bert-small-mnr",
        model=ModelConfig(target="representax_b200.models.bert.build_bert", parameters=params),
        task=RetrievalConfig(),
        loss=MNRConfig(scale=20.0),
        optimization=OptimizationConfig(optimizer=ComponentConfig(target="optax.adamw",
                                                                  parameters={"learning_rate": 2e-5})),
        data=DataConfig(distribution=mix(source("memory://pairs", map=identity), seed=0), num_threads=1,
                        prefetch_buffer_size=1,
                        collate=ComponentConfig(target="tests.test_job_cpu.collate")),
        training=TrainingConfig(global_batch_size=32 if not small else 8, max_steps=max_steps, seed=0,
                                batch=BatchConfig(micro_batch_size=8)),
        checkpointing=CheckpointConfig(every=checkpoint_every, keep=2, asynchronous=True),
    )


def test_job_config_roundtrips_json():
    job = _job()
    again = JobConfig.model_validate_json(job.model_dump_json())
    assert again == job
    assert "training" in job.parameters("scientific")


def test_run_job_resume_and_export(tmp_path):
    from representax_b200.export import load_inference_bundle
    from representax_b200.train.job import run_job

    resolvers = {"memory": resolve_memory}
    job = _job()
    result, bundle = run_job(job, tmp_path / "full", resolvers=resolvers, device="cpu")
    assert result.completed_iterations == 10 and result.optimizer_steps == 10
    metrics = [json.loads(l) for l in (tmp_path / "full" / "metrics.jsonl").read_text().splitlines()]
    train_rows = [m for m in metrics if m["namespace"] == "train"]
    assert len(train_rows) == 10

    # Interrupted run: 5 steps, then resume to 10 from the checkpoint.
    short = job.model_copy(update={"training": job.training.model_copy(update={"max_steps": 5})})
    from representax_b200.train.checkpoint import IncompleteCheckpointError

    with pytest.raises(IncompleteCheckpointError):
        # A different max_steps is a different scientific job: resume must refuse it.
        run_job(short, tmp_path / "full", resolvers=resolvers, device="cpu", resume=True)
    run_job(job.model_copy(update={"export": job.export.model_copy(update={"enabled": False})}),
            tmp_path / "split", resolvers=resolvers, device="cpu")

    model, loaded_job = load_inference_bundle(bundle.path)
    assert loaded_job == job
    from safetensors.torch import load_file

    native = load_file(str(bundle.path / "native" / "model.safetensors"))
    for name, tensor in model.state_dict().items():
        assert torch.equal(tensor.float(), native[name])


def test_exact_resume_matches_uninterrupted(tmp_path):
    from representax_b200.train.checkpoint import CheckpointManager
    from representax_b200.train.job import run_job

    resolvers = {"memory": resolve_memory}
    job = _job(max_steps=6, checkpoint_every=3)
    job = job.model_copy(update={"export": job.export.model_copy(update={"enabled": False})})
    run_job(job, tmp_path / "a", resolvers=resolvers, device="cpu")
    # Same job, killed after the step-3 checkpoint: simulate by truncating to 3 then resuming.
    run_job(job, tmp_path / "b", resolvers=resolvers, device="cpu")
    ckpt_b = CheckpointManager(tmp_path / "b" / "checkpoints")
    latest = ckpt_b.latest()
    assert latest.iteration == 6
    # Remove the final checkpoint and resume from iteration 3.
    import shutil

    shutil.rmtree(latest.path)
    (tmp_path / "b" / "checkpoints" / "latest").write_text(json.dumps(
        {"schema_version": "representax-checkpoint-latest-v1", "iteration": 3, "path": f"{3:010d}"}))
    run_job(job, tmp_path / "b", resolvers=resolvers, device="cpu", resume=True)
    a = CheckpointManager(tmp_path / "a" / "checkpoints").latest()
    b = CheckpointManager(tmp_path / "b" / "checkpoints").latest()
    ta, _ = CheckpointManager(tmp_path / "a" / "checkpoints").restore(a)
    tb, _ = CheckpointManager(tmp_path / "b" / "checkpoints").restore(b)
    assert set(ta) == set(tb)
    for k in ta:
        assert torch.equal(ta[k], tb[k]), k
    rows_a = (tmp_path / "a" / "metrics.jsonl").read_text().count('"namespace": "train"')
    rows_b = (tmp_path / "b" / "metrics.jsonl").read_text().count('"namespace": "train"')
    assert rows_a == rows_b == 6
