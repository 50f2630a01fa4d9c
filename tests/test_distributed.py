"""Multi-process data parallelism: CPU gloo ranks and (on >= 2 GPUs) the fused cross-rank MNR."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, backend):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from representax_b200.parallel.dist import init_from_env

    return init_from_env(backend=backend, timeout_s=60)


def _tiny_cfg():
    from representax_b200.models.bert import BertConfig

    return BertConfig(vocab_size=2000, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, max_position_embeddings=64, hidden_dropout_probability=0.0,
                      attention_dropout_probability=0.0)


def _step_master(batch, ctx, execution, device="cpu"):
    from representax_b200.models.bert import BertEncoder
    from representax_b200.precision import FP32_POLICY
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.optimizer import AdamW
    from representax_b200.train.step import TrainStep, init_train_state

    torch.use_deterministic_algorithms(True)
    state = init_train_state(BertEncoder(_tiny_cfg(), seed=0), device=device, precision=FP32_POLICY)
    step = TrainStep(state, MNRTask(scale=20.0, symmetric=True), optimizer=AdamW(learning_rate=1e-3),
                     precision=FP32_POLICY, execution=execution, dist=ctx)
    m = step(batch, 0)
    return state.store.grad.clone(), float(m.loss)


def _gloo_worker(rank, world, port, out):
    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.tasks._batch import slice_rows
    from representax_b200.train.execution import Direct, GradCache

    ctx = _init(rank, world, port, "gloo")
    full = retrieval_pairs(np.random.default_rng(0), 8, 32, vocab=2000, low=100, min_len=4)
    local = slice_rows(full, rank * 4, rank * 4 + 4)
    local.positive_mask = torch.eye(4, dtype=torch.bool)
    for name, execution in (("direct", Direct()), ("grad_cache", GradCache(query_chunk_size=3))):
        master, loss = _step_master(local, ctx, execution)
        if rank == 0:
            torch.save({"master": master, "loss": loss}, out + f".{name}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.distributed
def test_two_gloo_ranks_match_single_process(tmp_path):
    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.parallel.dist import LOCAL
    from representax_b200.train.execution import Direct

    out = str(tmp_path / "rank0")
    mp.spawn(_gloo_worker, args=(2, _port(), out), nprocs=2, join=True)
    full = retrieval_pairs(np.random.default_rng(0), 8, 32, vocab=2000, low=100, min_len=4)
    master, loss = _step_master(full, LOCAL, Direct())
    for name in ("direct", "grad_cache"):
        got = torch.load(out + f".{name}")
        assert abs(got["loss"] - loss) < 1e-5, name
        assert torch.allclose(got["master"], master, rtol=1e-4, atol=1e-6), name


def _fused_worker(rank, world, port, out, symmetric, hard_negatives=False):
    from representax_b200.parallel.fused_mnr import ShardedRetrievalBatch, sharded_mnr_loss
    from representax_b200.tasks.retrieval import retrieval_batch

    ctx = _init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    L, D = 96, 80
    Ld = 2 * L if hard_negatives else L  # documents: positives, then one hard negative per query
    g = torch.Generator().manual_seed(100 + rank)
    q = torch.randn(L, D, generator=g).to(dev).requires_grad_(True)
    d = torch.randn(Ld, D, generator=g).to(dev).requires_grad_(True)
    mask = torch.zeros(L, Ld, dtype=torch.bool)
    mask[:, :L] = torch.eye(L, dtype=torch.bool)
    local = retrieval_batch(query=q.detach(), document=d.detach(), positive_mask=mask)
    local = local.map_tensors(lambda t: t.to(dev))
    local.document_valid[5] = False
    sb = ShardedRetrievalBatch.from_local(local, ctx, symmetric=symmetric)
    loss, fwd, rev = sharded_mnr_loss(q, d, sb, scale=20.0, symmetric=symmetric)
    loss.backward()
    torch.cuda.synchronize()
    from representax_b200.ops._ext import check_status

    check_status(dev)
    parts = {k: [torch.empty_like(v) for _ in range(world)] for k, v in
             {"q": q.detach(), "d": d.detach(), "gq": q.grad, "gd": d.grad}.items()}
    for k, v in {"q": q.detach(), "d": d.detach(), "gq": q.grad, "gd": d.grad}.items():
        dist.all_gather(parts[k], v.contiguous())
    dv = [torch.empty_like(local.document_valid) for _ in range(world)]
    dist.all_gather(dv, local.document_valid)
    if rank == 0:
        torch.save({k: torch.cat(v).cpu() for k, v in parts.items()} | {"loss": float(loss), "dv": torch.cat(dv).cpu()},
                   out)
    dist.barrier()
    from representax_b200.parallel.peer import close_peer_groups

    close_peer_groups()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("hard_negatives", [False, True])
@pytest.mark.parametrize("symmetric", [False, True])
def test_fused_cross_rank_mnr_matches_gathered_reference(tmp_path, symmetric, hard_negatives):
    """Fused cross-rank MNR on every GPU of the box (2 to 4 ranks) against an fp64 gathered oracle."""

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    from representax_b200.ops.mnr import mnr_terms_reference

    out = str(tmp_path / "fused.pt")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_fused_worker, args=(world, _port(), out, symmetric, hard_negatives), nprocs=world, join=True)
    r = torch.load(out)
    q = r["q"].double().requires_grad_(True)
    d = r["d"].double().requires_grad_(True)
    n = q.shape[0]
    lq = n // world
    ld = d.shape[0] // world  # documents per rank (rank-major)
    w = torch.zeros(n, d.shape[0], dtype=torch.float64)
    for rank in range(world):
        w[rank * lq:(rank + 1) * lq, rank * ld:rank * ld + lq] = torch.eye(lq)
    qv = torch.ones(n, dtype=torch.bool)
    loss, *_ = mnr_terms_reference(q, d, w, qv, r["dv"], 20.0, symmetric)
    loss.backward()
    assert abs(r["loss"] - float(loss)) < 1e-4
    assert torch.allclose(r["gq"].double(), q.grad, rtol=1e-3, atol=1e-6)
    assert torch.allclose(r["gd"].double(), d.grad, rtol=1e-3, atol=1e-6)


def _sharded_worker(rank, world, port, out):
    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.models.bert import BertEncoder
    from representax_b200.precision import BF16_MIXED_POLICY
    from representax_b200.tasks._batch import slice_rows, to_device
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.execution import GradCache
    from representax_b200.train.optimizer import AdamW
    from representax_b200.train.step import TrainStep, init_train_state

    ctx = _init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    full = retrieval_pairs(np.random.default_rng(0), 16 * world, 48, vocab=2000, low=100, min_len=8)
    local = to_device(slice_rows(full, rank * 16, rank * 16 + 16), dev)
    local.positive_mask = torch.eye(16, dtype=torch.bool, device=dev)
    results = {}
    for sharded in (False, True):
        state = init_train_state(BertEncoder(_tiny_cfg(), seed=0, compute_dtype=torch.bfloat16), device=dev,
                                 precision=BF16_MIXED_POLICY, dist=ctx, sharded_optimizer=sharded)
        assert state.store.sharded == sharded
        step = TrainStep(state, MNRTask(scale=20.0), optimizer=AdamW(learning_rate=1e-3), precision=BF16_MIXED_POLICY,
                         execution=GradCache(query_chunk_size=8), dist=ctx, stochastic=False)
        for it in range(2):
            m = step(local, it)
        torch.cuda.synchronize()
        m_full, v_full = state.store.full_moments(ctx)
        results[sharded] = {"master": state.store.master[:state.store.numel].clone().cpu(), "m": m_full.cpu(),
                            "compute": state.store.compute.float().cpu(), "loss": float(m.loss)}
    if rank == 0:
        torch.save(results, out)
    dist.barrier()
    from representax_b200.parallel.peer import close_peer_groups

    close_peer_groups()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_optimizer_matches_ddp(tmp_path):
    """Fused peer reduce-scatter + sharded AdamW + all-gather == NCCL all-reduce + replicated AdamW."""

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "sharded.pt")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_sharded_worker, args=(world, _port(), out), nprocs=world, join=True)
    r = torch.load(out)
    a, b = r[True], r[False]
    assert abs(a["loss"] - b["loss"]) < 1e-3
    n = min(a["master"].numel(), b["master"].numel())
    diff = (a["master"][:n] - b["master"][:n]).abs()
    assert diff.max() <= 4.1e-3                       # at most a couple of lr-sized sign flips
    assert (diff <= 1e-5 + 1e-3 * b["master"][:n].abs()).float().mean() > 0.999
    torch.testing.assert_close(a["compute"][:n], a["master"][:n].bfloat16().float())
