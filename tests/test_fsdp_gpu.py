"""FSDP: the forward GEMM with the weight gather fused in, and the sharded layout.

``test_fused_gather_gemm_*`` runs on one GPU: the "owner shards" are separate
local buffers, so the kernel's per-chunk copies (split at shard boundaries),
readiness flags and tile waits run as on several GPUs, without a peer.
The two-rank test trains a small BERT with FSDP and with the replicated
sharded-optimizer layout from the same start and data and compares them.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("world,offset,n,k,epi", [(4, 64, 296, 256, "bias"), (3, 1024, 2304, 768, "none"),
                                                 (8, 0, 96, 128, "gelu")])
def test_fused_gather_gemm_matches_plain_gemm(world, offset, n, k, epi, variant):
    """variant 1: one CTA per tile; 2: CTA pairs (cta_group::2), the default for >= 256 rows."""

    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import check_status, ext, status

    torch.manual_seed(0)
    total = offset + n * k + 512
    seg = (total + world - 1) // world
    seg = (seg + 63) // 64 * 64
    flat = (torch.randn(world * seg, device=_dev()) * 0.05).to(torch.bfloat16)
    shards = [flat[r * seg:(r + 1) * seg].clone() for r in range(world)]  # each "rank" owns one segment
    weight_ref = flat[offset:offset + n * k].view(n, k)
    cache = torch.full((world * seg,), float("nan"), device=_dev()).to(torch.bfloat16)
    w_view = cache[offset:offset + n * k].view(n, k)
    x = (torch.randn(777, k, device=_dev()) * 0.5).to(torch.bfloat16)
    bias = (torch.randn(n, device=_dev()) * 0.1).to(torch.bfloat16)
    out = torch.empty(777, n, dtype=torch.bfloat16, device=_dev())
    ref = torch.empty_like(out)
    ready = torch.zeros(4096, dtype=torch.int32, device=_dev())
    code = {"none": G.EPI_NONE, "bias": G.EPI_BIAS, "gelu": G.EPI_BIAS | G.EPI_GELU}[epi]
    pre = torch.empty_like(out) if epi == "gelu" else None
    pre_ref = torch.empty_like(out) if epi == "gelu" else None
    ext().gemm_gather(x, w_view, out, code, G.OUT_BF16, 1.0, None if epi == "none" else bias, pre, None,
                      status(_dev()), 0, 0, 0.0, [t.data_ptr() for t in shards], seg, offset, ready, variant)
    G.gemm(x, weight_ref, ref, epi=code, bias=None if epi == "none" else bias, aux_out=pre_ref, variant=variant)
    torch.cuda.synchronize()
    check_status(_dev())
    assert torch.equal(w_view, weight_ref)  # the weight landed in the cache exactly
    assert torch.equal(out, ref)  # same kernel arithmetic on the same operands
    if pre is not None:
        assert torch.equal(pre, pre_ref)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fsdp_worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.models.bert import BertConfig, BertEncoder
    from representax_b200.ops._ext import check_status
    from representax_b200.parallel.dist import init_from_env
    from representax_b200.parallel.peer import close_peer_groups
    from representax_b200.precision import BF16_MIXED_POLICY
    from representax_b200.tasks._batch import slice_rows, to_device
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.checkpoint import load_training_tensors, training_tensors
    from representax_b200.train.execution import GradCache
    from representax_b200.train.optimizer import AdamW
    from representax_b200.train.step import TrainStep, init_train_state

    ctx = init_from_env(backend="nccl", timeout_s=120)
    dev = torch.device("cuda", rank)
    # The fused-gather GEMM picks the same tile variant as the plain GEMM for a
    # shape, so the two layouts run the same arithmetic.
    cfg = BertConfig(vocab_size=3000, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                     num_attention_heads=4, max_position_embeddings=128, hidden_dropout_probability=0.0,
                     attention_dropout_probability=0.0)
    full = retrieval_pairs(np.random.default_rng(3), 16 * world, 48, vocab=3000, low=100, min_len=8)
    local = to_device(slice_rows(full, rank * 16, rank * 16 + 16), dev)
    results = {}
    for mode in ("replicated", "fsdp"):
        model = BertEncoder(cfg, seed=0, compute_dtype=torch.bfloat16)
        state = init_train_state(model, device=dev, precision=BF16_MIXED_POLICY, dist=ctx,
                                 sharded_optimizer=True, fsdp=mode == "fsdp")
        step = TrainStep(state, MNRTask(scale=20.0), optimizer=AdamW(learning_rate=1e-3), precision=BF16_MIXED_POLICY,
                         execution=GradCache(query_chunk_size=8), dist=ctx, stochastic=False)
        losses = [float(step(local, it).loss) for it in range(3)]
        torch.cuda.synchronize()
        check_status(dev)
        store = state.store
        master = store.gather_master() if mode == "fsdp" else store.master[:store.numel].clone()
        results[mode] = {"losses": losses, "master": master.cpu()}
        if mode == "fsdp":
            fsdp = store.fsdp
            results[mode]["stats"] = dict(fsdp.stats)
            results[mode]["segment"] = store.master.numel()
            results[mode]["numel"] = store.numel
            # checkpoint round trip of this rank's segments
            saved = {k: v.clone() for k, v in training_tensors(state).items()}
            store.master.add_(1.0)
            load_training_tensors(state, saved)
            results[mode]["restored"] = bool(torch.equal(store.master, saved["model/master_segment"]))
    if rank == 0:
        torch.save(results, out)
    dist.barrier()
    close_peer_groups()
    dist.destroy_process_group()


def test_fsdp_ranks_match_replicated_layout(tmp_path):
    """FSDP on every GPU of the box (2 to 4 ranks) against the replicated layout."""

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    out = str(tmp_path / "fsdp.pt")
    mp.spawn(_fsdp_worker, args=(world, _port(), out), nprocs=world, join=True)
    r = torch.load(out)
    rep, fsdp = r["replicated"], r["fsdp"]
    assert fsdp["segment"] == -(-fsdp["numel"] // world)  # master weights: one 1/N segment per rank
    assert fsdp["stats"]["fused_gathers"] >= 8 * 2  # 4 GEMM weights per layer, 2 layers, from step 2 on
    assert fsdp["restored"]
    # Same kernels on the same operands; only the order of a few fp32 atomic
    # reductions (norm-parameter gradients) may differ between runs.
    for a, b in zip(rep["losses"], fsdp["losses"]):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (rep["losses"], fsdp["losses"])
    diff = (rep["master"] - fsdp["master"]).abs()
    assert diff.max().item() < 5e-4 and diff.mean().item() < 1e-6, (diff.max().item(), diff.mean().item())
