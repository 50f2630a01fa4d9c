"""Training benchmarks of the other reference configurations.

    python -m representax_b200.bench_models --config {mpnet,modernvbert,qwen3vl} --steps K --warmup W
    (N GPUs: python -m torch.distributed.run --nproc-per-node N -m representax_b200.bench_models ...)

Each configuration is one of the reference's benchmark workloads at its
named shape, with random-init weights and synthetic inputs:

* ``mpnet`` - MPNet-base (12 layers, hidden 768, 12 heads, FFN 3072, 32
  relative-position buckets, vocab 30527, mean pooling), bf16-mixed; 512
  (anchor, positive, hard-negative) triplets per rank of length 128, token ids
  uniform in [1000, 30527); symmetric MNR (scale 20) with Matryoshka over
  dimensions [768, 512, 256, 128, 64]; direct execution.
* ``modernvbert`` - ModernVBERT text-image retriever: ModernBERT text tower
  (22 layers, hidden 768, 12 heads, GeGLU FFN 1152, RoPE, global attention
  every 3rd layer, 128-token sliding window otherwise) and a SigLIP vision tower
  (12 layers, hidden 768, patch 16 at 512 x 512, pixel shuffle 4 -> 64 image
  tokens). Queries are text of length 128 (ids uniform over the 50368 vocab),
  documents are one N(0, 1) image each; cached MNR (GradCache) with global
  batch 2048 and mini-batch 64; block-scaled (MXFP8) linear layers
  (``--fp8 tensor``: the reference's per-tensor scaling).
* ``qwen3vl`` - Qwen3-VL-2B-style embedder: 28-layer decoder (hidden 2048,
  16 query / 8 KV heads of 128, SwiGLU 6144, M-RoPE, vocab 151936) with packed
  INT4 base weights and LoRA rank 16 on q/k/v/o/gate/up/down, and a 24-layer
  vision tower (hidden 1024, patch 16, 2 x 2 merge); queries are text of
  length 512, documents one 448 x 448 image (196 merged tokens) with a short
  text prompt; last-token pooling; cached MNR with global batch 1024 and
  mini-batch 16.

Multi-GPU runs are one process per GPU with cross-rank in-batch negatives
through the fused peer-memory MNR kernels; ``mpnet`` and ``modernvbert`` run
their named FSDP layout by default (``--layout``), ``qwen3vl`` runs data
parallel with a sharded optimizer (its TP x FSDP layout is not built); the
layout is recorded beside the number. Timing follows ``bench.py``: W untimed warm-up steps, then K steps
bracketed by a barrier and ``torch.cuda.synchronize()``, CUDA events on the
launching stream, maximum over ranks; rank 0 prints one JSON line.

Reference parity: the workloads of benchmarks/grad_cache_modernvbert.py,
benchmarks/dense_retrieval.py and benchmarks/results/qwen3-vl-2b-20260821
of the reference (their shapes, not their harness).
"""

from __future__ import annotations

import os

os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import argparse
import json

import numpy as np
import torch


def _mpnet(args, rng_for_rank):
    from representax_b200.data.synthetic import token_batch
    from representax_b200.models.mpnet import MPNetConfig, MPNetEncoder
    from representax_b200.precision import BF16_MIXED_POLICY
    from representax_b200.tasks.modifiers.task import MatryoshkaTask
    from representax_b200.tasks.retrieval import MNRTask, RetrievalBatch
    from representax_b200.train.execution import Direct

    per_rank, seq = args.rows or 512, 128
    cfg = MPNetConfig(hidden_dropout_probability=args.dropout, attention_dropout_probability=args.dropout)
    model = MPNetEncoder(cfg, seed=0, compute_dtype=torch.bfloat16)
    task = MatryoshkaTask(MNRTask(scale=20.0, symmetric=True), [768, 512, 256, 128, 64])

    def batch(rng):
        q = token_batch(rng, per_rank, seq, vocab=30527, low=1000, min_len=seq, max_len=seq, cls_id=0, sep_id=2)
        d = token_batch(rng, 2 * per_rank, seq, vocab=30527, low=1000, min_len=seq, max_len=seq, cls_id=0, sep_id=2)
        mask = torch.zeros(per_rank, 2 * per_rank, dtype=torch.bool)
        mask[:, :per_rank] = torch.eye(per_rank, dtype=torch.bool)  # documents: positives then hard negatives
        return RetrievalBatch(query=q, document=d, positive_mask=mask)

    info = {"model": "mpnet-base (12L, H768, 12 heads, FFN 3072, 32 relative buckets, vocab 30527, mean pooling)",
            "rows_per_rank": per_rank, "unit_rows": "triplets", "seq_len": seq,
            "loss": "symmetric MNR (scale 20) + Matryoshka [768, 512, 256, 128, 64], hard negatives",
            "execution": "direct", "reference_parallelism": "FSDP over 8 GPUs"}
    return model, task, Direct(), BF16_MIXED_POLICY, batch, per_rank, info


def _modernvbert(args, rng_for_rank):
    from representax_b200.data.synthetic import token_batch
    from representax_b200.models.modernvbert import ModernVBERTBatch, ModernVBERTConfig, ModernVBERTEncoder
    from representax_b200.precision import FP8_MIXED_POLICY, MXFP8_MIXED_POLICY
    from representax_b200.tasks.retrieval import MNRTask, RetrievalBatch
    from representax_b200.train.execution import GradCache

    world = int(os.environ.get("WORLD_SIZE", "1"))
    global_batch = args.rows or 2048
    per_rank, mini, seq = global_batch // world, 64, 128
    vocab = 50368
    # The image placeholder must be a row of the embedding table.
    cfg = ModernVBERTConfig(image_token_id=vocab - 1)
    model = ModernVBERTEncoder(cfg, seed=0, compute_dtype=torch.bfloat16)
    n_img = cfg.image_sequence_length
    task = MNRTask(scale=20.0)

    def batch(rng):
        q = token_batch(rng, per_rank, seq, vocab=vocab - 1, low=0, min_len=seq, max_len=seq, cls_id=50281,
                        sep_id=50282, pack=False)
        ids = np.full((per_rank, n_img + 2), cfg.image_token_id, dtype=np.int64)
        ids[:, 0], ids[:, -1] = 50281, 50282
        pixels = torch.from_numpy(rng.standard_normal((per_rank, 1, 3, 512, 512), dtype=np.float32))
        d = ModernVBERTBatch(torch.ones(per_rank, n_img + 2, dtype=torch.long), torch.from_numpy(ids), pixels).pack()
        qb = ModernVBERTBatch(q.attention_mask.long(), q.input_ids.long()).pack()
        return RetrievalBatch(query=qb, document=d, positive_mask=torch.eye(per_rank, dtype=torch.bool))

    info = {"model": "modernvbert (ModernBERT 22L H768 GeGLU 1152, sliding 128 / global every 3rd; SigLIP 12L H768 "
                     "patch 16 @ 512x512, pixel shuffle 4)",
            "global_batch": global_batch, "mini_batch": mini, "unit_rows": "pairs", "seq_len": seq,
            "documents": "one 512x512 N(0,1) image (64 image tokens) per document",
            "loss": "cached MNR (GradCache), scale 20",
            "precision": ("fp8 linear layers (MXFP8: E4M3 / E5M2 gradients with one UE8M0 scale per 32 values, "
                          "tcgen05 block-scaled MMA)" if args.fp8 == "block" else
                          "fp8 linear layers (per-tensor scaled E4M3 / E5M2 gradients)")
            + ", bf16 elsewhere, fp32 master", "reference_parallelism": "FSDP over 8 GPUs"}
    policy = MXFP8_MIXED_POLICY if args.fp8 == "block" else FP8_MIXED_POLICY
    return model, task, GradCache(query_chunk_size=mini, retain_bytes="auto"), policy, batch, per_rank, info


def _qwen3vl(args, rng_for_rank):
    from representax_b200.data.synthetic import token_batch
    from representax_b200.models.adapters import apply_quantized_lora
    from representax_b200.models.qwen3 import Qwen3TextConfig
    from representax_b200.models.qwen3_vl import Qwen3VLBatch, Qwen3VLConfig, Qwen3VLEncoder, Qwen3VLVisionConfig
    from representax_b200.precision import BF16_MIXED_POLICY
    from representax_b200.tasks.retrieval import MNRTask, RetrievalBatch
    from representax_b200.train.execution import GradCache

    world = int(os.environ.get("WORLD_SIZE", "1"))
    global_batch = args.rows or 1024
    per_rank, mini, seq = global_batch // world, 16, 512
    vocab = 151936
    cfg = Qwen3VLConfig(
        text=Qwen3TextConfig(vocab_size=vocab, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                             num_attention_heads=16, num_key_value_heads=8, head_dimension=128,
                             mrope_section=(24, 20, 20), pad_token_id=151643),
        vision=Qwen3VLVisionConfig(depth=24, hidden_size=1024, intermediate_size=4096, num_heads=16, patch_size=16,
                                   out_hidden_size=2048, num_position_embeddings=2304,
                                   deepstack_visual_indexes=(5, 11, 17)),
        image_token_id=151655)
    model = Qwen3VLEncoder(cfg, seed=0, compute_dtype=torch.bfloat16)
    # q/k/v are one fused [q; k; v] weight and gate/up one [gate; up] weight in this layout.
    apply_quantized_lora(model, rank=16, alpha=32.0, target_pattern=r"text\.layers\.\d+\.(qkv|o_proj|gate_up|down)")
    task = MNRTask(scale=20.0)
    grid_side = 448 // 16
    merged = (grid_side // 2) ** 2
    patch_dim = 3 * 2 * 16 * 16

    def batch(rng):
        q = token_batch(rng, per_rank, seq, vocab=151643, low=0, min_len=seq, max_len=seq, cls_id=151643,
                        sep_id=151645, pack=False)
        qb = Qwen3VLBatch(q.input_ids.long(), q.attention_mask.long()).prepare(cfg)
        prompt = 16
        ids = rng.integers(0, 151643, size=(per_rank, merged + prompt)).astype(np.int64)
        ids[:, 1:1 + merged] = cfg.image_token_id
        grid = torch.tensor([[1, grid_side, grid_side]] * per_rank)
        pixels = torch.from_numpy(rng.standard_normal((per_rank * grid_side * grid_side, patch_dim),
                                                      dtype=np.float32))
        d = Qwen3VLBatch(torch.from_numpy(ids), torch.ones(per_rank, merged + prompt, dtype=torch.long), pixels,
                         grid).prepare(cfg)
        return RetrievalBatch(query=qb, document=d, positive_mask=torch.eye(per_rank, dtype=torch.bool))

    info = {"model": "qwen3-vl-2b-style (28L H2048 16q/8kv hd128 SwiGLU 6144 M-RoPE vocab 151936; vision 24L H1024 "
                     "patch 16, 2x2 merge)",
            "global_batch": global_batch, "mini_batch": mini, "unit_rows": "pairs", "seq_len": seq,
            "documents": "one 448x448 N(0,1) image (196 merged tokens) + 16-token prompt",
            "adapters": "packed INT4 base weights + LoRA r16 (alpha 32) on q/k/v/o/gate/up/down",
            "loss": "cached MNR (GradCache), scale 20, last-token pooling",
            "reference_parallelism": "TP=2 x FSDP=4 on 8 GPUs"}
    return model, task, GradCache(query_chunk_size=mini, retain_bytes="auto"), BF16_MIXED_POLICY, batch, per_rank, info


BUILDERS = {"mpnet": _mpnet, "modernvbert": _modernvbert, "qwen3vl": _qwen3vl}


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--config", choices=sorted(BUILDERS), required=True)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--rows", type=int, default=None,
                        help="override the per-rank triplets (mpnet) or global batch (others)")
    parser.add_argument("--dropout", type=float, default=0.1, help="mpnet hidden / attention dropout")
    parser.add_argument("--fp8", choices=["block", "tensor"], default="block",
                        help="modernvbert fp8 scaling: MXFP8 blocks (default) or per tensor")
    parser.add_argument("--out", default=None, help="append the JSON line to this file (rank 0)")
    parser.add_argument("--layout", choices=["auto", "dp", "fsdp"], default="auto",
                        help="N > 1: dp = replicated weights + sharded optimizer; fsdp = master weights, moments and "
                             "bf16 owner copies sharded, weights gathered at first use (fused into the forward "
                             "GEMMs); auto = the configuration's named layout (FSDP for mpnet / modernvbert, dp for "
                             "qwen3vl, whose TP x FSDP layout is not built)")
    args = parser.parse_args(argv)

    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    from bench import ClockSampler  # noqa: E402  (the flagship bench's clock sampler)

    from representax_b200.ops._ext import check_status, launch_counter
    from representax_b200.parallel.dist import barrier, init_from_env
    from representax_b200.tasks._batch import to_device
    from representax_b200.train.optimizer import AdamW
    from representax_b200.train.step import TrainStep, init_train_state

    ctx = init_from_env(timeout_s=600.0)
    world = ctx.world_size
    device = torch.device("cuda", ctx.local_rank)
    torch.cuda.set_device(device)
    model, task, execution, policy, make_batch, rows, info = BUILDERS[args.config](args, None)
    layout = args.layout if args.layout != "auto" else ("dp" if args.config == "qwen3vl" else "fsdp")
    fsdp = layout == "fsdp" and world > 1
    state = init_train_state(model, device=device, precision=policy, dist=ctx, sharded_optimizer=world > 1,
                             fsdp=fsdp)
    step = TrainStep(state, task, optimizer=AdamW(learning_rate=2e-5, weight_decay=0.01), precision=policy,
                     execution=execution, max_gradient_norm=1.0, dist=ctx,
                     stochastic=args.config == "mpnet" and args.dropout > 0)
    rng = np.random.default_rng(4321 + ctx.rank)
    n_host = 2
    host = [make_batch(rng).map_tensors(lambda t: t.pin_memory()) for _ in range(n_host)]
    resident = [to_device(b, device) for b in host]
    torch.cuda.synchronize()

    it = 0
    for _ in range(args.warmup):
        step(resident[it % n_host], it)
        it += 1
    torch.cuda.synchronize()
    check_status(device)

    counter = launch_counter()
    sampler = ClockSampler(ctx.local_rank)
    barrier(ctx)
    torch.cuda.synchronize()
    sampler.start()
    counter.launches = 0
    counter.counting = True
    start_ev = torch.cuda.Event(enable_timing=True)
    end_ev = torch.cuda.Event(enable_timing=True)
    start_ev.record()
    for _ in range(args.steps):
        metrics = step(resident[it % n_host], it)
        it += 1
    end_ev.record()
    torch.cuda.synchronize()
    counter.counting = False
    barrier(ctx)
    clocks = sampler.stop()
    check_status(device)
    t = torch.tensor([start_ev.elapsed_time(end_ev) / 1e3], device=device)
    if ctx.enabled:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    elapsed = float(t)
    if ctx.rank == 0:
        global_rows = rows * world
        out = {"metric": f"train {info['unit_rows']}/sec (device-timed, max over ranks)",
               "value": global_rows * args.steps / elapsed, "unit": f"{info['unit_rows']}/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * elapsed / args.steps,
               "higher_is_better": True, "dtype": "bf16", "data": "synthetic inputs; random-init weights",
               "config": dict(info, name=args.config,
                              parallelism=(f"fsdp{world} (sharded master / moments / bf16 owner copy, fused "
                                           "gather-GEMM, cross-rank negatives)") if fsdp else
                              (f"dp{world}" + ("" if world == 1 else " (sharded optimizer, cross-rank negatives)"))),
               "clocks": clocks, "gpu_launches": counter.launches, "final_loss": float(metrics.loss),
               "peak_memory_gb": torch.cuda.max_memory_allocated(device) / 2**30, "impl": "ours"}
        line = json.dumps(out)
        print(line, flush=True)
        if args.out:
            with open(args.out, "a") as handle:
                handle.write(line + "\n")
    if ctx.enabled:
        from representax_b200.parallel.peer import close_peer_groups

        close_peer_groups()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
