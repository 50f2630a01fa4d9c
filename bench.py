"""Flagship benchmark: BERT-base cached-MNR (GradCache) training on 1..8 B200.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

Configuration: BERT-base (12 layers, hidden 768,
12 heads, FFN 3072, vocab 30522, mean pooling), bf16 compute with fp32
master weights and AdamW, cached MNR (scale 20) with global batch 4096
(anchor, positive) pairs, mini-batch 128, length 256, token ids uniform in
[1000, 30522) with [CLS]/[SEP], valid lengths uniform in [32, 256]. Data
parallel over N GPUs with cross-rank in-batch negatives (a 4096 x 4096
similarity per step). The global batch is fixed as N grows (strong scaling).

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the maximum over ranks is reported. Each step's working set
(weights, optimizer state, activations: several GB) exceeds the 126 MB L2, so
no explicit flush is inserted. A second timed phase ("e2e") runs the same
steps through the public API with every step's inputs copied host->device
from pinned memory and the loss read back to the host.
"""

from __future__ import annotations

import os

# Retained GradCache graphs fill most of HBM; expandable segments keep the
# caching allocator from fragmenting around them (must be set before CUDA init).
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

METRIC = "train pairs/sec (box, device-timed, max over ranks) at 1/2/4/8 B200 vs ref JAX/NCCL"
MODEL = "bert-base (12L, H768, 12 heads, FFN 3072, vocab 30522, mean pooling)"
GLOBAL_BATCH = 4096
MINI_BATCH = 128
SEQ = 256
MIN_LEN = 32
VOCAB = 30522


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--global-batch", type=int, default=GLOBAL_BATCH)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-strict", action="store_true",
                   help="skip the second timed phase with GradCache graph retention off")
    p.add_argument("--optimizer", choices=["sharded", "ddp"], default="sharded",
                   help="N>1: sharded = peer-memory reduce-scatter + sharded AdamW + all-gather kernels; "
                        "ddp = NCCL all-reduce + replicated AdamW")
    p.add_argument("--dropout", type=float, default=0.1,
                   help="hidden and attention dropout (BERT-base default 0.1; native Philox masks)")
    p.add_argument("--gemm-table", default=None,
                   help="write per-shape GEMM device times of one extra step to this markdown file (rank 0)")
    p.add_argument("--kernel-table", default=None,
                   help="after the timed steps, run one more step under torch.profiler (CUPTI) and write a "
                        "per-kernel device-time table to this path (rank 0); not part of the timed number")
    p.add_argument("--retain-gb", type=float, default=None,
                   help="GradCache graph-retention budget in GiB (default: free HBM minus a reserve; 0: replay "
                        "all chunks, the strict GradCache of the reference)")
    return p.parse_args()


def _reference_arm(args) -> None:
    """Run the unmodified reference (installed under baseline/_ref) on config 2, or say why it cannot.

    The reference is JAX/Equinox/Optax/Grain/Orbax code. This arm imports its
    runtime and the package from ``baseline/_ref`` and reports the import
    failures it actually caught; only when every import succeeds does it hand
    over to the reference's own public training API.
    """

    rank = int(os.environ.get("RANK", "0"))
    ref_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if os.path.isdir(ref_dir):
        sys.path.insert(0, ref_dir)
    failures = []
    for module in ("jax", "equinox", "optax", "grain", "orbax.checkpoint", "representax"):
        try:
            __import__(module)
        except Exception as error:  # ImportError, or a broken install raising at import time
            failures.append(f"{module}: {type(error).__name__}: {error}")
    if failures:
        if rank == 0:
            why = ("reference not runnable offline (pip install of /root/reference fails: build backend "
                   "hatchling absent from the wheelhouse); imports tried from baseline/_ref: " + "; ".join(failures))
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    from representax.train import run_job  # noqa: F401  (reference public API)

    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": "the reference imported, but its run_job needs a "
                          "dataset on disk; this arm has no synthetic-data adapter for it yet"}), flush=True)


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.device_index = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.handle = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.handle, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.handle.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for name, flag in zip(names, parts[5:9]):
                    if flag.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        loaded = [x for x in sm if mx and x > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _gemm_table(step, batch, it, path) -> None:
    """Device time of every tcgen05 GEMM launch of one training step, grouped by
    kind / shape / epilogue (CUDA events around each launch)."""

    from representax_b200.ops import gemm as G

    torch.cuda.synchronize()
    G.profile_gemms(True)
    step(batch, it)
    records = G.profile_gemms(False)
    rows = G.gemm_table(records)
    peak = _measured_bf16()
    total = sum(t for _, _, t in rows)
    with open(path, "w") as f:
        f.write("| GEMM (kind, M N K, epilogue bits, output mode) | launches | device ms | us per launch "
                "| TFLOP/s | of measured bf16 | share |\n|---|---|---|---|---|---|---|\n")
        for key, n, t in rows:
            m, nn, k = (int(tok[1:]) for tok in key.split()[1:4])  # "M.. N.. K.."
            flops = 2.0 * m * nn * k * n
            tf = flops / (t / 1e3) / 1e12
            f.write(f"| {key} | {n} | {t:.2f} | {1e3 * t / n:.1f} | {tf:.0f} | {tf * 1e12 / peak:.2f} | "
                    f"{t / total:.1%} |\n")
        f.write(f"| total | {sum(n for _, n, _ in rows)} | {total:.2f} | | | | 100% |\n")


def _measured_bf16() -> float:
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as handle:
            return float(json.load(handle)["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        return 1.59e15


def _kernel_table(step, batch, it, path) -> None:
    """Per-kernel device time of one training step (CUPTI via torch.profiler)."""

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step(batch, it)
        torch.cuda.synchronize()
    rows, examples = {}, {}
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        name = e.name
        for key, short in (("gemm_pair_kernel", "gemm_tcgen05_pair"), ("gemm_kernel", "gemm_tcgen05"),
                           ("attn_fwd", "attention_fwd"), ("attn_bwd", "attention_bwd"), ("attn_dvec", "attention_dvec"),
                           ("attn_dq_convert", "attention_dq_convert"), ("norm_fwd", "layernorm_fwd"),
                           ("norm_param_reduce", "layernorm_param_reduce"),
                           ("norm_bwd", "layernorm_bwd"), ("embed_ln", "embed_layernorm"), ("pool_", "pool"),
                           ("dropout_colsum", "dropout_colsum"), ("colsum", "colsum"), ("mnr", "mnr"), ("sgemm", "mnr_sgemm"), ("adamw", "adamw"),
                           ("grad_norm", "grad_norm"), ("cast_bf16", "cast_bf16")):
            if key in name:
                name = short
                break
        else:
            name = name[:60]
        t, n = rows.get(name, (0.0, 0))
        rows[name] = (t + e.device_time_total / 1e3, n + 1)
        examples.setdefault(name, set()).add(e.name[:90])
    total = sum(t for t, _ in rows.values())
    with open(path, "w") as f:
        f.write("| kernel | launches | device ms | us per launch | share |\n|---|---|---|---|---|\n")
        for name, (t, n) in sorted(rows.items(), key=lambda kv: -kv[1][0]):
            f.write(f"| {name} | {n} | {t:.2f} | {1e3 * t / n:.1f} | {t / total:.1%} |\n")
        f.write(f"| total | {sum(n for _, n in rows.values())} | {total:.2f} | | 100% |\n")
        f.write("\nKernels behind each label:\n\n")
        for name in sorted(examples):
            f.write(f"- {name}: " + "; ".join(sorted(examples[name])[:4]) + "\n")


def main() -> None:
    args = _args()
    if args.impl == "reference":
        _reference_arm(args)
        return

    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.models.bert import BertConfig, BertEncoder
    from representax_b200.ops._ext import check_status, launch_counter
    from representax_b200.parallel.dist import barrier, init_from_env
    from representax_b200.precision import BF16_MIXED_POLICY
    from representax_b200.tasks._batch import to_device
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.execution import GradCache
    from representax_b200.train.optimizer import AdamW
    from representax_b200.train.step import TrainStep, init_train_state

    ctx = init_from_env(timeout_s=600.0)
    world = ctx.world_size
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", ctx.local_rank)
    torch.cuda.set_device(device)
    if args.global_batch % world:
        raise SystemExit("global batch must divide evenly over ranks")
    local = args.global_batch // world

    config = BertConfig.base(hidden_dropout_probability=args.dropout, attention_dropout_probability=args.dropout)
    model = BertEncoder(config, seed=0, compute_dtype=torch.bfloat16)
    state = init_train_state(model, device=device, precision=BF16_MIXED_POLICY, dist=ctx,
                             sharded_optimizer=args.optimizer == "sharded")
    step = TrainStep(state, MNRTask(scale=20.0), optimizer=AdamW(learning_rate=2e-5, weight_decay=0.01),
                     precision=BF16_MIXED_POLICY,
                     execution=GradCache(query_chunk_size=MINI_BATCH,
                                         retain_bytes="auto" if args.retain_gb is None else int(args.retain_gb * 2**30)),
                     max_gradient_norm=1.0, dist=ctx, stochastic=args.dropout > 0)

    # Host batches (pinned), distinct per step; same shapes every step. Every rank
    # draws the same global batch and keeps its token-balanced share of the pairs
    # (equal pair counts, token counts within one pair of each other), so no rank
    # waits for a rank that drew longer sequences.
    from representax_b200.data.balance import pair_lengths, token_balanced_shards
    from representax_b200.models.text_batch import TokenBatch
    from representax_b200.tasks.retrieval import RetrievalBatch

    rng = np.random.default_rng(1234)
    n_host = 4
    host = []
    for _ in range(n_host):
        full = retrieval_pairs(rng, args.global_batch, SEQ, vocab=VOCAB, low=1000, min_len=MIN_LEN, max_len=SEQ,
                               pack=False)
        mine = torch.from_numpy(token_balanced_shards(
            pair_lengths(full.query.attention_mask.sum(1).numpy(), full.document.attention_mask.sum(1).numpy()),
            world)[ctx.rank])

        def rows(tb):
            return TokenBatch(input_ids=tb.input_ids[mine], attention_mask=tb.attention_mask[mine]).pack()

        b = RetrievalBatch(query=rows(full.query), document=rows(full.document),
                           positive_mask=torch.eye(local, dtype=torch.bool))
        b = b.map_tensors(lambda t: t.pin_memory())
        host.append(b)

    def h2d(b):
        return to_device(b, device)

    def packed_bytes(b):
        return b.query.packed.nbytes() + b.document.packed.nbytes() + sum(
            t.nbytes for t in (b.query.attention_mask, b.query.input_ids, b.document.attention_mask,
                               b.document.input_ids, b.positive_mask, b.query_valid, b.document_valid))

    resident = [h2d(b) for b in host]
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
    for k in range(args.steps):
        metrics = step(resident[it % n_host], it)
        it += 1
    end_ev.record()
    torch.cuda.synchronize()
    counter.counting = False
    barrier(ctx)
    clocks = sampler.stop()
    launches = counter.launches
    check_status(device)
    elapsed = start_ev.elapsed_time(end_ev) / 1e3
    t = torch.tensor([elapsed], device=device)
    if ctx.enabled:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    elapsed = float(t)
    final_loss = float(metrics.loss)

    if args.gemm_table and ctx.world_size == 1:
        _gemm_table(step, resident[it % n_host], it, args.gemm_table)
        it += 1
    if args.kernel_table and ctx.rank == 0:
        _kernel_table(step, resident[it % n_host], it, args.kernel_table)
        it += 1
    elif args.kernel_table:
        step(resident[it % n_host], it)
        it += 1

    # Strict GradCache (the reference's recompute-everything semantics): the same
    # steps with no first-pass graph kept, so every chunk is replayed. Reported
    # beside the headline so the 1 -> N curve can be read without HBM retention.
    strict = None
    if args.retain_gb is None and not args.no_strict:
        strict_step = TrainStep(state, MNRTask(scale=20.0), optimizer=AdamW(learning_rate=2e-5, weight_decay=0.01),
                                precision=BF16_MIXED_POLICY, execution=GradCache(query_chunk_size=MINI_BATCH,
                                                                                 retain_bytes=0),
                                max_gradient_norm=1.0, dist=ctx, stochastic=args.dropout > 0)
        strict_step(resident[it % n_host], it)
        it += 1
        barrier(ctx)
        torch.cuda.synchronize()
        s3 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        s3.record()
        for k in range(args.steps):
            strict_step(resident[it % n_host], it)
            it += 1
        e3.record()
        torch.cuda.synchronize()
        barrier(ctx)
        check_status(device)
        ts = torch.tensor([s3.elapsed_time(e3) / 1e3], device=device)
        if ctx.enabled:
            torch.distributed.all_reduce(ts, op=torch.distributed.ReduceOp.MAX)
        strict_elapsed = float(ts)
        strict = {"value": args.global_batch * args.steps / strict_elapsed, "unit": "pairs/s",
                  "ms_per_step": 1e3 * strict_elapsed / args.steps, "retained_chunks": 0,
                  "note": "GradCache replays every chunk (no first-pass graph kept), same kernels and steps"}
        del strict_step

    e2e = None
    if not args.no_e2e:
        barrier(ctx)
        torch.cuda.synchronize()
        s2 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        s2.record()
        for k in range(args.steps):
            batch = h2d(host[it % n_host])
            m = step(batch, it)
            loss_host = float(m.loss)  # device -> host read of the step's loss
            it += 1
        e2.record()
        torch.cuda.synchronize()
        barrier(ctx)
        te = torch.tensor([s2.elapsed_time(e2) / 1e3], device=device)
        if ctx.enabled:
            torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        e2e_elapsed = float(te)
        e2e = {"value": args.global_batch * args.steps / e2e_elapsed, "unit": "pairs/s",
               "h2d_bytes_per_step": int(packed_bytes(host[0])), "d2h_bytes_per_step": 4,
               "ms_per_step": 1e3 * e2e_elapsed / args.steps, "last_loss": loss_host}

    if ctx.rank == 0:
        value = args.global_batch * args.steps / elapsed
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "pairs/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": 1e3 * elapsed / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform token ids, uniform valid lengths); random-init weights",
            "config": {
                "model": MODEL,
                "global_batch": args.global_batch,
                "mini_batch": MINI_BATCH,
                "seq_len": SEQ,
                "valid_len": [MIN_LEN, SEQ],
                "grad_cache": ("exact cached MNR; first-pass graphs of {retained_chunks} of {chunks} chunks kept in "
                               "HBM ({gb:.0f} GB), their replay forward skipped; all other chunks replayed").format(
                                   gb=step.execution.stats.get("retained_bytes", 0) / 2**30, **{
                                       k: step.execution.stats.get(k, 0) for k in ("retained_chunks", "chunks")}),
                "parallelism": f"dp{world}" + ("" if world == 1 else " with cross-rank negatives"),
                "loss": "cached MNR (GradCache), scale 20, global negatives",
                "optimizer": "AdamW lr 2e-5 wd 0.01, clip 1.0, fp32 master, bf16 compute",
                "optimizer_step": ("single-GPU fused norm/clip/AdamW kernels" if world == 1 else
                                   "sharded: peer-memory gradient reduce-scatter + shard AdamW + parameter all-gather"
                                   if args.optimizer == "sharded" else "NCCL all-reduce + replicated fused AdamW"),
                "dropout": args.dropout,
                "padding": "packed (padding tokens are not computed)",
                "rank_assignment": ("one global batch per step, its pairs dealt to ranks token-balanced "
                                    "(serpentine over pairs sorted by length)"),
                "l2": "per-step working set > 126 MB L2; no explicit flush",
            },
            "clocks": clocks,
            "strict_grad_cache": strict,
            "e2e": e2e,
            "gpu_launches": launches,
            "final_loss": final_loss,
            "impl": "ours",
        }
        print(json.dumps(out), flush=True)
    if ctx.enabled:
        from representax_b200.parallel.peer import close_peer_groups

        close_peer_groups()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
