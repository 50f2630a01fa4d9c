"""Fused compute + collective kernels on N GPUs of one node.

    torchrun --nproc-per-node N -m representax_b200.bench_comm [--only mnr] [--rows 512]

Cases (config 2 per-rank shapes: 4096 pairs over N ranks, width 768):

* ``mnr_scores_fused``: one launch of the tcgen05 scoring kernel whose stager
  warps pull every peer's candidate rows over NVLink while the tensor cores
  multiply the blocks already staged (fused all-gather + GEMM).
* ``mnr_scores_nccl``: the same result the unfused way: NCCL all_gather of
  the candidate rows, then the same kernel on local memory only.
* ``mnr_backward_fused``: dQ from the staged candidates plus the candidate
  gradient written into the owners' slots by the GEMM epilogue (peer stores),
  device barrier, slot reduction.

Each is timed with CUDA events on the launching stream after warm-up, the
maximum over ranks is reported, and the roofline is the slower of the FLOPs
at the measured bf16 burst peak and the bytes that must cross NVLink at the
measured 770 GB/s per direction per GPU (the split-bf16 scheme issues three
MMAs per product; FLOPs count 2 M N K). Prints one JSON line per case (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def _peak_flops() -> float:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        return 1.59e15


def _time(fn, warmup=5, iters=20) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end) / 1e3 / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def bench_mnr(rows: int, width: int, report) -> None:
    from representax_b200.ops._ext import check_status, ext
    from representax_b200.ops.mnr import split_bf16, tc_gemm, tc_scores
    from representax_b200.parallel.dist import DistContext
    from representax_b200.parallel.peer import peer_group

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = DistContext(rank=rank, world_size=world, local_rank=dev.index)
    group = peer_group(ctx, dev)
    C = ext()
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    q = torch.nn.functional.normalize(torch.randn(rows, width, generator=g), dim=1).to(dev)
    d = torch.nn.functional.normalize(torch.randn(rows, width, generator=g), dim=1).to(dev)
    dbuf = group.cached(("bench_d", rows, width), rows * width)
    dbuf.tensor.copy_(d.reshape(-1))
    slots = group.cached(("bench_slots", rows, width), world * rows * width)
    group.barrier()
    n = world * rows
    flops = 2 * rows * n * width
    remote = (world - 1) * rows * width * 4  # fp32 candidate rows that must cross NVLink into this GPU
    peak = _peak_flops()

    def roofline(t):
        bound = max(flops / peak, remote / (NVLINK_GBS * 1e9))
        return {"ms": t * 1e3, "tflops": flops / t / 1e12, "nvlink_bytes_in": remote,
                "nvlink_gbs": remote / t / 1e9, "roofline_ms": bound * 1e3, "frac_of_roofline": bound / t}

    # fused: staged peer loads inside the scoring kernel
    t = _time(lambda: tc_scores(q, dbuf.peer_ptrs, rows, rank))
    report({"case": "mnr_scores_fused", "world": world, "M": rows, "N": n, "K": width, **roofline(t)})

    # unfused: NCCL all_gather then the same kernel on local rows
    gathered = torch.empty(n, width, device=dev)
    local_ptr = [gathered.data_ptr()]

    def unfused():
        dist.all_gather_into_tensor(gathered, d)
        tc_scores(q, local_ptr, n, 0)

    t = _time(unfused)
    report({"case": "mnr_scores_nccl_allgather_then_gemm", "world": world, "M": rows, "N": n, "K": width,
            **roofline(t)})

    # backward: dQ from staged candidates + routed candidate gradient + barrier + slot reduce
    _, q_split, d_all = tc_scores(q, dbuf.peer_ptrs, rows, rank)
    grad = torch.randn(rows, n, device=dev) * 1e-3
    dq = torch.empty(rows, width, device=dev)
    dd = torch.zeros(rows, width, device=dev)

    def backward():
        group.barrier()  # owners finished reducing the previous round (the forward's barrier in a step)
        gs = split_bf16(grad)
        tc_gemm(gs, False, d_all, True, rows, width, n, out=dq)
        tc_gemm(gs, True, q_split, True, n, width, rows, route=slots.peer_ptrs, route_rows=rows,
                route_offset=rank * rows * width, ldc=width)
        group.barrier()
        C.slot_reduce(slots.tensor, world, dd, False)

    t = _time(backward)
    out_bytes = (world - 1) * rows * width * 4  # candidate-gradient rows sent to their owners
    bound = max(2 * flops / peak, out_bytes / (NVLINK_GBS * 1e9))
    report({"case": "mnr_backward_fused", "world": world, "M": rows, "N": n, "K": width, "ms": t * 1e3,
            "nvlink_bytes_out": out_bytes, "roofline_ms": bound * 1e3, "frac_of_roofline": bound / t})
    torch.cuda.synchronize()
    check_status(dev)


def bench_fsdp(report) -> None:
    """First-use GEMMs of FSDP-sharded BERT-base weights on one GradCache chunk (18432 tokens).

    ``fsdp_gather_gemm_fused``: the weight's flat segments sit in their owners'
    IPC buffers; one tcgen05 launch copies the remote rows into this GPU's cache
    (epilogue warps, peer loads) while the producer starts tiles whose rows are
    in place. ``fsdp_gather_gemm_nccl``: NCCL all_gather of the bf16 weight, then
    the plain GEMM. ``gemm_local``: the GEMM alone on a local weight.
    """

    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import check_status, ext, status
    from representax_b200.parallel.dist import DistContext
    from representax_b200.parallel.peer import peer_group

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    group = peer_group(DistContext(rank=rank, world_size=world, local_rank=dev.index), dev)
    peak = _peak_flops()
    rows = 18432
    ready = torch.zeros(8192, dtype=torch.int32, device=dev)
    for name, n, k in (("qkv", 2304, 768), ("ffn_in", 3072, 768), ("ffn_out", 768, 3072)):
        numel = n * k
        seg = -(-numel // world)
        seg = (seg + 63) // 64 * 64
        owner = group.cached(("bench_fsdp", name), seg, torch.bfloat16)
        g = torch.Generator(device="cpu").manual_seed(11)
        full = (torch.randn(world * seg, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        owner.tensor.copy_(full[rank * seg:(rank + 1) * seg])
        group.barrier()
        cache = torch.empty(world * seg, dtype=torch.bfloat16, device=dev)
        w = cache[:numel].view(n, k)
        x = (torch.randn(rows, k, device=dev) * 0.5).to(torch.bfloat16)
        bias = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        out = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
        st = status(dev)
        flops = 2 * rows * n * k
        remote = (world - 1) * seg * 2

        def fused():
            ext().gemm_gather(x, w, out, G.EPI_BIAS, G.OUT_BF16, 1.0, bias, None, None, st, 0, 0, 0.0,
                              owner.peer_ptrs, seg, 0, ready, 0)

        t = _time(fused)
        bound = max(flops / peak, remote / (NVLINK_GBS * 1e9))
        report({"case": f"fsdp_gather_gemm_fused_{name}", "world": world, "M": rows, "N": n, "K": k,
                "ms": t * 1e3, "tflops": flops / t / 1e12, "nvlink_bytes_in": remote, "roofline_ms": bound * 1e3,
                "frac_of_roofline": bound / t})
        assert torch.equal(w, full[:numel].view(n, k))
        gathered = torch.empty(world * seg, dtype=torch.bfloat16, device=dev)
        wg = gathered[:numel].view(n, k)

        def nccl():
            dist.all_gather_into_tensor(gathered, owner.tensor[:seg])
            G.gemm(x, wg, out, epi=G.EPI_BIAS, bias=bias)

        t = _time(nccl)
        report({"case": f"fsdp_gather_gemm_nccl_{name}", "world": world, "M": rows, "N": n, "K": k,
                "ms": t * 1e3, "tflops": flops / t / 1e12, "roofline_ms": bound * 1e3, "frac_of_roofline": bound / t})
        t = _time(lambda: G.gemm(x, wg, out, epi=G.EPI_BIAS, bias=bias, variant=1))
        report({"case": f"gemm_local_single_cta_{name}", "world": world, "M": rows, "N": n, "K": k,
                "ms": t * 1e3, "tflops": flops / t / 1e12, "frac_of_peak": flops / t / peak})
        t = _time(lambda: G.gemm(x, wg, out, epi=G.EPI_BIAS, bias=bias))
        report({"case": f"gemm_local_pair_{name}", "world": world, "M": rows, "N": n, "K": k,
                "ms": t * 1e3, "tflops": flops / t / 1e12, "frac_of_peak": flops / t / peak})
    torch.cuda.synchronize()
    check_status(dev)


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--only", default="mnr,fsdp")
    parser.add_argument("--rows", type=int, default=None, help="rows per rank (default 4096 / world)")
    parser.add_argument("--width", type=int, default=768)
    parser.add_argument("--out", default=None)
    args = parser.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    import datetime

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    world = dist.get_world_size()
    lines = []

    def report(row):
        if dist.get_rank() == 0:
            lines.append(row)
            print(json.dumps(row), flush=True)

    if "mnr" in args.only.split(","):
        bench_mnr(args.rows or 4096 // world, args.width, report)
    if "fsdp" in args.only.split(","):
        bench_fsdp(report)
    if args.out and dist.get_rank() == 0:
        with open(args.out, "a") as handle:
            for row in lines:
                handle.write(json.dumps(row) + "\n")
    from representax_b200.parallel.peer import close_peer_groups

    close_peer_groups()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
