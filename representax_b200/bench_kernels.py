"""Kernel microbenchmarks: ``python -m representax_b200.bench_kernels``.

Times each hot kernel with CUDA events on the launching stream after warm-up,
flushing L2 between iterations with a 256 MB write, and prints one JSON line
per case with the achieved rate and its fraction of the measured device peaks
(``MEASURED_PEAKS.json`` when present; else 6.65 TB/s and 1.59 PFLOP/s).
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            data = json.load(handle)
        return float(data["hbm_gbs"]) * 1e9, float(data["bf16_tflops"]) * 1e12, "measured"
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15, "fallback"


class Timer:
    def __init__(self, warmup=3, iters=10):
        self.warmup = warmup
        self.iters = iters
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def __call__(self, fn):
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(self.iters):
            self.flush.fill_(1.0)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            torch.cuda.synchronize()
            times.append(start.elapsed_time(end) / 1e3)
        times.sort()
        return times[len(times) // 2]


CASE_FILTER = None


def bench_gemm(timer, hbm, flops_peak, tag, report):
    from representax_b200.ops import gemm as G

    shapes = [
        ("qkv_fwd", 18432, 2304, 768),
        ("ffn1_fwd", 18432, 3072, 768),
        ("ffn2_fwd", 18432, 768, 3072),
        ("square_8k", 8192, 8192, 8192),
    ]
    for name, m, n, k in shapes:
        if CASE_FILTER and CASE_FILTER not in name:
            continue
        a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        b = torch.randn(n, k, device="cuda").to(torch.bfloat16)
        c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        t = timer(lambda: G.gemm(a, b, c))
        t_ref = timer(lambda: torch.matmul(a, b.T))
        fl = 2.0 * m * n * k
        report({"kernel": "gemm_tcgen05_fwd", "case": name, "M": m, "N": n, "K": k, "ms": t * 1e3,
                "tflops": fl / t / 1e12, f"frac_of_{tag}_bf16": fl / t / flops_peak,
                "cublas_ms": t_ref * 1e3})
    for name, t_, n, k in [("qkv", 18432, 2304, 768), ("ffn2", 18432, 768, 3072)]:
        if CASE_FILTER:
            continue
        dy = torch.randn(t_, n, device="cuda").to(torch.bfloat16)
        w = torch.randn(n, k, device="cuda").to(torch.bfloat16)
        x = torch.randn(t_, k, device="cuda").to(torch.bfloat16)
        dx = torch.empty(t_, k, dtype=torch.bfloat16, device="cuda")
        gw = torch.zeros(n, k, device="cuda")
        fl = 2.0 * t_ * n * k
        t = timer(lambda: G.linear_dgrad(dy, w, out=dx))
        report({"kernel": "gemm_tcgen05_dgrad", "case": name, "ms": t * 1e3, "tflops": fl / t / 1e12,
                f"frac_of_{tag}_bf16": fl / t / flops_peak, "cublas_ms": timer(lambda: dy @ w) * 1e3})
        t = timer(lambda: G.linear_wgrad(dy, x, gw))
        report({"kernel": "gemm_tcgen05_wgrad", "case": name, "ms": t * 1e3, "tflops": fl / t / 1e12,
                f"frac_of_{tag}_bf16": fl / t / flops_peak, "cublas_ms": timer(lambda: dy.T @ x) * 1e3})


def bench_attention(timer, hbm, flops_peak, tag, report):
    from representax_b200.ops._ext import ext

    C = ext()
    torch.manual_seed(0)
    batch, heads = 128, 12
    lens = torch.randint(32, 257, (batch,))
    total = int(lens.sum())
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = lens.cumsum(0)
    cu = cu.cuda()
    qkv = torch.randn(total, 3 * 768, device="cuda").to(torch.bfloat16)
    q, k, v = qkv[:, :768], qkv[:, 768:1536], qkv[:, 1536:]
    o = torch.empty(total, 768, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(heads, total, device="cuda")
    fl = float(sum(4 * n * n * 64 * heads for n in lens.tolist()))
    do = torch.randn(total, 768, device="cuda").to(torch.bfloat16)
    dqkv = torch.empty_like(qkv)
    acc = torch.empty(total, 768, device="cuda")
    dvec = torch.empty(heads, total, device="cuda")
    # Minimum DRAM traffic: forward reads Q, K, V and writes O (bf16); backward
    # reads Q, K, V, O, dO and writes dQ, dK, dV (bf16).
    fwd_bytes = 4 * total * 768 * 2
    bwd_bytes = 8 * total * 768 * 2
    for impl in ("tcgen05", "mma_sync"):
        C.set_attention_tcgen05(impl == "tcgen05")
        t = timer(lambda: C.attention_forward(q, k, v, o, lse, cu, 256, heads, heads, 0.125, False, -1, 0, 0, 0.0,
                                              None))
        report({"kernel": "attention_fwd", "impl": impl, "case": "bert_b128_len32-256", "ms": t * 1e3,
                "tflops": fl / t / 1e12, f"frac_of_{tag}_bf16": fl / t / flops_peak,
                f"frac_of_{tag}_hbm": fwd_bytes / t / hbm})
        t = timer(lambda: C.attention_backward(do, q, k, v, o, lse, dqkv[:, :768], dqkv[:, 768:1536],
                                               dqkv[:, 1536:], acc, dvec, cu, 256, heads, heads, 0.125,
                                               False, -1, 0, 0, 0.0, None, None))
        report({"kernel": "attention_bwd", "impl": impl, "case": "bert_b128_len32-256", "ms": t * 1e3,
                "tflops": 2.5 * fl / t / 1e12, f"frac_of_{tag}_bf16": 2.5 * fl / t / flops_peak,
                f"frac_of_{tag}_hbm": bwd_bytes / t / hbm})
    C.set_attention_tcgen05(True)
    # Attention-probability dropout 0.1 (Philox masks regenerated in both passes).
    t = timer(lambda: C.attention_forward(q, k, v, o, lse, cu, 256, heads, heads, 0.125, False, -1, 7, 1, 0.1, None))
    report({"kernel": "attention_fwd", "impl": "tcgen05", "case": "bert_b128_len32-256_dropout0.1", "ms": t * 1e3,
            "tflops": fl / t / 1e12, f"frac_of_{tag}_hbm": fwd_bytes / t / hbm})
    t = timer(lambda: C.attention_backward(do, q, k, v, o, lse, dqkv[:, :768], dqkv[:, 768:1536], dqkv[:, 1536:],
                                           acc, dvec, cu, 256, heads, heads, 0.125, False, -1, 7, 1, 0.1, None,
                                           None))
    report({"kernel": "attention_bwd", "impl": "tcgen05", "case": "bert_b128_len32-256_dropout0.1", "ms": t * 1e3,
            "tflops": 2.5 * fl / t / 1e12, f"frac_of_{tag}_hbm": bwd_bytes / t / hbm})


def bench_norm(timer, hbm, flops_peak, tag, report):
    """LayerNorm forward / backward on one GradCache chunk's rows (18432 =
    128 sequences x 144 tokens, H 768) and on four chunks; the backward also
    sums the producing linear layer's bias gradient, as in the training step."""

    from representax_b200.ops._ext import ext

    C = ext()
    h = 768
    for rows in (18432, 18432 * 4):
        x = torch.randn(rows, h, device="cuda").to(torch.bfloat16)
        g = torch.ones(h, device="cuda", dtype=torch.bfloat16)
        b = torch.zeros(h, device="cuda", dtype=torch.bfloat16)
        y = torch.empty_like(x)
        mean = torch.empty(rows, device="cuda")
        rstd = torch.empty(rows, device="cuda")
        t = timer(lambda: C.norm_forward(x, g, b, y, mean, rstd, 1e-12, False))
        by = 2 * rows * h * 2
        report({"kernel": "layernorm_fwd", "rows": rows, "H": h, "ms": t * 1e3, "gbs": by / t / 1e9,
                f"frac_of_{tag}_hbm": by / t / hbm})
        dx = torch.empty_like(x)
        dg = torch.zeros(h, device="cuda")
        db = torch.zeros(h, device="cuda")
        dbp = torch.zeros(h, device="cuda")
        t = timer(lambda: C.norm_backward(y, x, mean, rstd, g, dx, dg, db, dbp, False))
        by = 3 * rows * h * 2
        report({"kernel": "layernorm_bwd", "rows": rows, "H": h, "ms": t * 1e3, "gbs": by / t / 1e9,
                f"frac_of_{tag}_hbm": by / t / hbm})
    # bias-gradient column sums of a QKV-shaped gradient (one GradCache chunk)
    g_qkv = torch.randn(18432, 2304, device="cuda").to(torch.bfloat16)
    acc = torch.zeros(2304, device="cuda")
    t = timer(lambda: C.colsum_accumulate(g_qkv, acc))
    by = g_qkv.numel() * 2
    report({"kernel": "colsum", "rows": 18432, "cols": 2304, "ms": t * 1e3, "gbs": by / t / 1e9,
            f"frac_of_{tag}_hbm": by / t / hbm})


def bench_mnr(timer, hbm, flops_peak, tag, report):
    """MNR similarity products (config 2: 4096 pairs, width 768).

    ``scores`` is the fused staging + tcgen05 scoring kernel; with ``owners`` > 1
    the candidate rows sit in that many separate buffers (a per-rank slice of
    an N-GPU run emulated on one GPU: staging, readiness counters and the
    owner-rotated tile order, but local instead of NVLink traffic). FLOPs are
    counted as 2 M N K (the split-bf16 scheme issues three MMAs per product).
    """

    from representax_b200.ops._ext import ext
    from representax_b200.ops.mnr import split_bf16, tc_gemm, tc_scores

    C = ext()
    width = 768
    for rows, owners, cand_rows in ((4096, 1, 4096), (512, 8, 512)):
        q = torch.nn.functional.normalize(torch.randn(rows, width, device="cuda"), dim=1)
        cands = [torch.nn.functional.normalize(torch.randn(cand_rows, width, device="cuda"), dim=1)
                 for _ in range(owners)]
        ptrs = [c.data_ptr() for c in cands]
        n = owners * cand_rows
        t = timer(lambda: tc_scores(q, ptrs, cand_rows, 0))
        flops = 2 * rows * n * width
        report({"kernel": "mnr_scores_tc", "M": rows, "N": n, "K": width, "owners": owners, "ms": t * 1e3,
                "tflops": flops / t / 1e12, f"frac_of_{tag}_bf16": flops / t / flops_peak})
        scores, qs, ds = tc_scores(q, ptrs, cand_rows, 0)
        g = torch.randn(rows, n, device="cuda") * 1e-3
        gs = split_bf16(g)
        dq = torch.empty(rows, width, device="cuda")
        dd = torch.empty(n, width, device="cuda")
        t = timer(lambda: tc_gemm(gs, False, ds, True, rows, width, n, out=dq))
        report({"kernel": "mnr_dq_tc", "M": rows, "N": width, "K": n, "ms": t * 1e3,
                "tflops": flops / t / 1e12, f"frac_of_{tag}_bf16": flops / t / flops_peak})
        t = timer(lambda: tc_gemm(gs, True, qs, True, n, width, rows, out=dd))
        report({"kernel": "mnr_dd_tc", "M": n, "N": width, "K": rows, "ms": t * 1e3,
                "tflops": flops / t / 1e12, f"frac_of_{tag}_bf16": flops / t / flops_peak})
        t = timer(lambda: split_bf16(g))
        by = g.numel() * 8
        report({"kernel": "mnr_split", "elements": g.numel(), "ms": t * 1e3, "gbs": by / t / 1e9,
                f"frac_of_{tag}_hbm": by / t / hbm})
        if owners == 1:  # the fp32 CUDA-core GEMM it replaces
            out = torch.empty(rows, n, device="cuda")
            cat = torch.cat(cands)
            t = timer(lambda: C.sgemm(q, False, cat, False, out, 1.0, False))
            report({"kernel": "mnr_scores_simt_fp32", "M": rows, "N": n, "K": width, "ms": t * 1e3,
                    "tflops": flops / t / 1e12})
            ref = q.double() @ cat.double().T
            report({"check": "mnr_scores_tc_max_abs_err_vs_fp64",
                    "value": (scores.double() - ref).abs().max().item()})


def bench_pool(timer, hbm, flops_peak, tag, report):
    """Mean pooling + L2 normalisation of one GradCache chunk (128 rows, 18432 packed tokens)."""

    from representax_b200.ops._ext import ext

    C = ext()
    h, rows = 768, 128
    lens = torch.full((rows,), 18432 // rows, dtype=torch.int32)
    cu = torch.zeros(rows + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    cu = cu.cuda()
    x = torch.randn(int(cu[-1]), h, device="cuda").to(torch.bfloat16)
    out = torch.empty(rows, h, device="cuda")
    norm = torch.empty(rows, device="cuda")
    t = timer(lambda: C.pool_forward(x, cu, out, norm, 0, True))
    by = x.numel() * 2
    report({"kernel": "pool_mean_fwd", "tokens": x.shape[0], "H": h, "ms": t * 1e3, "gbs": by / t / 1e9,
            f"frac_of_{tag}_hbm": by / t / hbm})
    g = torch.randn(rows, h, device="cuda")
    dh = torch.empty_like(x)
    t = timer(lambda: C.pool_backward(g, out, norm, cu, dh, 0, True))
    report({"kernel": "pool_mean_bwd", "tokens": x.shape[0], "H": h, "ms": t * 1e3, "gbs": by / t / 1e9,
            f"frac_of_{tag}_hbm": by / t / hbm})


def bench_mxfp8(timer, hbm, flops_peak, tag, report):
    """Block-scaled MXFP8 GEMM (tcgen05 kind::mxf8f6f4.block_scale) beside the
    per-tensor fp8 and bf16 tcgen05 GEMMs on the same shapes, plus the quantiser.
    Fractions are of the measured bf16 peak (nominal dense fp8 is twice bf16)."""

    from representax_b200.ops import gemm as G
    from representax_b200.ops import mxfp8 as MX
    from representax_b200.ops._ext import ext, status

    C = ext()
    for name, m, n, k in [("qkv", 18432, 2304, 768), ("ffn2", 18432, 768, 3072), ("square_8k", 8192, 8192, 8192)]:
        a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        b = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
        aq, _ = MX.quantize(a, MX.E4M3)
        bq, _ = MX.quantize(b, MX.E4M3)
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        fl = 2.0 * m * n * k
        t = timer(lambda: MX.gemm(aq, bq, y))
        t_q = timer(lambda: MX.quantize(a, MX.E4M3))
        # per-tensor fp8 on the same operands' bits (scales 1)
        ones = torch.ones(2, device="cuda")
        t_pt = timer(lambda: C.gemm_fp8(aq.data, bq.data, y, 0, 0, 0, 0, 1.0, ones, None, None, status(y.device)))
        t_bf = timer(lambda: G.gemm(a, b, y))
        report({"kernel": "mxfp8_gemm", "case": name, "M": m, "N": n, "K": k, "ms": t * 1e3,
                "tflops": fl / t / 1e12, f"frac_of_{tag}_bf16": fl / t / flops_peak,
                "fp8_per_tensor_ms": t_pt * 1e3, "bf16_tcgen05_ms": t_bf * 1e3,
                "quantize_A_ms": t_q * 1e3, "quantize_A_gbs": (a.numel() * 3 + a.numel() / 16) / t_q / 1e9})
    # hardest-negative mining: 8192 anchors x 8192 candidates, width 768
    from representax_b200.ops.mnr import hardest_candidates

    q = torch.randn(8192, 768, device="cuda")
    d = torch.randn(8192, 768, device="cuda")
    t = timer(lambda: hardest_candidates(q, d))

    def torch_mining():
        qn = torch.nn.functional.normalize(q, dim=1)
        dn = torch.nn.functional.normalize(d, dim=1)
        for s0 in range(0, 8192, 1024):
            sc = qn[s0:s0 + 1024] @ dn.T
            sc[torch.arange(1024, device="cuda"), torch.arange(s0, s0 + 1024, device="cuda")] = float("-inf")
            sc.argmax(1)

    report({"kernel": "mining_argmax_tcgen05", "M": 8192, "N": 8192, "K": 768, "ms": t * 1e3,
            "torch_fp32_chunked_ms": timer(torch_mining) * 1e3,
            "note": "split-bf16 scores (3 MMAs per product) reduced to a row argmax in the epilogue"})


def bench_int4(timer, hbm, flops_peak, tag, report):
    """Frozen INT4 base weight (QLoRA): the tcgen05 GEMM that expands packed
    nibbles in its main loop, beside dequantise-to-HBM + bf16 tcgen05 GEMM, on
    Qwen3-VL-2B-like projections (hidden 2048, MLP 6144), forward and dgrad."""

    from representax_b200.models.adapters import QuantizedLoRAWeight
    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import ext, status

    C = ext()
    st = status(torch.device("cuda", 0))
    cases = [("qkv", t, 4096, 2048) for t in (128, 512, 2048, 4096, 16384)]
    cases += [("up", 16384, 6144, 2048), ("down", 16384, 2048, 6144), ("down", 1024, 2048, 6144)]
    for name, t_rows, n, k in cases:
        if CASE_FILTER and CASE_FILTER not in f"{name}_t{t_rows}":
            continue
        q = QuantizedLoRAWeight(torch.randn(n, k) * 0.05, rank=16, alpha=32.0, seed=0).to("cuda")
        x = torch.randn(t_rows, k, device="cuda").to(torch.bfloat16)
        dy = torch.randn(t_rows, n, device="cuda").to(torch.bfloat16)
        y = torch.empty(t_rows, n, dtype=torch.bfloat16, device="cuda")
        dx = torch.empty(t_rows, k, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(n, k, dtype=torch.bfloat16, device="cuda")
        fl = 2.0 * t_rows * n * k
        t_f = timer(lambda: C.int4_gemm(x, q.packed_weight, q.scale_bits, k, y, None, None, False, st))
        t_d = timer(lambda: C.int4_gemm(dy, q.packed_weight, q.scale_bits, k, dx, None, None, True, st))

        def unfused_fwd():
            C.int4_dequantize(q.packed_weight, q.scale_bits, w)
            G.gemm(x, w, y)

        def unfused_dgrad():
            C.int4_dequantize(q.packed_weight, q.scale_bits, w)
            G.linear_dgrad(dy, w, out=dx)

        report({"kernel": "int4_gemm", "case": name, "T": t_rows, "N": n, "K": k, "fwd_ms": t_f * 1e3,
                "fwd_tflops": fl / t_f / 1e12, f"fwd_frac_of_{tag}_bf16": fl / t_f / flops_peak,
                "dgrad_ms": t_d * 1e3, "dgrad_tflops": fl / t_d / 1e12,
                "dequant_then_gemm_fwd_ms": timer(unfused_fwd) * 1e3,
                "dequant_then_gemm_dgrad_ms": timer(unfused_dgrad) * 1e3})


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--only", default="gemm,attention,norm")
    parser.add_argument("--out", default=None)
    parser.add_argument("--case", default=None, help="run only GEMM cases whose name contains this")
    args = parser.parse_args(argv)
    global CASE_FILTER
    CASE_FILTER = args.case
    hbm, flops_peak, tag = _peaks()
    timer = Timer()
    rows = []

    def report(row):
        rows.append(row)
        print(json.dumps(row), flush=True)

    selected = args.only.split(",")
    if "gemm" in selected:
        bench_gemm(timer, hbm, flops_peak, tag, report)
    if "attention" in selected:
        bench_attention(timer, hbm, flops_peak, tag, report)
    if "norm" in selected:
        bench_norm(timer, hbm, flops_peak, tag, report)
    if "mnr" in selected:
        bench_mnr(timer, hbm, flops_peak, tag, report)
    if "pool" in selected:
        bench_pool(timer, hbm, flops_peak, tag, report)
    if "mxfp8" in selected:
        bench_mxfp8(timer, hbm, flops_peak, tag, report)
    if "int4" in selected:
        bench_int4(timer, hbm, flops_peak, tag, report)
    from representax_b200.ops._ext import check_status

    torch.cuda.synchronize()
    check_status(torch.device("cuda", 0))
    if args.out:
        with open(args.out, "w") as handle:
            for row in rows:
                handle.write(json.dumps(row) + "\n")


if __name__ == "__main__":
    main()
