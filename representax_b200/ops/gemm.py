"""Python entry points of the tcgen05 GEMM (``csrc/gemm*.cu``).

All shapes follow the storage of the operands: a linear layer's forward is
``A=x [T, K]`` (K-major) times ``B=W [N, K]`` (K-major); its input gradient is
``dy [T, N]`` times ``W`` read MN-major; its weight gradient reads both ``dy``
and ``x`` MN-major, so no transpose is ever materialised.
"""

from __future__ import annotations

import torch

from representax_b200.parallel.fsdp import take_pending

from ._ext import ext, status

EPI_NONE = 0
EPI_BIAS = 1
EPI_GELU = 2
EPI_DGELU = 4
EPI_RESID = 8
EPI_DROP = 16
EPI_COLSUM = 32

OUT_BF16 = 0
OUT_F32 = 1
OUT_F32_ACC = 2
OUT_F32_ATOMIC = 3

# Opt-in per-call timing (``profile_gemms``): None, or a list that collects
# (shape / layout / epilogue key, start event, end event) for every launch.
_PROFILE: list | None = None


def profile_gemms(on: bool) -> list | None:
    """Start (on=True) or stop collecting CUDA-event timings of every GEMM launch;
    stopping returns the collected (key, start, end) records."""

    global _PROFILE
    records, _PROFILE = _PROFILE, ([] if on else None)
    return records


def gemm_table(records: list) -> list[tuple[str, int, float]]:
    """(key, launches, total device ms) per GEMM key, largest first (synchronises)."""

    torch.cuda.synchronize()
    rows: dict[str, list] = {}
    for key, start, end in records:
        r = rows.setdefault(key, [0, 0.0])
        r[0] += 1
        r[1] += start.elapsed_time(end)
    return sorted(((k, n, t) for k, (n, t) in rows.items()), key=lambda x: -x[2])


# Default tile variant for every GEMM (0 = automatic).
GEMM_VARIANT = 0


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    epi: int = EPI_NONE,
    out_mode: int = OUT_BF16,
    alpha: float = 1.0,
    bias: torch.Tensor | None = None,
    aux_in: torch.Tensor | None = None,
    aux_out: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    split_k: int = 0,
    variant: int | None = None,
    dropout: tuple[int, int, float] | None = None,
    colsum: torch.Tensor | None = None,
) -> torch.Tensor:
    """``variant``: 1 = one CTA per 128x256 tile, 2 = CTA pair per 256x256 tile
    (cta_group::2), 0/None = the default (``GEMM_VARIANT``, pair for >= 256 rows).
    ``colsum`` (fp32 [N]): accumulate the output's column sums into it."""

    seed, stream, p = dropout if dropout is not None else (0, 0, 0.0)
    if dropout is not None:
        epi |= EPI_DROP
    if colsum is not None:
        epi |= EPI_COLSUM
    pending = take_pending(b)
    if pending is not None:  # an FSDP weight whose first use in this version is this GEMM
        state, slot = pending
        if not a_mn and not b_mn and colsum is None and aux_in is None and out_mode in (OUT_BF16, OUT_F32):
            shards, shard_numel, offset, ready = state.gemm_gather_args(slot)
            ext().gemm_gather(a, b, out, epi, out_mode, alpha, bias, aux_out, residual, status(out.device), seed,
                              stream, p, shards, shard_numel, offset, ready,
                              GEMM_VARIANT if variant is None else variant)
            return out
        state._gather_slot(slot)
    if _PROFILE is not None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    ext().gemm(
        a, b, out, a_mn, b_mn, epi, out_mode, alpha, bias, aux_in, aux_out, residual,
        status(out.device), split_k, GEMM_VARIANT if variant is None else variant, seed, stream, p, colsum,
    )
    if _PROFILE is not None:
        end.record()
        m = a.shape[1] if a_mn else a.shape[0]
        k = a.shape[0] if a_mn else a.shape[1]
        n = b.shape[1] if b_mn else b.shape[0]
        kind = "wgrad" if (a_mn and b_mn) else ("dgrad" if b_mn else "fwd")
        _PROFILE.append((f"{kind} M{m} N{n} K{k} epi{epi} out{out_mode}", start, end))
    return out


def linear_forward(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    gelu_grad: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    dropout: tuple[int, int, float] | None = None,
) -> torch.Tensor:
    """``y = x W^T (+ b) (-> gelu, storing gelu'(pre-activation) into ``gelu_grad`` for the
    backward) (-> dropout) (+ residual)``.

    ``dropout = (seed, stream, p)`` drops elements of the biased product
    before the residual add (needs bias and residual)."""

    rows, n = x.shape[0], weight.shape[0]
    if out is None:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=x.device)
    epi = EPI_NONE
    if bias is not None:
        epi |= EPI_BIAS
    if gelu_grad is not None:
        epi |= EPI_GELU
    if residual is not None:
        epi |= EPI_RESID
    return gemm(x, weight, out, epi=epi, bias=bias, aux_out=gelu_grad, residual=residual, dropout=dropout)


def linear_dgrad(
    dy: torch.Tensor,
    weight: torch.Tensor,
    *,
    gelu_grad: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    colsum: torch.Tensor | None = None,
) -> torch.Tensor:
    """``dx = dy W`` (times the layer below's saved gelu derivative ``gelu_grad``) (+ residual);
    ``colsum``: also add dx's column sums into it (the lower layer's bias gradient)."""

    rows, k = dy.shape[0], weight.shape[1]
    if out is None:
        out = torch.empty((rows, k), dtype=torch.bfloat16, device=dy.device)
    epi = EPI_NONE
    if gelu_grad is not None:
        epi |= EPI_DGELU
    if residual is not None:
        epi |= EPI_RESID
    return gemm(
        dy, weight, out, b_mn=True, epi=epi, aux_in=gelu_grad, residual=residual, colsum=colsum
    )


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    """``grad += dy^T x`` into an fp32 accumulator (split-K with atomics)."""

    return gemm(dy, x, grad, a_mn=True, b_mn=True, out_mode=OUT_F32_ATOMIC)
