"""FP8 linear layers: per-tensor dynamically scaled E4M3 / E5M2 tcgen05 GEMMs.

Forward ``y = x W^T``: x and W quantised to E4M3 (scale = amax / 448), one
``kind::f8f6f4`` GEMM with the scale product applied to the fp32
accumulator. Backward: dy quantised to E5M2 (scale = amax / 57344);
``dx = dy W`` uses W^T re-quantised transposed (E4M3); ``dW += dy^T x`` uses
dy^T (E5M2) and x^T (E4M3) so every operand is K-major; the weight gradient
is accumulated in fp32. Scales never leave the device.

Parity: ``_fp8_linear_dot`` and its VJP (src/representax/precision.py:127-221).
"""

from __future__ import annotations

import torch

from ._ext import ext, status
from .functional import _colsum_into, _GradSink, compute_view

E4M3, E5M2 = 0, 1
EPI_BIAS, EPI_RESID = 1, 8
OUT_BF16, OUT_F32_ATOMIC = 0, 3


def _scaled(x: torch.Tensor, fmt: int, *, transpose: bool, scale_slot: torch.Tensor,
            scratch: torch.Tensor) -> torch.Tensor:
    C = ext()
    C.fp8_scale(x, scale_slot, scratch, fmt == E5M2)
    rows, cols = x.shape
    if transpose:
        # rows become the contraction dimension: pad the row stride to 16 bytes for TMA;
        # the padding is never read (the tensor map's K extent is ``rows``)
        out = torch.empty(cols, (rows + 15) // 16 * 16, dtype=torch.uint8, device=x.device)[:, :rows]
    else:
        out = torch.empty(rows, cols, dtype=torch.uint8, device=x.device)
    C.fp8_quantize(x, scale_slot, out, fmt == E5M2, transpose)
    return out


class LinearFP8Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        C = ext()
        dev = x.device
        wc = compute_view(w)
        scratch = torch.empty(1, dtype=torch.int32, device=dev)
        s_fwd = torch.empty(2, dtype=torch.float32, device=dev)      # [s_x, s_w]
        xq = _scaled(x, E4M3, transpose=False, scale_slot=s_fwd[0:1], scratch=scratch)
        wq = _scaled(wc, E4M3, transpose=False, scale_slot=s_fwd[1:2], scratch=scratch)
        y = torch.empty(x.shape[0], w.shape[0], dtype=torch.bfloat16, device=dev)
        epi = (EPI_BIAS if b is not None else 0) | (EPI_RESID if residual is not None else 0)
        C.gemm_fp8(xq, wq, y, E4M3, E4M3, epi, OUT_BF16, 1.0, s_fwd, None if b is None else compute_view(b),
                   residual, status(dev))
        ctx.save_for_backward(x, w, b if b is not None else torch.empty(0, device=dev))
        ctx.has_b, ctx.has_res = b is not None, residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        x, w, b = ctx.saved_tensors
        dy = dy.contiguous()
        dev = dy.device
        scratch = torch.empty(1, dtype=torch.int32, device=dev)
        scales = torch.empty(4, dtype=torch.float32, device=dev)     # [s_dy, s_w, s_dy, s_x]
        sw = _GradSink(w)
        dx = None
        if ctx.needs_input_grad[0]:
            dyq = _scaled(dy, E5M2, transpose=False, scale_slot=scales[0:1], scratch=scratch)
            wtq = _scaled(compute_view(w), E4M3, transpose=True, scale_slot=scales[1:2], scratch=scratch)
            dx = torch.empty(x.shape, dtype=torch.bfloat16, device=dev)
            C.gemm_fp8(dyq, wtq, dx, E5M2, E4M3, 0, OUT_BF16, 1.0, scales[0:2], None, None, status(dev))
        if sw.wanted:
            dytq = _scaled(dy, E5M2, transpose=True, scale_slot=scales[2:3], scratch=scratch)
            xtq = _scaled(x, E4M3, transpose=True, scale_slot=scales[3:4], scratch=scratch)
            C.gemm_fp8(dytq, xtq, sw.buffer(), E5M2, E4M3, 0, OUT_F32_ATOMIC, 1.0, scales[2:4], None, None,
                       status(dev))
        sb = _GradSink(b) if ctx.has_b else None
        if sb is not None:
            _colsum_into(dy, sb)
        return dx, sw.result(), (sb.result() if sb is not None else None), (dy if ctx.has_res else None)


def fp8_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """8-bit TMA rows must be 16-byte multiples: in_features and out_features % 16 == 0."""

    return x.shape[1] % 16 == 0 and weight.shape[0] % 16 == 0


def linear_fp8(x, weight, bias=None, residual=None):
    return LinearFP8Fn.apply(x.contiguous(), weight, bias, residual)


def quantize_reference(x: torch.Tensor, fmt: int) -> tuple[torch.Tensor, torch.Tensor]:
    """PyTorch statement of the per-tensor quantisation (fake-quantised fp32 values, scale)."""

    dtype = torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2
    maximum = torch.finfo(dtype).max
    xf = x.float()
    scale = torch.clamp(xf.abs().max() / maximum, min=torch.finfo(torch.float32).tiny)
    q = (xf / scale).clamp(-maximum, maximum).to(dtype).float()
    return q, scale


def linear_fp8_reference(x, weight, bias=None):
    """fp32 statement of the fp8 forward (quantise, multiply, rescale)."""

    xq, sx = quantize_reference(x, E4M3)
    wq, sw = quantize_reference(weight, E4M3)
    y = (xq @ wq.T) * (sx * sw)
    if bias is not None:
        y = y + bias.float()
    return y


__all__ = ["LinearFP8Fn", "fp8_supported", "linear_fp8", "linear_fp8_reference", "quantize_reference"]
