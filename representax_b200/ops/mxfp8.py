"""MXFP8 linear layers: block-scaled E4M3 / E5M2 tcgen05 GEMMs.

Every operand carries one power-of-two scale (UE8M0) per 32 consecutive
values along the contraction dimension, and the tensor core applies the
scales inside the MMA (``kind::mxf8f6f4.block_scale``). Forward
``y = x W^T``: x and W quantised row-wise to E4M3. Backward: dy quantised to
E5M2 both row-wise (for ``dx = dy W``, with W quantised transposed) and
transposed (for ``dW += dy^T x``, with x quantised transposed); the weight
gradient accumulates in fp32 in the GEMM epilogue. One quantiser launch per
tensor writes every layout it needs, with scales in the order the GEMM loads.

Parity: the reference's fp8 linear (src/representax/precision.py:127-221) is
the same E4M3-forward / E5M2-gradient recipe with one per-tensor scale; here
the scale is per 32-value block (the OCP MX layout), selected by
``PrecisionConfig(matrix_dtype="float8_e4m3fn", fp8_scaling="block")``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ._ext import ext, status
from .functional import _colsum_into, _GradSink, compute_view

E4M3, E5M2 = 0, 1
OUT_BF16, OUT_F32, OUT_F32_ACC = 0, 1, 2
FMAX = {E4M3: 448.0, E5M2: 57344.0}


def _scale_bytes(rows: int, k: int) -> int:
    """Size of a scale array: [ceil(k / 128)][ceil(rows / 128) + 1][512]."""

    return (k + 127) // 128 * ((rows + 127) // 128 + 1) * 512


@dataclass
class MXOperand:
    """8-bit data [rows, >= k] (K-major) with its block scales."""

    data: torch.Tensor
    scales: torch.Tensor
    fmt: int
    k: int


def quantize(x: torch.Tensor, fmt: int, *, rowwise: bool = True, transposed: bool = False):
    """bf16 ``x`` [R, C] -> (row-wise operand [R, C] or None, transposed operand [C, R] or None)."""

    x = x.contiguous()
    r, c = x.shape
    dev = x.device
    q = sf = qt = sft = None
    if rowwise:
        q = torch.empty(r, c, dtype=torch.uint8, device=dev)
        sf = torch.zeros(_scale_bytes(r, c), dtype=torch.uint8, device=dev)
    if transposed:
        qt = torch.empty(c, (r + 31) // 32 * 32, dtype=torch.uint8, device=dev)
        sft = torch.zeros(_scale_bytes(c, r), dtype=torch.uint8, device=dev)
    ext().mx_quantize(x, q, sf, qt, sft, fmt == E5M2)
    # the transposed operand contracts over R rounded up to a whole block: the
    # quantiser zero-fills the rows past R, so both sides of a product agree
    return (MXOperand(q, sf, fmt, c) if rowwise else None,
            MXOperand(qt, sft, fmt, (r + 31) // 32 * 32) if transposed else None)


def gemm(a: MXOperand, b: MXOperand, out: torch.Tensor, mode: int = OUT_BF16, bias=None, residual=None) -> None:
    """``out [M, N] (+)= A . B^T`` with both operands block-scaled along K."""

    assert a.k == b.k
    ext().mx_gemm(a.data, a.scales, a.fmt, b.data, b.scales, b.fmt, a.k, out, mode, bias, residual,
                  status(out.device))


class LinearMXFP8Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        dev = x.device
        xq, _ = quantize(x, E4M3)
        wq, _ = quantize(compute_view(w), E4M3)
        y = torch.empty(x.shape[0], w.shape[0], dtype=torch.bfloat16, device=dev)
        gemm(xq, wq, y, OUT_BF16, None if b is None else compute_view(b), residual)
        ctx.save_for_backward(x, w, b if b is not None else torch.empty(0, device=dev))
        ctx.has_b, ctx.has_res = b is not None, residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b = ctx.saved_tensors
        dy = dy.contiguous()
        sw = _GradSink(w)
        need_dx = ctx.needs_input_grad[0]
        dyq, dytq = quantize(dy, E5M2, rowwise=need_dx, transposed=sw.wanted)
        dx = None
        if need_dx:
            _, wtq = quantize(compute_view(w), E4M3, rowwise=False, transposed=True)
            dx = torch.empty(x.shape, dtype=torch.bfloat16, device=dy.device)
            gemm(dyq, wtq, dx, OUT_BF16)
        if sw.wanted:
            _, xtq = quantize(x, E4M3, rowwise=False, transposed=True)
            gemm(dytq, xtq, sw.buffer(), OUT_F32_ACC)
        sb = _GradSink(b) if ctx.has_b else None
        if sb is not None:
            _colsum_into(dy, sb)
        return dx, sw.result(), (sb.result() if sb is not None else None), (dy if ctx.has_res else None)


def mxfp8_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Blocks of 32 along both contraction dimensions (in_features and out_features),
    and 16-byte rows for the transposed token-major operands."""

    return x.shape[1] % 32 == 0 and weight.shape[0] % 32 == 0


def linear_mxfp8(x, weight, bias=None, residual=None):
    return LinearMXFP8Fn.apply(x.contiguous(), weight, bias, residual)


# ------------------------------------------------------------ PyTorch oracle
def quantize_reference(x: torch.Tensor, fmt: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Fake-quantised fp32 values and per-block exponents of a row-wise MX quantisation.

    e = ceil(log2(amax / FMAX)) read from the fp32 bits of amax / FMAX (as the
    kernel does), clamped to [-127, 126]; q = sat(x * 2^-e) in the 8-bit format."""

    dtype = torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2
    fmax = FMAX[fmt]
    xf = x.float()
    r, c = xf.shape
    blocks = xf.reshape(r, c // 32, 32)
    v = blocks.abs().amax(-1) / fmax
    bits = v.contiguous().view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    e = e.clamp(-127, 126)
    q = (blocks * torch.exp2(-e.float())[..., None]).clamp(-fmax, fmax).to(dtype).float()
    return (q * torch.exp2(e.float())[..., None]).reshape(r, c), e


def linear_mxfp8_reference(x, weight, bias=None):
    """fp32 statement of the MXFP8 forward (block fake-quantisation, fp32 product)."""

    xq, _ = quantize_reference(x, E4M3)
    wq, _ = quantize_reference(weight, E4M3)
    y = xq @ wq.T
    if bias is not None:
        y = y + bias.float()
    return y


__all__ = ["LinearMXFP8Fn", "MXOperand", "gemm", "linear_mxfp8", "linear_mxfp8_reference", "mxfp8_supported",
           "quantize", "quantize_reference"]
