"""Packed INT4 base weights with trainable low-rank (LoRA) adapters.

Parity: ``_pack_int4_rows`` / ``_unpack_int4_rows``, ``QuantizedLoRALinear``,
``apply_quantized_lora``, ``merge_quantized_lora`` and
``lora_parameter_filter`` of src/representax/models/adapters.py:30-267.

The storage format is kept identical so adapter bundles interoperate: each
output row has a symmetric bf16 scale ``max|w| / 7`` (stored as its uint16
bit pattern), values are rounded and clipped to [-7, 7], and two 4-bit
two's-complement values share one uint8 with the even column in the low
nibble. ``lora_a [rank, in]`` starts ~ N(0, in^-1/2) (or the configured
scale) and ``lora_b [out, rank]`` at zero, so the adapted model starts equal
to the quantized base. The forward is
``x W_q^T + ((x A^T) B^T) * alpha / rank (+ bias)``.

Models in this package hold linear weights as ``<name>_weight`` parameters;
``apply_quantized_lora`` swaps each matching 2-D weight for a
:class:`QuantizedLoRAWeight` submodule under the same attribute name, and
the models' linear helpers dispatch on it.
"""

from __future__ import annotations

import re

import torch
from torch import nn


def _bf16_bits(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).view(torch.int16).view(torch.uint16) if hasattr(torch, "uint16") else \
        x.to(torch.bfloat16).view(torch.int16)


def _from_bf16_bits(bits: torch.Tensor) -> torch.Tensor:
    return bits.view(torch.int16).view(torch.bfloat16) if bits.dtype != torch.int16 else bits.view(torch.bfloat16)


def pack_int4_rows(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize ``[..., out, in]`` rows to packed int4 plus bf16 row scales."""

    numeric = weight.to(torch.bfloat16)
    maximum = numeric.abs().amax(dim=-1).to(torch.float32)
    scale = torch.where(maximum > 0, maximum / 7.0, torch.ones_like(maximum)).to(torch.bfloat16)
    q = torch.clamp(torch.round(numeric.float() / scale.float()[..., None]), -7, 7).to(torch.int8)
    unsigned = (q & 0x0F).to(torch.uint8)
    if unsigned.shape[-1] % 2:
        unsigned = torch.nn.functional.pad(unsigned, (0, 1))
    pairs = unsigned.reshape(*unsigned.shape[:-1], -1, 2)
    packed = pairs[..., 0] | (pairs[..., 1] << 4)
    return packed.contiguous(), _bf16_bits(scale)


def unpack_int4_rows(packed: torch.Tensor, scale_bits: torch.Tensor, input_size: int) -> torch.Tensor:
    low = packed & 0x0F
    high = packed >> 4
    unsigned = torch.stack((low, high), dim=-1).reshape(*packed.shape[:-1], -1)[..., :input_size].to(torch.int16)
    signed = torch.where(unsigned < 8, unsigned, unsigned - 16)
    scale = _from_bf16_bits(scale_bits)
    return signed.to(torch.bfloat16) * scale[..., None]


class QuantizedLoRAWeight(nn.Module):
    """Frozen packed-int4 weight plus trainable fp32 LoRA factors."""

    def __init__(self, weight: torch.Tensor, *, rank: int, alpha: float, seed: int = 0,
                 initialization_scale: float | None = None) -> None:
        super().__init__()
        out_f, in_f = weight.shape[-2:]
        if rank <= 0 or rank > min(out_f, in_f):
            raise ValueError("adapter rank must fit both linear dimensions")
        if alpha <= 0:
            raise ValueError("adapter alpha must be positive")
        packed, scales = pack_int4_rows(weight.detach())
        self.register_buffer("packed_weight", packed)
        self.register_buffer("scale_bits", scales)
        g = torch.Generator().manual_seed(seed)
        scale = in_f ** -0.5 if initialization_scale is None else initialization_scale
        self.lora_a = nn.Parameter(scale * torch.randn(*weight.shape[:-2], rank, in_f, generator=g))
        self.lora_b = nn.Parameter(torch.zeros(*weight.shape[:-2], out_f, rank))
        self.input_size, self.output_size, self.rank, self.alpha = in_f, out_f, rank, float(alpha)
        self.shape = tuple(weight.shape)

    def base_weight(self) -> torch.Tensor:
        return unpack_int4_rows(self.packed_weight, self.scale_bits, self.input_size)

    def merged_weight(self) -> torch.Tensor:
        return self.base_weight().float() + (self.lora_b @ self.lora_a) * (self.alpha / self.rank)

    def base_weight_bf16(self) -> torch.Tensor:
        """The dequantised base weight (bf16); one kernel on CUDA."""

        if self.packed_weight.is_cuda and self.input_size % 16 == 0 and self.packed_weight.dim() == 2:
            from representax_b200.ops._ext import ext

            out = torch.empty(self.output_size, self.input_size, dtype=torch.bfloat16, device=self.packed_weight.device)
            ext().int4_dequantize(self.packed_weight, self.scale_bits, out)
            return out
        return self.base_weight().to(torch.bfloat16)

    # Expand the packed weight inside the GEMM's main loop instead of
    # dequantising it to a bf16 temporary first. Off by default: on B200 the
    # one-pass dequantisation (a few microseconds, one layer's weight at a
    # time) plus the CTA-pair bf16 GEMM measured faster at every token count
    # tried (128 to 16384 tokens, Qwen3-VL-2B projections), because every M
    # tile re-expands its B tiles and that costs as much issue time as the MMAs.
    mainloop_dequant: bool = False

    def fused_int4(self) -> bool:
        """Whether the tcgen05 GEMM can expand this packed weight in its main
        loop: 16-byte packed rows (in_features % 32) and 16-byte output rows."""

        p = self.packed_weight
        return (p.is_cuda and p.dim() == 2 and self.input_size % 32 == 0 and self.output_size % 8 == 0
                and p.stride(1) == 1 and p.stride(0) % 16 == 0 and p.data_ptr() % 16 == 0
                and self.scale_bits.data_ptr() % 16 == 0)

    def linear_native(self, x: torch.Tensor, bias: torch.Tensor | None = None,
                      residual: torch.Tensor | None = None) -> torch.Tensor:
        """Packed-row bf16 path: ``x W_q^T + bias + residual + ((x A^T) * alpha / r) B^T``.

        The LoRA product is added by the base GEMM's residual epilogue. The
        frozen base weight (only dx flows through it) is dequantised by one
        kernel per use into a bf16 temporary for the tcgen05 GEMM, or, with
        ``mainloop_dequant``, expanded from its packed nibbles inside the
        GEMM's main loop so that no bf16 copy reaches HBM.
        """

        from representax_b200.ops import nn as N

        u = N.linear(x, self.lora_a) * (self.alpha / self.rank)
        lora = N.linear(u, self.lora_b, residual=residual)
        return _FrozenLinearFn.apply(x, self, bias, lora)

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        dtype = x.dtype
        out = torch.nn.functional.linear(x, self.base_weight().to(dtype))
        hidden = torch.nn.functional.linear(x, self.lora_a.to(dtype))
        out = out + torch.nn.functional.linear(hidden, self.lora_b.to(dtype)) * (self.alpha / self.rank)
        if bias is not None:
            out = out + bias.to(dtype)
        return out


class _FrozenLinearFn(torch.autograd.Function):
    """``x W^T (+ b) + residual`` with a frozen weight produced on demand (bf16)."""

    @staticmethod
    def forward(ctx, x, owner, bias, residual):
        from representax_b200.ops import gemm as G
        from representax_b200.ops.functional import compute_view

        x = x.contiguous()
        b = None if bias is None else compute_view(bias)
        if owner.mainloop_dequant and owner.fused_int4():
            # the packed weight is expanded inside the GEMM's main loop
            from representax_b200.ops._ext import ext, status

            y = torch.empty(x.shape[0], owner.output_size, dtype=torch.bfloat16, device=x.device)
            ext().int4_gemm(x, owner.packed_weight, owner.scale_bits, owner.input_size, y, b,
                            None if residual is None else residual.contiguous(), False, status(x.device))
        else:
            y = G.linear_forward(x, owner.base_weight_bf16(), b, residual=residual)
        ctx.owner = owner
        ctx.save_for_backward(bias if bias is not None else torch.empty(0, device=x.device))
        ctx.has_b = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        from representax_b200.ops import gemm as G
        from representax_b200.ops.functional import _colsum_into, _GradSink

        (bias,) = ctx.saved_tensors
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            owner = ctx.owner
            if owner.mainloop_dequant and owner.fused_int4():
                from representax_b200.ops._ext import ext, status

                dx = torch.empty(dy.shape[0], owner.input_size, dtype=torch.bfloat16, device=dy.device)
                ext().int4_gemm(dy, owner.packed_weight, owner.scale_bits, owner.input_size, dx, None, None, True,
                                status(dy.device))
            else:
                dx = G.linear_dgrad(dy, owner.base_weight_bf16())
        sb = _GradSink(bias) if ctx.has_b else None
        if sb is not None:
            _colsum_into(dy, sb)
        return dx, None, (sb.result() if sb is not None else None), dy


def linear(x: torch.Tensor, weight, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x W^T + b`` for a plain weight or a :class:`QuantizedLoRAWeight`."""

    if isinstance(weight, QuantizedLoRAWeight):
        return weight.linear(x, bias)
    return torch.nn.functional.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))


def apply_quantized_lora(model: nn.Module, *, rank: int, alpha: float, seed: int = 0, target_pattern: str = ".*",
                         initialization_scale: float | None = None) -> nn.Module:
    """Quantize matching 2-D ``*_weight`` / ``weight`` parameters and freeze everything else."""

    pattern = re.compile(target_pattern)
    targets = []
    skip = re.compile(r"embed|embeddings\.|\.word$|^word$|position|pos_embed|class_embedding|patch_w$|connector")
    for mod_name, module in model.named_modules():
        for attr, p in list(module._parameters.items()):
            if p is None or p.ndim != 2:
                continue
            full = f"{mod_name}.{attr}" if mod_name else attr
            if skip.search(full):
                continue
            if pattern.fullmatch(full) or pattern.search(full):
                targets.append((module, attr, full))
    if not targets:
        raise ValueError(f"no linear weights match adapter target_pattern {target_pattern!r}")
    for p in model.parameters():
        p.requires_grad_(False)
    for i, (module, attr, _) in enumerate(targets):
        weight = module._parameters.pop(attr)
        adapter = QuantizedLoRAWeight(weight, rank=rank, alpha=alpha, seed=seed + i,
                                      initialization_scale=initialization_scale)
        module.add_module(attr, adapter)
    return model


def merge_quantized_lora(model: nn.Module) -> nn.Module:
    """Replace every adapter by its merged fp32 weight (a plain parameter)."""

    for module in list(model.modules()):
        for name, child in list(module._modules.items()):
            if isinstance(child, QuantizedLoRAWeight):
                del module._modules[name]
                module.register_parameter(name, nn.Parameter(child.merged_weight().detach().float()))
    return model


def lora_parameter_filter(model: nn.Module) -> dict[str, bool]:
    """Trainability of every parameter: only LoRA factors train once adapted."""

    return {name: ("lora_a" in name or "lora_b" in name) for name, _ in model.named_parameters()}


__all__ = ["QuantizedLoRAWeight", "apply_quantized_lora", "linear", "lora_parameter_filter", "merge_quantized_lora",
           "pack_int4_rows", "unpack_int4_rows"]
