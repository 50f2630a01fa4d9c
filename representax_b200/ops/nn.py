"""Packed-row building blocks shared by the encoder and decoder families.

Every op takes packed token rows (``[T, features]``, sequences delimited by
``cu_seqlens``) and dispatches on the input: bf16 CUDA tensors run the
sm_100a extension kernels (tcgen05 GEMMs, fused RoPE/q-k-norm, packed flash
attention with windows / causal / GQA, fused norms, gated activations) and
write parameter gradients into fp32 accumulators (``param.main_grad`` when
the parameter lives in a flat store); anything else runs the plain PyTorch
statement of the same math, which is also the numerics oracle in tests.

Parity: the shared components of src/representax/models/components.py
(Linear, LayerNorm/RMSNorm, attention, activations), RoPE / M-RoPE of
src/representax/models/qwen3_vl/text.py:30-61 and
src/representax/models/modernvbert/model.py:82-112.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import gemm as G
from ._ext import ext
from .functional import _colsum_into, _GradSink, compute_view

ACT_CODES = {"gelu": 0, "gelu_erf": 0, "gelu_pytorch_tanh": 1, "gelu_tanh": 1, "silu": 2, "swish": 2,
             "quick_gelu": 3}


def native(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16


def weight_as(param: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """The parameter in the compute dtype of ``x`` (the bf16 copy on the native path)."""

    return compute_view(param) if native(x) else param.to(x.dtype)


@dataclass
class Segments:
    """Sequence boundaries of packed rows (host list + device int32 tensor)."""

    cu_host: list[int]
    cu_seqlens: torch.Tensor

    @classmethod
    def from_lengths(cls, lengths, device) -> "Segments":
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + int(n))
        return cls(cu, torch.tensor(cu, dtype=torch.int32, device=device))

    @property
    def max_len(self) -> int:
        return max((b - a for a, b in zip(self.cu_host, self.cu_host[1:])), default=0)

    @property
    def total(self) -> int:
        return self.cu_host[-1]

    @property
    def batch(self) -> int:
        return len(self.cu_host) - 1

    def lengths(self) -> list[int]:
        return [b - a for a, b in zip(self.cu_host, self.cu_host[1:])]


# ------------------------------------------------------------------ linear
class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        y = G.linear_forward(x, compute_view(w, fused_gather=True), None if b is None else compute_view(b),
                             residual=residual)
        ctx.save_for_backward(x, w, b if b is not None else torch.empty(0, device=x.device))
        ctx.has_b, ctx.has_res = b is not None, residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b = ctx.saved_tensors
        dy = dy.contiguous()
        sw = _GradSink(w)
        if sw.wanted:
            G.linear_wgrad(dy, x, sw.buffer())
        sb = _GradSink(b) if ctx.has_b else None
        if sb is not None:
            _colsum_into(dy, sb)
        dx = G.linear_dgrad(dy, compute_view(w)) if ctx.needs_input_grad[0] else None
        return dx, sw.result(), (sb.result() if sb is not None else None), (dy if ctx.has_res else None)


def _fp8_matrices() -> bool:
    from representax_b200.precision import active_policy

    return active_policy().matrix_dtype == torch.float8_e4m3fn


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           residual: torch.Tensor | None = None) -> torch.Tensor:
    """``x W^T (+ b) (+ residual)``; W in the Hugging Face ``[out, in]`` layout.

    Under a precision policy whose matrix dtype is ``float8_e4m3fn`` the
    native path runs the per-tensor-scaled FP8 GEMMs of ``ops.fp8``, or the
    block-scaled MXFP8 GEMMs of ``ops.mxfp8`` when the policy asks for block
    scaling."""

    from representax_b200.models.adapters import QuantizedLoRAWeight

    if isinstance(weight, QuantizedLoRAWeight):
        if native(x) and x.shape[1] % 16 == 0 and weight.output_size % 8 == 0:
            return weight.linear_native(x.contiguous(), bias, residual)
        y = weight.linear(x, bias)
        return y if residual is None else y + residual
    if native(x) and _fp8_matrices():
        from representax_b200.precision import active_policy

        if active_policy().fp8_block_scaled:
            from .mxfp8 import linear_mxfp8, mxfp8_supported

            if mxfp8_supported(x, weight):
                return linear_mxfp8(x, weight, bias, residual)
        else:
            from .fp8 import fp8_supported, linear_fp8

            if fp8_supported(x, weight):
                return linear_fp8(x, weight, bias, residual)
    if native(x) and x.shape[1] % 8 == 0 and weight.shape[0] % 8 == 0:
        return _LinearFn.apply(x.contiguous(), weight, bias, residual)
    y = torch.nn.functional.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))
    return y if residual is None else y + residual


# ------------------------------------------------------------------- norms
class _NormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, eps, rms):
        C = ext()
        rows = x.shape[0]
        y = torch.empty_like(x)
        mean = None if rms else torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        C.norm_forward(x, compute_view(gamma), None if beta is None else compute_view(beta), y, mean, rstd, eps, rms)
        empty = torch.empty(0, device=x.device)
        ctx.save_for_backward(x, empty if mean is None else mean, rstd, gamma, empty if beta is None else beta)
        ctx.rms, ctx.has_beta = rms, beta is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        x, mean, rstd, gamma, beta = ctx.saved_tensors
        sg = _GradSink(gamma)
        sb = _GradSink(beta) if ctx.has_beta else None
        dx = torch.empty_like(x)
        C.norm_backward(dy.contiguous(), x, None if ctx.rms else mean, rstd, compute_view(gamma), dx,
                        sg.buffer() if sg.wanted else None,
                        sb.buffer() if (sb is not None and sb.wanted) else None, None, ctx.rms)
        return dx, sg.result(), (sb.result() if sb is not None else None), None, None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, eps: float) -> torch.Tensor:
    if native(x) and x.shape[1] % 8 == 0 and x.shape[1] <= 2048:
        return _NormFn.apply(x.contiguous(), weight, bias, eps, False)
    y = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), weight.float(),
                                       None if bias is None else bias.float(), eps)
    return y.to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if native(x) and x.shape[1] % 8 == 0 and x.shape[1] <= 2048:
        return _NormFn.apply(x.contiguous(), weight, None, eps, True)
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return y.to(x.dtype)


# -------------------------------------------------------------------- RoPE
def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    """``theta^(-2i/D)`` for i < D/2, computed in float64 then rounded once."""

    i = torch.arange(0, head_dim, 2, dtype=torch.float64)
    return (1.0 / theta ** (i / head_dim)).to(torch.float32).to(device)


def mrope_axis_table(head_dim: int, sections: tuple[int, ...], *, interleaved: bool) -> list[int]:
    """Axis (0 = temporal, 1 = height, 2 = width) read by each frequency.

    Interleaved (Qwen3-VL): frequency f takes H when f % 3 == 1 and
    f < 3 * sections[1], W when f % 3 == 2 and f < 3 * sections[2], else T.
    Sectioned (Qwen2.5-Omni / Qwen2-VL): contiguous runs of sections[0] T,
    sections[1] H and sections[2] W frequencies.
    """

    half = head_dim // 2
    if interleaved:
        table = [0] * half
        for axis in (1, 2):
            for f in range(axis, min(half, 3 * sections[axis]), 3):
                table[f] = axis
        return table
    if sum(sections) != half:
        raise ValueError("M-RoPE sections must sum to head_dim / 2")
    table = []
    for axis, n in enumerate(sections):
        table += [axis] * n
    return table


def _rope_reference(x, pos, axis_of, inv_freq, heads, norm_w, eps):
    T = x.shape[0]
    D = x.shape[1] // heads
    v = x.float().reshape(T, heads, D)
    if norm_w is not None:
        v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
    if pos.shape[0] > 1:
        p = pos.float()[torch.as_tensor(axis_of, device=x.device).long()].T  # [T, D/2]
    else:
        p = pos[0].float()[:, None].expand(T, D // 2)
    ang = p * inv_freq.to(x.device)[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    a, b = v[..., : D // 2], v[..., D // 2:]
    out = torch.cat([a * cos - b * sin, b * cos + a * sin], -1)
    return out.reshape(T, heads * D).to(x.dtype)


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, norm_w, pos, axis_of, inv_freq, heads, eps):
        C = ext()
        y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        w = None if norm_w is None else norm_w.float()
        C.rope_forward(x, y, pos, axis_of, inv_freq, heads, w, eps)
        ctx.save_for_backward(x if norm_w is not None else torch.empty(0, device=x.device),
                              norm_w if norm_w is not None else torch.empty(0, device=x.device), pos,
                              axis_of if axis_of is not None else torch.empty(0, device=x.device), inv_freq)
        ctx.meta = (heads, eps, norm_w is not None, axis_of is not None, x.shape)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        x, norm_w, pos, axis_of, inv_freq = ctx.saved_tensors
        heads, eps, has_norm, has_axis, shape = ctx.meta
        dx = torch.empty(shape, dtype=dy.dtype, device=dy.device)
        sw = _GradSink(norm_w) if has_norm else None
        dw = None
        if sw is not None:
            dw = sw.buffer() if sw.wanted else torch.zeros(norm_w.shape, dtype=torch.float32, device=dy.device)
        C.rope_backward(dy.contiguous(), dx, x if has_norm else None, pos, axis_of if has_axis else None, inv_freq,
                        heads, norm_w.float() if has_norm else None, eps, dw)
        return dx, (sw.result() if sw is not None else None), None, None, None, None, None


def rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, heads: int, *,
         axis_of: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
         eps: float = 1e-6) -> torch.Tensor:
    """Rotate-half RoPE of ``x`` ([T, heads*D]) at int32 positions ``pos`` ([axes, T]).

    ``norm_weight`` applies a per-head RMSNorm first (Qwen3 q/k norm).
    """

    if pos.dim() == 1:
        pos = pos[None]
    D = x.shape[1] // heads
    if native(x) and D in (64, 128):
        axis = None if pos.shape[0] == 1 else axis_of.to(device=x.device, dtype=torch.int32).contiguous()
        return _RopeFn.apply(x, norm_weight, pos.to(device=x.device, dtype=torch.int32).contiguous(),
                             axis, inv_freq.to(x.device).float().contiguous(), heads, eps)
    return _rope_reference(x, pos, axis_of, inv_freq, heads, norm_weight, eps)


# --------------------------------------------------------------- attention
class _AttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_len, heads, kv_heads, scale, causal, window):
        C = ext()
        T = q.shape[0]
        o = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
        lse = torch.empty(heads, T, dtype=torch.float32, device=q.device)
        C.attention_forward(q, k, v, o, lse, cu_seqlens, max_len, heads, kv_heads, scale, causal, window, 0, 0, 0.0, None)
        ctx.save_for_backward(q, k, v, o, lse, cu_seqlens)
        ctx.meta = (max_len, heads, kv_heads, scale, causal, window)
        return o

    @staticmethod
    def backward(ctx, do):
        C = ext()
        q, k, v, o, lse, cu = ctx.saved_tensors
        max_len, heads, kv_heads, scale, causal, window = ctx.meta
        T = q.shape[0]
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dq_acc = torch.empty(T, q.shape[1], dtype=torch.float32, device=q.device)
        dvec = torch.empty(heads, T, dtype=torch.float32, device=q.device)
        C.attention_backward(do.contiguous(), q, k, v, o, lse, dq, dk, dv, dq_acc, dvec, cu, max_len, heads, kv_heads,
                             scale, causal, window, 0, 0, 0.0, None, None)
        return dq, dk, dv, None, None, None, None, None, None, None


def _attention_reference(q, k, v, seg: Segments, heads, kv_heads, scale, causal, window, bias=None):
    D = q.shape[1] // heads
    out = torch.empty_like(q)
    rep = heads // kv_heads
    for b, (a, e) in enumerate(zip(seg.cu_host, seg.cu_host[1:])):
        n = e - a
        if n == 0:
            continue
        qq = q[a:e].float().reshape(n, heads, D).transpose(0, 1)
        kk = k[a:e].float().reshape(n, kv_heads, D).transpose(0, 1).repeat_interleave(rep, 0)
        vv = v[a:e].float().reshape(n, kv_heads, D).transpose(0, 1).repeat_interleave(rep, 0)
        s = qq @ kk.transpose(-1, -2) * scale
        if bias is not None:
            s = s + bias(b, n)
        i = torch.arange(n, device=q.device)
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device)
        if causal:
            mask &= i[None, :] <= i[:, None]
        if window >= 0:
            mask &= (i[None, :] - i[:, None]).abs() <= window
        s = s.masked_fill(~mask, float("-inf"))
        out[a:e] = (torch.softmax(s, -1) @ vv).transpose(0, 1).reshape(n, heads * D).to(q.dtype)
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seg: Segments, *, heads: int,
              kv_heads: int | None = None, causal: bool = False, window: int = -1,
              scale: float | None = None) -> torch.Tensor:
    """Packed multi-head attention; ``window`` >= 0 keeps keys with |i - j| <= window."""

    kv_heads = kv_heads or heads
    D = q.shape[1] // heads
    scale = D ** -0.5 if scale is None else scale
    if native(q) and D in (64, 128):
        return _AttentionFn.apply(q, k, v, seg.cu_seqlens, seg.max_len, heads, kv_heads, scale, causal, window)
    return _attention_reference(q, k, v, seg, heads, kv_heads, scale, causal, window)


class _QKVAttentionFn(torch.autograd.Function):
    """RoPE (+ q/k RMSNorm) on the q/k slices of a fused projection, attention,
    and a backward that writes one ``dqkv`` buffer (no per-slice gradients)."""

    @staticmethod
    def forward(ctx, qkv, q_norm, k_norm, cu_seqlens, max_len, heads, kv_heads, scale, causal, window, pos, axis_of,
                inv_freq, eps):
        C = ext()
        T, width = qkv.shape
        D = width // (heads + 2 * kv_heads)
        qd, kd = heads * D, kv_heads * D
        q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
        if pos is not None:
            q_r = torch.empty(T, qd, dtype=qkv.dtype, device=qkv.device)
            k_r = torch.empty(T, kd, dtype=qkv.dtype, device=qkv.device)
            C.rope_forward(q, q_r, pos, axis_of, inv_freq, heads, None if q_norm is None else q_norm.float(), eps)
            C.rope_forward(k, k_r, pos, axis_of, inv_freq, kv_heads, None if k_norm is None else k_norm.float(), eps)
        else:
            q_r, k_r = q, k
        o = torch.empty(T, qd, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(heads, T, dtype=torch.float32, device=qkv.device)
        C.attention_forward(q_r, k_r, v, o, lse, cu_seqlens, max_len, heads, kv_heads, scale, causal, window, 0, 0, 0.0, None)
        e = torch.empty(0, device=qkv.device)
        ctx.save_for_backward(qkv, q_r, k_r, o, lse, cu_seqlens, e if q_norm is None else q_norm,
                              e if k_norm is None else k_norm, e if pos is None else pos,
                              e if axis_of is None else axis_of, e if inv_freq is None else inv_freq)
        ctx.meta = (max_len, heads, kv_heads, scale, causal, window, eps, q_norm is not None, k_norm is not None,
                    pos is not None, axis_of is not None, D)
        return o

    @staticmethod
    def backward(ctx, do):
        C = ext()
        qkv, q_r, k_r, o, lse, cu, q_norm, k_norm, pos, axis_of, inv_freq = ctx.saved_tensors
        max_len, heads, kv_heads, scale, causal, window, eps, has_qn, has_kn, has_pos, has_axis, D = ctx.meta
        T = qkv.shape[0]
        qd, kd = heads * D, kv_heads * D
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = dqkv[:, :qd], dqkv[:, qd:qd + kd], dqkv[:, qd + kd:]
        dq_acc = torch.empty(T, qd, dtype=torch.float32, device=qkv.device)
        dvec = torch.empty(heads, T, dtype=torch.float32, device=qkv.device)
        C.attention_backward(do.contiguous(), q_r, k_r, qkv[:, qd + kd:], o, lse, dq, dk, dv, dq_acc, dvec, cu,
                             max_len, heads, kv_heads, scale, causal, window, 0, 0, 0.0, None, None)
        grads = []
        if has_pos:
            axis = axis_of if has_axis else None
            for sl, x, nw, has_n, nh in ((dq, qkv[:, :qd], q_norm, has_qn, heads),
                                         (dk, qkv[:, qd:qd + kd], k_norm, has_kn, kv_heads)):
                sink = _GradSink(nw) if has_n else None
                dw = None
                if sink is not None:
                    dw = sink.buffer() if sink.wanted else torch.zeros(nw.shape, dtype=torch.float32,
                                                                        device=qkv.device)
                C.rope_backward(sl, sl, x if has_n else None, pos, axis, inv_freq, nh,
                                nw.float() if has_n else None, eps, dw)
                grads.append(sink.result() if sink is not None else None)
        else:
            grads = [None, None]
        return (dqkv, grads[0], grads[1]) + (None,) * 11


def qkv_attention(qkv: torch.Tensor, seg: Segments, *, heads: int, kv_heads: int | None = None,
                  pos: torch.Tensor | None = None, inv_freq: torch.Tensor | None = None,
                  axis_of: torch.Tensor | None = None, q_norm: torch.Tensor | None = None,
                  k_norm: torch.Tensor | None = None, norm_eps: float = 1e-6, causal: bool = False,
                  window: int = -1, scale: float | None = None) -> torch.Tensor:
    """Attention over a fused ``[T, (heads + 2 kv_heads) * D]`` projection.

    With ``pos``/``inv_freq`` the q and k slices are rotated first (after a
    per-head RMSNorm when ``q_norm``/``k_norm`` are given).
    """

    kv_heads = kv_heads or heads
    D = qkv.shape[1] // (heads + 2 * kv_heads)
    scale = D ** -0.5 if scale is None else scale
    if pos is not None and pos.dim() == 1:
        pos = pos[None]
    if native(qkv) and D in (64, 128):
        p = None if pos is None else pos.to(device=qkv.device, dtype=torch.int32).contiguous()
        a = None
        if p is not None and p.shape[0] > 1:
            a = axis_of.to(device=qkv.device, dtype=torch.int32).contiguous()
        f = None if inv_freq is None else inv_freq.to(qkv.device).float().contiguous()
        return _QKVAttentionFn.apply(qkv.contiguous(), q_norm, k_norm, seg.cu_seqlens, seg.max_len, heads, kv_heads,
                                     scale, causal, window, p, a, f, norm_eps)
    qd, kd = heads * D, kv_heads * D
    q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
    if pos is not None:
        q = _rope_reference(q, pos, axis_of, inv_freq, heads, q_norm, norm_eps)
        k = _rope_reference(k, pos, axis_of, inv_freq, kv_heads, k_norm, norm_eps)
    return _attention_reference(q, k, v, seg, heads, kv_heads, scale, causal, window)


# ------------------------------------------------------------- activations
class _ActFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, code, gated):
        C = ext()
        width = z.shape[1] // 2 if gated else z.shape[1]
        y = torch.empty(z.shape[0], width, dtype=z.dtype, device=z.device)
        C.activation_forward(z, y, code, gated)
        ctx.save_for_backward(z)
        ctx.meta = (code, gated)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        (z,) = ctx.saved_tensors
        code, gated = ctx.meta
        dz = torch.empty_like(z)
        C.activation_backward(dy.contiguous(), z, dz, code, gated)
        return dz, None, None


def _act_reference(x: torch.Tensor, name: str) -> torch.Tensor:
    if name in ("gelu", "gelu_erf"):
        return torch.nn.functional.gelu(x)
    if name in ("gelu_pytorch_tanh", "gelu_tanh"):
        return torch.nn.functional.gelu(x, approximate="tanh")
    if name in ("silu", "swish"):
        return torch.nn.functional.silu(x)
    if name == "quick_gelu":
        return x * torch.sigmoid(1.702 * x)
    raise ValueError(f"unsupported activation {name!r}")


def activation(z: torch.Tensor, name: str) -> torch.Tensor:
    if native(z) and z.shape[1] % 8 == 0:
        return _ActFn.apply(z.contiguous(), ACT_CODES[name], False)
    return _act_reference(z.float(), name).to(z.dtype)


def gated_activation(z: torch.Tensor, name: str) -> torch.Tensor:
    """``act(z[:, :I]) * z[:, I:]`` (GeGLU / SwiGLU)."""

    width = z.shape[1] // 2
    if native(z) and width % 8 == 0:
        return _ActFn.apply(z.contiguous(), ACT_CODES[name], True)
    zf = z.float()
    return (_act_reference(zf[:, :width], name) * zf[:, width:]).to(z.dtype)


# ---------------------------------------------------------------- pooling
def pool_rows(h: torch.Tensor, seg: Segments, mode: str = "mean", normalize: bool = True) -> torch.Tensor:
    """Per-sequence mean / first / last row of packed hidden states (fp32)."""

    if native(h) and mode in ("mean", "first", "cls", "last", "lasttoken"):
        from .functional import POOL_MODES, PoolFn

        return PoolFn.apply(h, seg.cu_seqlens, POOL_MODES[mode], normalize)
    outs = []
    for a, e in zip(seg.cu_host, seg.cu_host[1:]):
        rows = h[a:e].float()
        if mode == "mean":
            outs.append(rows.mean(0) if e > a else torch.zeros(h.shape[1], device=h.device))
        elif mode in ("first", "cls"):
            outs.append(rows[0])
        else:
            outs.append(rows[-1])
    out = torch.stack(outs)
    return out / out.norm(dim=-1, keepdim=True).clamp_min(1e-12) if normalize else out


def scatter_rows(h: torch.Tensor, seg: Segments, max_len: int | None = None) -> torch.Tensor:
    """Packed rows -> zero-padded ``[batch, sequence, features]``."""

    S = max_len or seg.max_len
    out = h.new_zeros(seg.batch, S, h.shape[1])
    for b, (a, e) in enumerate(zip(seg.cu_host, seg.cu_host[1:])):
        out[b, : e - a] = h[a:e]
    return out


def sinusoid_table(n: int, dim: int) -> torch.Tensor:
    """Fixed sin/cos position table (first half sin, second half cos)."""

    log_step = math.log(10000.0) / (dim // 2 - 1)
    inv = torch.exp(-log_step * torch.arange(dim // 2, dtype=torch.float64))
    ang = torch.arange(n, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.sin(ang), torch.cos(ang)], 1).float()


__all__ = ["ACT_CODES", "Segments", "activation", "attention", "gated_activation", "layer_norm", "linear",
           "mrope_axis_table", "native", "pool_rows", "qkv_attention", "rms_norm", "rope", "rope_inv_freq", "scatter_rows",
           "sinusoid_table", "weight_as"]
