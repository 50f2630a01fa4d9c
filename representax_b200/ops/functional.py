"""Native (sm_100a) transformer building blocks as autograd functions.

Each block runs entirely in the extension kernels on packed token rows
([T, hidden] bf16, sequences delimited by ``cu_seqlens``) and writes its
parameter gradients straight into fp32 accumulators: ``param.main_grad`` when
the parameter lives in a flat store, otherwise a fresh fp32 tensor returned
through autograd. Parameters are read through their bf16 compute copy
(``param.compute``), refreshed by the fused optimizer step.

Blocks:
  attention_block   s = x + Attn(x Wqkv^T + bqkv) Wo^T + bo
  mlp_block         s = x + act(x W1^T + b1) W2^T + b2     (act = exact GELU)
  layer_norm        y = LN(s) (or RMSNorm), fp32 statistics
  embed_layer_norm  y = LN(word[ids] + pos[pids] + type[tids])
  pool              e = normalize(mean / first / last token of each sequence)
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import gemm as G
from ._ext import ext


@dataclass
class Packed:
    """Device-side description of a packed batch of sequences."""

    cu_seqlens: torch.Tensor  # [B + 1] int32 on device
    max_len: int
    total: int

    @property
    def batch(self) -> int:
        return self.cu_seqlens.numel() - 1


def compute_view(param: torch.Tensor, *, fused_gather: bool = False) -> torch.Tensor:
    """The bf16 compute copy of a parameter.

    Under FSDP the copy is this GPU's cache of the sharded weights: it is
    gathered here on first use in a parameter version, or, with
    ``fused_gather`` (the caller feeds it straight to a forward GEMM), by that
    GEMM's kernel itself.
    """

    state = getattr(param, "fsdp_state", None)
    if state is not None:
        return state.view(param, fused=fused_gather)
    copy = getattr(param, "compute", None)
    if copy is not None:
        return copy
    return param.detach().to(torch.bfloat16)


class _GradSink:
    """fp32 accumulator for one parameter's gradient."""

    def __init__(self, param: torch.Tensor):
        self.param = param
        self.main = getattr(param, "main_grad", None)
        self.fresh = None

    @property
    def wanted(self) -> bool:
        return self.param.requires_grad

    def buffer(self) -> torch.Tensor:
        if self.main is not None:
            return self.main
        if self.fresh is None:
            self.fresh = torch.zeros(self.param.shape, dtype=torch.float32, device=self.param.device)
        return self.fresh

    def result(self):
        if self.main is not None or self.fresh is None:
            return None
        return self.fresh.to(self.param.dtype)


def _colsum_into(x: torch.Tensor, sink: _GradSink) -> None:
    if sink.wanted:
        ext().colsum_accumulate(x, sink.buffer())


@dataclass(frozen=True)
class Dropout:
    """Dropout of one block: Philox seed, the block's first site id, probabilities."""

    seed: int
    site: int
    attention: float = 0.0
    hidden: float = 0.0

    def hidden_args(self, offset: int):
        return (self.seed, self.site + offset, self.hidden) if self.hidden > 0 else None


def _hidden_backward(ds: torch.Tensor, drop: "Dropout | None", offset: int,
                     colsum: torch.Tensor | None = None) -> torch.Tensor:
    """Gradient through an inverted-dropout site (the same Philox mask as the
    forward); ``colsum`` also receives the result's column sums (a bias gradient)."""

    if drop is None or drop.hidden <= 0:
        return ds
    out = torch.empty_like(ds)
    ext().dropout_apply(ds, out, drop.seed, drop.site + offset, drop.hidden, colsum)
    return out


class AttentionBlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_qkv, b_qkv, w_o, b_o, cu_seqlens, max_len, heads, kv_heads, causal, window,
                out_bias_grad_fused=False, dropout=None, rel_table=None, rel_buckets=None):
        C = ext()
        T, H = x.shape
        head_dim = 64
        wq, bq = compute_view(w_qkv, fused_gather=True), compute_view(b_qkv)
        wo, bo = compute_view(w_o, fused_gather=True), compute_view(b_o)
        qkv = G.linear_forward(x, wq, bq)
        qd, kd = heads * head_dim, kv_heads * head_dim
        q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
        a = torch.empty(T, qd, dtype=torch.bfloat16, device=x.device)
        lse = torch.empty(heads, T, dtype=torch.float32, device=x.device)
        scale = head_dim ** -0.5
        pa = dropout.attention if dropout is not None else 0.0
        seed = dropout.seed if dropout is not None else 0
        site = dropout.site if dropout is not None else 0
        lut = None
        if rel_table is not None:  # [buckets, heads] -> [heads, 2 L - 1] over signed distances
            lut = rel_table.detach().float()[rel_buckets].T.contiguous()
        C.attention_forward(q, k, v, a, lse, cu_seqlens, max_len, heads, kv_heads, scale, causal, window, seed, site,
                            pa, lut)
        s = G.linear_forward(a, wo, bo, residual=x, dropout=None if dropout is None else dropout.hidden_args(1))
        ctx.save_for_backward(x, qkv, a, lse, cu_seqlens, w_qkv, b_qkv, w_o, b_o)
        ctx.rel = (rel_table, rel_buckets, lut)
        ctx.meta = (max_len, heads, kv_heads, causal, window, scale)
        ctx.out_bias_grad_fused = out_bias_grad_fused
        ctx.dropout = dropout
        return s

    @staticmethod
    def backward(ctx, ds):
        C = ext()
        x, qkv, a, lse, cu, w_qkv, b_qkv, w_o, b_o = ctx.saved_tensors
        max_len, heads, kv_heads, causal, window, scale = ctx.meta
        drop = ctx.dropout
        ds = ds.contiguous()
        T = x.shape[0]
        qd, kd = heads * 64, kv_heads * 64
        g_wo, g_bo, g_wqkv, g_bqkv = _GradSink(w_o), _GradSink(b_o), _GradSink(w_qkv), _GradSink(b_qkv)
        dropped = drop is not None and drop.hidden > 0
        # gradient of the pre-dropout projection; its column sums are the out-bias gradient
        dpre = _hidden_backward(ds, drop, 1, g_bo.buffer() if (dropped and g_bo.wanted) else None)
        if g_wo.wanted:
            G.linear_wgrad(dpre, a, g_wo.buffer())
        if not ctx.out_bias_grad_fused and not dropped:
            _colsum_into(dpre, g_bo)
        da = G.linear_dgrad(dpre, compute_view(w_o))
        dqkv = torch.empty_like(qkv)
        q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
        dq_acc = torch.empty(T, qd, dtype=torch.float32, device=x.device)
        dvec = torch.empty(heads, T, dtype=torch.float32, device=x.device)
        rel_table, rel_buckets, lut = ctx.rel
        drel = None if lut is None else torch.zeros_like(lut)
        # the QKV bias gradient (column sums of dq | dk | dv) is taken inside the
        # backward's dQ conversion and dK / dV epilogue
        C.attention_backward_bias(da, q, k, v, a, lse, dqkv[:, :qd], dqkv[:, qd:qd + kd], dqkv[:, qd + kd:],
                                  dq_acc, dvec, cu, max_len, heads, kv_heads, scale, causal, window,
                                  drop.seed if drop is not None else 0, drop.site if drop is not None else 0,
                                  drop.attention if drop is not None else 0.0, lut, drel,
                                  g_bqkv.buffer() if g_bqkv.wanted else None)
        g_rel = None
        if drel is not None and rel_table.requires_grad:
            sink = _GradSink(rel_table)
            sink.buffer().index_add_(0, rel_buckets, drel.T)
            g_rel = sink.result()
        if g_wqkv.wanted:
            G.linear_wgrad(dqkv, x, g_wqkv.buffer())
        dx = G.linear_dgrad(dqkv, compute_view(w_qkv), residual=ds)
        return (dx, g_wqkv.result(), g_bqkv.result(), g_wo.result(), g_bo.result(), None, None, None, None, None,
                None, None, None, g_rel, None)


class MlpBlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, out_bias_grad_fused=False, dropout=None):
        T = x.shape[0]
        inter = w1.shape[0]
        z = torch.empty(T, inter, dtype=torch.bfloat16, device=x.device)
        g = G.linear_forward(x, compute_view(w1, fused_gather=True), compute_view(b1), gelu_grad=z)
        s = G.linear_forward(g, compute_view(w2, fused_gather=True), compute_view(b2), residual=x,
                             dropout=None if dropout is None else dropout.hidden_args(2))
        ctx.save_for_backward(x, z, g, w1, b1, w2, b2)
        ctx.out_bias_grad_fused = out_bias_grad_fused
        ctx.dropout = dropout
        return s

    @staticmethod
    def backward(ctx, ds):
        x, z, g, w1, b1, w2, b2 = ctx.saved_tensors
        ds = ds.contiguous()
        s_w1, s_b1, s_w2, s_b2 = _GradSink(w1), _GradSink(b1), _GradSink(w2), _GradSink(b2)
        dropped = ctx.dropout is not None and ctx.dropout.hidden > 0
        dpre = _hidden_backward(ds, ctx.dropout, 2, s_b2.buffer() if (dropped and s_b2.wanted) else None)
        if s_w2.wanted:
            G.linear_wgrad(dpre, g, s_w2.buffer())
        if not ctx.out_bias_grad_fused and not dropped:
            _colsum_into(dpre, s_b2)
        # dz = (dpre W2) * gelu'(z); the GEMM epilogue also sums dz's columns (the ffn-in bias gradient)
        dz = G.linear_dgrad(dpre, compute_view(w2), gelu_grad=z, colsum=s_b1.buffer() if s_b1.wanted else None)
        if s_w1.wanted:
            G.linear_wgrad(dz, x, s_w1.buffer())
        dx = G.linear_dgrad(dz, compute_view(w1), residual=ds)
        return dx, s_w1.result(), s_b1.result(), s_w2.result(), s_b2.result(), None, None


class LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, s, gamma, beta, eps, rms, producer_bias=None):
        C = ext()
        rows = s.shape[0]
        y = torch.empty_like(s)
        mean = None if rms else torch.empty(rows, dtype=torch.float32, device=s.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=s.device)
        C.norm_forward(s, compute_view(gamma), None if beta is None else compute_view(beta), y, mean, rstd, eps, rms)
        ctx.save_for_backward(s, mean if mean is not None else torch.empty(0, device=s.device), rstd, gamma,
                              beta if beta is not None else torch.empty(0, device=s.device),
                              producer_bias if producer_bias is not None else torch.empty(0, device=s.device))
        ctx.has_producer_bias = producer_bias is not None
        ctx.rms = rms
        ctx.has_beta = beta is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        s, mean, rstd, gamma, beta, pbias = ctx.saved_tensors
        dy = dy.contiguous()
        sg = _GradSink(gamma)
        sb = _GradSink(beta) if ctx.has_beta else None
        sp = _GradSink(pbias) if ctx.has_producer_bias else None
        dx = torch.empty_like(s)
        C.norm_backward(dy, s, None if ctx.rms else mean, rstd, compute_view(gamma), dx,
                        sg.buffer() if sg.wanted else None,
                        sb.buffer() if (sb is not None and sb.wanted) else None,
                        sp.buffer() if (sp is not None and sp.wanted) else None, ctx.rms)
        return (dx, sg.result(), (sb.result() if sb is not None else None), None, None,
                sp.result() if sp is not None else None)


class EmbedLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, pos_ids, type_ids, word, pos, typ, gamma, beta, eps, pad_id, dropout=None):
        C = ext()
        rows, H = ids.numel(), word.shape[1]
        y = torch.empty(rows, H, dtype=torch.bfloat16, device=ids.device)
        mean = torch.empty(rows, dtype=torch.float32, device=ids.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=ids.device)
        C.embed_ln_forward(ids, pos_ids, type_ids, compute_view(word), compute_view(pos), compute_view(typ),
                           compute_view(gamma), compute_view(beta), y, mean, rstd, eps)
        ctx.dropout = dropout
        if dropout is not None and dropout.hidden > 0:
            C.dropout_apply(y, y, dropout.seed, dropout.site, dropout.hidden, None)
        ctx.save_for_backward(ids, pos_ids, type_ids if type_ids is not None else torch.empty(0, device=ids.device),
                              mean, rstd, word, pos, typ, gamma, beta)
        ctx.has_types = type_ids is not None
        ctx.pad_id = pad_id
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        ids, pos_ids, type_ids, mean, rstd, word, pos, typ, gamma, beta = ctx.saved_tensors
        sinks = [_GradSink(p) for p in (word, pos, typ, gamma, beta)]
        bufs = [s.buffer() for s in sinks]
        dy = _hidden_backward(dy.contiguous(), ctx.dropout, 0)
        C.embed_ln_backward(dy, ids, pos_ids, type_ids if ctx.has_types else None,
                            compute_view(word), compute_view(pos), compute_view(typ), compute_view(gamma),
                            mean, rstd, bufs[0], bufs[1], bufs[2], bufs[3], bufs[4], ctx.pad_id)
        return (None, None, None) + tuple(s.result() for s in sinks) + (None, None, None)


POOL_MODES = {"mean": 0, "first": 1, "cls": 1, "last": 2, "lasttoken": 2}


class PoolFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, cu_seqlens, mode, normalize):
        C = ext()
        B = cu_seqlens.numel() - 1
        out = torch.empty(B, h.shape[1], dtype=torch.float32, device=h.device)
        norm = torch.empty(B, dtype=torch.float32, device=h.device)
        C.pool_forward(h.contiguous(), cu_seqlens, out, norm, mode, normalize)
        ctx.save_for_backward(out, norm, cu_seqlens)
        ctx.meta = (mode, normalize, h.shape)
        return out

    @staticmethod
    def backward(ctx, dout):
        C = ext()
        out, norm, cu = ctx.saved_tensors
        mode, normalize, shape = ctx.meta
        dh = torch.empty(shape, dtype=torch.bfloat16, device=out.device)
        C.pool_backward(dout.contiguous().to(torch.float32), out, norm, cu, dh, mode, normalize)
        return dh, None, None, None


def attention_block(x, w_qkv, b_qkv, w_o, b_o, packed: Packed, *, heads, kv_heads=None, causal=False, window=-1,
                    out_bias_grad_fused: bool = False, dropout: Dropout | None = None, rel_table=None,
                    rel_buckets=None):
    """``out_bias_grad_fused``: the following layer_norm was given ``producer_bias=b_o``
    and reduces its gradient in its own backward kernel (not with hidden dropout).
    ``dropout``: attention-probability dropout (site) and output dropout (site + 1).
    ``rel_table`` ([buckets, heads]) with ``rel_buckets`` (bucket of each signed
    distance -(L-1)..L-1): an additive relative-position bias (MPNet)."""

    return AttentionBlockFn.apply(x, w_qkv, b_qkv, w_o, b_o, packed.cu_seqlens, packed.max_len, heads,
                                  kv_heads or heads, causal, window, out_bias_grad_fused, dropout, rel_table,
                                  rel_buckets)


def mlp_block(x, w1, b1, w2, b2, *, out_bias_grad_fused: bool = False, dropout: Dropout | None = None):
    """``dropout``: output dropout at site + 2."""

    return MlpBlockFn.apply(x, w1, b1, w2, b2, out_bias_grad_fused, dropout)


def layer_norm(s, gamma, beta, eps: float, rms: bool = False, *, producer_bias=None):
    """``producer_bias``: bias of the linear layer that produced ``s``; its
    gradient (the column sum of ds) is accumulated by the norm's backward."""

    return LayerNormFn.apply(s, gamma, beta, eps, rms, producer_bias)


def embed_layer_norm(ids, pos_ids, type_ids, word, pos, typ, gamma, beta, eps: float, pad_id: int,
                     dropout: Dropout | None = None):
    return EmbedLayerNormFn.apply(ids, pos_ids, type_ids, word, pos, typ, gamma, beta, eps, pad_id, dropout)


def pool(h, packed: Packed, mode: str = "mean", normalize: bool = True):
    return PoolFn.apply(h, packed.cu_seqlens, POOL_MODES[mode], normalize)


__all__ = [
    "Dropout",
    "Packed",
    "attention_block",
    "compute_view",
    "embed_layer_norm",
    "layer_norm",
    "mlp_block",
    "pool",
]
