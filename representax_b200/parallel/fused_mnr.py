"""Cross-rank MNR with the all-gather and reduce-scatter fused into the kernels.

Each rank holds its own Lq query and Ld document embeddings (rank-major global
order; Ld > Lq with hard negatives). Instead of all-gathering the embeddings, computing the whole
[N*L, N*L] objective on every rank and slicing the gradient, every rank:

  forward   writes its normalised rows into its peer buffers, barriers, and
            computes its own L score rows against all N*L candidates with a
            GEMM whose candidate tiles are loaded directly from the owning
            ranks' buffers (fused all-gather), then the masked LSE /
            cross-entropy / logit-gradient row kernel.
  backward  dQ_local = G D_all reads peers again; the candidate-side product
            G^T Q_local is written by the GEMM straight into each owner's slot
            buffer (slot = this rank), and after a device barrier every owner
            sums its N slots in rank order (fused, deterministic
            reduce-scatter). Symmetric mode runs the transposed direction the
            same way.

The value returned is the global loss; its gradient flows only through this
rank's partial, so ``loss.backward()`` on every rank yields exactly the
gradient of the global objective with respect to each rank's embeddings.
Scalars (active-row counts, loss values) use tiny NCCL all-reduces.

Parity: global in-batch negatives of src/representax/tasks/retrieval/mnr.py
under the SPMD sharding of src/representax/train/sharding.py (the reference
all-gathers candidates and reduce-scatters their cotangents through XLA).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from representax_b200.ops._ext import ext

from .dist import DistContext, gather_rows
from .peer import PeerGroup, peer_group


@dataclass
class ShardedRetrievalBatch:
    """A rank's rows of a retrieval batch whose negatives span all ranks.

    ``forward_weights`` [Lq, N*Ld]: positive weights of local queries over all
    documents; ``reverse_weights`` [Ld, N*Lq]: of local documents over all
    queries (only needed in symmetric mode).
    """

    ctx: DistContext
    forward_weights: torch.Tensor
    reverse_weights: torch.Tensor | None
    query_valid: torch.Tensor          # [Lq]
    document_valid: torch.Tensor       # [Ld]
    query_valid_all: torch.Tensor      # [N*Lq]
    document_valid_all: torch.Tensor   # [N*Ld]

    @classmethod
    def from_local(cls, batch, ctx: DistContext, *, symmetric: bool) -> "ShardedRetrievalBatch":
        local_d = batch.document_valid.shape[0]
        global_d = local_d * ctx.world_size
        w = batch.weights().to(torch.float32)
        if w.shape[1] == local_d:
            wide = torch.zeros(w.shape[0], global_d, dtype=w.dtype, device=w.device)
            wide[:, ctx.rank * local_d:(ctx.rank + 1) * local_d] = w
            w = wide
        elif w.shape[1] != global_d:
            raise ValueError("positive_mask columns must cover the local or the global documents")
        reverse = None
        if symmetric:
            w_all = gather_rows(w.contiguous(), ctx)  # [N*L, N*L]
            reverse = w_all[:, ctx.rank * local_d:(ctx.rank + 1) * local_d].T.contiguous()
        qv_all = gather_rows(batch.query_valid.to(torch.uint8), ctx).bool()
        dv_all = gather_rows(batch.document_valid.to(torch.uint8), ctx).bool()
        return cls(ctx, w.contiguous(), reverse, batch.query_valid.bool(), batch.document_valid.bool(), qv_all, dv_all)


def _active(weights, row_valid, col_valid, ctx):
    w = weights * col_valid[None, :].to(weights.dtype)
    count = (row_valid & (w.sum(1) > 0)).sum().to(torch.float32).reshape(1)
    dist.all_reduce(count)
    return torch.clamp(count, min=1.0)


class _ShardedMNR(torch.autograd.Function):
    @staticmethod
    def forward(ctx_, qn, dn, sb: ShardedRetrievalBatch, scale: float, symmetric: bool, group: PeerGroup,
                n_f, n_r):
        C = ext()
        Lq, D = qn.shape
        Ld = dn.shape[0]
        world, rank = group.world, group.rank
        dev = qn.device
        half = 0.5 if symmetric else 1.0
        qbuf = group.cached(("mnr_q", Lq, D), Lq * D)
        dbuf = group.cached(("mnr_d", Ld, D), Ld * D)
        qslots = group.cached(("mnr_qs", Lq, D), world * Lq * D)
        dslots = group.cached(("mnr_ds", Ld, D), world * Ld * D)
        group.barrier()  # peers are done reading the previous contents
        qbuf.tensor.copy_(qn.reshape(-1))
        dbuf.tensor.copy_(dn.reshape(-1))
        group.barrier()  # every rank's rows are published

        def direction(rows, cands_buf, n_cands, weights, row_valid, col_valid, n_active):
            n_rows = rows.shape[0]
            scores = torch.empty(n_rows, world * n_cands, device=dev, dtype=torch.float32)
            C.peer_sgemm(rows, False, cands_buf.ptrs, n_cands, D, False, False, n_rows, world * n_cands, D, scores,
                         None, 1, 0, 1.0, False)
            grad = torch.empty_like(scores)
            row_loss = torch.empty(n_rows, device=dev)
            row_active = torch.empty(n_rows, device=dev)
            coef = (half / n_active).reshape(1)
            C.mnr_rows(scores, weights, row_valid, col_valid, grad, row_loss, row_active, float(scale), coef)
            return (row_loss * row_active).sum() / n_active.reshape(()), grad

        fwd_local, g_f = direction(qn, dbuf, Ld, sb.forward_weights, sb.query_valid, sb.document_valid_all, n_f)
        if symmetric:
            rev_local, g_r = direction(dn, qbuf, Lq, sb.reverse_weights, sb.document_valid, sb.query_valid_all,
                                       n_r)
        else:
            rev_local, g_r = torch.zeros((), device=dev), torch.empty(0, device=dev)
        ctx_.save_for_backward(qn, dn, g_f, g_r)
        ctx_.meta = (group, symmetric, Lq, Ld, D, qbuf, dbuf, qslots, dslots)
        return fwd_local, rev_local

    @staticmethod
    def backward(ctx_, grad_fwd, grad_rev):
        C = ext()
        qn, dn, g_f, g_r = ctx_.saved_tensors
        group, symmetric, Lq, Ld, D, qbuf, dbuf, qslots, dslots = ctx_.meta
        world, rank = group.world, group.rank
        half = 0.5 if symmetric else 1.0
        # g_* hold d(loss)/d(score) for loss = half * (fwd + rev); rescale by the upstream gradients.
        g_f = g_f * (grad_fwd / half)
        dq = torch.empty_like(qn)
        C.peer_sgemm(g_f, False, dbuf.ptrs, Ld, D, True, True, Lq, D, world * Ld, dq, None, 1, 0, 1.0, False)
        local_q = torch.tensor([qn.data_ptr()], dtype=torch.int64, device=qn.device)
        C.peer_sgemm(g_f, True, local_q, D, D, True, False, world * Ld, D, Lq, dq, dslots.ptrs, Ld, rank, 1.0,
                     False)
        dd = torch.zeros_like(dn)
        if symmetric:
            g_r = g_r * (grad_rev / half)
            C.peer_sgemm(g_r, False, qbuf.ptrs, Lq, D, True, True, Ld, D, world * Lq, dd, None, 1, 0, 1.0, False)
            local_d = torch.tensor([dn.data_ptr()], dtype=torch.int64, device=dn.device)
            C.peer_sgemm(g_r, True, local_d, D, D, True, False, world * Lq, D, Ld, dd, qslots.ptrs, Lq, rank, 1.0,
                         False)
        group.barrier()  # every rank's slot contributions have landed
        C.slot_reduce(dslots.tensor, world, dd, True)
        if symmetric:
            C.slot_reduce(qslots.tensor, world, dq, True)
        return dq, dd, None, None, None, None, None, None


def sharded_mnr_loss(q: torch.Tensor, d: torch.Tensor, sb: ShardedRetrievalBatch, *, scale: float,
                     symmetric: bool):
    """Global MNR loss (value) whose gradient reaches only this rank's rows."""

    from representax_b200.ops.mnr import normalize

    group = peer_group(sb.ctx, q.device)
    qn, dn = normalize(q).contiguous(), normalize(d).contiguous()
    n_f = _active(sb.forward_weights, sb.query_valid, sb.document_valid_all, sb.ctx)
    n_r = _active(sb.reverse_weights, sb.document_valid, sb.query_valid_all, sb.ctx) if symmetric else n_f
    fwd_local, rev_local = _ShardedMNR.apply(qn, dn, sb, scale, symmetric, group, n_f, n_r)
    values = torch.stack([fwd_local.detach(), rev_local.detach()])
    dist.all_reduce(values)
    fwd = fwd_local + (values[0] - fwd_local.detach())
    rev = rev_local + (values[1] - rev_local.detach())
    loss = (fwd + rev) / 2.0 if symmetric else fwd
    return loss, values[0], values[1]


__all__ = ["ShardedRetrievalBatch", "sharded_mnr_loss"]
