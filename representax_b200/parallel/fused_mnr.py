"""Cross-rank MNR with the all-gather and reduce-scatter fused into the kernels.

Each rank holds its own Lq query and Ld document embeddings (rank-major global
order; Ld > Lq with hard negatives). Instead of all-gathering the embeddings, computing the whole
[N*L, N*L] objective on every rank and slicing the gradient, every rank:

  forward   writes its normalised rows into its peer buffers, barriers, and
            computes its own L score rows against all N*L candidates in one
            tcgen05 kernel whose stager warps pull the owners' rows over
            NVLink into local split-bf16 operands while the tensor cores
            multiply the blocks already staged (fused all-gather), then the
            masked LSE / cross-entropy / logit-gradient row kernel.
  backward  dQ_local = G D_all reuses the candidates staged in the forward
            (no second transfer); the candidate-side product G^T Q_local is
            written by the tcgen05 epilogue straight into each owner's slot
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
from representax_b200.ops.mnr import split_bf16, tc_gemm, tc_scores

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


def _local_active(weights, row_valid, col_valid):
    w = weights * col_valid[None, :].to(weights.dtype)
    return (row_valid & (w.sum(1) > 0)).sum().to(torch.float32).reshape(1)


def _active_counts(sb: "ShardedRetrievalBatch", symmetric: bool):
    """Global active-row counts of both directions in one 8-byte all-reduce."""

    f = _local_active(sb.forward_weights, sb.query_valid, sb.document_valid_all)
    r = _local_active(sb.reverse_weights, sb.document_valid, sb.query_valid_all) if symmetric else f
    counts = torch.cat([f, r])
    dist.all_reduce(counts)
    counts = torch.clamp(counts, min=1.0)
    return counts[0:1], counts[1:2]


class _ShardedMNR(torch.autograd.Function):
    @staticmethod
    def forward(ctx_, qn, dn, sb: ShardedRetrievalBatch, scale: float, symmetric: bool, group: PeerGroup,
                n_f, n_r):
        C = ext()
        Lq, D = qn.shape
        Ld = dn.shape[0]
        if Lq % 8 or Ld % 8:
            raise ValueError(f"fused cross-rank MNR needs per-rank query and document counts divisible by 8 "
                             f"(got {Lq} and {Ld})")
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
            # scores against every rank's candidates; the kernel pulls the peers'
            # rows over NVLink into local split operands while it multiplies
            scores, own, cands = tc_scores(rows, cands_buf.peer_ptrs, n_cands, rank)
            grad = torch.empty_like(scores)
            row_loss = torch.empty(rows.shape[0], device=dev)
            row_active = torch.empty(rows.shape[0], device=dev)
            coef = (half / n_active).reshape(1)
            C.mnr_rows(scores, weights, row_valid, col_valid, grad, row_loss, row_active, float(scale), coef)
            return (row_loss * row_active).sum() / n_active.reshape(()), grad, own, cands

        fwd_local, g_f, q_own, d_all = direction(qn, dbuf, Ld, sb.forward_weights, sb.query_valid,
                                                 sb.document_valid_all, n_f)
        if symmetric:
            rev_local, g_r, d_own, q_all = direction(dn, qbuf, Lq, sb.reverse_weights, sb.document_valid,
                                                     sb.query_valid_all, n_r)
        else:
            rev_local = torch.zeros((), device=dev)
            empty = torch.empty(0, device=dev)
            g_r, d_own, q_all = empty, (empty, empty), (empty, empty)
        ctx_.save_for_backward(g_f, g_r, *q_own, *d_all, *d_own, *q_all)
        ctx_.meta = (group, symmetric, Lq, Ld, D, qslots, dslots)
        return fwd_local, rev_local

    @staticmethod
    def backward(ctx_, grad_fwd, grad_rev):
        C = ext()
        g_f, g_r, q_hi, q_lo, da_hi, da_lo, d_hi, d_lo, qa_hi, qa_lo = ctx_.saved_tensors
        group, symmetric, Lq, Ld, D, qslots, dslots = ctx_.meta
        world, rank = group.world, group.rank
        half = 0.5 if symmetric else 1.0
        # g_* hold d(loss)/d(score) for loss = half * (fwd + rev); rescale by the upstream gradients.
        gf = split_bf16(g_f * (grad_fwd / half))
        dq = torch.empty(Lq, D, dtype=torch.float32, device=g_f.device)
        # dQ = G_f . D_all from the candidates staged on this GPU in the forward (no NVLink)
        tc_gemm(gf, False, (da_hi, da_lo), True, Lq, D, world * Ld, out=dq)
        # G_f^T . Q: candidate-gradient rows of owner r go straight into slot `rank` of r's buffer
        tc_gemm(gf, True, (q_hi, q_lo), True, world * Ld, D, Lq, route=dslots.peer_ptrs, route_rows=Ld,
                route_offset=rank * Ld * D, ldc=D)
        dd = torch.zeros(Ld, D, dtype=torch.float32, device=g_f.device)
        if symmetric:
            gr = split_bf16(g_r * (grad_rev / half))
            tc_gemm(gr, False, (qa_hi, qa_lo), True, Ld, D, world * Lq, out=dd)
            tc_gemm(gr, True, (d_hi, d_lo), True, world * Lq, D, Ld, route=qslots.peer_ptrs, route_rows=Lq,
                    route_offset=rank * Lq * D, ldc=D)
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
    n_f, n_r = _active_counts(sb, symmetric)
    fwd_local, rev_local = _ShardedMNR.apply(qn, dn, sb, scale, symmetric, group, n_f, n_r)
    values = torch.stack([fwd_local.detach(), rev_local.detach()])
    dist.all_reduce(values)
    fwd = fwd_local + (values[0] - fwd_local.detach())
    rev = rev_local + (values[1] - rev_local.detach())
    loss = (fwd + rev) / 2.0 if symmetric else fwd
    return loss, values[0], values[1]


__all__ = ["ShardedRetrievalBatch", "sharded_mnr_loss"]
