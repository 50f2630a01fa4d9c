"""Multiple-negatives ranking objective: reference and native paths.

``mnr_loss`` computes the query-balanced cosine MNR of
src/representax/tasks/retrieval/mnr.py:123-379:

    logits = scale * cos(q_i, d_j), invalid documents masked to -inf
    row_loss_i = sum_j w_ij (lse_i - raw_ij) / max(sum_j w_ij, 1)
    loss = mean of row_loss over active rows (valid, with positive weight)

(symmetric mode averages it with the transposed direction). On CUDA the
similarity matrices and both gradient products run in the fp32 tiled GEMM of
``csrc/mnr.cu`` and the masked log-sum-exp / cross-entropy / logit gradient in
one row kernel; elsewhere the same formula runs in PyTorch.
"""

from __future__ import annotations

import torch

from ._ext import ext


def normalize(values: torch.Tensor) -> torch.Tensor:
    values = values.to(torch.float32)
    norm = torch.linalg.vector_norm(values, dim=1, keepdim=True)
    return values / torch.clamp(norm, min=1e-12)


def _direction_reference(rows, cands, weights, row_valid, cand_valid, scale):
    cosine = rows @ cands.T
    raw = cosine * scale
    logits = raw.masked_fill(~cand_valid[None, :], float("-inf"))
    active = (weights > 0) & row_valid[:, None] & cand_valid[None, :]
    w = torch.where(active, weights, torch.zeros_like(weights))
    lse = torch.logsumexp(logits, dim=1)
    row_weight = w.sum(1)
    terms = torch.where(active, w * (lse[:, None] - raw), torch.zeros_like(raw))
    row_losses = terms.sum(1) / torch.clamp(row_weight, min=1.0)
    active_rows = row_valid & (row_weight > 0)
    loss = torch.where(active_rows, row_losses, torch.zeros_like(row_losses)).sum() / torch.clamp(
        active_rows.sum(), min=1
    ).to(torch.float32)
    return loss, row_losses, active_rows, cosine, logits


def mnr_terms_reference(q, d, weights, q_valid, d_valid, scale, symmetric):
    qn, dn = normalize(q), normalize(d)
    forward, row_f, _, cosine, logits = _direction_reference(qn, dn, weights, q_valid, d_valid, scale)
    if symmetric:
        reverse, row_r, _, _, _ = _direction_reference(dn, qn, weights.T, d_valid, q_valid, scale)
        loss = (forward + reverse) / 2.0
    else:
        reverse = torch.zeros((), dtype=torch.float32, device=q.device)
        row_r = torch.zeros(d.shape[0], dtype=torch.float32, device=q.device)
        loss = forward
    return loss, forward, reverse, row_f, row_r, cosine, logits


def _active_count(weights, row_valid, cand_valid):
    w = weights * cand_valid[None, :].to(weights.dtype)
    return (row_valid & (w.sum(1) > 0)).sum().clamp(min=1).to(torch.float32)


class _NativeMNR(torch.autograd.Function):
    """Normalised embeddings in, (loss, forward, reverse) out."""

    @staticmethod
    def forward(ctx, qn, dn, weights, q_valid, d_valid, scale, symmetric):
        C = ext()
        dev = qn.device
        half = 0.5 if symmetric else 1.0
        qn = qn.contiguous()
        dn = dn.contiguous()
        weights = weights.to(torch.float32).contiguous()

        def direction(rows, cands, w, rv, cv):
            cos = torch.empty(rows.shape[0], cands.shape[0], device=dev, dtype=torch.float32)
            C.sgemm(rows, False, cands, False, cos, 1.0, False)
            n_active = _active_count(w, rv, cv)
            coef = (half / n_active).reshape(1)
            grad = torch.empty_like(cos)
            row_loss = torch.empty(rows.shape[0], device=dev)
            row_active = torch.empty(rows.shape[0], device=dev)
            C.mnr_rows(cos, w, rv, cv, grad, row_loss, row_active, float(scale), coef)
            loss = (row_loss * row_active).sum() / n_active
            return loss, grad

        forward_loss, grad_f = direction(qn, dn, weights, q_valid, d_valid)
        if symmetric:
            reverse_loss, grad_r = direction(dn, qn, weights.T.contiguous(), d_valid, q_valid)
            loss = (forward_loss + reverse_loss) / 2.0
        else:
            reverse_loss = torch.zeros((), device=dev)
            grad_r = None
            loss = forward_loss.clone()
        ctx.save_for_backward(qn, dn, grad_f, grad_r if grad_r is not None else torch.empty(0, device=dev))
        ctx.symmetric = symmetric
        ctx.mark_non_differentiable(forward_loss, reverse_loss)
        return loss, forward_loss, reverse_loss

    @staticmethod
    def backward(ctx, grad_loss, _gf, _gr):
        C = ext()
        qn, dn, grad_f, grad_r = ctx.saved_tensors
        dq = torch.empty_like(qn)
        dd = torch.empty_like(dn)
        # dq = G_f dn ; dd = G_f^T qn  (+ reverse direction terms)
        C.sgemm(grad_f, False, dn, True, dq, 1.0, False)
        C.sgemm(grad_f, True, qn, True, dd, 1.0, False)
        if ctx.symmetric:
            C.sgemm(grad_r, False, qn, True, dd, 1.0, True)
            C.sgemm(grad_r, True, dn, True, dq, 1.0, True)
        dq = dq * grad_loss
        dd = dd * grad_loss
        return dq, dd, None, None, None, None, None


def mnr_loss(q, d, weights, q_valid, d_valid, *, scale: float = 20.0, symmetric: bool = False):
    """Return ``(loss, forward_loss, reverse_loss)`` of the MNR objective."""

    if q.is_cuda:
        qn, dn = normalize(q), normalize(d)
        return _NativeMNR.apply(qn, dn, weights, q_valid, d_valid, scale, symmetric)
    loss, forward, reverse, *_ = mnr_terms_reference(q, d, weights, q_valid, d_valid, scale, symmetric)
    return loss, forward, reverse


__all__ = ["mnr_loss", "mnr_terms_reference", "normalize"]
