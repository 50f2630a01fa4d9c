"""Multiple-negatives ranking objective: reference and native paths.

``mnr_loss`` computes the query-balanced cosine MNR of
src/representax/tasks/retrieval/mnr.py:123-379:

    logits = scale * cos(q_i, d_j), invalid documents masked to -inf
    row_loss_i = sum_j w_ij (lse_i - raw_ij) / max(sum_j w_ij, 1)
    loss = mean of row_loss over active rows (valid, with positive weight)

(symmetric mode averages it with the transposed direction). On CUDA the
similarity matrices and both gradient products run on the tcgen05 tensor cores
(``csrc/mnr_tc.cu``: split-bf16 operands, fp32 accumulation) and the masked
log-sum-exp / cross-entropy / logit gradient in one row kernel
(``csrc/mnr.cu``); elsewhere the same formula runs in PyTorch.
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


# --------------------------------------------------------------------------- tensor-core path
# The similarity products run on tcgen05 with every fp32 operand split into a
# bf16 (hi, lo) pair (three MMAs per K step, ~1e-5 agreement with fp32). The
# operands' row counts are padded to multiples of 8 (16-byte TMA strides);
# padded candidates are invalid (masked out of the log-sum-exp, zero gradient).

_READY: dict[int, torch.Tensor] = {}


def _ready(device: torch.device) -> torch.Tensor:
    buf = _READY.get(device.index)
    if buf is None:
        buf = torch.zeros(32, dtype=torch.int32, device=device)
        _READY[device.index] = buf
    return buf


def _status(device: torch.device) -> torch.Tensor:
    from ._ext import status

    return status(device)


def split_bf16(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``x`` -> (hi, lo) bf16 with hi = bf16(x), lo = bf16(x - hi)."""

    x = x.contiguous()
    hi = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    lo = torch.empty_like(hi)
    ext().mnr_split(x, hi, lo)
    return hi, lo


def tc_scores(rows: torch.Tensor, cand_ptrs: list[int], cand_rows: int, rank: int):
    """``rows . candidates^T`` where rank r's candidates start at ``cand_ptrs[r]``.

    Returns the fp32 scores and the split operands (rows, all candidates) that
    the kernel staged on this GPU, for the gradient products.
    """

    m, k = rows.shape
    n = len(cand_ptrs) * cand_rows
    dev = rows.device
    a = (torch.empty(m, k, dtype=torch.bfloat16, device=dev), torch.empty(m, k, dtype=torch.bfloat16, device=dev))
    b = (torch.empty(n, k, dtype=torch.bfloat16, device=dev), torch.empty(n, k, dtype=torch.bfloat16, device=dev))
    scores = torch.empty(m, n, dtype=torch.float32, device=dev)
    ext().mnr_tc_scores(rows.contiguous(), [int(p) for p in cand_ptrs], cand_rows, rank, a[0], a[1], b[0], b[1],
                        _ready(dev), scores, 1.0, _status(dev))
    return scores, a, b


def hardest_candidates(anchor: torch.Tensor, candidates: torch.Tensor, valid: torch.Tensor | None = None,
                       *, exclude_offset: int | None = 0) -> torch.Tensor:
    """Index of each anchor row's most cosine-similar candidate (int64 [M]).

    Candidates with ``valid[n]`` false are skipped, and so is column
    ``m + exclude_offset`` for row m (the row's own pair; ``None`` keeps every
    column). Ties go to the smaller index; a row without any candidate gets 0.
    On CUDA one tcgen05 launch scores the unit vectors in split bf16 (near
    fp32) and reduces every tile to its rows' best candidate in the epilogue,
    so the [M, N] score matrix is never written. Parity:
    src/representax/train/mega_batch.py:27-55 (row-chunked masked argmax).
    """

    a = torch.nn.functional.normalize(anchor.detach().float(), dim=1, eps=1e-12)
    c = torch.nn.functional.normalize(candidates.detach().float(), dim=1, eps=1e-12)
    m, n = a.shape[0], c.shape[0]
    if not a.is_cuda:
        out = []
        cols = torch.arange(n)
        for s in range(0, m, 1024):
            scores = a[s:s + 1024] @ c.T
            if valid is not None:
                scores[:, ~valid.bool().cpu()] = float("-inf")
            if exclude_offset is not None:
                rows = torch.arange(s, min(m, s + 1024)) + exclude_offset
                scores[cols[None, :] == rows[:, None]] = float("-inf")
            out.append(scores.argmax(1))
        return torch.cat(out) if out else torch.zeros(0, dtype=torch.long)
    k = a.shape[1]
    if k % 8:  # 16-byte rows for the split operands
        a = torch.nn.functional.pad(a, (0, 8 - k % 8))
        c = torch.nn.functional.pad(c, (0, 8 - k % 8))
    ah, al = split_bf16(a)
    ch, cl = split_bf16(c)
    best = torch.empty(m, dtype=torch.long, device=a.device)
    v = None if valid is None else valid.to(device=a.device, dtype=torch.bool).contiguous()
    off = (1 << 40) if exclude_offset is None else int(exclude_offset)
    ext().mnr_tc_argmax(ah, al, ch, cl, best, v, off, _status(a.device))
    return torch.where(best == 0, torch.zeros_like(best), 0xFFFFFFFF - (best & 0xFFFFFFFF))


def tc_gemm(a, a_mn: bool, b, b_mn: bool, m: int, n: int, k: int, *, out: torch.Tensor | None = None,
            route: list[int] | None = None, route_rows: int = 1, route_offset: int = 0, ldc: int | None = None,
            accumulate: bool = False) -> None:
    """``out (+)= A . B^T`` on split operands (A [m, k] or [k, m], B [n, k] or [k, n]).

    With ``route`` the output rows go to other ranks' memory: row i lands at
    ``route[i // route_rows] + route_offset + (i % route_rows) * ldc`` (fp32).
    """

    dev = a[0].device
    ext().mnr_tc_gemm(a[0], a[1], a_mn, b[0], b[1], b_mn, m, n, k, out, [int(p) for p in (route or [])],
                      route_rows, route_offset, ldc if ldc is not None else n, 1.0, accumulate, _status(dev))


def _pad_rows(x: torch.Tensor, rows: int, value=0) -> torch.Tensor:
    if x.shape[0] == rows:
        return x.contiguous()
    pad = torch.full((rows - x.shape[0], *x.shape[1:]), value, dtype=x.dtype, device=x.device)
    return torch.cat([x, pad]).contiguous()


def _up8(n: int) -> int:
    return (n + 7) // 8 * 8


class _NativeMNR(torch.autograd.Function):
    """Normalised embeddings in, (loss, forward, reverse) out."""

    @staticmethod
    def forward(ctx, qn, dn, weights, q_valid, d_valid, scale, symmetric):
        C = ext()
        dev = qn.device
        half = 0.5 if symmetric else 1.0
        lq, ld = qn.shape[0], dn.shape[0]
        pq, pd = _up8(lq), _up8(ld)
        qp, dp = _pad_rows(qn.float(), pq), _pad_rows(dn.float(), pd)
        qv, dv = _pad_rows(q_valid.bool(), pq, False), _pad_rows(d_valid.bool(), pd, False)
        w = torch.zeros(pq, pd, dtype=torch.float32, device=dev)
        w[:lq, :ld] = weights.to(torch.float32)

        def direction(scores, w_dir, rv, cv):
            n_active = _active_count(w_dir, rv, cv)
            coef = (half / n_active).reshape(1)
            grad = torch.empty_like(scores)
            row_loss = torch.empty(scores.shape[0], device=dev)
            row_active = torch.empty(scores.shape[0], device=dev)
            C.mnr_rows(scores, w_dir, rv, cv, grad, row_loss, row_active, float(scale), coef)
            return (row_loss * row_active).sum() / n_active, grad

        scores_f, q_split, d_split = tc_scores(qp, [dp.data_ptr()], pd, 0)
        forward_loss, grad_f = direction(scores_f, w, qv, dv)
        del scores_f
        if symmetric:
            scores_r, _, _ = tc_scores(dp, [qp.data_ptr()], pq, 0)
            reverse_loss, grad_r = direction(scores_r, w.T.contiguous(), dv, qv)
            del scores_r
            loss = (forward_loss + reverse_loss) / 2.0
        else:
            reverse_loss = torch.zeros((), device=dev)
            grad_r = torch.empty(0, device=dev)
            loss = forward_loss.clone()
        ctx.save_for_backward(grad_f, grad_r, *q_split, *d_split)
        ctx.meta = (symmetric, lq, ld, pq, pd, qn.shape[1])
        ctx.mark_non_differentiable(forward_loss, reverse_loss)
        return loss, forward_loss, reverse_loss

    @staticmethod
    def backward(ctx, grad_loss, _gf, _gr):
        grad_f, grad_r, q_hi, q_lo, d_hi, d_lo = ctx.saved_tensors
        symmetric, lq, ld, pq, pd, width = ctx.meta
        qs, ds = (q_hi, q_lo), (d_hi, d_lo)
        dev = grad_f.device
        dq = torch.empty(pq, width, dtype=torch.float32, device=dev)
        dd = torch.empty(pd, width, dtype=torch.float32, device=dev)
        gf = split_bf16(grad_f)
        tc_gemm(gf, False, ds, True, pq, width, pd, out=dq)  # dq = G_f . D
        tc_gemm(gf, True, qs, True, pd, width, pq, out=dd)   # dd = G_f^T . Q
        if symmetric:
            gr = split_bf16(grad_r)
            tc_gemm(gr, False, qs, True, pd, width, pq, out=dd, accumulate=True)  # dd += G_r . Q
            tc_gemm(gr, True, ds, True, pq, width, pd, out=dq, accumulate=True)   # dq += G_r^T . D
        dq = dq[:lq] * grad_loss
        dd = dd[:ld] * grad_loss
        return dq, dd, None, None, None, None, None


def mnr_loss(q, d, weights, q_valid, d_valid, *, scale: float = 20.0, symmetric: bool = False):
    """Return ``(loss, forward_loss, reverse_loss)`` of the MNR objective."""

    if q.is_cuda:
        qn, dn = normalize(q), normalize(d)
        return _NativeMNR.apply(qn, dn, weights, q_valid, d_valid, scale, symmetric)
    loss, forward, reverse, *_ = mnr_terms_reference(q, d, weights, q_valid, d_valid, scale, symmetric)
    return loss, forward, reverse


__all__ = ["mnr_loss", "mnr_terms_reference", "normalize", "split_bf16", "tc_gemm", "tc_scores"]
