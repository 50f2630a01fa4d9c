"""tcgen05 split-bf16 MNR kernels against fp32 / fp64 PyTorch references.

The scoring kernel is checked with several "ranks" whose candidate rows are
separate local buffers: the stager warps, the per-owner readiness counters and
the owner-rotated tile order run exactly as on several GPUs, without a peer.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _unit(n, k, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, k, generator=g, dtype=torch.float64)
    return (x / x.norm(dim=1, keepdim=True)).to(torch.float32).to(_dev())


@pytest.mark.parametrize("world,rank,rows,cand_rows,k", [(1, 0, 256, 384, 768), (4, 1, 136, 96, 768),
                                                         (3, 2, 40, 200, 96)])
def test_staged_scores_match_fp64(world, rank, rows, cand_rows, k):
    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mnr import tc_scores

    q = _unit(rows, k, 1)
    owners = [_unit(cand_rows, k, 10 + r) for r in range(world)]
    scores, (a_hi, a_lo), (b_hi, b_lo) = tc_scores(q, [t.data_ptr() for t in owners], cand_rows, rank)
    torch.cuda.synchronize()
    check_status(_dev())
    cands = torch.cat(owners)
    ref = q.double() @ cands.double().T
    err = (scores.double() - ref).abs().max().item()
    assert err < 2e-5, err
    # the staged split operands reconstruct the inputs to ~2^-16
    assert (a_hi.float() + a_lo.float() - q).abs().max().item() < 1e-5
    assert (b_hi.float() + b_lo.float() - cands).abs().max().item() < 1e-5


@pytest.mark.parametrize("a_mn,b_mn,m,n,k", [(False, False, 200, 136, 328), (False, True, 200, 136, 328),
                                             (True, True, 200, 136, 328), (True, False, 200, 136, 328),
                                             (False, True, 104, 72, 2048), (True, True, 64, 768, 4096)])
def test_split_gemm_layouts_and_accumulate(a_mn, b_mn, m, n, k):
    """The last two cases have too few tiles for the GPU and run split-K (fp32 atomics)."""

    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mnr import split_bf16, tc_gemm

    torch.manual_seed(3)
    a = torch.randn(m, k, device=_dev())
    b = torch.randn(n, k, device=_dev())
    a_store = a.T.contiguous() if a_mn else a
    b_store = b.T.contiguous() if b_mn else b
    out = torch.randn(m, n, device=_dev())
    base = out.clone()
    tc_gemm(split_bf16(a_store), a_mn, split_bf16(b_store), b_mn, m, n, k, out=out, accumulate=True)
    torch.cuda.synchronize()
    check_status(_dev())
    ref = base.double() + a.double() @ b.double().T
    rel = ((out.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 3e-5, rel
    fresh = torch.full((m, n), float("nan"), device=_dev())
    tc_gemm(split_bf16(a_store), a_mn, split_bf16(b_store), b_mn, m, n, k, out=fresh)
    torch.cuda.synchronize()
    rel = ((fresh.double() - a.double() @ b.double().T).abs().max() / ref.abs().max()).item()
    assert rel < 3e-5, rel


def test_routed_rows_land_in_owner_slots():
    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mnr import split_bf16, tc_gemm

    torch.manual_seed(4)
    world, seg, width, k, rank = 3, 64, 128, 96, 1
    g = torch.randn(k, world * seg, device=_dev())   # stored [K, M]: A is MN-major
    q = torch.randn(k, width, device=_dev())         # stored [K, N]: B is MN-major
    slots = [torch.full((world, seg, width), -7.0, device=_dev()) for _ in range(world)]
    tc_gemm(split_bf16(g), True, split_bf16(q), True, world * seg, width, k,
            route=[t.data_ptr() for t in slots], route_rows=seg, route_offset=rank * seg * width, ldc=width)
    torch.cuda.synchronize()
    check_status(_dev())
    full = g.double().T @ q.double()
    for owner in range(world):
        got = slots[owner][rank].double()
        want = full[owner * seg:(owner + 1) * seg]
        assert ((got - want).abs().max() / want.abs().max()).item() < 3e-5
        others = torch.cat([slots[owner][r] for r in range(world) if r != rank])
        assert torch.all(others == -7.0)  # only this rank's slot is written


def test_unaligned_batch_mnr_matches_reference():
    """Odd query / document counts go through the padded tensor-core path."""

    from representax_b200.ops.mnr import _NativeMNR, mnr_terms_reference, normalize

    torch.manual_seed(5)
    q = torch.randn(37, 64, device=_dev(), requires_grad=True)
    d = torch.randn(53, 64, device=_dev(), requires_grad=True)
    w = torch.zeros(37, 53, device=_dev())
    w[torch.arange(37), torch.arange(37)] = 1.0
    qv = torch.ones(37, dtype=torch.bool, device=_dev())
    dv = torch.ones(53, dtype=torch.bool, device=_dev())
    loss, _, _ = _NativeMNR.apply(normalize(q), normalize(d), w, qv, dv, 20.0, True)
    loss.backward()
    q2 = q.detach().double().requires_grad_(True)
    d2 = d.detach().double().requires_grad_(True)
    ref, *_ = mnr_terms_reference(q2, d2, w.double(), qv, dv, 20.0, True)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-4
    assert (q.grad.double() - q2.grad).abs().max().item() < 1e-5 + 1e-3 * q2.grad.abs().max().item()
    assert (d.grad.double() - d2.grad).abs().max().item() < 1e-5 + 1e-3 * d2.grad.abs().max().item()


@pytest.mark.parametrize("m,n,k,offset,masked", [(1000, 1000, 64, 0, True), (300, 2048, 768, 100, False),
                                                 (129, 77, 20, None, True)])
def test_mining_argmax_matches_fp64(m, n, k, offset, masked):
    """Fused mining kernel: each row's best allowed candidate without storing scores."""

    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mnr import hardest_candidates

    g = torch.Generator(device="cpu").manual_seed(17)
    a = (torch.randn(m, k, generator=g) * 3).to(_dev())
    c = torch.randn(n, k, generator=g).to(_dev())
    valid = (torch.rand(n, generator=g) > 0.25).to(_dev()) if masked else None
    got = hardest_candidates(a, c, valid, exclude_offset=offset)
    torch.cuda.synchronize()
    check_status(_dev())
    cos = torch.nn.functional.normalize(a.double(), dim=1) @ torch.nn.functional.normalize(c.double(), dim=1).T
    if valid is not None:
        cos[:, ~valid] = float("-inf")
    if offset is not None:
        rows = torch.arange(m, device=_dev())
        keep = rows + offset < n
        cos[rows[keep], rows[keep] + offset] = float("-inf")
    want = cos.argmax(1)
    best = cos.max(1).values
    picked = cos.gather(1, got[:, None])[:, 0]
    # the picked candidate is allowed and within split-bf16 rounding of the best
    assert torch.isfinite(picked).all()
    assert (best - picked).max().item() < 2e-5
    assert (got != want).float().mean().item() < 0.01
