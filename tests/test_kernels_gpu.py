"""Numerics of every sm_100a kernel against plain fp32 PyTorch references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[1, 2], ids=["cta1", "cta_pair"])
def gemm_variant(request, monkeypatch):
    from representax_b200.ops import gemm as G

    monkeypatch.setattr(G, "GEMM_VARIANT", request.param)
    return request.param


@pytest.fixture(scope="module")
def C():
    from representax_b200.ops._ext import ext

    return ext()


def _dev():
    return torch.device("cuda", 0)


def _rand(*shape, dtype=torch.bfloat16, scale=1.0, gen=None):
    return (torch.randn(*shape, generator=gen, device=_dev()) * scale).to(dtype)


def _close(actual, expected, rtol, atol, what=""):
    actual = actual.float()
    expected = expected.float()
    err = (actual - expected).abs()
    tol = atol + rtol * expected.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad} elements off; max err {err.max().item():.3e}"


GEMM_SHAPES = [(128, 256, 64), (300, 520, 200), (2048, 768, 768), (1000, 2304, 768), (4096, 3072, 768)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_gemm_forward_plain(m, n, k, gemm_variant):
    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import check_status

    torch.manual_seed(0)
    a = _rand(m, k)
    b = _rand(n, k)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=_dev())
    G.gemm(a, b, out)
    torch.cuda.synchronize()
    check_status(_dev())
    ref = a.float() @ b.float().T
    _close(out, ref, rtol=1e-2, atol=1e-2 * math.sqrt(k), what="gemm")


@pytest.mark.parametrize("m,n,k", [(333, 600, 256), (2048, 3072, 768)])
def test_gemm_forward_epilogues(m, n, k, gemm_variant):
    from representax_b200.ops import gemm as G

    torch.manual_seed(1)
    x = _rand(m, k, scale=0.5)
    w = _rand(n, k, scale=0.05)
    bias = _rand(n, scale=0.1)
    grad = torch.empty(m, n, dtype=torch.bfloat16, device=_dev())
    y = G.linear_forward(x, w, bias, gelu_grad=grad)
    ref_pre = x.float() @ w.float().T + bias.float()
    # the epilogue saves gelu'(z) = Phi(z) + z phi(z) for the backward
    ref_grad = 0.5 * (1 + torch.erf(ref_pre * 0.7071067811865476)) + ref_pre * torch.exp(-0.5 * ref_pre ** 2) * 0.3989422804014327
    _close(grad, ref_grad, rtol=1e-2, atol=2e-2, what="gelu derivative")
    _close(y, torch.nn.functional.gelu(ref_pre), rtol=1e-2, atol=2e-2, what="gelu")
    res = _rand(m, n)
    y2 = G.linear_forward(x, w, bias, residual=res)
    _close(y2, ref_pre + res.float(), rtol=1e-2, atol=3e-2, what="bias+residual")
    y3 = torch.empty(m, n, dtype=torch.float32, device=_dev())
    G.gemm(x, w, y3, epi=G.EPI_BIAS, out_mode=G.OUT_F32, bias=bias)
    _close(y3, ref_pre, rtol=1e-3, atol=1e-3, what="f32 out")


@pytest.mark.parametrize("m,n,k", [(300, 520, 200), (2048, 768, 3072)])
def test_gemm_dgrad(m, n, k, gemm_variant):
    # dx[m, k] = dy[m, n] @ W[n, k]
    from representax_b200.ops import gemm as G

    torch.manual_seed(2)
    dy = _rand(m, n)
    w = _rand(n, k, scale=0.05)
    dx = G.linear_dgrad(dy, w)
    ref = dy.float() @ w.float()
    _close(dx, ref, rtol=1e-2, atol=2e-2, what="dgrad")
    saved = _rand(m, k)  # a saved gelu derivative: the epilogue multiplies by it
    dz = G.linear_dgrad(dy, w, gelu_grad=saved)
    _close(dz, ref * saved.float(), rtol=2e-2, atol=3e-2, what="dgrad*gelu'")
    # round trip: forward GELU epilogue saves gelu'(z), the dgrad epilogue applies it
    x = _rand(m, n, scale=0.5)
    w1 = _rand(k, n, scale=0.1)
    grad = torch.empty(m, k, dtype=torch.bfloat16, device=_dev())
    G.linear_forward(x, w1, torch.zeros(k, dtype=torch.bfloat16, device=_dev()), gelu_grad=grad)
    z = (x.float() @ w1.float().T).requires_grad_(True)
    torch.nn.functional.gelu(z).backward(ref)
    dz2 = G.linear_dgrad(dy, w, gelu_grad=grad)
    _close(dz2, z.grad, rtol=3e-2, atol=4e-2, what="gelu forward -> backward")
    res = _rand(m, k)
    dr = G.linear_dgrad(dy, w, residual=res)
    _close(dr, ref + res.float(), rtol=1e-2, atol=3e-2, what="dgrad+res")


@pytest.mark.parametrize("t,n,k", [(300, 520, 200), (4096, 768, 768), (9000, 3072, 768)])
def test_gemm_wgrad_accumulates(t, n, k, gemm_variant):
    from representax_b200.ops import gemm as G

    torch.manual_seed(3)
    dy = _rand(t, n, scale=0.1)
    x = _rand(t, k, scale=0.1)
    grad = torch.full((n, k), 0.5, dtype=torch.float32, device=_dev())
    G.linear_wgrad(dy, x, grad)
    G.linear_wgrad(dy, x, grad)
    ref = 0.5 + 2 * (dy.float().T @ x.float())
    _close(grad, ref, rtol=1e-3, atol=1e-3, what="wgrad")


@pytest.mark.parametrize("rows,h", [(1, 384), (777, 768), (64, 1024)])
def test_layernorm_fwd_bwd(C, rows, h):
    torch.manual_seed(4)
    x = _rand(rows, h, scale=2.0)
    g = _rand(h, scale=0.5) + 1
    b = _rand(h, scale=0.1)
    y = torch.empty_like(x)
    mean = torch.empty(rows, device=_dev())
    rstd = torch.empty(rows, device=_dev())
    C.norm_forward(x, g.to(torch.bfloat16), b, y, mean, rstd, 1e-12, False)
    xf = x.float().requires_grad_(True)
    gf = g.float().requires_grad_(True)
    bf = b.float().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xf, (h,), gf, bf, 1e-12)
    _close(y, ref, rtol=1e-2, atol=2e-2, what="ln fwd")
    dy = _rand(rows, h)
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dg = torch.zeros(h, device=_dev())
    db = torch.zeros(h, device=_dev())
    dprev = torch.zeros(h, device=_dev())
    C.norm_backward(dy, x, mean, rstd, g, dx, dg, db, dprev, False)
    _close(dx, xf.grad, rtol=2e-2, atol=3e-2, what="ln dx")
    _close(dg, gf.grad, rtol=1e-3, atol=1e-2, what="ln dgamma")
    _close(db, bf.grad, rtol=1e-3, atol=1e-2, what="ln dbeta")
    _close(dprev, xf.grad.sum(0), rtol=2e-2, atol=5e-2, what="ln dbias_prev")


def test_rmsnorm_fwd_bwd(C):
    torch.manual_seed(5)
    rows, h = 500, 768
    x = _rand(rows, h)
    g = _rand(h, scale=0.2) + 1
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device=_dev())
    C.norm_forward(x, g, None, y, None, rstd, 1e-6, True)
    xf = x.float().requires_grad_(True)
    gf = g.float().requires_grad_(True)
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * gf
    _close(y, ref, rtol=1e-2, atol=2e-2, what="rms fwd")
    dy = _rand(rows, h)
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dg = torch.zeros(h, device=_dev())
    C.norm_backward(dy, x, None, rstd, g, dx, dg, None, None, True)
    _close(dx, xf.grad, rtol=2e-2, atol=3e-2, what="rms dx")
    _close(dg, gf.grad, rtol=1e-3, atol=1e-2, what="rms dgamma")


def test_embedding_ln(C):
    torch.manual_seed(6)
    vocab, npos, h, rows = 1000, 512, 384, 3000
    word = _rand(vocab, h, scale=0.1)
    pos = _rand(npos, h, scale=0.1)
    typ = _rand(2, h, scale=0.1)
    g = _rand(h, scale=0.1) + 1
    b = _rand(h, scale=0.1)
    ids = torch.randint(0, vocab, (rows,), device=_dev(), dtype=torch.int32)
    ids[::7] = 0
    pids = torch.randint(0, npos, (rows,), device=_dev(), dtype=torch.int32)
    y = torch.empty(rows, h, dtype=torch.bfloat16, device=_dev())
    mean = torch.empty(rows, device=_dev())
    rstd = torch.empty(rows, device=_dev())
    C.embed_ln_forward(ids, pids, None, word, pos, typ, g, b, y, mean, rstd, 1e-12)
    wf = word.float().requires_grad_(True)
    pf = pos.float().requires_grad_(True)
    tf = typ.float().requires_grad_(True)
    gf = g.float().requires_grad_(True)
    bf = b.float().requires_grad_(True)
    s = wf[ids.long()] + pf[pids.long()] + tf[0]
    ref = torch.nn.functional.layer_norm(s, (h,), gf, bf, 1e-12)
    _close(y, ref, rtol=1e-2, atol=2e-2, what="embed fwd")
    dy = _rand(rows, h)
    ref.backward(dy.float())
    wg = torch.zeros(vocab, h, device=_dev())
    pg = torch.zeros(npos, h, device=_dev())
    tg = torch.zeros(2, h, device=_dev())
    dg = torch.zeros(h, device=_dev())
    db = torch.zeros(h, device=_dev())
    C.embed_ln_backward(dy, ids, pids, None, word, pos, typ, g, mean, rstd, wg, pg, tg, dg, db, 0)
    expected_wg = wf.grad.clone()
    expected_wg[0] = 0  # padding row receives no gradient
    _close(wg, expected_wg, rtol=2e-2, atol=5e-2, what="word grad")
    _close(pg, pf.grad, rtol=2e-2, atol=5e-2, what="pos grad")
    _close(tg, tf.grad, rtol=2e-2, atol=2e-1, what="type grad")
    _close(dg, gf.grad, rtol=1e-3, atol=5e-2, what="dgamma")


def _attn_ref(q, k, v, lens, heads, kv_heads, scale, causal, window, d=64):
    outs = []
    start = 0
    for n in lens:
        qs = q[start:start + n].float().view(n, heads, d).transpose(0, 1)
        ks = k[start:start + n].float().view(n, kv_heads, d).transpose(0, 1)
        vs = v[start:start + n].float().view(n, kv_heads, d).transpose(0, 1)
        rep = heads // kv_heads
        ks = ks.repeat_interleave(rep, 0)
        vs = vs.repeat_interleave(rep, 0)
        s = (qs @ ks.transpose(1, 2)) * scale
        i = torch.arange(n, device=q.device)[:, None]
        j = torch.arange(n, device=q.device)[None, :]
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device)
        if causal:
            mask &= j <= i
        if window >= 0:
            mask &= (j - i).abs() <= window
        s = s.masked_fill(~mask, float("-inf"))
        o = torch.softmax(s, -1) @ vs
        outs.append(o.transpose(0, 1).reshape(n, heads * d))
        start += n
    return torch.cat(outs)


@pytest.fixture(params=["tcgen05", "tcgen05_per_tile", "mma_sync"])
def attn_impl(request, C):
    """tcgen05: the warp-specialised persistent kernels at head dim 64;
    tcgen05_per_tile: the one-CTA-per-tile tcgen05 kernels; mma_sync: legacy."""
    fwd_default = C.attention_forward_ws_enabled()
    C.set_attention_tcgen05(request.param != "mma_sync")
    C.set_attention_backward_ws(request.param == "tcgen05")
    C.set_attention_forward_ws(request.param == "tcgen05")
    yield request.param
    C.set_attention_tcgen05(True)
    C.set_attention_backward_ws(True)
    C.set_attention_forward_ws(fwd_default)


@pytest.mark.parametrize(
    "lens,heads,kv_heads,causal,window,d,q_gain",
    [
        ([1, 17, 64, 65, 200, 256], 12, 12, False, -1, 64, 1.0),
        ([300, 129], 4, 4, False, 64, 64, 1.0),
        ([100, 257], 4, 2, True, -1, 64, 1.0),
        # several key blocks with sharp scores: exercises the running-max moves
        ([513, 40, 384], 2, 2, False, -1, 64, 4.0),
        ([1, 130, 256], 4, 4, False, -1, 128, 1.0),
        ([200, 77, 300], 4, 2, True, -1, 128, 2.0),
    ],
)
def test_attention_fwd_bwd(C, attn_impl, lens, heads, kv_heads, causal, window, d, q_gain):
    torch.manual_seed(7)
    total = sum(lens)
    hd = heads * d
    kvd = kv_heads * d
    qkv = _rand(total, hd + 2 * kvd)
    qkv[:, :hd] = (qkv[:, :hd].float() * q_gain).to(torch.bfloat16)
    q, k, v = qkv[:, :hd], qkv[:, hd:hd + kvd], qkv[:, hd + kvd:]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())
    scale = 1 / math.sqrt(d)
    o = torch.empty(total, hd, dtype=torch.bfloat16, device=_dev())
    lse = torch.empty(heads, total, device=_dev())
    C.attention_forward(q, k, v, o, lse, cu, max(lens), heads, kv_heads, scale, causal, window, 0, 0, 0.0, None)
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    ref = _attn_ref(qf, kf, vf, lens, heads, kv_heads, scale, causal, window, d)
    _close(o, ref, rtol=2e-2, atol=2e-2, what=f"attn fwd ({attn_impl})")
    do = _rand(total, hd)
    ref.backward(do.float())
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = dqkv[:, :hd], dqkv[:, hd:hd + kvd], dqkv[:, hd + kvd:]
    dq_acc = torch.empty(total, hd, device=_dev())
    dvec = torch.empty(heads, total, device=_dev())
    C.attention_backward(do, q, k, v, o, lse, dq, dk, dv, dq_acc, dvec, cu, max(lens), heads,
                         kv_heads, scale, causal, window, 0, 0, 0.0, None, None)
    torch.cuda.synchronize()
    gain = max(1.0, q_gain)
    _close(dq, qf.grad, rtol=3e-2, atol=3e-2 * gain, what=f"dq ({attn_impl})")
    _close(dk, kf.grad, rtol=3e-2, atol=3e-2 * gain, what=f"dk ({attn_impl})")
    _close(dv, vf.grad, rtol=3e-2, atol=3e-2 * gain, what=f"dv ({attn_impl})")


@pytest.mark.parametrize(
    "lens,heads,kv_heads,causal,window,drop",
    [
        ([1, 17, 64, 65, 200, 256, 31, 128, 129], 12, 12, False, -1, 0.0),
        ([1, 17, 64, 65, 200, 256], 12, 12, False, -1, 0.1),
        ([100, 257, 640], 4, 2, True, -1, 0.1),
        ([300, 129, 5], 4, 1, False, 64, 0.0),
        ([700, 3], 2, 2, True, 40, 0.2),
    ],
)
def test_attention_backward_ws_matches_per_tile_kernel(C, lens, heads, kv_heads, causal, window, drop):
    """The warp-specialised persistent backward (pipelined S / softmax / gradient
    MMAs, dQ drained by its own warps) against the per-key-tile tcgen05 backward
    on the same forward, dropout masks included; both also fuse the QKV bias
    gradient, checked against the column sums of the gradients they wrote."""
    torch.manual_seed(5)
    d = 64
    total = sum(lens)
    hd, kvd = heads * d, kv_heads * d
    qkv = _rand(total, hd + 2 * kvd)
    q, k, v = qkv[:, :hd], qkv[:, hd:hd + kvd], qkv[:, hd + kvd:]
    do = _rand(total, hd)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())
    o = torch.empty(total, hd, dtype=torch.bfloat16, device=_dev())
    lse = torch.empty(heads, total, device=_dev())
    C.attention_forward(q, k, v, o, lse, cu, max(lens), heads, kv_heads, d ** -0.5, causal, window, 99, 3, drop, None)
    out, bias = {}, {}
    for ws in (True, False):
        C.set_attention_backward_ws(ws)
        dqkv = torch.full_like(qkv, float("nan"))
        acc = torch.empty(total, hd, device=_dev())
        dvec = torch.empty(heads, total, device=_dev())
        db = torch.full((hd + 2 * kvd,), 0.5, device=_dev())  # accumulates onto what is there
        C.attention_backward_bias(do, q, k, v, o, lse, dqkv[:, :hd], dqkv[:, hd:hd + kvd], dqkv[:, hd + kvd:], acc,
                                  dvec, cu, max(lens), heads, kv_heads, d ** -0.5, causal, window, 99, 3, drop, None,
                                  None, db)
        out[ws] = dqkv.float()
        bias[ws] = db
    C.set_attention_backward_ws(True)
    torch.cuda.synchronize()
    from representax_b200.ops._ext import check_status

    check_status(_dev())  # no bounded wait ran out
    assert torch.isfinite(out[True]).all(), "ws backward left unwritten gradient rows"
    _close(out[True], out[False], rtol=1e-2, atol=1e-2, what="ws vs per-tile backward")
    for ws in (True, False):  # fused bias gradient == column sums of the bf16 gradients
        want = out[ws].double().sum(0) + 0.5
        _close(bias[ws], want, rtol=1e-4, atol=1e-3 * float(want.abs().max()), what=f"qkv bias grad (ws={ws})")


@pytest.mark.parametrize(
    "lens,heads,kv_heads,causal,window,drop,q_gain",
    [
        ([1, 17, 64, 65, 200, 256, 31, 128, 129], 12, 12, False, -1, 0.0, 1.0),
        ([1, 17, 64, 65, 200, 256], 12, 12, False, -1, 0.1, 1.0),
        ([100, 257, 640], 4, 2, True, -1, 0.1, 1.0),
        ([300, 129, 5], 4, 1, False, 64, 0.0, 1.0),
        ([513, 40, 384], 2, 2, False, -1, 0.0, 4.0),  # sharp scores: running-max moves, O rescales
        ([700, 3], 2, 2, True, 40, 0.2, 1.0),
    ],
)
def test_attention_forward_ws_matches_per_tile_kernel(C, lens, heads, kv_heads, causal, window, drop, q_gain):
    """The warp-specialised persistent forward (two pipelines per SM, score MMAs
    of the next block overlapping the softmax) against the per-tile tcgen05
    forward: outputs and log-sum-exps, dropout masks included."""
    torch.manual_seed(9)
    d = 64
    total = sum(lens)
    hd, kvd = heads * d, kv_heads * d
    qkv = _rand(total, hd + 2 * kvd)
    qkv[:, :hd] = (qkv[:, :hd].float() * q_gain).to(torch.bfloat16)
    q, k, v = qkv[:, :hd], qkv[:, hd:hd + kvd], qkv[:, hd + kvd:]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())
    default = C.attention_forward_ws_enabled()
    res = {}
    for ws in (True, False):
        C.set_attention_forward_ws(ws)
        o = torch.full((total, hd), float("nan"), dtype=torch.bfloat16, device=_dev())
        lse = torch.full((heads, total), float("nan"), device=_dev())
        C.attention_forward(q, k, v, o, lse, cu, max(lens), heads, kv_heads, d ** -0.5, causal, window, 77, 2, drop,
                            None)
        res[ws] = (o.float(), lse)
    C.set_attention_forward_ws(default)
    torch.cuda.synchronize()
    from representax_b200.ops._ext import check_status

    check_status(_dev())
    assert torch.isfinite(res[True][0]).all() and torch.isfinite(res[True][1]).all()
    _close(res[True][0], res[False][0], rtol=1e-2, atol=1e-2, what="ws vs per-tile forward O")
    _close(res[True][1], res[False][1], rtol=1e-4, atol=1e-3, what="ws vs per-tile forward lse")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("variant", ["relative_bias"])
def test_attention_variants_match_across_kernels(C, d, variant):
    """The tcgen05 and mma.sync kernels agree on MPNet's relative position bias and its gradient."""
    torch.manual_seed(11)
    lens, heads = [90, 130, 33, 257], 2
    total = sum(lens)
    hd = heads * d
    qkv = _rand(total, 3 * hd)
    q, k, v = qkv[:, :hd], qkv[:, hd:2 * hd], qkv[:, 2 * hd:]
    do = _rand(total, hd)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())
    drop = 0.15 if variant == "dropout" else 0.0
    lut = torch.randn(heads, 2 * 300 - 1, device=_dev()) if variant == "relative_bias" else None
    results = {}
    for impl in ("tcgen05", "mma_sync"):
        C.set_attention_tcgen05(impl == "tcgen05")
        o = torch.empty(total, hd, dtype=torch.bfloat16, device=_dev())
        lse = torch.empty(heads, total, device=_dev())
        C.attention_forward(q, k, v, o, lse, cu, max(lens), heads, heads, d ** -0.5, False, -1, 4321, 5, drop, lut)
        dqkv = torch.empty_like(qkv)
        acc = torch.empty(total, hd, device=_dev())
        dvec = torch.empty(heads, total, device=_dev())
        drel = None if lut is None else torch.zeros_like(lut)
        C.attention_backward(do, q, k, v, o, lse, dqkv[:, :hd], dqkv[:, hd:2 * hd], dqkv[:, 2 * hd:], acc, dvec, cu,
                             max(lens), heads, heads, d ** -0.5, False, -1, 4321, 5, drop, lut, drel)
        results[impl] = (o.float(), dqkv.float(), drel)
    C.set_attention_tcgen05(True)
    _close(results["tcgen05"][0], results["mma_sync"][0], rtol=2e-2, atol=2e-2, what=f"{variant} fwd")
    _close(results["tcgen05"][1], results["mma_sync"][1], rtol=3e-2, atol=3e-2, what=f"{variant} grads")
    if lut is not None:
        ref = results["mma_sync"][2]
        _close(results["tcgen05"][2], ref, rtol=2e-2, atol=2e-2 * float(ref.abs().max()), what="relative-bias grad")


@pytest.mark.parametrize("d", [64, 128])
def test_attention_dropout_mask_statistics(C, d):
    """Read the tcgen05 kernels' dropout mask back: with equal scores and V = I, O[i, j] is
    keep(i, j) * scale / L. The kept fraction matches 1 - p, kept values carry the unbiased scale,
    the mask is reproducible, and another seed gives another mask."""
    torch.manual_seed(3)
    heads, L, p = 4, 64, 0.25
    lens = [L] * 6
    total = sum(lens)
    hd = heads * d
    q = torch.zeros(total, hd, dtype=torch.bfloat16, device=_dev())
    k = _rand(total, hd)
    v = torch.zeros(total, hd, dtype=torch.bfloat16, device=_dev())
    eye = torch.eye(L, d, device=_dev()).to(torch.bfloat16)
    for s in range(len(lens)):
        for h in range(heads):
            v[s * L:(s + 1) * L, h * d:(h + 1) * d] = eye
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())

    def masks(seed):
        o = torch.empty(total, hd, dtype=torch.bfloat16, device=_dev())
        lse = torch.empty(heads, total, device=_dev())
        C.attention_forward(q, k, v, o, lse, cu, L, heads, heads, d ** -0.5, False, -1, seed, 2, p, None)
        return o.float().view(total, heads, d)[:, :, :L] * L

    m = masks(17)
    t8 = round(p * 256)  # 8-bit keep decisions
    scale = 256 / (256 - t8)
    kept = m > 0
    assert torch.allclose(m[kept], torch.full_like(m[kept], scale), rtol=1e-2)
    frac = kept.float().mean().item()
    n = kept.numel()
    assert abs(frac - (1 - p)) < 5 * (p * (1 - p) / n) ** 0.5, frac
    assert torch.equal(m, masks(17))
    other = masks(18) > 0
    assert (other != kept).float().mean().item() > 0.2


def test_attention_tcgen05_is_default(C):
    import os

    if os.environ.get("RX_ATTENTION_TC", "1") == "0":
        pytest.skip("tcgen05 attention switched off by RX_ATTENTION_TC=0")
    assert C.attention_tcgen05_enabled()


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("lens,h", [([3, 1, 50, 128], 768), ([40, 0, 33, 7], 4096), ([300], 2048)])
def test_pool(C, mode, lens, h):
    """Slices of 32 packed rows cross sequence boundaries; an empty sequence pools to zero."""

    torch.manual_seed(8)
    total = sum(lens)
    x = _rand(total, h)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=_dev())
    out = torch.empty(len(lens), h, device=_dev())
    norm = torch.empty(len(lens), device=_dev())
    C.pool_forward(x, cu, out, norm, mode, True)
    xf = x.float().requires_grad_(True)
    pooled = []
    s = 0
    for n in lens:
        seg = xf[s:s + n]
        if n == 0:
            pooled.append(torch.zeros(h, device=xf.device))
        else:
            pooled.append(seg.mean(0) if mode == 0 else seg[0] if mode == 1 else seg[-1])
        s += n
    ref = torch.nn.functional.normalize(torch.stack(pooled), dim=-1, eps=1e-12)
    _close(out, ref, rtol=1e-3, atol=1e-4, what="pool fwd")
    g = torch.randn_like(out)
    ref.backward(g)
    dh = torch.empty_like(x)
    C.pool_backward(g, out, norm, cu, dh, mode, True)
    _close(dh, xf.grad, rtol=2e-2, atol=1e-3, what="pool bwd")


def test_colsum_and_cast(C):
    for rows, cols, ld in ((1000, 768, 768), (37, 2304, 2304), (5000, 3072, 3072), (129, 8, 8),
                           (300, 4096, 4104), (70, 10240, 10240), (18432, 2304, 2304)):
        x = _rand(rows, ld)[:, :cols]
        out = torch.ones(cols, device=_dev())
        C.colsum_accumulate(x, out)
        _close(out, 1 + x.float().sum(0), rtol=1e-4, atol=2e-3, what=f"colsum {cols}")
    src = torch.randn(1001, device=_dev())
    dst = torch.empty(1001, dtype=torch.bfloat16, device=_dev())
    C.cast_bf16(src, dst)
    assert torch.equal(dst, src.to(torch.bfloat16))


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_sgemm(C, a_mn, b_mn):
    torch.manual_seed(9)
    m, n, k = 300, 257, 129
    a = torch.randn(k, m, device=_dev()) if a_mn else torch.randn(m, k, device=_dev())
    b = torch.randn(k, n, device=_dev()) if b_mn else torch.randn(n, k, device=_dev())
    c = torch.ones(m, n, device=_dev())
    C.sgemm(a, a_mn, b, b_mn, c, 0.5, True)
    am = a.T if a_mn else a
    bm = b if b_mn else b.T
    ref = 1 + 0.5 * (am.double() @ bm.double())
    _close(c, ref, rtol=1e-5, atol=1e-4, what="sgemm")


def test_mnr_rows(C):
    torch.manual_seed(10)
    r, c = 37, 50
    cos = torch.rand(r, c, device=_dev()) * 2 - 1
    w = (torch.rand(r, c, device=_dev()) < 0.1).float() * torch.rand(r, c, device=_dev()) * 2
    rv = torch.rand(r, device=_dev()) < 0.9
    cv = torch.rand(c, device=_dev()) < 0.9
    scale = 20.0
    n_active = ((w * cv[None].float() * rv[:, None].float()).sum(1) > 0).sum().clamp(min=1)
    coef = (1.0 / n_active.float()).reshape(1)
    grad = torch.empty(r, c, device=_dev())
    row_loss = torch.empty(r, device=_dev())
    row_active = torch.empty(r, device=_dev())
    C.mnr_rows(cos, w, rv, cv, grad, row_loss, row_active, scale, coef)
    x = cos.double().requires_grad_(True)
    raw = scale * x
    logits = raw.masked_fill(~cv[None], float("-inf"))
    lse = torch.logsumexp(logits, 1)
    act = w.double() * rv[:, None].double() * cv[None].double()
    rw = act.sum(1)
    rl = (act * (lse[:, None] - raw)).nan_to_num(0).sum(1) / rw.clamp(min=1)
    active = rv & (rw > 0)
    loss = (rl * active).sum() / active.sum().clamp(min=1)
    loss.backward()
    _close(row_loss * row_active, (rl * active).float(), rtol=1e-4, atol=1e-4, what="row loss")
    _close(grad, x.grad.float(), rtol=1e-4, atol=1e-6, what="mnr grad")


def test_adamw_clip_gate(C):
    torch.manual_seed(11)
    n = 10_001
    p = torch.randn(n, device=_dev())
    g = torch.randn(n, device=_dev()) * 3
    m = torch.zeros(n, device=_dev())
    v = torch.zeros(n, device=_dev())
    copy = torch.empty(n, dtype=torch.bfloat16, device=_dev())
    scalars = torch.zeros(8, device=_dev())
    nsq = torch.zeros(1, dtype=torch.float64, device=_dev())
    loss = torch.tensor([1.0], device=_dev())
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    lr, b1, b2, eps, wd, max_norm = 1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0
    for step in range(1, 4):
        C.grad_norm_sq(g, nsq)
        C.finalize_clip(nsq, scalars, loss, max_norm, 1)
        C.adamw_step(p, g, m, v, copy, scalars, lr, b1, b2, eps, wd)
        norm = g.double().norm()
        coef = min(1.0, max_norm / (norm.item() + 1e-6))
        gc = g * coef
        mr = b1 * mr + (1 - b1) * gc
        vr = b2 * vr + (1 - b2) * gc * gc
        upd = (mr / (1 - b1**step)) / ((vr / (1 - b2**step)).sqrt() + eps) + wd * pr
        pr = pr - lr * upd
    _close(p, pr, rtol=1e-5, atol=1e-6, what="adamw")
    assert torch.equal(copy, p.to(torch.bfloat16))
    assert scalars[2].item() == 3.0
    # A non-finite loss skips the update and keeps the step count.
    before = p.clone()
    C.grad_norm_sq(g, nsq)
    C.finalize_clip(nsq, scalars, torch.tensor([float("nan")], device=_dev()), max_norm, 1)
    C.adamw_step(p, g, m, v, copy, scalars, lr, b1, b2, eps, wd)
    assert torch.equal(p, before)
    assert scalars[2].item() == 3.0 and scalars[4].item() == 1.0


@pytest.mark.parametrize("symmetric", [False, True])
def test_native_mnr_loss_matches_reference(symmetric):
    from representax_b200.ops.mnr import _NativeMNR, mnr_terms_reference, normalize

    torch.manual_seed(12)
    q = torch.randn(70, 96, device=_dev(), requires_grad=True)
    d = torch.randn(70, 96, device=_dev(), requires_grad=True)
    w = torch.eye(70, device=_dev())
    w[3, 5] = 0.5
    qv = torch.ones(70, dtype=torch.bool, device=_dev())
    dv = torch.ones(70, dtype=torch.bool, device=_dev())
    dv[7] = False
    loss, fwd, rev = _NativeMNR.apply(normalize(q), normalize(d), w, qv, dv, 20.0, symmetric)
    loss.backward()
    gq, gd = q.grad.clone(), d.grad.clone()
    q2 = q.detach().double().requires_grad_(True)
    d2 = d.detach().double().requires_grad_(True)
    ref, rf, rr, *_ = mnr_terms_reference(q2, d2, w.double(), qv, dv, 20.0, symmetric)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-4
    assert abs(fwd.item() - rf.item()) < 1e-4
    _close(gq, q2.grad, rtol=1e-3, atol=1e-5, what="dq")
    _close(gd, d2.grad, rtol=1e-3, atol=1e-5, what="dd")


@pytest.mark.parametrize("t,n,k", [(300, 384, 256), (1000, 2112, 960), (129, 256, 2048)])
def test_int4_mainloop_gemm_forward_and_dgrad(C, t, n, k):
    """Packed INT4 weight expanded inside the tcgen05 main loop == dequantised weight product."""

    from representax_b200.models.adapters import QuantizedLoRAWeight

    g = torch.Generator().manual_seed(t + n)
    q = QuantizedLoRAWeight(torch.randn(n, k, generator=g) * 0.05, rank=4, alpha=8.0, seed=1).to(_dev())
    assert q.fused_int4()
    w = torch.empty(n, k, dtype=torch.bfloat16, device=_dev())
    C.int4_dequantize(q.packed_weight, q.scale_bits, w)
    x = _rand(t, k)
    bias = _rand(n)
    res = _rand(t, n)
    st = torch.zeros(1, dtype=torch.int32, device=_dev())
    y = torch.empty(t, n, dtype=torch.bfloat16, device=_dev())
    C.int4_gemm(x, q.packed_weight, q.scale_bits, k, y, bias, res, False, st)
    ref = x.double() @ w.double().T + bias.double() + res.double()
    _close(y, ref, rtol=1e-2, atol=2e-2, what="int4 fwd")
    dy = _rand(t, n)
    dx = torch.empty(t, k, dtype=torch.bfloat16, device=_dev())
    C.int4_gemm(dy, q.packed_weight, q.scale_bits, k, dx, None, None, True, st)
    _close(dx, dy.double() @ w.double(), rtol=1e-2, atol=2e-2, what="int4 dgrad")
    torch.cuda.synchronize()
    assert int(st.item()) == 0
