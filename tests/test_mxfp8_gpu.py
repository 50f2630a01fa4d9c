"""MXFP8 (block-scaled) quantiser, tcgen05 GEMM and linear layer against
PyTorch fp32 statements of the same recipe (``ops.mxfp8.quantize_reference``)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _unpack_scales(sf, rows, k):
    """Block exponents [rows, k / 32] from the tensor-core scale atoms."""

    groups, rt = (k + 127) // 128, (rows + 127) // 128 + 1
    a = sf.view(groups, rt, 32, 4, 4).permute(1, 3, 2, 0, 4).reshape(rt * 128, groups * 4)
    return a[:rows, : k // 32].int() - 127


def _decode(op, rows, fmt):
    from representax_b200.ops.mxfp8 import E4M3

    dtype = torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2
    q = op.data[:rows, : op.k].contiguous().view(dtype).float()
    e = _unpack_scales(op.scales, rows, op.k)
    return q * torch.exp2(e.float()).repeat_interleave(32, dim=1), e


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("r,c", [(64, 128), (300, 96), (129, 2304)])
def test_quantize_matches_reference(fmt, r, c):
    from representax_b200.ops.mxfp8 import quantize, quantize_reference

    g = torch.Generator().manual_seed(r + c + fmt)
    # rows of very different magnitudes, so block scales differ
    x = (torch.randn(r, c, generator=g) * torch.logspace(-3, 3, r)[:, None]).to(torch.bfloat16).to(_dev())
    row, col = quantize(x, fmt, rowwise=True, transposed=True)
    want, e_want = quantize_reference(x, fmt)
    got, e_got = _decode(row, r, fmt)
    assert torch.equal(e_got, e_want)
    assert torch.equal(got, want)
    want_t, e_want_t = quantize_reference(x.T.contiguous(), fmt) if r % 32 == 0 else (None, None)
    if want_t is not None:
        got_t, e_got_t = _decode(col, c, fmt)
        assert torch.equal(e_got_t, e_want_t)
        assert torch.equal(got_t, want_t)
    else:  # R not a multiple of 32: the last block of each column is zero-padded
        assert col.k == r + (-r) % 32
        pad = torch.zeros(col.k, c, dtype=torch.bfloat16, device=_dev())
        pad[:r] = x
        want_t, e_want_t = quantize_reference(pad.T.contiguous(), fmt)
        got_t, e_got_t = _decode(col, c, fmt)
        assert torch.equal(e_got_t, e_want_t)
        assert torch.equal(got_t, want_t)


@pytest.mark.parametrize("m,n,k", [(300, 200, 96), (1024, 768, 768), (512, 2304, 768), (130, 1152, 3072)])
def test_gemm_matches_fake_quant_product(m, n, k):
    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mxfp8 import E4M3, E5M2, OUT_BF16, OUT_F32, OUT_F32_ACC, gemm, quantize

    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).to(_dev())
    b = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16).to(_dev())
    aq, _ = quantize(a, E5M2)
    bq, _ = quantize(b, E4M3)
    af, _ = _decode(aq, m, E5M2)
    bf, _ = _decode(bq, n, E4M3)
    ref = af.double() @ bf.double().T
    out = torch.empty(m, n, device=_dev())
    gemm(aq, bq, out, OUT_F32)
    torch.cuda.synchronize()
    check_status(_dev())
    scale = ref.abs().max().item()
    assert (out.double() - ref).abs().max().item() < 1e-5 * scale
    gemm(aq, bq, out, OUT_F32_ACC)
    assert (out.double() - 2 * ref).abs().max().item() < 2e-5 * scale
    if n % 8 == 0:
        bias = torch.randn(n, generator=g).to(torch.bfloat16).to(_dev())
        res = torch.randn(m, n, generator=g).to(torch.bfloat16).to(_dev())
        y = torch.empty(m, n, dtype=torch.bfloat16, device=_dev())
        gemm(aq, bq, y, OUT_BF16, bias, res)
        want = ref + bias.double() + res.double()
        assert torch.allclose(y.double(), want, rtol=1e-2, atol=1e-2 * scale)
    torch.cuda.synchronize()
    check_status(_dev())


def test_linear_forward_backward_against_fake_quant():
    from representax_b200.ops._ext import check_status
    from representax_b200.ops.mxfp8 import E4M3, E5M2, linear_mxfp8, quantize_reference

    g = torch.Generator().manual_seed(3)
    m, k, n = 700, 768, 384
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(_dev()).requires_grad_(True)
    w = (torch.randn(n, k, generator=g) * 0.03).to(_dev()).requires_grad_(True)
    b = torch.randn(n, generator=g).to(_dev()).requires_grad_(True)
    y = linear_mxfp8(x, w, b)
    dy = torch.randn(m, n, generator=g).to(torch.bfloat16).to(_dev())
    y.backward(dy)
    torch.cuda.synchronize()
    check_status(_dev())
    xb, wb = x.detach(), w.detach().to(torch.bfloat16)
    xq, _ = quantize_reference(xb, E4M3)
    wq, _ = quantize_reference(wb, E4M3)
    y_ref = xq.double() @ wq.double().T + b.detach().to(torch.bfloat16).double()
    assert torch.allclose(y.double(), y_ref, rtol=1e-2, atol=1e-2)
    dyq, _ = quantize_reference(dy, E5M2)
    wtq, _ = quantize_reference(wb.T.contiguous(), E4M3)
    dx_ref = dyq.double() @ wtq.double().T
    assert torch.allclose(x.grad.double(), dx_ref, rtol=1e-2, atol=1e-2 * dx_ref.abs().max().item())
    pad = (-m) % 32
    dyt = torch.nn.functional.pad(dy.T, (0, pad))
    xt = torch.nn.functional.pad(xb.T, (0, pad))
    dytq, _ = quantize_reference(dyt.contiguous(), E5M2)
    xtq, _ = quantize_reference(xt.contiguous(), E4M3)
    dw_ref = dytq.double() @ xtq.double().T
    assert (w.grad.double() - dw_ref).abs().max().item() < 1e-5 * dw_ref.abs().max().item()
    assert torch.allclose(b.grad.double(), dy.double().sum(0), rtol=1e-3, atol=1e-2)
    # the block recipe tracks the exact product far closer than bf16 rounding of W would suggest
    exact = xb.double() @ w.detach().double().T
    rel = ((y.double() - b.detach().double() - exact).norm() / exact.norm()).item()
    assert rel < 0.08, rel
