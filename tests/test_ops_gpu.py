"""Native packed-row ops (bf16, sm_100a kernels) against their fp32 PyTorch statements."""

from __future__ import annotations

import pytest
import torch

from representax_b200.ops import nn as N

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err:.3e} vs scale {scale:.3e}"


def _pair(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x32 = (torch.randn(*shape, device=DEV, generator=g) * scale).requires_grad_()
    x16 = x32.detach().to(torch.bfloat16).requires_grad_()
    return x32, x16


def _seg(lengths):
    return N.Segments.from_lengths(lengths, DEV)


@pytest.mark.parametrize("bias,residual", [(False, False), (True, True)])
def test_linear(bias, residual):
    x32, x16 = _pair(300, 256)
    w = torch.nn.Parameter(torch.randn(384, 256, device=DEV) * 0.05)
    b = torch.nn.Parameter(torch.randn(384, device=DEV)) if bias else None
    r32, r16 = _pair(300, 384, seed=1) if residual else (None, None)
    y32 = N.linear(x32, w, b, r32)
    y16 = N.linear(x16, w, b, r16)
    _close(y16, y32, 2e-2)
    g = torch.randn_like(y32)
    grads32 = torch.autograd.grad(y32, [x32, w] + ([b] if bias else []), g)
    grads16 = torch.autograd.grad(y16, [x16, w] + ([b] if bias else []), g.to(torch.bfloat16))
    for a, c in zip(grads16, grads32):
        _close(a, c, 3e-2)


@pytest.mark.parametrize("rms", [False, True])
def test_norms(rms):
    x32, x16 = _pair(257, 1024, scale=3.0)
    w = torch.nn.Parameter(1 + 0.1 * torch.randn(1024, device=DEV))
    f = (lambda x: N.rms_norm(x, w, 1e-6)) if rms else (lambda x: N.layer_norm(x, w, None, 1e-5))
    y32, y16 = f(x32), f(x16)
    _close(y16, y32, 2e-2)
    g = torch.randn_like(y32)
    a = torch.autograd.grad(y16, [x16, w], g.to(torch.bfloat16))
    c = torch.autograd.grad(y32, [x32, w], g)
    for u, v in zip(a, c):
        _close(u, v, 3e-2)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("axes,norm", [(1, False), (1, True), (3, False)])
def test_rope(D, axes, norm):
    heads, T = 3, 200
    x32, x16 = _pair(T, heads * D, scale=2.0)
    pos = torch.randint(0, 5000, (axes, T), device=DEV, dtype=torch.int32)
    inv = N.rope_inv_freq(D, 10000.0, DEV)
    axis = torch.tensor(N.mrope_axis_table(D, (D // 8, D // 8 * 3 // 2, D // 8 * 3 // 2), interleaved=True),
                        device=DEV, dtype=torch.int32) if axes > 1 else None
    w = torch.nn.Parameter(1 + 0.1 * torch.randn(D, device=DEV)) if norm else None
    y32 = N.rope(x32, pos, inv, heads, axis_of=axis, norm_weight=w)
    y16 = N.rope(x16, pos, inv, heads, axis_of=axis, norm_weight=w)
    _close(y16, y32, 2e-2)
    g = torch.randn_like(y32)
    ins32 = [x32] + ([w] if norm else [])
    ins16 = [x16] + ([w] if norm else [])
    for a, c in zip(torch.autograd.grad(y16, ins16, g.to(torch.bfloat16)), torch.autograd.grad(y32, ins32, g)):
        _close(a, c, 3e-2)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("heads,kv,causal,window", [(4, 4, False, -1), (4, 2, True, -1), (4, 1, False, 20),
                                                    (2, 2, False, 64)])
def test_attention(D, heads, kv, causal, window):
    lengths = [130, 1, 77, 256, 64]
    T = sum(lengths)
    seg = _seg(lengths)
    q32, q16 = _pair(T, heads * D, seed=1)
    k32, k16 = _pair(T, kv * D, seed=2)
    v32, v16 = _pair(T, kv * D, seed=3)
    o32 = N.attention(q32, k32, v32, seg, heads=heads, kv_heads=kv, causal=causal, window=window)
    o16 = N.attention(q16, k16, v16, seg, heads=heads, kv_heads=kv, causal=causal, window=window)
    _close(o16, o32, 2e-2)
    g = torch.randn_like(o32)
    a = torch.autograd.grad(o16, [q16, k16, v16], g.to(torch.bfloat16))
    c = torch.autograd.grad(o32, [q32, k32, v32], g)
    for u, w in zip(a, c):
        _close(u, w, 4e-2)


@pytest.mark.parametrize("D,heads,kv", [(64, 4, 4), (128, 4, 2)])
def test_qkv_attention_with_rope_and_norm(D, heads, kv):
    lengths = [100, 37, 128]
    T = sum(lengths)
    seg = _seg(lengths)
    x32, x16 = _pair(T, (heads + 2 * kv) * D)
    pos = torch.cat([torch.arange(n) for n in lengths]).to(DEV, torch.int32)
    inv = N.rope_inv_freq(D, 1e6, DEV)
    qn = torch.nn.Parameter(1 + 0.1 * torch.randn(D, device=DEV))
    kn = torch.nn.Parameter(1 + 0.1 * torch.randn(D, device=DEV))
    kw = dict(heads=heads, kv_heads=kv, pos=pos, inv_freq=inv, q_norm=qn, k_norm=kn, causal=True)
    o32 = N.qkv_attention(x32, seg, **kw)
    o16 = N.qkv_attention(x16, seg, **kw)
    _close(o16, o32, 2e-2)
    g = torch.randn_like(o32)
    a = torch.autograd.grad(o16, [x16, qn, kn], g.to(torch.bfloat16))
    c = torch.autograd.grad(o32, [x32, qn, kn], g)
    for u, w in zip(a, c):
        _close(u, w, 4e-2)


@pytest.mark.parametrize("name", ["gelu", "gelu_pytorch_tanh", "silu", "quick_gelu"])
@pytest.mark.parametrize("gated", [False, True])
def test_activations(name, gated):
    z32, z16 = _pair(123, 512, scale=2.0)
    f = N.gated_activation if gated else N.activation
    y32, y16 = f(z32, name), f(z16, name)
    _close(y16, y32, 1e-2)
    g = torch.randn_like(y32)
    _close(torch.autograd.grad(y16, z16, g.to(torch.bfloat16))[0], torch.autograd.grad(y32, z32, g)[0], 2e-2)


def test_modernvbert_native_matches_reference():
    from representax_b200.models.modernvbert import ModernVBERTBatch, ModernVBERTConfig, ModernVBERTEncoder
    from representax_b200.models.modernvbert.config import ModernVBERTTextConfig, SigLIPVisionConfig

    cfg = ModernVBERTConfig(
        text=ModernVBERTTextConfig(vocab_size=512, hidden_size=256, intermediate_size=384, num_hidden_layers=4,
                                   num_attention_heads=4, local_attention=16, pad_token_id=0),
        vision=SigLIPVisionConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                                  image_size=64, patch_size=16),
        image_token_id=500, pixel_shuffle_factor=2)
    m32 = ModernVBERTEncoder(cfg, seed=0).to(DEV)
    m16 = ModernVBERTEncoder(cfg, seed=0, compute_dtype=torch.bfloat16).to(DEV)
    ids = torch.randint(3, 490, (3, 40))
    ids[:, 1:5] = 500
    mask = torch.ones_like(ids)
    mask[2, 30:] = 0
    pixels = torch.randn(3, 1, 3, 64, 64)
    b = ModernVBERTBatch(mask, ids, pixels).pack().map_tensors(lambda t: t.to(DEV))
    e32 = m32.encode(b)
    e16 = m16.encode(b)
    cos = torch.nn.functional.cosine_similarity(e16.float(), e32.float(), dim=-1)
    assert cos.min().item() > 0.995, cos
    e16.sum().backward()
    assert m16.vision.layers[0].qkv_w.grad is not None


def test_qwen3_vl_native_matches_reference():
    from representax_b200.models.qwen3 import Qwen3TextConfig
    from representax_b200.models.qwen3_vl import Qwen3VLBatch, Qwen3VLConfig, Qwen3VLEncoder, Qwen3VLVisionConfig

    cfg = Qwen3VLConfig(
        text=Qwen3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                             num_attention_heads=4, num_key_value_heads=2, head_dimension=64, mrope_section=(8, 12, 12),
                             pad_token_id=0),
        vision=Qwen3VLVisionConfig(depth=2, hidden_size=128, intermediate_size=256, num_heads=2, patch_size=8,
                                   out_hidden_size=256, num_position_embeddings=64, deepstack_visual_indexes=(0,)),
        image_token_id=500)
    m32 = Qwen3VLEncoder(cfg, seed=0).to(DEV)
    m16 = Qwen3VLEncoder(cfg, seed=0, compute_dtype=torch.bfloat16).to(DEV)
    ids = torch.randint(1, 490, (2, 48))
    ids[0, 2:18] = 500      # 8x8 patch grid -> 16 merged tokens
    ids[1, 5:21] = 500
    mask = torch.ones_like(ids)
    mask[1, 40:] = 0
    grid = torch.tensor([[1, 8, 8], [1, 8, 8]])
    pixels = torch.randn(128, 3 * 2 * 8 * 8)
    b = Qwen3VLBatch(ids, mask, pixels, grid).prepare(cfg)
    e32 = m32.encode(b)
    e16 = m16.encode(b)
    cos = torch.nn.functional.cosine_similarity(e16.float(), e32.float(), dim=-1)
    assert cos.min().item() > 0.99, cos
    e16.sum().backward()
    assert m16.text.layers[0].q_norm.grad is not None


@pytest.mark.parametrize("bias", [False, True])
def test_fp8_linear_matches_fake_quant_reference(bias):
    from representax_b200.ops.fp8 import linear_fp8, linear_fp8_reference, quantize_reference

    g = torch.Generator(device=DEV).manual_seed(3)
    x = (torch.randn(500, 384, device=DEV, generator=g) * 2).to(torch.bfloat16).requires_grad_()
    w = torch.nn.Parameter(torch.randn(640, 384, device=DEV, generator=g) * 0.05)
    b = torch.nn.Parameter(torch.randn(640, device=DEV, generator=g)) if bias else None
    # 500 rows: not a multiple of 16, exercising the padded transposed operands
    y = linear_fp8(x, w, b)
    ref = linear_fp8_reference(x.detach(), w.detach().to(torch.bfloat16), None if b is None else b.detach())
    _close(y, ref, 1e-2)
    # the fp8 product is close to the exact product too
    _close(y, x.float() @ w.T.float() + (0 if b is None else b.float()), 8e-2)
    dy = torch.randn_like(y)
    dx, dw = torch.autograd.grad(y, [x, w], dy)
    dyq, sdy = quantize_reference(dy, 1)
    wq, sw = quantize_reference(w.detach().to(torch.bfloat16), 0)
    xq, sx = quantize_reference(x.detach(), 0)
    _close(dx, (dyq @ wq) * (sdy * sw), 2e-2)
    _close(dw, (dyq.T @ xq) * (sdy * sx), 2e-2)


def test_fp8_policy_routes_modernvbert_linears():
    from representax_b200.models.modernvbert import ModernVBERTConfig, ModernVBERTEncoder
    from representax_b200.models.modernvbert.config import ModernVBERTTextConfig, SigLIPVisionConfig
    from representax_b200.models.text_batch import TokenBatch
    from representax_b200.precision import BF16_MIXED_POLICY, FP8_MIXED_POLICY, precision_context

    cfg = ModernVBERTConfig(
        text=ModernVBERTTextConfig(vocab_size=512, hidden_size=256, intermediate_size=384, num_hidden_layers=2,
                                   num_attention_heads=4, local_attention=16, pad_token_id=0),
        vision=SigLIPVisionConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=1, num_attention_heads=4,
                                  image_size=64, patch_size=16), image_token_id=500, pixel_shuffle_factor=2)
    m = ModernVBERTEncoder(cfg, seed=0, compute_dtype=torch.bfloat16).to(DEV)
    ids = torch.randint(3, 490, (4, 64))
    b = TokenBatch(attention_mask=torch.ones_like(ids), input_ids=ids).pack().map_tensors(lambda t: t.to(DEV))
    with precision_context(BF16_MIXED_POLICY):
        e16 = m.encode(b)
    with precision_context(FP8_MIXED_POLICY):
        e8 = m.encode(b)
        e8.sum().backward()
    cos = torch.nn.functional.cosine_similarity(e8.float(), e16.float(), dim=-1)
    assert cos.min().item() > 0.98, cos
    assert m.text.layers[0].Wqkv.grad is not None


@pytest.mark.parametrize("mainloop", [False, True])
def test_int4_lora_linear_native_matches_reference(mainloop):
    from representax_b200.models.adapters import QuantizedLoRAWeight, unpack_int4_rows

    g = torch.Generator().manual_seed(0)
    w = torch.randn(384, 256, generator=g) * 0.05
    q = QuantizedLoRAWeight(w, rank=16, alpha=32.0, seed=1).to(DEV)
    q.mainloop_dequant = mainloop  # packed nibbles expanded inside the tcgen05 main loop
    assert q.fused_int4()
    with torch.no_grad():
        q.lora_b.normal_(0, 0.02, generator=torch.Generator(device=DEV).manual_seed(2))
    base = q.base_weight_bf16()
    torch.testing.assert_close(base.float(), unpack_int4_rows(q.packed_weight, q.scale_bits, 256).float())
    x32, x16 = _pair(300, 256)
    bias = torch.nn.Parameter(torch.randn(384, device=DEV) * 0.1)
    y32 = q.linear(x32, bias)
    y16 = N.linear(x16, q, bias)
    _close(y16, y32, 2e-2)
    dy = torch.randn_like(y32)
    a = torch.autograd.grad(y16, [x16, q.lora_a, q.lora_b, bias], dy.to(torch.bfloat16))
    c = torch.autograd.grad(y32, [x32, q.lora_a, q.lora_b, bias], dy)
    for u, v in zip(a, c):
        _close(u, v, 4e-2)


def test_dropout_epilogue_and_pointwise_share_masks():
    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import ext

    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(700, 256, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(384, 256, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(384, device=DEV, generator=g).to(torch.bfloat16)
    r = torch.randn(700, 384, device=DEV, generator=g).to(torch.bfloat16)
    p = 0.25
    y0 = G.linear_forward(x, w, b).float()
    y1 = G.linear_forward(x, w, b, residual=r, dropout=(1234, 7, p)).float() - r.float()
    ones = torch.ones(700, 384, device=DEV, dtype=torch.bfloat16)
    mask = torch.empty_like(ones)
    ext().dropout_apply(ones, mask, 1234, 7, p, None)
    keep = mask.float() > 0
    assert abs(1 - keep.float().mean().item() - p) < 0.01
    torch.testing.assert_close(mask.float()[keep], torch.full_like(mask.float()[keep], 1 / (1 - p)), rtol=1e-2, atol=0)
    _close(y1, y0 * keep / (1 - p), 3e-2)
    other = torch.empty_like(ones)
    ext().dropout_apply(ones, other, 1235, 7, p, None)
    assert (other != mask).any()


@pytest.mark.parametrize("D", [64, 128])
def test_attention_dropout_gradient_is_consistent(D):
    """Directional derivative of the dropped-out attention matches its backward (same Philox mask)."""

    from representax_b200.ops._ext import ext

    C = ext()
    lengths = [90, 130, 33]
    T, heads = sum(lengths), 2
    seg = _seg(lengths)
    g = torch.Generator(device=DEV).manual_seed(1)
    q, k, v = (torch.randn(T, heads * D, device=DEV, generator=g) for _ in range(3))
    do = torch.randn(T, heads * D, device=DEV, generator=g)
    dirs = [torch.randn(T, heads * D, device=DEV, generator=g) for _ in range(3)]
    scale, p, seed = D ** -0.5, 0.2, 99

    def fwd(qq, kk, vv):
        o = torch.empty(T, heads * D, device=DEV, dtype=torch.bfloat16)
        lse = torch.empty(heads, T, device=DEV)
        C.attention_forward(qq.bfloat16(), kk.bfloat16(), vv.bfloat16(), o, lse, seg.cu_seqlens, seg.max_len, heads,
                            heads, scale, False, -1, seed, 3, p, None)
        return o, lse

    o, lse = fwd(q, k, v)
    o_again, _ = fwd(q, k, v)
    assert torch.equal(o, o_again)
    dq, dk, dv = (torch.empty(T, heads * D, device=DEV, dtype=torch.bfloat16) for _ in range(3))
    acc = torch.empty(T, heads * D, device=DEV)
    dvec = torch.empty(heads, T, device=DEV)
    C.attention_backward(do.bfloat16(), q.bfloat16(), k.bfloat16(), v.bfloat16(), o, lse, dq, dk, dv, acc, dvec,
                         seg.cu_seqlens, seg.max_len, heads, heads, scale, False, -1, seed, 3, p, None, None)
    eps = 0.25
    base = [x.bfloat16().float() for x in (q, k, v)]
    for i, grad in enumerate((dq, dk, dv)):
        args_p, args_m = list(base), list(base)
        # the perturbation actually seen by the bf16 kernel
        plus = (base[i] + eps * dirs[i]).bfloat16().float()
        minus = (base[i] - eps * dirs[i]).bfloat16().float()
        args_p[i], args_m[i] = plus, minus
        eff = (plus - minus) / (2 * eps)
        num = ((fwd(*args_p)[0].float() - fwd(*args_m)[0].float()) * do).sum() / (2 * eps)
        o_b, lse_b = fwd(*base)
        C.attention_backward(do.bfloat16(), *(x.bfloat16() for x in base), o_b, lse_b, dq, dk, dv, acc, dvec,
                             seg.cu_seqlens, seg.max_len, heads, heads, scale, False, -1, seed, 3, p, None, None)
        ana = (grad.float() * eff).sum()
        assert abs(num - ana) <= 0.1 * abs(ana) + 1.0, (i, float(num), float(ana))


def test_bert_native_dropout_replays_exactly():
    from representax_b200.models.bert import BertConfig, BertEncoder
    from representax_b200.models.text_batch import TokenBatch
    from representax_b200.train.rng import generator

    cfg = BertConfig(vocab_size=1000, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                     intermediate_size=512, max_position_embeddings=128)   # dropout 0.1 / 0.1
    m = BertEncoder(cfg, seed=0, compute_dtype=torch.bfloat16).to(DEV)
    ids = torch.randint(5, 900, (6, 40))
    mask = torch.ones_like(ids)
    mask[3, 25:] = 0
    b = TokenBatch(attention_mask=mask, input_ids=ids).pack().map_tensors(lambda t: t.to(DEV))
    e1 = m.encode(b, generator=generator(DEV, 1, "x"))
    e2 = m.encode(b, generator=generator(DEV, 1, "x"))
    e3 = m.encode(b, generator=generator(DEV, 2, "x"))
    e0 = m.encode(b)
    assert torch.equal(e1, e2)
    assert not torch.equal(e1, e3)
    cos = torch.nn.functional.cosine_similarity(e1, e0, dim=-1)
    assert 0.8 < cos.min().item() < 0.99999


def test_mpnet_native_relative_bias_matches_reference():
    from representax_b200.models.mpnet import MPNetConfig, MPNetEncoder
    from representax_b200.models.text_batch import TokenBatch

    cfg = MPNetConfig(vocab_size=600, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      intermediate_size=512, max_position_embeddings=300, hidden_dropout_probability=0.0,
                      attention_dropout_probability=0.0)
    m32 = MPNetEncoder(cfg, seed=0).to(DEV)
    m16 = MPNetEncoder(cfg, seed=0, compute_dtype=torch.bfloat16).to(DEV)
    with torch.no_grad():  # a bias large enough to matter
        for m in (m32, m16):
            m.relative_attention_bias.normal_(0, 1.0, generator=torch.Generator(device=DEV).manual_seed(5))
    ids = torch.randint(5, 590, (5, 200))
    mask = torch.ones_like(ids)
    mask[1, 150:] = 0
    mask[4, 30:] = 0
    ids[mask == 0] = cfg.pad_token_id
    host = TokenBatch(attention_mask=mask, input_ids=ids)
    e32 = m32.encode(host.map_tensors(lambda t: t.to(DEV)))
    b16 = host.pack().map_tensors(lambda t: t.to(DEV))
    assert m16._native(b16)
    e16 = m16.encode(b16)
    cos = torch.nn.functional.cosine_similarity(e16.float(), e32.float(), dim=-1)
    assert cos.min().item() > 0.995, cos
    (e32 * torch.arange(256, device=DEV)).sum().backward()
    (e16 * torch.arange(256, device=DEV)).sum().backward()
    g32 = m32.relative_attention_bias.grad
    g16 = m16.relative_attention_bias.grad
    assert torch.nn.functional.cosine_similarity(g16.flatten(), g32.flatten(), dim=0) > 0.98


def test_fused_column_sums_match():
    from representax_b200.ops import gemm as G
    from representax_b200.ops._ext import ext

    g = torch.Generator(device=DEV).manual_seed(4)
    dy = torch.randn(900, 768, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(768, 3072, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    z = torch.randn(900, 3072, device=DEV, generator=g).to(torch.bfloat16)
    cs = torch.zeros(3072, device=DEV)
    dz = G.linear_dgrad(dy, w, gelu_grad=z, colsum=cs)
    _close(cs, dz.float().sum(0), 2e-3)
    small = torch.zeros(3072, device=DEV)  # < 256 rows: the column sums run after the GEMM
    dz_s = G.linear_dgrad(dy[:100], w, gelu_grad=z[:100], colsum=small)
    _close(small, dz_s.float().sum(0), 2e-3)
    x = torch.randn(1000, 768, device=DEV, generator=g).to(torch.bfloat16)
    out = torch.empty_like(x)
    cs2 = torch.zeros(768, device=DEV)
    ext().dropout_apply(x, out, 7, 3, 0.1, cs2)
    ref = torch.empty_like(x)
    ext().dropout_apply(x, ref, 7, 3, 0.1, None)
    assert torch.equal(out, ref)
    _close(cs2, out.float().sum(0), 2e-3)
