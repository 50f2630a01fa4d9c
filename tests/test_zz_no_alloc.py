"""The allocation-free attention backward, called through its exported C symbol.

``rx_attention_backward_noalloc`` serves callers that may not allocate device
memory during a step (a host runtime that owns a fixed pool, or an embedder
without a device allocator): it takes its scratch from a static array inside
the library. This test loads the symbol with ctypes, runs it twice in a row
(the second call must not see the first call's leftover scratch) and compares
its dQ/dK/dV with the regular entry point, which allocates its scratch through
PyTorch, for full, causal and windowed attention; it checks that a call after
the first one changes neither PyTorch's allocations nor the device's free
memory, and that an oversized problem is rejected.

This file is named to be collected last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

RX_NOALLOC_OK = 0
RX_NOALLOC_TOO_LARGE = 1


def _entry():
    from representax_b200 import _C  # noqa: F401  (loads the library into the process)

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.rx_attention_backward_noalloc
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    fn.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, vp, i64, vp, i64,
                   vp, i64, vp]
    fn.restype = ctypes.c_int
    err = lib.rx_noalloc_error_string
    err.argtypes = [ctypes.c_int]
    err.restype = ctypes.c_char_p
    lib.rx_noalloc_last_cuda_error.restype = ctypes.c_int
    return fn, err


def _problem(seed, lens, heads):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    total = sum(lens)
    hd = heads * 64
    qkv = torch.randn(total, 3 * hd, generator=g, device=dev).to(torch.bfloat16)
    do = torch.randn(total, hd, generator=g, device=dev).to(torch.bfloat16)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
    return qkv, do, cu, total, hd


def _reference(C, qkv, do, cu, total, hd, heads, lens, causal=False, window=-1):
    q, k, v = qkv[:, :hd], qkv[:, hd:2 * hd], qkv[:, 2 * hd:]
    o = torch.empty(total, hd, dtype=torch.bfloat16, device=qkv.device)
    lse = torch.empty(heads, total, device=qkv.device)
    C.attention_forward(q, k, v, o, lse, cu, max(lens), heads, heads, 0.125, causal, window, 0, 0, 0.0, None)
    dqkv = torch.empty_like(qkv)
    acc = torch.empty(total, hd, device=qkv.device)
    dvec = torch.empty(heads, total, device=qkv.device)
    C.attention_backward(do, q, k, v, o, lse, dqkv[:, :hd], dqkv[:, hd:2 * hd], dqkv[:, 2 * hd:], acc, dvec,
                         cu, max(lens), heads, heads, 0.125, causal, window, 0, 0, 0.0, None, None)
    return o, lse, dqkv


def _call(fn, qkv, do, o, lse, cu, total, hd, heads, lens, out, causal=False, window=-1, stream=None):
    q, k, v = qkv[:, :hd], qkv[:, hd:2 * hd], qkv[:, 2 * hd:]
    ld = qkv.stride(0)
    stream = torch.cuda.current_stream().cuda_stream if stream is None else stream
    return fn(do.data_ptr(), do.stride(0), q.data_ptr(), ld, k.data_ptr(), ld, v.data_ptr(), ld,
              o.data_ptr(), o.stride(0), lse.data_ptr(), cu.data_ptr(), len(lens), total, max(lens), heads,
              0.125, int(causal), window, out[:, :hd].data_ptr(), out.stride(0), out[:, hd:2 * hd].data_ptr(),
              out.stride(0), out[:, 2 * hd:].data_ptr(), out.stride(0), stream)


def _close(actual, expected, rtol=3e-2, atol=3e-2):
    err = (actual.float() - expected.float()).abs()
    assert bool((err <= atol + rtol * expected.float().abs()).all()), f"max err {err.max().item():.3e}"


def test_noalloc_attention_backward_matches_regular_entry_point():
    from representax_b200.ops._ext import ext

    C = ext()
    fn, err = _entry()
    heads = 4
    # Two different problems back to back: the second runs on the scratch the
    # first one left behind.
    cases = ((0, [1, 17, 64, 65, 200], False, -1), (1, [130, 3, 256, 40], False, -1),
             (2, [90, 200, 7], True, -1), (3, [150, 64, 33], False, 24))
    for i, (seed, lens, causal, window) in enumerate(cases):
        qkv, do, cu, total, hd = _problem(seed, lens, heads)
        o, lse, ref = _reference(C, qkv, do, cu, total, hd, heads, lens, causal, window)
        out = torch.full_like(qkv, float("nan"))
        torch.cuda.synchronize()
        allocated, (free, _) = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()
        rc = _call(fn, qkv, do, o, lse, cu, total, hd, heads, lens, out, causal, window)
        torch.cuda.synchronize()
        assert rc == RX_NOALLOC_OK, err(rc).decode()
        if i > 0:  # the first call on the device may set up its module state; later calls allocate nothing
            assert torch.cuda.memory_allocated() == allocated
            assert torch.cuda.mem_get_info()[0] == free
        _close(out, ref)


def test_noalloc_rejects_problems_beyond_its_scratch():
    fn, err = _entry()
    heads = 12
    lens = [256] * 64  # 16,384 tokens x 12 heads needs about 49 MiB of scratch
    qkv, do, cu, total, hd = _problem(2, lens, heads)
    o = torch.zeros(total, hd, dtype=torch.bfloat16, device=qkv.device)
    lse = torch.zeros(heads, total, device=qkv.device)
    out = torch.zeros_like(qkv)
    rc = _call(fn, qkv, do, o, lse, cu, total, hd, heads, lens, out)
    assert rc == RX_NOALLOC_TOO_LARGE
    assert b"static array" in err(rc)


def test_noalloc_rejects_a_stream_of_another_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    fn, err = _entry()
    heads, lens = 2, [64, 32]
    qkv, do, cu, total, hd = _problem(4, lens, heads)
    o = torch.zeros(total, hd, dtype=torch.bfloat16, device=qkv.device)
    lse = torch.zeros(heads, total, device=qkv.device)
    out = torch.zeros_like(qkv)
    other = torch.cuda.Stream(device=1)
    rc = _call(fn, qkv, do, o, lse, cu, total, hd, heads, lens, out, stream=other.cuda_stream)
    assert rc == 2 and b"stream" in err(rc)
