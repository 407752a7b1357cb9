"""Allocation-free decode attention, checked against the allocating entry point.

Some callers of this library cannot call cudaMalloc: code that runs inside another
framework's CUDA-graph capture or private memory pool, or a host whose allocator
owns all device memory.  For them, rngd_attn_decode_noalloc keeps its chunk
partials in a scratch array built into the library instead of a buffer the caller
allocates.  These tests call it through the C ABI and compare its output with
rngd_attn_decode given caller-owned scratch and with fp32 numpy attention (up to S=1024),
on two calls in a row with different
shapes (the second call must not be affected by what the first left in the shared
scratch), and check that a request larger than the built-in scratch is refused.
This file sorts last so that a run stopping at the first failure has already run
every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 8, 128


def _inputs(seed, B, S, positions):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, NH * HD, generator=g).cuda()
    K = torch.randn(B, NKV, S, HD, generator=g).to(torch.bfloat16).cuda()
    V = torch.randn(B, NKV, S, HD, generator=g).to(torch.bfloat16).cuda()
    pos = torch.tensor(positions, dtype=torch.int32).cuda()
    return q, K, V, pos


def _attn_with_scratch(q, K, V, pos, B, S):
    from rngd_pd import _lib
    part = torch.empty(B, NH, S // 128, HD + 2, device="cuda")
    ao = torch.empty(B, NH * HD, device="cuda")
    _lib.call("rngd_attn_decode", _lib.ptr(q), _lib.ptr(K), _lib.ptr(V), _lib.ptr(pos), B, B, NH, NKV, HD, S,
              _lib.ptr(part), _lib.ptr(ao), _lib.stream_handle())
    return ao


def _attn_noalloc(q, K, V, pos, B, S):
    from rngd_pd import _lib
    ao = torch.empty(B, NH * HD, device="cuda")
    _lib.call("rngd_attn_decode_noalloc", _lib.ptr(q), _lib.ptr(K), _lib.ptr(V), _lib.ptr(pos), B, B, NH, NKV,
              HD, S, _lib.ptr(ao), _lib.stream_handle())
    return ao


def _attn_numpy(q, K, V, positions):
    """Softmax attention over positions 0..pos of each stream, in fp32 numpy."""
    B = len(positions)
    Kf, Vf = K.float().cpu().numpy(), V.float().cpu().numpy()
    qn = q.cpu().numpy().reshape(B, NKV, NH // NKV, HD)
    out = np.empty((B, NH * HD), np.float32)
    for b, p in enumerate(positions):
        sc = np.einsum("kgh,ksh->kgs", qn[b], Kf[b][:, :p + 1]) / np.sqrt(HD)
        sc -= sc.max(-1, keepdims=True)
        pr = np.exp(sc)
        pr /= pr.sum(-1, keepdims=True)
        out[b] = np.einsum("kgs,ksh->kgh", pr, Vf[b][:, :p + 1]).reshape(-1)
    return out


def test_noalloc_attention_matches_allocating_entry_point():
    # first call: the config-4 shape (16 streams, S=512, long contexts);
    # second call: fewer streams, a wider cache, short contexts, so most of the
    # scratch the first call filled is stale and must not leak into the result
    cases = [(1, 16, 512, [100 + 25 * b for b in range(16)]),
             (2, 5, 1024, [0, 3, 127, 128, 700])]
    for seed, B, S, positions in cases:
        q, K, V, pos = _inputs(seed, B, S, positions)
        want = _attn_with_scratch(q, K, V, pos, B, S)
        got = _attn_noalloc(q, K, V, pos, B, S)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(got.cpu().numpy(), _attn_numpy(q, K, V, positions), rtol=1e-4, atol=1e-5)


def test_noalloc_refuses_requests_beyond_its_scratch():
    from rngd_pd import _lib
    B, S = 16, 2048                      # 16 x 32 x 16 = 8192 partial records > 4096
    q, K, V, pos = _inputs(3, B, S, [5] * B)
    with pytest.raises(_lib.RngdError) as e:
        _attn_noalloc(q, K, V, pos, B, S)
    assert e.value.status == _lib.RNGD_ERR_ARG
    assert "exceed the built-in scratch" in str(e.value)
