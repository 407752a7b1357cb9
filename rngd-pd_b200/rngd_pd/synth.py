"""Seeded synthetic Llama weights and KV, generated on the device.

BASELINE.json measures random-init bf16 weights ~N(0, 0.02), seeded bf16 KV
~N(0, 1) and uniform token ids, since no checkpoint is available.  A
``SyntheticState`` stands in for the reference engines' HF state dict (`sd`,
src/rngd_pd/engines/decode_batch.py:175-219): the engines recognise it and
fill their HBM layouts directly with the kernel rngd_synth_gauss_bf16 (integer
splitmix64 / Irwin-Hall recipe of include/rngd_b200.h), so an 8B model
materialises in milliseconds instead of a 16 GB host upload.

Tensor ids (shared with the test oracle's CPU generator): layer l, kind k ->
l*16 + k with k = q, k, v, o, gate, up, down = 0..6; embed 0x7000;
lm_head 0x7001; KV cache K/V 0x8000/0x8001; tokens 0x9000; lengths 0x9001.
RMSNorm weights are 1.0 (HF initialisation).
"""
import math

from rngd_pd import _lib

T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN = range(7)
T_EMBED, T_LMHEAD = 0x7000, 0x7001
T_KCACHE, T_VCACHE = 0x8000, 0x8001
T_TOKENS, T_CTXLEN = 0x9000, 0x9001


def gauss_scale(sigma):
    """fp32 multiplier giving the Irwin-Hall(4) sum a standard deviation of sigma."""
    import numpy as np
    return float(np.float32(sigma / math.sqrt(4.0 * (65536.0 ** 2 - 1.0) / 12.0)))


def fill_gauss(t, seed, tid, sigma, start=0, stream=None):
    """Fill a contiguous bf16 device tensor with the seeded recipe (flat C-order index)."""
    import torch
    assert t.dtype == torch.bfloat16 and t.is_cuda and t.is_contiguous()
    _lib.call("rngd_synth_gauss_bf16", _lib.ptr(t), t.numel(), seed, tid, start, gauss_scale(sigma),
              _lib.stream_handle(stream))
    return t


def uniform_i32(n, seed, tid, hi, device="cuda", start=0):
    import torch
    t = torch.empty(n, dtype=torch.int32, device=device)
    _lib.call("rngd_synth_uniform_i32", _lib.ptr(t), n, seed, tid, start, hi, _lib.stream_handle())
    return t


def tokens(n, seed=2, vocab=128256):
    """Token ids U[0, vocab) (config 1: seed 2)."""
    return [int(v) for v in uniform_i32(n, seed, T_TOKENS, vocab).cpu()]


def context_lengths(n, seed=3, lo=64, hi=384):
    """Per-sequence past lengths U[lo, hi] (config 4 reading: L + 128 <= 512)."""
    return [lo + int(v) for v in uniform_i32(n, seed, T_CTXLEN, hi - lo + 1).cpu()]


class SyntheticState:
    """Stand-in for an HF state dict: describes seeded random-init weights."""

    def __init__(self, cfg, seed=0, sigma=0.02):
        self.cfg, self.seed, self.sigma = cfg, seed, sigma


def request_kv(cfg, S, seed, length, device="cuda", sigma=1.0):
    """One request's past KV in the reference layout K [L, NKV, HD, S], V [L, NKV, S, HD] (bf16).

    Positions < length are ~N(0, sigma) drawn in [L, NKV, pos, HD] order under
    the request's own seed; the tail is zero (the decode step's one-hot
    injection needs it, src/rngd_pd/engines/prefill_full.py:287-289).
    """
    import torch
    shape = (cfg.n_layers, cfg.n_kv, S, cfg.head_dim)
    K = fill_gauss(torch.empty(shape, dtype=torch.bfloat16, device=device), seed, T_KCACHE, sigma)
    V = fill_gauss(torch.empty(shape, dtype=torch.bfloat16, device=device), seed, T_VCACHE, sigma)
    K[:, :, length:] = 0
    V[:, :, length:] = 0
    return K.transpose(2, 3).contiguous(), V


def handoff_kv(cfg, S, seed, device="cuda", sigma=1.0):
    """One request's cache in the prefill layout [L, 2, NKV, S, HD] bf16, every position
    ~N(0, sigma) under the request's seed: K from the (seed, 0x8000) stream and V from
    (seed, 0x8001), each drawn in [L, NKV, S, HD] order (the KV handoff workload)."""
    import torch
    shape = (cfg.n_layers, cfg.n_kv, S, cfg.head_dim)
    kv = torch.empty((cfg.n_layers, 2) + shape[1:], dtype=torch.bfloat16, device=device)
    kv[:, 0] = fill_gauss(torch.empty(shape, dtype=torch.bfloat16, device=device), seed, T_KCACHE, sigma)
    kv[:, 1] = fill_gauss(torch.empty(shape, dtype=torch.bfloat16, device=device), seed, T_VCACHE, sigma)
    return kv
