"""numpy fp32 restatement of the reference's CPU path (test infrastructure only).

Each function names the reference lines it follows.  ``kv_bf16=False`` gives
the reference's arithmetic exactly (fp32 k/v); ``kv_bf16=True`` additionally
rounds every k/v written to the cache to bf16 before attention reads it, which
is what the device path stores (the reference's device graph also emits bf16
K/V: src/rngd_pd/kernels/decode_batch.py:78-82).  Everything else stays fp32.

Layouts follow the reference: decode caches K [B, NKV, HD, S], V [B, NKV, S, HD]
(kernels/decode_batch.py:81-82); prefill emits kT [NKV, HD, C], vT [NKV, C, HD]
(kernels/prefill_full.py:64-65).
"""
import math
from dataclasses import dataclass

import numpy as np

from oracle import synth_np as sy


@dataclass(frozen=True)
class Dims:
    H: int = 4096
    M: int = 14336
    NH: int = 32
    NKV: int = 8
    HD: int = 128
    L: int = 32
    V: int = 128256
    eps: float = 1e-5
    theta: float = 500000.0

    @property
    def G(self):
        return self.NH // self.NKV


LLAMA8B = Dims()


def inv_freq(d: Dims):
    """kernels/decode_batch.py:197 (float64 power, cast to fp32)."""
    return (1.0 / (d.theta ** (np.arange(0, d.HD, 2) / d.HD))).astype(np.float32)


def rms(t, g, eps):
    """kernels/decode_batch.py:130."""
    return t * (1.0 / np.sqrt((t * t).mean(-1, keepdims=True) + eps)) * g


def _rope_rows(t, pos_list, inv, nh, HD):
    """kernels/decode_batch.py:133-142 (HF rotate-half), one position per row."""
    R = t.shape[0]
    t = t.reshape(R, nh, HD).copy()
    half = HD // 2
    for r in range(R):
        ang = np.float32(pos_list[r]) * inv
        cs, sn = np.cos(ang), np.sin(ang)
        a, bb = t[r, :, :half].copy(), t[r, :, half:].copy()
        t[r, :, :half] = a * cs - bb * sn
        t[r, :, half:] = bb * cs + a * sn
    return t


def cpu_layer(x, w, Kp, Vp, inv, positions, S, eps, d: Dims = LLAMA8B, kv_bf16=False):
    """Batched decode layer: restates kernels/decode_batch.py:126-161.

    w = (n1, wq, wk, wv, wo, n2, wgu, wd) with HF [out, in] weights and
    wgu = [gate; up] stacked [2M, H] (kernels/decode_batch.py:128,159-161).
    """
    n1, wq, wk, wv, wo, n2, wgu, wd = w
    B = x.shape[0]
    NH, NKV, HD, G, M = d.NH, d.NKV, d.HD, d.G, d.M
    h = rms(x, n1, eps)
    q = _rope_rows(h @ wq.T, positions, inv, NH, HD)
    k = _rope_rows(h @ wk.T, positions, inv, NKV, HD)
    v = (h @ wv.T).reshape(B, NKV, HD)
    if kv_bf16:
        k, v = sy.bf16_round(k), sy.bf16_round(v)
    K, V = Kp.copy(), Vp.copy()
    for b in range(B):
        K[b, :, :, positions[b]] = k[b]
        V[b, :, positions[b], :] = v[b]
    sc = np.einsum("bkgh,bkhs->bkgs", q.reshape(B, NKV, G, HD), K) / math.sqrt(HD)
    for b in range(B):
        sc[b, :, :, positions[b] + 1:] = -1e4
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    ao = np.einsum("bkgs,bksh->bkgh", p, V).reshape(B, NH * HD)
    x2 = ao @ wo.T + x
    h2 = rms(x2, n2, eps)
    gu = h2 @ wgu.T
    g_, u_ = gu[:, :M], gu[:, M:]
    return (g_ / (1 + np.exp(-g_)) * u_) @ wd.T + x2, K, V


def cpu_layer_p(x, w, inv, C, eps, d: Dims = LLAMA8B, kv_bf16=False):
    """KV-free whole-prompt prefill layer: restates kernels/prefill_full.py:97-128."""
    n1, wq, wk, wv, wo, n2, wgu, wd = w
    NH, NKV, HD, G, M = d.NH, d.NKV, d.HD, d.G, d.M
    h = rms(x, n1, eps)
    pos = list(range(C))
    q = _rope_rows(h @ wq.T, pos, inv, NH, HD)
    k = _rope_rows(h @ wk.T, pos, inv, NKV, HD)
    v = (h @ wv.T).reshape(C, NKV, HD)
    if kv_bf16:
        k, v = sy.bf16_round(k), sy.bf16_round(v)
    kT, vT = k.transpose(1, 2, 0), v.transpose(1, 0, 2)
    qk = q.reshape(C, NKV, G, HD).transpose(1, 2, 0, 3)
    sc = np.einsum("kgch,khd->kgcd", qk, kT) / math.sqrt(HD)
    m = np.triu(np.full((C, C), -1e4, np.float32), 1)
    sc = sc + m[None, None]
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    ao = np.einsum("kgcd,kdh->kgch", p, vT).transpose(2, 0, 1, 3).reshape(C, NH * HD)
    x2 = ao @ wo.T + x
    h2 = rms(x2, n2, eps)
    gu = h2 @ wgu.T
    g_, u_ = gu[:, :M], gu[:, M:]
    return (g_ / (1 + np.exp(-g_)) * u_) @ wd.T + x2, kT, vT


def cpu_layer_chunk(x, w, Kp, Vp, inv, base, C, S, eps, d: Dims = LLAMA8B, kv_bf16=False):
    """Chunked prefill against a live S-wide cache: restates kernels/prefill_chunk.py:198-232."""
    n1, wq, wk, wv, wo, n2, wgu, wd = w
    NH, NKV, HD, G, M = d.NH, d.NKV, d.HD, d.G, d.M
    h = rms(x, n1, eps)
    pos = [base + c for c in range(C)]
    q = _rope_rows(h @ wq.T, pos, inv, NH, HD)
    k = _rope_rows(h @ wk.T, pos, inv, NKV, HD)
    v = (h @ wv.T).reshape(C, NKV, HD)
    if kv_bf16:
        k, v = sy.bf16_round(k), sy.bf16_round(v)
    Kf, Vf = Kp.copy(), Vp.copy()
    Kf[:, :, base:base + C] = k.transpose(1, 2, 0)
    Vf[:, base:base + C, :] = v.transpose(1, 0, 2)
    qk = q.reshape(C, NKV, G, HD).transpose(1, 2, 0, 3)
    sc = np.einsum("kgch,khs->kgcs", qk, Kf) / math.sqrt(HD)
    m = np.full((C, S), -1e4, np.float32)
    for c in range(C):
        m[c, :base + c + 1] = 0.0
    sc = sc + m[None, None]
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    ao = np.einsum("kgcs,ksh->kgch", p, Vf).transpose(2, 0, 1, 3).reshape(C, NH * HD)
    x2 = ao @ wo.T + x
    h2 = rms(x2, n2, eps)
    gu = h2 @ wgu.T
    g_, u_ = gu[:, :M], gu[:, M:]
    return (g_ / (1 + np.exp(-g_)) * u_) @ wd.T + x2, Kf, Vf


def rot_batch(inv, positions, HD=128):
    """[B, HD, HD] block rotations: restates kernels/decode_batch.py:112-123."""
    half = HD // 2
    ang = np.asarray(positions)[:, None] * inv[None, :]
    cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out = np.zeros((len(positions), HD, HD), np.float32)
    i = np.arange(half)
    out[:, i, i] = cs
    out[:, i + half, i + half] = cs
    out[:, i, i + half] = sn
    out[:, i + half, i] = -sn
    return out


def lm_logits(x, norm, lm, eps):
    """Final rms + lm_head: engines/model.py:117 batched (engines/decode_batch.py:127-129)."""
    return rms(x, norm, eps) @ lm.T


def greedy(logits):
    """First-max argmax per row: engines/decode_batch.py:162-171."""
    return [int(i) for i in np.argmax(logits, axis=-1)]


# ---------------------------------------------------------------------------
# synthetic model (random-init Llama shape) in the reference's cpu_layer format
# ---------------------------------------------------------------------------
class SynthModel:
    """Seeded random-init weights, bf16-valued fp32, HF [out, in] layout.

    Projections ~N(0, sigma) through oracle.synth_np; RMSNorm weights = 1.0
    (the HF initialisation; the reference's own validation scripts draw them
    at random, kernels/decode_batch.py:186-193).
    """

    def __init__(self, d: Dims, seed=0, sigma=0.02):
        self.d, self.seed, self.sigma = d, seed, sigma
        self._layers = {}

    def w(self, layer, kind):
        d = self.d
        shape = {sy.T_Q: (d.NH * d.HD, d.H), sy.T_K: (d.NKV * d.HD, d.H),
                 sy.T_V: (d.NKV * d.HD, d.H), sy.T_O: (d.H, d.NH * d.HD),
                 sy.T_GATE: (d.M, d.H), sy.T_UP: (d.M, d.H), sy.T_DOWN: (d.H, d.M)}[kind]
        return sy.gauss_bf16(self.seed, sy.layer_tid(layer, kind), shape, self.sigma)

    def layer(self, i):
        """(n1, wq, wk, wv, wo, n2, wgu, wd) for cpu_layer / cpu_layer_p."""
        if i not in self._layers:
            d = self.d
            ones = np.ones(d.H, np.float32)
            wgu = np.concatenate([self.w(i, sy.T_GATE), self.w(i, sy.T_UP)], 0)
            self._layers[i] = (ones, self.w(i, sy.T_Q), self.w(i, sy.T_K), self.w(i, sy.T_V),
                               self.w(i, sy.T_O), ones.copy(), wgu, self.w(i, sy.T_DOWN))
        return self._layers[i]

    def embed(self):
        return sy.gauss_bf16(self.seed, sy.T_EMBED, (self.d.V, self.d.H), self.sigma)

    def lm_head(self):
        return sy.gauss_bf16(self.seed, sy.T_LMHEAD, (self.d.V, self.d.H), self.sigma)

    def norm(self):
        return np.ones(self.d.H, np.float32)

    def state_dict(self):
        """HF-named fp32 (bf16-valued) arrays, the `sd` the reference engines take."""
        d = self.d
        sd = {"model.embed_tokens.weight": self.embed(), "lm_head.weight": self.lm_head(),
              "model.norm.weight": self.norm()}
        names = {sy.T_Q: "self_attn.q_proj", sy.T_K: "self_attn.k_proj", sy.T_V: "self_attn.v_proj",
                 sy.T_O: "self_attn.o_proj", sy.T_GATE: "mlp.gate_proj", sy.T_UP: "mlp.up_proj",
                 sy.T_DOWN: "mlp.down_proj"}
        for i in range(d.L):
            p = f"model.layers.{i}."
            for k, n in names.items():
                sd[p + n + ".weight"] = self.w(i, k)
            sd[p + "input_layernorm.weight"] = np.ones(d.H, np.float32)
            sd[p + "post_attention_layernorm.weight"] = np.ones(d.H, np.float32)
        return sd


def synth_kv(d: Dims, S, seed, length, sigma=1.0):
    """One request's past KV in the reference layout: K [L, NKV, HD, S], V [L, NKV, S, HD].

    Values for positions < length are bf16 ~N(0, sigma) drawn in [L, NKV, pos, HD]
    order (tids T_KCACHE / T_VCACHE, `seed` per request); the tail is zero, which
    the decode step's one-hot injection requires (engines/prefill_full.py:287-289).
    """
    shape = (d.L, d.NKV, S, d.HD)
    K = sy.gauss_bf16(seed, sy.T_KCACHE, shape, sigma)
    V = sy.gauss_bf16(seed, sy.T_VCACHE, shape, sigma)
    K[:, :, length:, :] = 0.0
    V[:, :, length:, :] = 0.0
    return np.ascontiguousarray(K.transpose(0, 1, 3, 2)), V


def decode_step(model: SynthModel, toks, positions, Ks, Vs, S, kv_bf16=True):
    """One batched decode step over all layers (engines/decode_batch.py:427-442 semantics).

    Ks/Vs: per-layer lists of [B, NKV, HD, S] / [B, NKV, S, HD] caches, updated in
    place.  Returns fp32 logits [B, V].
    """
    d = model.d
    inv = inv_freq(d)
    x = model.embed()[list(toks)].astype(np.float32)
    for i in range(d.L):
        x, Ks[i], Vs[i] = cpu_layer(x, model.layer(i), Ks[i], Vs[i], inv, list(positions), S,
                                    d.eps, d, kv_bf16=kv_bf16)
    return lm_logits(x, model.norm(), model.lm_head(), d.eps)


def prefill(model: SynthModel, tokens, S, kv_bf16=True):
    """Whole-prompt prefill over all layers; returns (K [L,NKV,HD,S], V [L,NKV,S,HD], logits_last).

    Follows engines/prefill_full.py:337-388 for an exact-fit prompt (C = P): the
    cache is zero past P and the next token comes from the last position.
    """
    d = model.d
    inv = inv_freq(d)
    P = len(tokens)
    x = model.embed()[list(tokens)].astype(np.float32)
    K = np.zeros((d.L, d.NKV, d.HD, S), np.float32)
    V = np.zeros((d.L, d.NKV, S, d.HD), np.float32)
    for i in range(d.L):
        x, kT, vT = cpu_layer_p(x, model.layer(i), inv, P, d.eps, d, kv_bf16=kv_bf16)
        K[i, :, :, :P] = kT
        V[i, :, :P, :] = vT
    return K, V, lm_logits(x[P - 1:P], model.norm(), model.lm_head(), d.eps)[0]


def prefill_chunked(model: SynthModel, tokens, S, C, kv_bf16=True):
    """Chunked prefill of one prompt, C positions per pass, against a cache that starts empty;
    returns (K [L,NKV,HD,S], V [L,NKV,S,HD], logits_last).

    Follows engines/prefill_chunk.py:108-142: the prompt is padded with its last token to a
    whole number of chunks (the pad positions' K/V are written too), every layer of a chunk
    runs cpu_layer_chunk at base = the chunk's first position, and the next token comes from
    the last prompt position's hidden state through the final norm and lm_head.
    """
    d = model.d
    inv = inv_freq(d)
    P = len(tokens)
    pad = (-P) % C
    toks = list(tokens) + [tokens[-1]] * pad
    K = np.zeros((d.L, d.NKV, d.HD, S), np.float32)
    V = np.zeros((d.L, d.NKV, S, d.HD), np.float32)
    emb = model.embed()
    hid = None
    for base in range(0, len(toks), C):
        x = emb[toks[base:base + C]].astype(np.float32)
        for i in range(d.L):
            x, K[i], V[i] = cpu_layer_chunk(x, model.layer(i), K[i], V[i], inv, base, C, S, d.eps, d,
                                            kv_bf16=kv_bf16)
        hid = x
    h = hid[(P - 1) % C:(P - 1) % C + 1]
    return K, V, lm_logits(h, model.norm(), model.lm_head(), d.eps)[0]
