"""Batched decode as a layer-group module (the names of src/rngd_pd/kernels/decode_batch.py:
DecodeModel, rot_batch and the shape constants), over the B200 decode kernels.

`DecodeModel(B, S, nl)` is called as the reference calls its compiled graph
(src/rngd_pd/engines/decode_batch.py:436-439): the hidden state x [B, H] of B streams, the
rms inputs, the group's weight stacks, the group's caches K [nl, B, NKV, HD, S] / V [nl, B,
NKV, S, HD], and the per-stream rotation, mask and one-hot rows of the step.  It returns the
new hidden state and the updated caches, K/V of the step written at each stream's position.
Underneath, the group runs as rngd_decode_begin + rngd_decode_layers (tcgen05 weight-streaming
GEMMs with RoPE / KV-append / residual / SwiGLU epilogues and the fused split-S attention),
on the caller's current CUDA stream.

The reference's graph is a generic tensor program: its one-hot row adds k into whatever the
cache holds, and its mask and rotation may be anything.  The kernels implement the decode
step those inputs encode, so each call checks on the device that the one-hot row names one
position per stream, that the mask is zero up to it and negative after it, that the rotation
is RoPE's at that position (for the module's inverse frequencies, `inv`), and that the cache
slot being written is empty; anything else raises ValueError instead of computing something
different.  The BatchDecodeEngine (rngd_pd.engines.decode_batch) drives the same kernels on a
resident cache without these conversions; this module is for callers written against the
reference's graph interface.
"""
import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.kernels._graph import (BF, G, H, HD, HINT, M, MAX_SHAPES, NH, NKV, Dims, PackCache, check_rows,
                                    default_inv, rotation_tables, scalar_eps, stacked)

MAXB = 16


class _StepBuffers:
    """The decode io struct's scratch for B streams of an S-wide cache (zeroed once)."""

    def __init__(self, model, dims, B, S, dev):
        f32 = dict(dtype=torch.float32, device=dev)
        pf, ct, act_cols, act2_cols = _lib.decode_workspace(model, S)
        self.x = torch.zeros((MAXB, dims.H), **f32)
        self.q = torch.zeros((MAXB, dims.QN), **f32)
        self.act = torch.zeros((2 * MAXB, act_cols), dtype=BF, device=dev)
        self.act_o = torch.zeros((2 * MAXB, dims.QN), dtype=BF, device=dev)
        self.act2 = torch.zeros((2 * MAXB, act2_cols), dtype=BF, device=dev)
        self.ss = torch.zeros((dims.H // 128, MAXB), **f32)
        self.logits = torch.zeros((B, 128), **f32)
        self.part = torch.zeros(_lib.decode_attn_workspace(model, B, S), **f32)
        self.partial = torch.zeros(max(pf, 1), **f32)
        self.counters = torch.zeros(max(ct, 1), dtype=torch.int32, device=dev)
        self.best = torch.zeros(MAXB, dtype=torch.int64, device=dev)
        self.toks = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.next = torch.zeros(B, dtype=torch.int32, device=dev)

    def io(self, B, S, nl, kc, vc, lanes=None, Bcap=None):
        p = lambda t: t.data_ptr()
        return _lib.DecodeIO(B=B, Bcap=Bcap or B, S=S, kv_layers=nl, kcache=p(kc), vcache=p(vc), toks=p(self.toks),
                             pos=p(self.pos), x=p(self.x), q=p(self.q), act=p(self.act), act_o=p(self.act_o),
                             act2=p(self.act2), ss=p(self.ss), logits=p(self.logits), attn_part=p(self.part),
                             partial=p(self.partial), counters=p(self.counters), best=p(self.best),
                             next=p(self.next), lanes=0 if lanes is None else p(lanes))


class DecodeModel(torch.nn.Module):
    """`nl` decode layers for B streams (<= 16) of an S-wide cache (S a multiple of 128).

    inv: RoPE inverse frequencies the rotation inputs were built from (default theta 5e5);
    pack_capacity: packed weight groups kept (see rngd_pd.kernels._graph.PackCache)."""

    def __init__(self, B, S, nl, inv=None, pack_capacity=8):
        super().__init__()
        if not 1 <= B <= MAXB:
            raise ValueError(f"B={B}: the decode kernels step 1..{MAXB} streams")
        if S % 128 or S <= 0:
            raise ValueError(f"S={S} must be a positive multiple of 128")
        self.B, self.S, self.nl = int(B), int(S), int(nl)
        self.inv = default_inv() if inv is None else np.asarray(inv, np.float32)
        self._packs = PackCache(pack_capacity)
        self._buffers = {}

    def _scratch(self, group, dims, dev):
        key = (str(dev), dims.H, dims.QN, dims.KN, dims.M)
        if key not in self._buffers:
            self._buffers[key] = _StepBuffers(group.model, dims, self.B, self.S, dev)
        return self._buffers[key]

    def forward(self, x, eps, nh, an1, aq, ak, av, ao, an2, awg, awu, awd, Kp, Vp, rot, mask, oh):
        """-> (x' [B, H] bf16, Kf [nl, B, NKV, HD, S], Vf [nl, B, NKV, S, HD]) as the reference's
        DecodeModel.forward (kernels/decode_batch.py:100-109)."""
        B, S, nl = self.B, self.S, self.nl
        if not x.is_cuda:
            raise ValueError("DecodeModel runs on a CUDA device: pass device tensors")
        dev = x.device
        an1, aq, ak, av, ao, an2, awg, awu, awd, Kp, Vp = map(stacked, (an1, aq, ak, av, ao, an2, awg, awu,
                                                                      awd, Kp, Vp))
        if aq.shape[0] != nl or tuple(x.shape[:1]) != (B,):
            raise ValueError(f"expected {nl} layers and {B} streams, got {aq.shape[0]} and {tuple(x.shape)}")
        dims = Dims(x, aq, ak, awg, rot.shape[-1])
        if tuple(Kp.shape) != (nl, B, dims.NKV, dims.HD, S) or tuple(Vp.shape) != (nl, B, dims.NKV, S, dims.HD):
            raise ValueError(f"caches must be K [{nl}, {B}, {dims.NKV}, {dims.HD}, {S}] and "
                             f"V [{nl}, {B}, {dims.NKV}, {S}, {dims.HD}]")
        with torch.cuda.device(dev):
            e = scalar_eps(eps, nh, dims.H)
            group = self._packs.get(dims, (an1, aq, ak, av, ao, an2, awg, awu, awd), e, self.inv, dev)
            kc = Kp.to(dev, BF).transpose(-1, -2).contiguous()          # [nl, B, NKV, S, HD]
            vc = Vp.to(dev, BF).contiguous()
            pos = oh.to(torch.float32).argmax(-1)
            at = pos.view(1, B, 1, 1, 1).expand(nl, B, dims.NKV, 1, dims.HD)
            check_rows(pos, oh, mask.reshape(B, S), rot, group.inv, kc.gather(3, at), vc.gather(3, at), S)
            buf = self._scratch(group, dims, dev)
            buf.x[:B].copy_(x)
            buf.pos.copy_(pos)
            io = buf.io(B, S, nl, kc, vc)
            h = _lib.stream_handle(torch.cuda.current_stream(dev))
            _lib.call("rngd_decode_begin", group.model, io, 0, h)
            _lib.call("rngd_decode_layers", group.model, io, 0, nl, h)
            return buf.x[:B].to(BF), kc.transpose(-1, -2).contiguous(), vc


def rot_batch(inv, positions):
    """[B, HD, HD] fp32 rotations, one per stream's position (kernels/decode_batch.py:112-123)."""
    return rotation_tables(inv, positions)


__all__ = ["BF", "H", "M", "NH", "NKV", "HD", "G", "HINT", "MAX_SHAPES", "DecodeModel", "rot_batch"]
