"""KV-free whole-prompt prefill as a layer-group module (the names of
src/rngd_pd/kernels/prefill_full.py: PrefillModel and the shape constants), over the B200
prefill kernels.

`PrefillModel(C, nl)` is called as the reference calls its compiled graph
(src/rngd_pd/engines/prefill_full.py:210-214): the hidden state x [C, H] of the C prompt
positions, the rms inputs, the group's weight stacks, the rotation of every position and the
causal mask.  It returns the new hidden state and the group's kT [nl, NKV, HD, C] and vT
[nl, NKV, C, HD].  Underneath, the group runs as rngd_prefill_begin + rngd_prefill_layers
(tcgen05 token-tile GEMMs with RoPE / KV-emission / residual / SwiGLU epilogues and the
tcgen05 causal attention) on the caller's current CUDA stream; C must be a multiple of 128.

The rotation input must be RoPE's at positions 0..C-1 for the module's inverse frequencies
and the mask causal (0 on and below the diagonal, negative above); anything else raises
ValueError, because the kernels implement exactly that step.  FullPrefillEngine
(rngd_pd.engines.prefill_full) drives the same kernels from token ids with buckets; this
module is for callers written against the reference's graph interface.
"""
import ctypes

import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.kernels._graph import (BF, G, H, HD, HINT, M, NH, NKV, Dims, PackCache, check_rows, default_inv,
                                    rotation_tables, scalar_eps, stacked)


class _PassBuffers:
    def __init__(self, model, dims, C, dev):
        f32 = dict(dtype=torch.float32, device=dev)
        pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.call("rngd_prefill_workspace", ctypes.byref(model), C, ctypes.byref(pf), ctypes.byref(ct))
        ld = max(dims.H, dims.QN)
        self.toks = torch.zeros(C, dtype=torch.int32, device=dev)
        self.x = torch.zeros((C, dims.H), **f32)
        self.q = torch.zeros((C, dims.QN), **f32)
        self.act = torch.zeros((2 * C, ld), dtype=BF, device=dev)
        self.act_o = torch.zeros((2 * C, dims.QN), dtype=BF, device=dev)
        self.act2 = torch.zeros((2 * C, dims.M), dtype=BF, device=dev)
        self.ss = torch.zeros((dims.H // 128, C), **f32)
        self.partial = torch.zeros(max(pf.value, 1), **f32)
        self.counters = torch.zeros(max(ct.value, 1), dtype=torch.int32, device=dev)

    def io(self, C, nl, kv):
        p = lambda t: t.data_ptr()
        return _lib.PrefillIO(C=C, P=C, S=C, kv_layers=nl, kv=p(kv), toks=p(self.toks), x=p(self.x), q=p(self.q),
                              operand_lo=1,
                              act=p(self.act), act_o=p(self.act_o), act2=p(self.act2), ss=p(self.ss),
                              partial=p(self.partial), counters=p(self.counters))


class PrefillModel(torch.nn.Module):
    """`nl` prefill layers over C prompt positions (C a multiple of 128).

    inv: RoPE inverse frequencies the rotation input was built from (default theta 5e5)."""

    def __init__(self, C, nl, inv=None, pack_capacity=8):
        super().__init__()
        if C % 128 or C <= 0:
            raise ValueError(f"C={C}: the prefill kernels take a positive multiple of 128 positions")
        self.C, self.nl = int(C), int(nl)
        self.inv = default_inv() if inv is None else np.asarray(inv, np.float32)
        self._packs = PackCache(pack_capacity)
        self._buffers = {}

    def forward(self, x, eps, nh, an1, aq, ak, av, ao, an2, awg, awu, awd, rot, mask):
        """-> (x' [C, H] bf16, kT [nl, NKV, HD, C], vT [nl, NKV, C, HD]) as the reference's
        PrefillModel.forward (kernels/prefill_full.py:79-94)."""
        C, nl = self.C, self.nl
        if not x.is_cuda:
            raise ValueError("PrefillModel runs on a CUDA device: pass device tensors")
        dev = x.device
        an1, aq, ak, av, ao, an2, awg, awu, awd = map(stacked, (an1, aq, ak, av, ao, an2, awg, awu, awd))
        if aq.shape[0] != nl or x.shape[0] != C:
            raise ValueError(f"expected {nl} layers and {C} positions, got {aq.shape[0]} and {x.shape[0]}")
        dims = Dims(x, aq, ak, awg, rot.shape[-1])
        with torch.cuda.device(dev):
            e = scalar_eps(eps, nh, dims.H)
            group = self._packs.get(dims, (an1, aq, ak, av, ao, an2, awg, awu, awd), e, self.inv, dev)
            # the mask arrives as [1, G*C, C] (G copies of the C x C causal rows); check the first copy
            rows = mask.reshape(-1, C, C)[0]
            pos = torch.arange(C, device=dev)
            check_rows(pos, torch.eye(C, device=dev), rows, rot, group.inv, None, None, C)
            key = (str(dev), dims.H, dims.QN, dims.KN, dims.M)
            buf = self._buffers.get(key)
            if buf is None:
                buf = self._buffers[key] = _PassBuffers(group.model, dims, C, dev)
            kv = torch.zeros((nl, 2, dims.NKV, C, dims.HD), dtype=BF, device=dev)
            buf.x.copy_(x)
            io = buf.io(C, nl, kv)
            h = _lib.stream_handle(torch.cuda.current_stream(dev))
            _lib.call("rngd_prefill_begin", group.model, io, 0, h)
            _lib.call("rngd_prefill_layers", group.model, io, 0, nl, h)
            return buf.x.to(BF), kv[:, 0].transpose(-1, -2).contiguous(), kv[:, 1].contiguous()


def rot_matrices(inv, C):
    """[C, HD, HD] rotations of positions 0..C-1 (the table the reference's prefill engine builds)."""
    return rotation_tables(inv, np.arange(C))


__all__ = ["BF", "H", "M", "NH", "NKV", "HD", "G", "HINT", "PrefillModel", "rot_matrices"]
