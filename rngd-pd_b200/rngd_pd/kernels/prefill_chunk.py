"""Chunked prefill against a live cache as a layer-group module (the names of
src/rngd_pd/kernels/prefill_chunk.py: ChunkModel, rot_matrices and the shape constants), over
the B200 decode kernels.

`ChunkModel(C, S, nl)` is called as the reference calls its compiled graph
(src/rngd_pd/engines/prefill_chunk.py:109-142): the hidden state x [C, H] of the chunk's C
positions base .. base+C-1 of one sequence, the rms inputs, the group's weight stacks, the
sequence's caches K [nl, NKV, HD, S] / V [nl, NKV, S, HD], the chunk's rotations, its one-hot
columns ohK [C, S] and their transpose ohV [S, C], and the mask [1, G*C, S].  It returns the
new hidden state and the caches with the chunk's K/V written.

Underneath, a chunk is one decode step of C streams (C <= 16) that share one cache lane
(rngd_decode_io_t.lanes): stream c holds position base + c, its K/V is appended to the lane
and its attention reads the lane up to its own position, the chunk's causal mask over the
earlier chunks.  The inputs must encode exactly that (one-hot columns at consecutive
positions, ohV their transpose, a causal mask, RoPE's rotations, an empty slot at each
position written); anything else raises ValueError.
"""
import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.kernels._graph import (BF, G, H, HD, HINT, M, NH, NKV, Dims, PackCache, check_rows, default_inv,
                                    rotation_tables, scalar_eps, stacked)
from rngd_pd.kernels.decode_batch import MAXB, _StepBuffers


class ChunkModel(torch.nn.Module):
    """`nl` layers advancing C (<= 16) positions of one sequence in an S-wide cache."""

    def __init__(self, C, S, nl, inv=None, pack_capacity=8):
        super().__init__()
        if not 1 <= C <= MAXB:
            raise ValueError(f"C={C}: a chunk is one step of at most {MAXB} streams")
        if S % 128 or S <= 0:
            raise ValueError(f"S={S} must be a positive multiple of 128")
        self.C, self.S, self.nl = int(C), int(S), int(nl)
        self.inv = default_inv() if inv is None else np.asarray(inv, np.float32)
        self._packs = PackCache(pack_capacity)
        self._buffers = {}

    def forward(self, x, eps, nh, an1, aq, ak, av, ao, an2, awg, awu, awd, Kp, Vp, rot, ohK, ohV, mask):
        """-> (x' [C, H] bf16, Kf [nl, NKV, HD, S], Vf [nl, NKV, S, HD]) as the reference's
        ChunkModel.forward (kernels/prefill_chunk.py:164-180)."""
        C, S, nl = self.C, self.S, self.nl
        if not x.is_cuda:
            raise ValueError("ChunkModel runs on a CUDA device: pass device tensors")
        dev = x.device
        an1, aq, ak, av, ao, an2, awg, awu, awd, Kp, Vp = map(stacked, (an1, aq, ak, av, ao, an2, awg, awu,
                                                                      awd, Kp, Vp))
        if aq.shape[0] != nl or x.shape[0] != C:
            raise ValueError(f"expected {nl} layers and {C} positions, got {aq.shape[0]} and {x.shape[0]}")
        dims = Dims(x, aq, ak, awg, rot.shape[-1])
        if tuple(Kp.shape) != (nl, dims.NKV, dims.HD, S) or tuple(Vp.shape) != (nl, dims.NKV, S, dims.HD):
            raise ValueError(f"caches must be K [{nl}, {dims.NKV}, {dims.HD}, {S}] and V [{nl}, {dims.NKV}, {S}, "
                             f"{dims.HD}]")
        with torch.cuda.device(dev):
            e = scalar_eps(eps, nh, dims.H)
            group = self._packs.get(dims, (an1, aq, ak, av, ao, an2, awg, awu, awd), e, self.inv, dev)
            kc = Kp.to(dev, BF).transpose(-1, -2).contiguous().unsqueeze(1)     # [nl, 1, NKV, S, HD]
            vc = Vp.to(dev, BF).contiguous().unsqueeze(1)
            pos = ohK.to(torch.float32).argmax(-1)
            if not torch.equal(ohV.to(torch.float32), ohK.to(torch.float32).t()):
                raise ValueError("ohV must be the transpose of ohK")
            if C > 1 and not bool((pos[1:] - pos[:-1] == 1).all()):
                raise ValueError("a chunk's one-hot columns must name consecutive positions")
            at = pos.view(1, 1, 1, C, 1).expand(nl, 1, dims.NKV, C, dims.HD)
            check_rows(pos, ohK, mask.reshape(-1, C, S)[0], rot, group.inv, kc.gather(3, at), vc.gather(3, at), S)
            key = (str(dev), dims.H, dims.QN, dims.KN, dims.M)
            buf = self._buffers.get(key)
            if buf is None:
                buf = self._buffers[key] = _StepBuffers(group.model, dims, C, S, dev)
                buf.lanes = torch.zeros(C, dtype=torch.int32, device=dev)    # every stream on lane 0
            buf.x[:C].copy_(x)
            buf.pos.copy_(pos)
            io = buf.io(C, S, nl, kc, vc, lanes=buf.lanes, Bcap=1)
            h = _lib.stream_handle(torch.cuda.current_stream(dev))
            _lib.call("rngd_decode_begin", group.model, io, 0, h)
            _lib.call("rngd_decode_layers", group.model, io, 0, nl, h)
            return buf.x[:C].to(BF), kc[:, 0].transpose(-1, -2).contiguous(), vc[:, 0].contiguous()


def rot_matrices(inv, base, C):
    """[C, HD, HD] rotations of positions base .. base+C-1 (kernels/prefill_chunk.py:185-195)."""
    return rotation_tables(inv, np.arange(base, base + C, dtype=np.float32))


__all__ = ["BF", "H", "M", "NH", "NKV", "HD", "G", "HINT", "ChunkModel", "rot_matrices"]
