"""Chunked prefill against a live cache on B200 (API of src/rngd_pd/engines/prefill_chunk.py:36-142).

The reference advances one sequence C positions per compiled-graph call (ChunkLayer,
src/rngd_pd/kernels/prefill_chunk.py:117-161): the chunk's C tokens are written into the
cache at positions base .. base+C-1 by a one-hot matmul, and token c attends to every
cached position <= base + c.

Here a chunk of C <= 16 tokens is one decode step over C streams that share one cache
lane (rngd_decode_io_t.lanes): stream c carries token base + c at position base + c, the
QKV epilogue appends its K/V to the shared lane, and the attention that follows reads the
lane up to the stream's own position -- the chunk's causal mask with the rows of earlier
chunks in front.  The last chunk also runs the final norm + lm_head, whose first-max argmax
at the prompt's last position is the next token.  The prompt is padded with its last token
to a whole number of chunks, as in the reference (the pad positions' K/V are written too).
"""
import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.engines.decode_batch import BF, MAXB, BatchDecodeEngine


class _SharedLaneSteps(BatchDecodeEngine):
    """Decode-step machinery for C streams over a one-lane cache ([NG][1][NKV][S][HD])."""

    def __init__(self, cfg, sd, C, S, group, chip, share=None):
        super().__init__(cfg, sd, B=C, S=S, group=group, chip=chip, share=share)
        self._lanes = torch.zeros(C, dtype=torch.int32, device=self.dev)
        c = self.cfg
        self._group_numel = self.NG * c.n_kv * S * c.head_dim

    def _io(self, Kg, Vg):
        io = super()._io(Kg, Vg)
        io.Bcap = 1
        io.lanes = self._lanes.data_ptr()
        return io

    def _check_cache(self, Kd, Vd):
        c = self.cfg
        shape = (self.NG, 1, c.n_kv, self.S, c.head_dim)
        if len(Kd) != self.ngroups or len(Vd) != self.ngroups:
            raise ValueError(f"expected {self.ngroups} cache groups")
        for t in list(Kd) + list(Vd):
            if tuple(t.shape) != shape or t.dtype != BF or not t.is_contiguous() or t.device != self.dev:
                raise ValueError(f"cache group must be a contiguous bf16 {shape} tensor on {self.dev}, "
                                 f"got {tuple(t.shape)} {t.dtype} on {t.device}")

    def _alloc_cache(self, ipc=False):
        c = self.cfg
        K = torch.zeros((self.nl, 1, c.n_kv, self.S, c.head_dim), dtype=BF, device=self.dev)
        V = torch.zeros_like(K)
        return ([K[g * self.NG:(g + 1) * self.NG] for g in range(self.ngroups)],
                [V[g * self.NG:(g + 1) * self.NG] for g in range(self.ngroups)])

    def run_chunk(self, toks, positions, Kd, Vd, lmhead):
        """One chunk on self.stream: embedding, every layer, and (last chunk) the lm_head."""
        toks, positions = self._validate(toks, positions)
        self._check_cache(Kd, Vd)
        self._copied.synchronize()
        self._in_np[0] = toks
        self._in_np[1] = positions
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self._tp.copy_(self._in_host, non_blocking=True)
            self._copied.record(s)
            h = _lib.stream_handle(s)
            io = self._io(Kd[0], Vd[0])
            _lib.call("rngd_decode_embed", self._m, io, h)
            for g in range(self.ngroups):
                io.kcache, io.vcache = Kd[g].data_ptr(), Vd[g].data_ptr()
                _lib.call("rngd_decode_layers", self._m, io, g * self.NG, (g + 1) * self.NG, h)
            if lmhead:
                _lib.call("rngd_decode_lmhead", self._m, io, h)

    def next_tokens(self):
        with torch.cuda.stream(self.stream):
            self._out_host.copy_(self._next, non_blocking=True)
        self.stream.synchronize()
        return self._out_host.tolist()


class ChunkPrefillEngine:
    """Same constructor and methods as the reference's ChunkPrefillEngine
    (engines/prefill_chunk.py:36-142): `fresh_kv()` and `prefill(tokens) -> (K, V, next)`
    with K [L, NKV, HD, S] and V [L, NKV, S, HD] float32 (bf16 values) on the host.
    `cache_dir` is accepted for signature compatibility; `share` reuses the weights of
    another engine on the same card (BatchDecodeEngine(share=...))."""

    def __init__(self, cfg, sd, S=256, C=16, group=2, chip=1, cache_dir=None, share=None):
        if not 1 <= C <= MAXB:
            raise ValueError(f"C={C}: a chunk is one step of at most {MAXB} streams")
        self.cfg, self.S, self.C, self.NG = cfg, S, C, group
        self.nl = cfg.n_layers
        if self.nl % group:
            raise ValueError("layer count must divide into whole groups")
        self.ngroups = self.nl // group
        self._e = _SharedLaneSteps(cfg, sd, C, S, group, chip, share=share)
        self.dev = self._e.dev

    @_lib.on_device
    def fresh_kv(self):
        """An empty one-sequence cache (opaque group lists, as the decode engine's)."""
        return self._e._alloc_cache()

    @_lib.on_device
    def prefill_device(self, tokens):
        """The whole prompt, C positions per step, into a fresh device cache.
        Returns (Kd, Vd, next_token)."""
        C, S = self.C, self.S
        P = len(tokens)
        if P < 1:
            raise ValueError("empty prompt")
        pad = (-P) % C
        if P + pad > S:
            raise ValueError(f"prompt {P} (+{pad} pad) exceeds the cache size S={S}")
        toks = [int(t) for t in tokens] + [int(tokens[-1])] * pad   # last chunk padded
        Kd, Vd = self.fresh_kv()
        for base in range(0, len(toks), C):
            self._e.run_chunk(toks[base:base + C], list(range(base, base + C)), Kd, Vd,
                              lmhead=base + C >= len(toks))
        nxt = self._e.next_tokens()[(P - 1) % C]
        return Kd, Vd, nxt

    @_lib.on_device
    def prefill(self, tokens):
        """Whole prompt, C positions per pass. Returns (K, V, next_token) on the host."""
        Kd, Vd, nxt = self.prefill_device(tokens)
        K = torch.cat([k[:, 0].transpose(-1, -2).float().cpu() for k in Kd], 0).numpy()
        V = torch.cat([v[:, 0].float().cpu() for v in Vd], 0).numpy()
        return K, V, nxt


__all__ = ["ChunkPrefillEngine"]
