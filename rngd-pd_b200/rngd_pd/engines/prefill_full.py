"""Serving wrapper for the KV-free whole-prompt prefill on B200
(API of src/rngd_pd/engines/prefill_full.py:119-400).

Same constructor, buckets, `pick`, `prefill`, `prefill_device`,
`begin_device_prefill` (resumable stage with `advance(n)` / `result()`) and
`prefill_stream(tokens, sink)` as the reference's FullPrefillEngine; the compiled
NPU graph is replaced by the sm_100a kernels of _rngd_b200.so
(rngd_prefill_embed / rngd_prefill_layers / rngd_lmhead_rows).

The cache is produced in the prefill layout kv [L][2][NKV][S][HD] (K then V per
layer, one 256-byte row per position; `prefill_kv_device`), which is what the
NVLink handoff moves.  The reference layouts K [nl, NKV, HD, S] / V [nl, NKV, S, HD]
are produced at the API boundary (`prefill`, `prefill_device`, `prefill_stream`).
"""
import os
import time

import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.engines.decode_batch import _dev
from rngd_pd.engines.weights import DeviceWeights

BF = torch.bfloat16


class _DevicePrefillStage:
    """One prefill advanced a layer group at a time (engines/prefill_full.py:77-116):
    advance() runs the next groups and returns True when the pass is done."""

    def __init__(self, eng, tokens):
        self.e, self.P = eng, len(tokens)
        self.C = eng.pick(self.P)
        if self.P > self.C:
            raise ValueError(f"prompt {self.P} exceeds the widest compiled bucket C={self.C}")
        self._b = eng.buckets[self.C]
        self.kv = eng._new_kv()
        eng._begin(self._b, tokens, self.kv)
        self.g = 0

    @_lib.on_device
    def advance(self, n=1):
        for _ in range(n):
            self.e._group(self._b, self.g, self.kv)
            self.g += 1
            if self.g >= self.e.ngroups:
                return True
        return False

    @_lib.on_device
    def result(self):
        nxt = self.e._finish(self._b)
        K, V = self.e.reference_layout(self.kv)
        return K, V, nxt

    @_lib.on_device
    def result_kv(self):
        """(kv in the prefill layout [L][2][NKV][S][HD], next token), without a relayout."""
        return self.kv, self.e._finish(self._b)


class FullPrefillEngine:
    def __init__(self, cfg, sd, C=256, group=2, chip=0, cache_dir=None, S=0):
        """C: widest prompt of the first bucket; S: the decode cache width the KV is padded
        to (engines/prefill_full.py:120-125).  `sd` may be an HF state dict, a
        SyntheticState, or the DeviceWeights of another engine on the same card.
        `cache_dir` is accepted for signature compatibility (no compiled artifacts)."""
        if C % 128:
            raise ValueError(f"bucket width C={C} must be a multiple of 128")
        self.C, self.NG = C, group
        self.S = S or C
        self.cfg = cfg
        self.nl = cfg.n_layers
        if self.nl % group:
            raise ValueError("layer count must divide into whole groups")
        self.ngroups = self.nl // group
        self.dev = sd.device if isinstance(sd, DeviceWeights) else _dev(chip)
        self.eps = cfg.eps
        self.V = cfg.vocab
        self.w = sd if isinstance(sd, DeviceWeights) else DeviceWeights(cfg, sd, self.dev)
        self._m = self.w.model_struct()
        self.stream = torch.cuda.Stream(device=self.dev)
        # GEMM operand precision ($RNGD_PREFILL_OPERAND): "hilo" = bf16 hi + lo rows (fp32-level),
        # "bf16" = one bf16 row, as the reference's graph takes its activations
        mode = os.environ.get("RNGD_PREFILL_OPERAND", "hilo")
        if mode not in ("hilo", "bf16"):
            raise ValueError(f"RNGD_PREFILL_OPERAND={mode!r}: expected 'hilo' or 'bf16'")
        self.operand_lo = 1 if mode == "hilo" else 0
        self.buckets = {}
        self.last_C = None
        self.last_compute_ms = self.last_download_ms = 0.0
        t0 = time.time()
        self.add_bucket(C)
        self.compile_s = time.time() - t0
        self._build_lmhead()

    # ------------------------------------------------------------- buckets
    @_lib.on_device
    def add_bucket(self, C):
        """Buffers for one prefill width (engines/prefill_full.py:168-203)."""
        if C in self.buckets:
            return self.buckets[C]
        if C % 128:
            raise ValueError(f"bucket width C={C} must be a multiple of 128")
        if C > self.S:
            raise ValueError(f"bucket width C={C} exceeds the cache width S={self.S}")
        import ctypes
        c, d = self.cfg, self.dev
        H, M = c.hidden, c.inter
        QN = c.n_heads * c.head_dim
        ld = max(H, QN)
        pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.call("rngd_prefill_workspace", ctypes.byref(self._m), C, ctypes.byref(pf), ctypes.byref(ct))
        f32 = dict(dtype=torch.float32, device=d)
        b = {"C": C,
             "toks": torch.zeros(C, dtype=torch.int32, device=d),
             "toks_host": torch.zeros(C, dtype=torch.int32).pin_memory(),
             "x": torch.zeros((C, H), **f32), "q": torch.zeros((C, QN), **f32),
             "act": torch.zeros((2 * C, ld), dtype=BF, device=d),
             "act_o": torch.zeros((2 * C, QN), dtype=BF, device=d),
             "act2": torch.zeros((2 * C, M), dtype=BF, device=d),
             "ss": torch.zeros((H // 128, C), **f32),
             "partial": torch.zeros(max(pf.value, 1), **f32),
             "counters": torch.zeros(max(ct.value, 1), dtype=torch.int32, device=d)}
        self.buckets[C] = b
        self.C = max(self.buckets)
        return b

    def pick(self, P):
        """The narrowest width that swallows this prompt (engines/prefill_full.py:205-208)."""
        fits = [c for c in sorted(self.buckets) if c >= P]
        return fits[0] if fits else max(self.buckets)

    @_lib.on_device
    def _build_lmhead(self):
        import ctypes
        c, d = self.cfg, self.dev
        pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.call("rngd_lmhead_workspace", ctypes.byref(self._m), ctypes.byref(pf), ctypes.byref(ct))
        self._lm = {"act": torch.zeros((32, c.hidden), dtype=BF, device=d),
                    "ss": torch.zeros((c.hidden // 128, 16), dtype=torch.float32, device=d),
                    "logits": torch.zeros((1, self.V), dtype=torch.float32, device=d),
                    "best": torch.zeros(16, dtype=torch.int64, device=d),
                    "next": torch.zeros(1, dtype=torch.int32, device=d),
                    "partial": torch.zeros(max(pf.value, 1), dtype=torch.float32, device=d),
                    "counters": torch.zeros(max(ct.value, 1), dtype=torch.int32, device=d)}

    # ---------------------------------------------------------------- pass
    def _new_kv(self):
        c = self.cfg
        return torch.zeros((self.nl, 2, c.n_kv, self.S, c.head_dim), dtype=BF, device=self.dev)

    def _io(self, b, kv_group, P):
        p = lambda t: t.data_ptr()
        return _lib.PrefillIO(C=b["C"], P=P, S=self.S, kv_layers=self.NG, kv=p(kv_group), toks=p(b["toks"]),
                              operand_lo=self.operand_lo,
                              x=p(b["x"]), q=p(b["q"]), act=p(b["act"]), act_o=p(b["act_o"]), act2=p(b["act2"]),
                              ss=p(b["ss"]), partial=p(b["partial"]), counters=p(b["counters"]))

    def _begin(self, b, tokens, kv):
        """Pad the prompt with its last token to the bucket (engines/prefill_full.py:356) and embed."""
        tokens = [int(t) for t in tokens]
        for t in tokens:
            if not 0 <= t < self.V:
                raise ValueError(f"token {t} outside the vocabulary")
        C, P = b["C"], len(tokens)
        b["P"] = P
        b["toks_host"][:] = torch.tensor(tokens + [tokens[-1]] * (C - P), dtype=torch.int32)
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            b["toks"].copy_(b["toks_host"], non_blocking=True)
            _lib.call("rngd_prefill_embed", self._m, self._io(b, kv[0], P), _lib.stream_handle(s))

    def _group(self, b, g, kv):
        s = self.stream
        with torch.cuda.stream(s):
            io = self._io(b, kv[g * self.NG], b["P"])
            _lib.call("rngd_prefill_layers", self._m, io, g * self.NG, (g + 1) * self.NG, _lib.stream_handle(s))

    def _finish(self, b):
        """Last prompt position -> next token on the device (engines/prefill_full.py:265-270)."""
        s, lm = self.stream, self._lm
        P = b["P"]
        with torch.cuda.stream(s):
            xrow = b["x"][P - 1:P]
            _lib.call("rngd_lmhead_rows", self._m, _lib.ptr(xrow), self.cfg.hidden, 1, _lib.ptr(lm["act"]),
                      _lib.ptr(lm["ss"]), _lib.ptr(lm["logits"]), _lib.ptr(lm["best"]), _lib.ptr(lm["next"]),
                      _lib.ptr(lm["partial"]), _lib.ptr(lm["counters"]), _lib.stream_handle(s))
        self.last_C = b["C"]
        s.synchronize()
        return int(lm["next"].item())

    @_lib.on_device
    def prefill_kv_device(self, tokens, kv=None):
        """The whole pass; returns (kv [L, 2, NKV, S, HD] bf16 on the device, next token).
        `kv` may be a caller-owned zeroed buffer of that shape (e.g. a decode-side landing zone)."""
        P = len(tokens)
        C = self.pick(P)
        if P > C:
            raise ValueError(f"prompt {P} exceeds the widest compiled bucket C={C}")
        if P > self.S:
            raise ValueError(f"prompt {P} exceeds the cache width S={self.S}")
        b = self.buckets[C]
        kv = self._new_kv() if kv is None else kv
        t0 = time.perf_counter()
        self._begin(b, tokens, kv)
        for g in range(self.ngroups):
            self._group(b, g, kv)
        nxt = self._finish(b)
        self.last_compute_ms = (time.perf_counter() - t0) * 1e3
        return kv, nxt

    @_lib.on_device
    def logits(self):
        """fp32 logits [V] of the last prefill's final position (device)."""
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        return self._lm["logits"][0]

    @staticmethod
    def reference_layout(kv):
        """prefill layout [L, 2, NKV, S, HD] -> reference K [L, NKV, HD, S], V [L, NKV, S, HD] (views)."""
        return kv[:, 0].transpose(-1, -2), kv[:, 1]

    @_lib.on_device
    def prefill_device(self, tokens):
        """Prefill and leave the cache on the device in the reference layout (bf16), padded to S
        with zeros past the prompt (engines/prefill_full.py:278-304)."""
        kv, nxt = self.prefill_kv_device(tokens)
        K, V = self.reference_layout(kv)
        return K.contiguous(), V.contiguous(), nxt

    @_lib.on_device
    def begin_device_prefill(self, tokens):
        """Prefill as resumable layer-group steps (engines/prefill_full.py:306-317)."""
        return _DevicePrefillStage(self, tokens)

    @_lib.on_device
    def prefill_stream(self, tokens, sink):
        """Hand each layer group's cache over as it exists (engines/prefill_full.py:337-388):
        sink(g, kh, vh) with host float32 kh [NG, NKV, HD, S], vh [NG, NKV, S, HD]."""
        P = len(tokens)
        C = self.pick(P)
        if P > C:
            raise ValueError(f"prompt {P} exceeds the widest compiled bucket C={C}")
        b = self.buckets[C]
        kv = self._new_kv()
        t_c = t_d = 0.0
        self._begin(b, tokens, kv)
        for g in range(self.ngroups):
            t0 = time.perf_counter()
            self._group(b, g, kv)
            self.stream.synchronize()
            t1 = time.perf_counter()
            grp = kv[g * self.NG:(g + 1) * self.NG]
            kh = grp[:, 0].transpose(-1, -2).float().cpu().numpy()
            vh = grp[:, 1].float().cpu().numpy()
            t2 = time.perf_counter()
            sink(g, kh, vh)
            t_c += t1 - t0
            t_d += t2 - t1
        self.last_compute_ms = t_c * 1e3
        self.last_download_ms = t_d * 1e3
        return self._finish(b)

    @_lib.on_device
    def prefill_stream_device(self, tokens, sink):
        """The same with device views: sink(g, kv_group [NG, 2, NKV, S, HD]) right after the group's
        kernels are queued on self.stream (the sink orders its own work after that stream)."""
        P = len(tokens)
        C = self.pick(P)
        if P > C:
            raise ValueError(f"prompt {P} exceeds the widest compiled bucket C={C}")
        b = self.buckets[C]
        kv = self._new_kv()
        self._begin(b, tokens, kv)
        for g in range(self.ngroups):
            self._group(b, g, kv)
            sink(g, kv[g * self.NG:(g + 1) * self.NG])
        return self._finish(b)

    @_lib.on_device
    def prefill(self, tokens):
        """The same pass, handed back as host float32 arrays in the reference layout
        (engines/prefill_full.py:390-400)."""
        K, V, nxt = self.prefill_device(tokens)
        return K.float().cpu().numpy(), V.float().cpu().numpy(), nxt
