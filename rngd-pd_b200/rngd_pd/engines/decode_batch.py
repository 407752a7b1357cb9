"""Serving wrapper for batched decode on B200 (API of src/rngd_pd/engines/decode_batch.py:174-442).

Same constructor, same methods, same return shapes as the reference's
BatchDecodeEngine; the compiled NPU graph is replaced by the sm_100a kernels
of _rngd_b200.so (rngd_decode_embed / rngd_decode_layers /
rngd_decode_lmhead), and the whole step is captured once into a CUDA graph per
cache binding.

Resident cache.  Kd / Vd are lists of per-group device tensors, opaque to
callers exactly as in the reference (src/rngd_pd/engines/tiers.py:15-17).
Their layout is the decode layout [NG][B][NKV][S][HD] for BOTH K and V (a
position's 128-dim key is one 256-byte row, which is what the attention
kernel streams); the reference's K [NKV][HD][S] layout is used only at the
host/connector boundary (load_kv, write_slot_kv, download_kv, upload_kv).
"""
import ctypes
import os

import numpy as np
import torch

from rngd_pd import _lib
from rngd_pd.engines.weights import DeviceWeights

BF = torch.bfloat16
MAXB = 16          # lanes a single step kernel set handles
ATTN_CHUNK = 128   # split-S chunk of the decode attention kernel


class PrefillKV:
    """A request's cache as a prefill engine leaves it on the device: kv bf16 [L][2][NKV][S][HD]
    (K then V per layer, FullPrefillEngine.prefill_kv_device) and the prompt length `tokens`.
    BatchDecodeEngine.write_slot_kv moves its positions [0, tokens) straight into a decode lane
    with the handoff kernel (one launch per layer group, no relayout on the host or through
    torch); positions past the prompt keep whatever the lane held, which no step reads before
    the step at that position writes it."""

    __slots__ = ("kv", "tokens")

    def __init__(self, kv, tokens):
        self.kv, self.tokens = kv, int(tokens)


def greedy_tokens(logits, Vp, V, B):
    """First-max argmax per stream of logits in the reference layout [NG, Vp/NG, B]
    (engines/decode_batch.py:162-171)."""
    lg = logits.detach().cpu().reshape(Vp, B)[:V]
    return torch.argmax(lg, dim=0).tolist()


def _dev(chip):
    if isinstance(chip, torch.device):
        return chip
    if isinstance(chip, str):
        return torch.device(chip)
    return torch.device("cuda", int(chip) if torch.cuda.device_count() > int(chip) else 0)


class BatchDecodeEngine:
    def __init__(self, cfg, sd, B=2, S=256, group=2, chip=0, cache_dir=None, share=None, hint=None):
        """`share`: another BatchDecodeEngine on the same device whose weights this one
        reuses (engines/decode_batch.py:175-181); `cache_dir` and `hint` are accepted for
        signature compatibility (there is no compiled-graph artifact or tactic search:
        the kernels are built ahead of time)."""
        if not 1 <= B <= MAXB:
            raise ValueError(f"B={B}: the decode kernels take 1..{MAXB} lanes")
        if S % ATTN_CHUNK:
            raise ValueError(f"S={S} must be a multiple of {ATTN_CHUNK}")
        group = share.NG if share is not None else group
        self.hint = hint
        self.B, self.S, self.NG = B, S, group
        self.cfg = cfg
        self.nl = cfg.n_layers
        if self.nl % group:
            raise ValueError("layer count must divide into whole groups")
        self.ngroups = self.nl // group
        if share is not None:
            self.dev = share.dev
        elif isinstance(sd, DeviceWeights):
            self.dev = sd.device
        else:
            self.dev = _dev(chip)
        self.eps = cfg.eps
        self.V = cfg.vocab
        self.NGV = 32
        self.Vp = (self.V + self.NGV - 1) // self.NGV * self.NGV
        if share is not None:
            self.w = share.w
        elif isinstance(sd, DeviceWeights):   # weights already on this card (another engine / width)
            self.w = sd
        else:
            self.w = DeviceWeights(cfg, sd, self.dev)
        self._m = self.w.model_struct()
        c, d = cfg, self.dev
        H, M = c.hidden, c.inter
        QN, KN = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        f32 = dict(dtype=torch.float32, device=d)
        partial_floats, counters, act_cols, act2_cols = _lib.decode_workspace(self._m, S)
        self._x = torch.zeros((MAXB, H), **f32)
        self._q = torch.zeros((MAXB, QN), **f32)
        # hi/lo bf16 GEMM operands: rows of streams >= B must stay zero
        self._act = torch.zeros((2 * MAXB, act_cols), dtype=BF, device=d)
        self._act_o = torch.zeros((2 * MAXB, QN), dtype=BF, device=d)
        self._act2 = torch.zeros((2 * MAXB, act2_cols), dtype=BF, device=d)
        self._ss = torch.zeros((H // 128, MAXB), **f32)
        self._logits = torch.zeros((B, self.V), **f32)
        # fused attention: chunk records ({value, flag} words) and per-(stream, kv head) epochs
        self._part = torch.zeros(_lib.decode_attn_workspace(self._m, B, S), **f32)
        self._partial = torch.zeros(max(partial_floats, 1), **f32)
        self._counters = torch.zeros(max(counters, 1), dtype=torch.int32, device=d)
        self._best = torch.zeros(MAXB, dtype=torch.int64, device=d)
        # tokens and positions side by side, so one host->device copy carries both
        self._tp = torch.zeros((2, B), dtype=torch.int32, device=d)
        self._toks, self._pos = self._tp[0], self._tp[1]
        self._next = torch.zeros(B, dtype=torch.int32, device=d)
        self._in_host = torch.zeros((2, B), dtype=torch.int32).pin_memory()
        self._in_np = self._in_host.numpy()   # the pinned buffer, written in place
        self._out_host = torch.zeros(B, dtype=torch.int32).pin_memory()
        self._checked = set()                 # cache bindings (data pointers) already validated
        self._group_numel = self.NG * B * c.n_kv * S * c.head_dim
        self.stream = torch.cuda.Stream(device=d)
        self.use_graph = os.environ.get("RNGD_CUDA_GRAPH", "1") != "0"
        self._graphs = {}
        self._copied = torch.cuda.Event()
        self._fill = None                     # lane-fill state: private flags, counter, item, sequence
        # embed + operand; per layer: QKV gemm, fused attention, O gemm, gate/up gemm, down gemm;
        # lm_head gemm, argmax finalize; advance
        self.launches_per_step = 2 + self.nl * 5 + 2 + 1

    # ------------------------------------------------------------ buffers
    def _io(self, Kg, Vg):
        p = lambda t: t.data_ptr()
        return _lib.DecodeIO(B=self.B, Bcap=self.B, S=self.S, kv_layers=self.NG, kcache=p(Kg), vcache=p(Vg),
                             toks=p(self._toks), pos=p(self._pos), x=p(self._x), q=p(self._q),
                             act=p(self._act), act_o=p(self._act_o), act2=p(self._act2), ss=p(self._ss),
                             logits=p(self._logits),
                             attn_part=p(self._part), partial=p(self._partial), counters=p(self._counters),
                             best=p(self._best), next=p(self._next))

    def _check_cache(self, Kd, Vd):
        c = self.cfg
        shape = (self.NG, self.B, c.n_kv, self.S, c.head_dim)
        if len(Kd) != self.ngroups or len(Vd) != self.ngroups:
            raise ValueError(f"expected {self.ngroups} cache groups")
        for t in list(Kd) + list(Vd):
            if tuple(t.shape) != shape or t.dtype != BF or not t.is_contiguous() or t.device != self.dev:
                raise ValueError(f"cache group must be a contiguous bf16 {shape} tensor on {self.dev}, "
                                 f"got {tuple(t.shape)} {t.dtype} on {t.device}")

    def _alloc_cache(self, ipc=False):
        c = self.cfg
        shape = (self.nl, self.B, c.n_kv, self.S, c.head_dim)
        if ipc:
            from rngd_pd.nvlink import ipc_empty
            K, V = ipc_empty(shape, BF, self.dev), ipc_empty(shape, BF, self.dev)
        else:
            K = torch.zeros(shape, dtype=BF, device=self.dev)
            V = torch.zeros_like(K)
        return ([K[g * self.NG:(g + 1) * self.NG] for g in range(self.ngroups)],
                [V[g * self.NG:(g + 1) * self.NG] for g in range(self.ngroups)])

    @_lib.on_device
    def full_kv(self, Kd, Vd):
        """The whole resident cache (K, V) [L][B][NKV][S][HD] behind a group list from blank_kv /
        adopt_kv_device / load_kv: what a KV transport binds to write requests into lanes."""
        self._check_cache(Kd, Vd)
        c = self.cfg
        shape = (self.nl, self.B, c.n_kv, self.S, c.head_dim)
        out = []
        for groups in (Kd, Vd):
            g0 = groups[0]
            step = g0.numel() * g0.element_size()
            if any(t.data_ptr() != g0.data_ptr() + g * step for g, t in enumerate(groups)):
                raise ValueError("full_kv: cache groups are not consecutive slices of one allocation")
            out.append(torch.empty(0, dtype=BF, device=self.dev).set_(g0.untyped_storage(), g0.storage_offset(),
                                                                      shape))
        return out[0], out[1]

    # ---------------------------------------------------------- KV intake
    @staticmethod
    def _bf16_host(a):
        return a if torch.is_tensor(a) else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(BF)

    @_lib.on_device
    def prepare_kv(self, Ks, Vs):
        """Host-side stack + cast, off the device (engines/decode_batch.py:305-330).
        Ks/Vs: per-stream K [nl, NKV, HD, S] / V [nl, NKV, S, HD], padded to B lanes
        by repeating the last."""
        Ks, Vs = list(Ks), list(Vs)
        while len(Ks) < self.B:
            Ks.append(Ks[-1])
            Vs.append(Vs[-1])
        K = torch.stack([self._bf16_host(a) for a in Ks], 1)   # [nl, B, NKV, HD, S]
        V = torch.stack([self._bf16_host(a) for a in Vs], 1)   # [nl, B, NKV, S, HD]
        return K, V

    @staticmethod
    def stage_host_kv(K, V):
        """float32 host arrays -> bfloat16 host tensors (engines/decode_batch.py:332-341)."""
        return (torch.from_numpy(np.ascontiguousarray(K, dtype=np.float32)).to(BF),
                torch.from_numpy(np.ascontiguousarray(V, dtype=np.float32)).to(BF))

    @_lib.on_device
    def upload_prepared_kv(self, prepared):
        """Transfer + relayout to the decode layout (engines/decode_batch.py:343-351)."""
        K, V = prepared
        Kd, Vd = self._alloc_cache()
        Kdev = K.to(self.dev, non_blocking=False).transpose(-1, -2)      # -> [nl, B, NKV, S, HD]
        Vdev = V.to(self.dev, non_blocking=False)
        for g in range(self.ngroups):
            sl = slice(g * self.NG, (g + 1) * self.NG)
            Kd[g].copy_(Kdev[sl])
            Vd[g].copy_(Vdev[sl])
        return Kd, Vd

    @_lib.on_device
    def load_kv(self, Ks, Vs):
        return self.upload_prepared_kv(self.prepare_kv(Ks, Vs))

    @_lib.on_device
    def write_slot_kv(self, Kd, Vd, idx, K, V):
        """Replace lane idx of the resident cache in place (engines/decode_batch.py:357-377).
        K [nl, NKV, HD, S] / V [nl, NKV, S, HD]: host float32/bf16 or device tensors; or K a
        PrefillKV (a prefill-layout cache on this device, V unused), moved by the handoff kernel."""
        if not 0 <= idx < self.B:
            raise IndexError(f"lane {idx} outside 0..{self.B - 1}")
        if isinstance(K, PrefillKV):
            return self._fill_lane(Kd, Vd, idx, K)
        Kt = (K if torch.is_tensor(K) else self._bf16_host(K)).to(self.dev, BF).transpose(-1, -2)
        Vt = (V if torch.is_tensor(V) else self._bf16_host(V)).to(self.dev, BF)
        for g in range(self.ngroups):
            sl = slice(g * self.NG, (g + 1) * self.NG)
            Kd[g][:, idx].copy_(Kt[sl])
            Vd[g][:, idx].copy_(Vt[sl])
        return Kd, Vd

    def _fill_lane(self, Kd, Vd, idx, pk):
        """Positions [0, pk.tokens) of a prefill-layout cache into lane idx, on self.stream: one
        rngd_kv_handoff_batch launch per layer group with this GPU's cache as the destination.
        The kernel's layer flags go to a private array nobody waits on: the steps that read the
        lane are queued after the fill on the same stream."""
        c = self.cfg
        kv, tokens = pk.kv, pk.tokens
        want = (self.nl, 2, c.n_kv, self.S, c.head_dim)
        if kv.dtype != BF or kv.device != self.dev or not kv.is_contiguous() or tuple(kv.shape) != want:
            raise ValueError(f"PrefillKV: kv must be a contiguous bf16 {want} tensor on {self.dev}, "
                             f"got {tuple(kv.shape)} {kv.dtype} on {kv.device}")
        if not 1 <= tokens <= self.S:
            raise ValueError(f"PrefillKV: {tokens} tokens outside 1..{self.S}")
        self._check_cache(Kd, Vd)
        if self._fill is None:
            self._fill = {"flags": torch.zeros((self.B, self.NG), dtype=torch.int64, device=self.dev),
                          "done": torch.zeros(_lib.KV_MAX_BATCH, dtype=torch.int32, device=self.dev),
                          "item": (_lib.KvItem * 1)(), "seq": 0}
        f = self._fill
        f["seq"] += 1
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.dev))
        kv.record_stream(s)                   # the caller may drop kv before the fill has read it
        plane = c.n_kv * self.S * c.head_dim  # elements of one layer's K (or V) block
        h = _lib.stream_handle(s)
        it = f["item"][0]
        for g in range(self.ngroups):
            base = kv.data_ptr() + g * self.NG * 2 * plane * 2
            it.src_k, it.src_v, it.lane, it.tokens, it.seq = base, base + plane * 2, idx, tokens, f["seq"]
            _lib.call("rngd_kv_handoff_batch", f["item"], 1, 2 * plane, ctypes.c_void_p(Kd[g].data_ptr()),
                      ctypes.c_void_p(Vd[g].data_ptr()), self.NG, c.n_kv, self.S, c.head_dim, self.B, 0, self.NG,
                      _lib.ptr(f["done"]), _lib.ptr(f["flags"]), h)
        return Kd, Vd

    @_lib.on_device
    def download_kv(self, Kd, Vd):
        """Resident cache -> host [nl, B, NKV, HD, S] / [nl, B, NKV, S, HD] float32."""
        K = torch.cat([k.transpose(-1, -2).float().cpu() for k in Kd], 0).numpy()
        V = torch.cat([v.float().cpu() for v in Vd], 0).numpy()
        return K, V

    @_lib.on_device
    def upload_kv(self, K, V):
        """[nl, B, ...] host arrays (reference layout) back onto the device, per group."""
        return self.upload_prepared_kv((self._bf16_host(K), self._bf16_host(V)))

    @_lib.on_device
    def adopt_kv_device(self, Ks, Vs):
        """Per-request device caches (prefill on this card, reference layout) batched in place
        (engines/decode_batch.py:399-414)."""
        Ks, Vs = list(Ks), list(Vs)
        while len(Ks) < self.B:
            Ks.append(Ks[-1])
            Vs.append(Vs[-1])
        Kd, Vd = self._alloc_cache()
        for b in range(self.B):
            self.write_slot_kv(Kd, Vd, b, Ks[b], Vs[b])
        return Kd, Vd

    @_lib.on_device
    def blank_kv(self, ipc=False):
        """An empty resident cache: every slot free (engines/decode_batch.py:416-420).
        ipc=True allocates it so that a prefill process can map it (rngd_pd.nvlink)."""
        return self._alloc_cache(ipc)

    # ---------------------------------------------------------------- step
    def _launch(self, Kd, Vd, stream):
        h = _lib.stream_handle(stream)
        m = self._m
        io = self._io(Kd[0], Vd[0])
        _lib.call("rngd_decode_embed", m, io, h)
        for g in range(self.ngroups):
            io.kcache, io.vcache = Kd[g].data_ptr(), Vd[g].data_ptr()
            _lib.call("rngd_decode_layers", m, io, g * self.NG, (g + 1) * self.NG, h)
        _lib.call("rngd_decode_lmhead", m, io, h)
        _lib.call("rngd_decode_advance", io, h)   # next -> toks, pos + 1 (used by step_device)

    def _validate(self, toks, positions):
        toks, positions = list(toks), list(positions)
        if len(toks) != self.B or len(positions) != self.B:
            raise ValueError(f"expected {self.B} tokens and positions")
        for p in positions:
            if not 0 <= int(p) < self.S:
                raise ValueError(f"position {p} outside the {self.S}-wide cache")
        for t in toks:
            if not 0 <= int(t) < self.V:
                raise ValueError(f"token {t} outside the vocabulary")
        return toks, positions

    def _run(self, toks, positions, Kd, Vd):
        """Upload this step's tokens/positions and run the (captured) step on self.stream."""
        groups = list(Kd) + list(Vd)
        key = tuple(t.data_ptr() for t in groups)
        # a binding (its data pointers) gets the full check once; later steps re-check size and
        # dtype only, which still catches a smaller tensor allocated at a freed address
        if key not in self._checked or any(t.numel() != self._group_numel or t.dtype != BF for t in groups):
            self._check_cache(Kd, Vd)
            self._checked.add(key)
        self._copied.synchronize()            # the previous step's upload has left the pinned buffer
        self._in_np[0] = toks
        self._in_np[1] = positions
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.dev))
        def upload():
            self._tp.copy_(self._in_host, non_blocking=True)
            self._copied.record(s)

        with torch.cuda.stream(s):
            g = self._graphs.get(key) if self.use_graph else None
            upload()
            if self.use_graph and g is None:
                # first use of this cache binding: one eager run with this step's inputs loads
                # the kernels, then the step is captured.  The run below recomputes the same
                # step from the same inputs (its k/v land at the same positions), so the eager
                # run leaves no trace.
                self._launch(Kd, Vd, s)
                g = torch.cuda.CUDAGraph()
                # thread_local: a CUDA call made meanwhile by another thread (a producer copying
                # flags or allocating on another GPU) is legal and does not void this capture
                with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                    self._launch(Kd, Vd, s)
                self._graphs[key] = g
                # the step ends by advancing toks/pos on the device (for step_device):
                # put this step's inputs back before the replay
                upload()
            if g is not None:
                g.replay()
            else:
                self._launch(Kd, Vd, s)

    @_lib.on_device
    def step(self, toks, positions, Kd, Vd):
        """One token for each of B streams. Returns next tokens and the cache."""
        toks, positions = self._validate(toks, positions)
        self._run(toks, positions, Kd, Vd)
        with torch.cuda.stream(self.stream):
            self._out_host.copy_(self._next, non_blocking=True)
        self.stream.synchronize()
        return self._out_host.tolist(), Kd, Vd

    @_lib.on_device
    def step_logits(self, toks, positions, Kd, Vd):
        """The same step returning fp32 logits in the reference layout [NG, Vp/NG, B]
        (zero-padded past V) on the device, for teacher-forced comparisons."""
        toks, positions = self._validate(toks, positions)
        self._run(toks, positions, Kd, Vd)
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        lg = torch.zeros((self.Vp, self.B), dtype=torch.float32, device=self.dev)
        lg[:self.V] = self._logits.t()
        return lg.view(self.NGV, self.Vp // self.NGV, self.B), Kd, Vd

    @_lib.on_device
    def set_inputs(self, toks, positions):
        """Upload tokens/positions for step_device() (validated like step())."""
        toks, positions = self._validate(toks, positions)
        self._copied.synchronize()
        self._in_np[0] = toks
        self._in_np[1] = positions
        with torch.cuda.stream(self.stream):
            self._tp.copy_(self._in_host, non_blocking=True)
            self._copied.record(self.stream)

    @_lib.on_device
    def step_device(self, Kd, Vd, n=1):
        """n greedy steps entirely on the device: each step's argmax becomes the next
        step's token and every position advances by one (no host round trip).  The
        caller keeps positions < S (set_inputs first).  Returns immediately; the work
        is queued on self.stream."""
        self._check_cache(Kd, Vd)
        key = tuple(t.data_ptr() for t in list(Kd) + list(Vd))
        g = self._graphs.get(key)
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                if g is None:
                    self._launch(Kd, Vd, self.stream)
                else:
                    g.replay()

    @_lib.on_device
    def next_tokens_device(self):
        return self._next

    @_lib.on_device
    def logits_bv(self):
        """The last step's logits as [B, V] fp32 (device)."""
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        return self._logits
