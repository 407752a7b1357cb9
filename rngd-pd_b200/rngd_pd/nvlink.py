"""`nvlink` KV transport: prefill GPU -> decode GPU over NVLink peer-to-peer stores.

New next to the reference's host-staged `shm` / `tcp` paths (src/rngd_pd/connector/
transport.py:80-235) and modelled on the fence/ownership contract of its NIXL
transport (src/rngd_pd/kv_nixl.py:145-369: bind / plan / submit / wait, no silent
fallback, in-flight work drained before release).

Roles.
  * Decode side (receiver) owns the destination: its resident K / V caches
    [L][Bcap][NKV][S][HD] and an int64 flag array [Bcap][L].  It `bind_cache()`s them,
    `reserve(req_id, lane)`s a lane for a request before prefill writes (a lease with a
    sequence number that only grows, so a stale flag from the lane's previous request
    never satisfies a new wait), and publishes `handshake_metadata()`.
  * Prefill side (sender) `set_remote_handshake(meta)`s and `push_device()`s a request's
    cache (prefill layout [L][2][NKV][S][HD]) or single layers into the leased lane.  One
    fused kernel (rngd_kv_handoff) stores the bytes into the peer's lane and publishes the
    per-layer flags with a system-scope release.
  * `wait()` (host, bounded, TimeoutError: polls the lane's flags with small device->host
    copies, no kernel) or `wait_stream()` (a bounded device wait ordered before the decode
    stream's next step) observes arrival.  The device wait is used only for a lease whose
    sender was declared to run on another GPU: a spinning kernel must never depend on a
    kernel of its own GPU, which nothing guarantees to run beside it.  A decode worker
    never frees memory prefill may write; prefill never frees decode memory.

Peers in one process use direct device pointers (peer access enabled); peers in other
processes map the receiver's buffers through CUDA IPC handles carried in the handshake
metadata (buffers allocated by `ipc_empty`).
"""
import collections
import ctypes
import os
import socket
import threading
import time
import weakref

import torch

from rngd_pd import _lib
from rngd_pd.connector.transport import Transport

BF = torch.bfloat16
_HSIZE = None


def _handle_size():
    global _HSIZE
    if _HSIZE is None:
        _HSIZE = _lib.lib.rngd_ipc_handle_size()
    return _HSIZE


class IpcBuffer:
    """cudaMalloc'ed, zeroed device memory with a CUDA IPC handle.  `tensor()` views keep it alive."""

    def __init__(self, nbytes, device):
        self.device = torch.device(device)
        self.nbytes = int(nbytes)
        self.handle = ctypes.create_string_buffer(_handle_size())
        p = ctypes.c_void_p(0)
        with torch.cuda.device(self.device):
            _lib.call("rngd_ipc_alloc", self.nbytes, ctypes.byref(p), self.handle)
        self.ptr = p.value

    @property
    def handle_hex(self):
        return self.handle.raw.hex()

    def tensor(self, shape, dtype):
        buf = self

        class _View:
            __cuda_array_interface__ = {"shape": tuple(shape), "typestr": {BF: "<f2", torch.int64: "<i8",
                                                                           torch.float32: "<f4"}[dtype],
                                        "data": (buf.ptr, False), "version": 3, "strides": None}
            owner = buf

        t = torch.as_tensor(_View(), device=self.device)
        return t.view(dtype) if dtype == BF else t

    def __del__(self):
        if getattr(self, "ptr", None):
            try:
                with torch.cuda.device(self.device):
                    _lib.lib.rngd_ipc_free(ctypes.c_void_p(self.ptr))
            except Exception:
                pass
            self.ptr = None


_IPC_TENSORS = weakref.WeakValueDictionary()  # data_ptr -> IpcBuffer, for handle lookup


def ipc_empty(shape, dtype, device):
    """A zeroed tensor whose memory can be mapped by another process (CUDA IPC)."""
    esize = torch.empty((), dtype=dtype).element_size()
    n = 1
    for d in shape:
        n *= int(d)
    buf = IpcBuffer(max(n * esize, 256), device)
    t = buf.tensor(shape, dtype)
    _IPC_TENSORS[t.data_ptr()] = buf
    return t


def ipc_handle(t):
    buf = _IPC_TENSORS.get(t.data_ptr())
    return buf.handle_hex if buf is not None else None


class _Peer:
    """A receiver as seen by a sender: device pointers of its K, V caches and flags."""

    def __init__(self, meta, local_device):
        self.meta = meta
        self.L, self.Bcap, self.NKV, self.S, self.HD = meta["shape"]
        self.device = meta["device"]
        self._opened = []
        same_process = meta["pid"] == os.getpid() and meta["host"] == socket.gethostname()
        if same_process:
            self.k, self.v, self.flags = meta["ptrs"]["k"], meta["ptrs"]["v"], meta["ptrs"]["flags"]
            if self.device != local_device.index:
                _lib.call("rngd_peer_enable", local_device.index, self.device)
        else:
            hs = meta.get("handles") or {}
            if not all(hs.get(n) for n in ("k", "v", "flags")):
                raise _lib.RngdError(_lib.RNGD_ERR_ARG, "nvlink: the receiver's buffers are not IPC-exportable "
                                     "(allocate its cache with rngd_pd.nvlink.ipc_empty)")
            ptrs = {}
            with torch.cuda.device(local_device):
                for n in ("k", "v", "flags"):
                    p = ctypes.c_void_p(0)
                    _lib.call("rngd_ipc_open", bytes.fromhex(hs[n]), ctypes.byref(p))
                    ptrs[n] = p.value
                    self._opened.append(p.value)
            self.k, self.v, self.flags = ptrs["k"], ptrs["v"], ptrs["flags"]
        self._local_device = local_device

    def close(self):
        with torch.cuda.device(self._local_device):
            for p in self._opened:
                _lib.lib.rngd_ipc_close(ctypes.c_void_p(p))
        self._opened = []


class LaneLeases:
    """The receiver's lease book (host-only state; the flags themselves live wherever the
    caller keeps them).

    A lane is leased to one request at a time.  Every lease takes the lane's next sequence
    number, and the sender publishes that number into the lane's per-layer flags after the
    layer's bytes have landed.  A layer has arrived for a lease when its flag is >= the lease's
    number; because numbers only grow, whatever an earlier request left in the flags never
    satisfies a later lease of the same lane.  `start_after(lane, n)` continues after the
    numbers already present in existing flags."""

    def __init__(self, lanes):
        self.lanes = int(lanes)
        self._lock = threading.Lock()
        self._seq = [0] * self.lanes
        self._held = {}              # req_id -> (lane, seq)
        self._sender = {}            # req_id -> sender device index, when declared

    def start_after(self, lane, n):
        with self._lock:
            self._seq[lane] = max(self._seq[lane], int(n))

    def reserve(self, req_id, lane, sender_device=None):
        if not 0 <= lane < self.lanes:
            raise IndexError(f"lane {lane} outside 0..{self.lanes - 1}")
        with self._lock:
            if any(l == lane for l, _ in self._held.values()):
                raise ValueError(f"nvlink: lane {lane} is already leased")
            if req_id in self._held:
                raise ValueError(f"nvlink: request {req_id!r} already holds lane {self._held[req_id][0]}")
            self._seq[lane] += 1
            self._held[req_id] = (lane, self._seq[lane])
            self._sender[req_id] = sender_device
            return {"req": req_id, "lane": lane, "seq": self._seq[lane]}

    def release(self, req_id):
        with self._lock:
            self._held.pop(req_id, None)
            self._sender.pop(req_id, None)

    def lookup(self, req_id):
        """(lane, seq, sender device or None) of a held lease; KeyError if none."""
        with self._lock:
            if req_id not in self._held:
                raise KeyError(f"nvlink: no lease for request {req_id!r}")
            lane, seq = self._held[req_id]
            return lane, seq, self._sender.get(req_id)

    def snapshot(self):
        with self._lock:
            return {r: [lane, seq] for r, (lane, seq) in self._held.items()}

    def clear(self):
        with self._lock:
            self._held.clear()
            self._sender.clear()

    @staticmethod
    def landed(flag_row, seq, layer0, layer1):
        """Whether layers [layer0, layer1) of a lane's flags (a sequence of ints) reached seq."""
        row = flag_row[layer0:layer1]
        return len(row) == 0 or int(min(row)) >= seq


class SenderLeases:
    """The sender's view of leases: request -> (receiver key, lane, seq), learned from a
    receiver's handshake metadata or from tickets forwarded with requests."""

    def __init__(self):
        self._lock = threading.Lock()
        self._known = {}

    def learn(self, peer_key, leases):
        with self._lock:
            for r, (lane, seq) in leases.items():
                self._known[r] = (peer_key, lane, seq)

    def add(self, peer_key, ticket):
        with self._lock:
            self._known[ticket["req"]] = (peer_key, ticket["lane"], ticket["seq"])

    def find(self, req_id):
        with self._lock:
            return self._known.get(req_id)

    def clear(self):
        with self._lock:
            self._known.clear()


def poll_until(check, timeout, what, pause=20e-6, spin=2e-3):
    """Call check() until it is true; TimeoutError naming `what` after `timeout` seconds.
    Returns the seconds waited.  For the first `spin` seconds the checks run back to back (a
    check is itself a device->host copy of ~10 us, while time.sleep rounds a pause this short up
    to ~60 us, which would dominate a handoff of tens of microseconds); after that each check
    is followed by a pause."""
    t0 = time.perf_counter()
    while not check():
        waited = time.perf_counter() - t0
        if waited > timeout:
            raise TimeoutError(f"nvlink: {what} did not arrive within {timeout}s")
        if waited > spin:
            time.sleep(pause)
    return time.perf_counter() - t0


class NvlinkTransport(Transport):
    """GPU -> GPU KV transport over NVLink (`airm.kv_transports` name `nvlink`)."""

    name = "nvlink"
    shared = True

    def __init__(self, device=None, wait_slice_s=1.0):
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.wait_slice_s = wait_slice_s
        self._lock = threading.RLock()
        # receiver state
        self._cache = None          # (K, V, flags) tensors
        self.leases = LaneLeases(0)
        self._status_host = self._status_dev = None
        self._status_next = 0
        self._poll_stream = None
        self._poll_all = self._poll_np = None
        # sender state
        self._peers = {}            # peer key -> _Peer
        self.remote_leases = SenderLeases()
        self._done = {}             # stream handle -> completion counter of that stream's handoffs
        self._items = None          # the launch's rngd_kv_item_t array, reused
        self.measurements = collections.deque(maxlen=1024)

    # ------------------------------------------------------------- receiver
    def bind_cache(self, K, V, flags=None):
        """Register the decode cache this transport writes into: K, V bf16 [L][Bcap][NKV][S][HD]
        (contiguous, on this device; from `ipc_empty` when senders live in other processes)."""
        if K.shape != V.shape or K.dim() != 5 or K.dtype != BF or not (K.is_contiguous() and V.is_contiguous()):
            raise ValueError("bind_cache: K and V must be contiguous bf16 [L, Bcap, NKV, S, HD] tensors")
        if K.device != self.device or V.device != self.device:
            raise ValueError(f"bind_cache: the cache must live on {self.device}")
        L, Bcap = K.shape[0], K.shape[1]
        if flags is None:
            flags = ipc_empty((Bcap, L), torch.int64, self.device) if ipc_handle(K) else \
                torch.zeros((Bcap, L), dtype=torch.int64, device=self.device)
        elif (tuple(flags.shape) != (Bcap, L) or flags.dtype != torch.int64 or not flags.is_contiguous()
              or flags.device != self.device):
            raise ValueError(f"bind_cache: flags must be a contiguous int64 [{Bcap}, {L}] tensor on {self.device}")
        with self._lock:
            self._cache = (K, V, flags)
            self.leases = LaneLeases(Bcap)
            for b in range(Bcap):   # continue after whatever the flags already hold
                self.leases.start_after(b, int(flags[b].max().item()))

    def reserve(self, req_id, lane, sender_device=None):
        """Lease `lane` to `req_id` before prefill writes it; returns the ticket {req, lane, seq}.
        `sender_device`: the GPU the prefill side pushes from, when known; only a sender on
        another GPU lets wait_stream() order the decode stream with a device-side wait."""
        if self._cache is None:
            raise RuntimeError("nvlink: reserve() before bind_cache()")
        return self.leases.reserve(req_id, lane, sender_device)

    def release(self, req_id):
        self.leases.release(req_id)

    def handshake_metadata(self):
        if self._cache is None:
            return {"transport": self.name, "pid": os.getpid(), "host": socket.gethostname()}
        K, V, flags = self._cache
        leases = self.leases.snapshot()
        return {"transport": self.name, "pid": os.getpid(), "host": socket.gethostname(),
                "device": self.device.index, "shape": list(K.shape),
                "ptrs": {"k": K.data_ptr(), "v": V.data_ptr(), "flags": flags.data_ptr()},
                "handles": {"k": ipc_handle(K), "v": ipc_handle(V), "flags": ipc_handle(flags)},
                "leases": leases}

    _NSTATUS = 256

    def _status(self):
        """One host-mapped status word from a pool (rotating; 256 waits may be outstanding)."""
        with self._lock:
            if self._status_host is None:
                h, d = ctypes.c_void_p(0), ctypes.c_void_p(0)
                _lib.call("rngd_host_alloc_mapped", 4 * self._NSTATUS, ctypes.byref(h), ctypes.byref(d))
                self._status_host, self._status_dev = h.value, d.value
            i = self._status_next
            self._status_next = (i + 1) % self._NSTATUS
        return self._status_host + 4 * i, self._status_dev + 4 * i

    def _lease(self, req_id, layer0, layer1):
        if self._cache is None:
            raise RuntimeError("nvlink: wait before bind_cache()")
        L = self._cache[0].shape[0]
        layer1 = L if layer1 is None else layer1
        if not 0 <= layer0 < layer1 <= L:
            raise ValueError(f"nvlink: layers [{layer0}, {layer1}) outside [0, {L})")
        lane, seq, sender = self.leases.lookup(req_id)
        return lane, seq, layer1, sender

    def _read_all_flags(self):
        """Every lane's per-layer flags on the host, a [Bcap][L] int64 array: one device->host copy
        of the whole flag block on a side stream (rngd_kv_read_flags), into a pinned buffer."""
        flags = self._cache[2]
        with self._lock:
            if self._poll_all is None or tuple(self._poll_all.shape) != tuple(flags.shape):
                if self._poll_stream is None:
                    self._poll_stream = torch.cuda.Stream(device=self.device)
                self._poll_all = torch.zeros(flags.shape, dtype=torch.int64).pin_memory()
                self._poll_np = self._poll_all.numpy()
            _lib.call("rngd_kv_read_flags", _lib.ptr(flags), _lib.ptr(self._poll_all), flags.numel(),
                      _lib.stream_handle(self._poll_stream))
            return self._poll_np.copy()

    def _read_flags(self, lane):
        """The lane's per-layer flags on the host."""
        return self._read_all_flags()[lane]

    def arrived_all(self, req_ids, layer0=0, layer1=None):
        """Whether every request of `req_ids` has layers [layer0, layer1) landed."""
        leases = [self._lease(r, layer0, layer1) for r in req_ids]
        rows = self._read_all_flags()
        return all(LaneLeases.landed(rows[lane], seq, layer0, l1) for lane, seq, l1, _ in leases)

    def wait_all(self, req_ids, layer0=0, layer1=None, timeout=5.0):
        """wait() for several requests at once: each poll reads every lane's flags in one copy."""
        req_ids = list(req_ids)
        for r in req_ids:
            self._lease(r, layer0, layer1)
        return poll_until(lambda: self.arrived_all(req_ids, layer0, layer1), timeout,
                          f"requests {req_ids[:3]}{'...' if len(req_ids) > 3 else ''} layers [{layer0}, {layer1})")

    def arrived(self, req_id, layer0=0, layer1=None):
        """Whether the request's layers [layer0, layer1) have landed."""
        lane, seq, layer1, _ = self._lease(req_id, layer0, layer1)
        return LaneLeases.landed(self._read_flags(lane), seq, layer0, layer1)

    def wait(self, req_id, layer0=0, layer1=None, timeout=5.0):
        """Block until the request's layers [layer0, layer1) have landed; TimeoutError after
        `timeout` seconds.  Host polling of the flags: no kernel waits on another kernel."""
        self._lease(req_id, layer0, layer1)
        return poll_until(lambda: self.arrived(req_id, layer0, layer1), timeout,
                          f"request {req_id!r} layers [{layer0}, {layer1})")

    def wait_stream(self, req_id, stream=None, layer0=0, layer1=None, timeout=5.0):
        """Order `stream` after the arrival of the request's layers [layer0, layer1); returns a
        callable outcome(block=True) that reports True or raises TimeoutError.

        Sender declared on another GPU (reserve(..., sender_device=d), d != this device): a
        bounded one-warp device wait on the flags (rngd_kv_wait) is enqueued on `stream`, so
        the host does not block.  Sender on this GPU or not declared: the host waits first
        (wait()), since a spinning kernel must not depend on another kernel of the same GPU."""
        lane, seq, layer1, sender = self._lease(req_id, layer0, layer1)
        if sender is None or sender == self.device.index:
            self.wait(req_id, layer0, layer1, timeout)
            return lambda block=True: True
        hptr, dptr = self._status()
        word = ctypes.c_int32.from_address(hptr)
        word.value = -99
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        fl = self._cache[2][lane]
        with torch.cuda.device(self.device):
            _lib.call("rngd_kv_wait", _lib.ptr(fl), layer0, layer1, seq, int(timeout * 1e9), ctypes.c_void_p(dptr),
                      _lib.stream_handle(s))

        def outcome(block=True):
            t0 = time.time()
            while word.value == -99:
                if not block:
                    return None
                if time.time() - t0 > timeout + 5.0:
                    raise TimeoutError(f"nvlink: wait for {req_id!r} did not report")
                time.sleep(20e-6)
            if word.value != 0:
                raise TimeoutError(f"nvlink: request {req_id!r} layers [{layer0}, {layer1}) did not arrive "
                                   f"within {timeout}s")
            return True

        return outcome

    def lane_views(self, req_id):
        """(K, V) device views of the leased lane, [L, NKV, S, HD] each."""
        K, V, _ = self._cache
        lane, _, _ = self.leases.lookup(req_id)
        return K[:, lane], V[:, lane]

    # ---------------------------------------------------------------- sender
    def set_remote_handshake(self, meta):
        """Register a receiver (its buffers and current leases)."""
        if meta.get("transport") != self.name or "shape" not in meta:
            raise ValueError("nvlink: not an nvlink receiver's handshake metadata")
        key = (meta["host"], meta["pid"], meta["device"], meta["ptrs"]["k"])
        with self._lock:
            if key not in self._peers:
                self._peers[key] = _Peer(meta, self.device)
        self.remote_leases.learn(key, meta.get("leases", {}))
        return key

    def add_lease(self, peer_key, ticket):
        """Learn one lease (e.g. a ticket forwarded with the request) for a registered receiver."""
        self.remote_leases.add(peer_key, ticket)

    def _target(self, req_id):
        known = self.remote_leases.find(req_id)
        if known is not None:
            key, lane, seq = known
            with self._lock:
                return self._peers[key], lane, seq
        if self._cache is not None:                      # sender and receiver in one object
            try:
                lane, seq, _ = self.leases.lookup(req_id)
            except KeyError:
                pass
            else:
                meta = self.handshake_metadata()
                key = (meta["host"], meta["pid"], meta["device"], meta["ptrs"]["k"])
                with self._lock:
                    if key not in self._peers:
                        self._peers[key] = _Peer(meta, self.device)
                    return self._peers[key], lane, seq
        raise KeyError(f"nvlink: no lease known for request {req_id!r} (set_remote_handshake/add_lease first)")

    def push_device(self, req_id, kv, layer0=0, layer1=None, stream=None, tokens=None):
        """Move a request's cache (prefill layout [L][2][NKV][S][HD] bf16 on this device, or the
        layer block [layer1-layer0][2][NKV][S][HD] starting at layer0) into its leased lane.
        tokens: move positions [0, tokens) only (the prompt); default all S.  Returns the bytes moved."""
        return self.push_many([(req_id, kv, tokens)], layer0, layer1, stream)

    def push_many(self, items, layer0=0, layer1=None, stream=None):
        """push_device for several requests [(req_id, kv, tokens or None), ...]: one launch per
        receiver and per 16 requests (rngd_kv_handoff_batch).  Returns the bytes moved.

        The host path stays short: K / V source addresses are computed from the cache tensor's
        address (no views are made), each cache is recorded once on the launch stream, and the
        launch's item array is a reused ctypes buffer."""
        groups = {}
        for req_id, kv, tokens in items:
            peer, lane, seq = self._target(req_id)
            l1 = peer.L if layer1 is None else layer1
            nl = l1 - layer0
            if kv.dtype != BF or kv.device != self.device or not kv.is_contiguous():
                raise ValueError(f"nvlink: kv must be a contiguous bf16 tensor on {self.device}")
            shape = kv.shape
            if shape[1:] != (2, peer.NKV, peer.S, peer.HD) or shape[0] not in (nl, peer.L):
                raise ValueError(f"nvlink: kv layer block {tuple(shape)} does not match the receiver's "
                                 f"[{nl}, 2, {peer.NKV}, {peer.S}, {peer.HD}]")
            plane = peer.NKV * peer.S * peer.HD * 2                     # bytes of one layer's K (or V)
            k_ptr = kv.data_ptr() + (0 if shape[0] == nl else layer0) * 2 * plane
            groups.setdefault(id(peer), (peer, l1, []))[2].append((lane, seq, k_ptr, k_ptr + plane, tokens, kv))
        moved = 0
        for peer, l1, reqs in groups.values():
            for i in range(0, len(reqs), _lib.KV_MAX_BATCH):
                moved += self._launch(peer, reqs[i:i + _lib.KV_MAX_BATCH], 2 * peer.NKV * peer.S * peer.HD, layer0,
                                      l1, stream)
        return moved

    def push_layer(self, req_id, layer, k, v, stream=None, tokens=None):
        """Move one layer's k [NKV][S][HD] and v [NKV][S][HD] (the connector's save_kv_layer)."""
        peer, lane, seq = self._target(req_id)
        for t in (k, v):
            if t.dtype != BF or not t.is_contiguous() or t.device != self.device or \
                    tuple(t.shape) != (peer.NKV, peer.S, peer.HD):
                raise ValueError(f"nvlink: layer tensors must be contiguous bf16 [{peer.NKV}, {peer.S}, "
                                 f"{peer.HD}] on {self.device}")
        return self._launch(peer, [(lane, seq, k.data_ptr(), v.data_ptr(), tokens, k, v)], 0, layer, layer + 1,
                            stream)

    def _counter(self, s):
        key = s.cuda_stream
        with self._lock:
            c = self._done.get(key)
            if c is None:
                c = self._done[key] = torch.zeros(_lib.KV_MAX_BATCH, dtype=torch.int32, device=self.device)
        return c

    def _launch(self, peer, reqs, stride, layer0, layer1, stream):
        """One rngd_kv_handoff_batch launch: reqs = [(lane, seq, k address, v address, tokens,
        *tensors the addresses point into), ...] (<= 16)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with self._lock:
            arr = self._items
            if arr is None:
                arr = self._items = (_lib.KvItem * _lib.KV_MAX_BATCH)()
            moved = 0
            for i, (lane, seq, k_ptr, v_ptr, tokens, *owners) in enumerate(reqs):
                tokens = peer.S if tokens is None else int(tokens)
                # the caller may drop its cache right after this call: keep the allocator from
                # handing the memory to other work before the handoff kernel on `s` has read it
                for t in owners:
                    t.record_stream(s)
                it = arr[i]
                it.src_k, it.src_v, it.lane, it.tokens, it.seq = k_ptr, v_ptr, lane, tokens, seq
                moved += (layer1 - layer0) * 2 * peer.NKV * tokens * peer.HD * 2
            args = (arr, len(reqs), stride, ctypes.c_void_p(peer.k), ctypes.c_void_p(peer.v), peer.L, peer.NKV,
                    peer.S, peer.HD, peer.Bcap, layer0, layer1, _lib.ptr(self._counter(s)),
                    ctypes.c_void_p(peer.flags), _lib.stream_handle(s))
            if torch.cuda.current_device() == self.device.index:
                _lib.call("rngd_kv_handoff_batch", *args)
            else:
                with torch.cuda.device(self.device):
                    _lib.call("rngd_kv_handoff_batch", *args)
        return moved

    def record(self, seconds, nbytes):
        """Log one transfer under rm-core's measurement names."""
        from rngd_pd.airm import Measurement
        tags = {"component": "rngd-pd", "kv_transport": self.name}
        self.measurements.append(Measurement("kv_transfer_ms", seconds * 1e3, dict(tags)).validate())
        self.measurements.append(Measurement("kv_transfer_gbps", nbytes / seconds / 1e9, dict(tags)).validate())

    # ------------------------------------------------ key -> bytes interface
    def push(self, key, buf):
        from rngd_pd.airm import TransportError
        raise TransportError("nvlink moves device KV (push_device / push_layer); host bytes go through shm")

    def pull(self, key, timeout=5.0):
        from rngd_pd.airm import TransportError
        raise TransportError("nvlink delivers into the receiver's bound cache (wait / lane_views), not bytes")

    def close(self):
        with self._lock:
            for p in self._peers.values():
                p.close()
            self._peers.clear()
        self.remote_leases.clear()
        self.leases.clear()
        if self._status_host is not None:
            _lib.lib.rngd_host_free(ctypes.c_void_p(self._status_host))
            self._status_host = self._status_dev = None
