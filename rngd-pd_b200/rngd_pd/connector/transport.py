"""KV transport abstraction for the connector (API of src/rngd_pd/connector/transport.py).

One interface, swappable backends, chosen by name:

  Transport (ABC): push(key, buf) / pull(key, timeout) / close()
    + the NIXL-parity handshake hooks handshake_metadata() / set_remote_handshake()
    ├─ InProcTransport   in-process dict (tests, single process)
    ├─ ShmTransport      /dev/shm files, atomic publish (cross-process, same host)
    ├─ TcpTransport      a TcpKVServer relay (rngd_pd.connector.tcpkv): cross-node, host-staged
    ├─ NixlUcxTransport  NIXL UCX one-sided READ between registered host arenas, descriptors
    │                    through the relay (rngd_pd.connector.ucxkv): cross-node, host-staged
    └─ NvlinkTransport   GPU -> GPU peer-to-peer stores over NVLink (rngd_pd.nvlink),
                         registered as `nvlink`; moves device KV with push_device()

`ser` / `deser` are byte-compatible with the reference's wire (fp16 default, `bf16` =
fp32 bits >> 16), so pods on the reference's code and on this build interoperate over
the same shm directory or TCP relay.  `ser_tensor` / `deser_into` give the same bytes
straight from and into torch tensors: a bf16 tensor on the bf16 wire crosses the bus as its
raw bits, with no fp32 pass on the host.  `select_transport(name)` resolves a name through rm-core's
`airm.kv_transports` entry points when rm-core is installed, else through this
package's own table; an unknown name raises KeyError, never a fallback.
"""
import os
import pickle
import threading
import time
from abc import ABC, abstractmethod

import numpy as np

WIRE = "fp16"


def ser(arr, wire=None):
    """Array -> wire bytes (connector/transport.py:29-37): pickled fp16, or a dict of
    bf16 bits (fp32 bits >> 16, exact for bf16-valued data)."""
    a = np.ascontiguousarray(arr)
    if (wire or WIRE) == "bf16":
        f = a if a.dtype == np.float32 else a.astype(np.float32)
        u = (f.view(np.uint32) >> 16).astype(np.uint16)
        return pickle.dumps({"bf16": u, "shape": a.shape}, protocol=4)
    return pickle.dumps(a.astype(np.float16), protocol=4)


def deser(buf):
    """Wire bytes -> float32 array (connector/transport.py:39-43)."""
    o = pickle.loads(buf)
    if isinstance(o, dict) and "bf16" in o:
        return (o["bf16"].astype(np.uint32) << 16).view(np.float32).reshape(o["shape"])
    return o.astype(np.float32)


def _host_view(t):
    """A contiguous torch tensor -> a numpy view of it in host memory (device tensors are copied
    into a pinned buffer first)."""
    import torch
    if t.is_cuda:
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h.numpy()
    return t.numpy()


def ser_tensor(t, wire=None):
    """A torch tensor (any device) -> the bytes ser(t.float().numpy(), wire) gives.  On the bf16
    wire a bf16 tensor is staged as its raw bits (2 bytes per element cross the bus); on the fp16
    wire the device converts (round to nearest even, as numpy's astype does from the exact fp32
    value); other cases go through ser()."""
    import torch
    w = wire or WIRE
    t = t.detach()
    if w == "bf16" and t.dtype == torch.bfloat16:
        bits = _host_view(t.contiguous().view(torch.int16)).view(np.uint16)
        return pickle.dumps({"bf16": bits, "shape": tuple(int(d) for d in t.shape)}, protocol=4)
    if w != "bf16" and t.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return pickle.dumps(_host_view(t.contiguous().to(torch.float16)), protocol=4)
    return ser(t.float().cpu().numpy(), wire=w)


def deser_into(buf, dst):
    """Wire bytes -> dst (a torch tensor, any device) in place; returns dst.  bf16 wire bytes into
    a bf16 tensor are copied as raw bits; everything else goes through deser()'s float32 values.
    ValueError if the element counts differ."""
    import torch
    o = pickle.loads(buf)
    if isinstance(o, dict) and "bf16" in o:
        bits = np.ascontiguousarray(o["bf16"]).reshape(-1)
        if bits.size != dst.numel():
            raise ValueError(f"wire holds {bits.size} elements, destination {tuple(dst.shape)}")
        if dst.dtype == torch.bfloat16:
            dst.view(torch.int16).copy_(torch.from_numpy(bits.view(np.int16)).view(dst.shape))
            return dst
        vals = (bits.astype(np.uint32) << 16).view(np.float32)
    else:
        vals = np.ascontiguousarray(o, dtype=np.float32).reshape(-1)
        if vals.size != dst.numel():
            raise ValueError(f"wire holds {vals.size} elements, destination {tuple(dst.shape)}")
    dst.copy_(torch.from_numpy(vals).view(dst.shape))
    return dst


class Transport(ABC):
    """Key -> bytes KV transport (connector/transport.py:46-60)."""

    @abstractmethod
    def push(self, key: str, buf: bytes) -> None: ...

    @abstractmethod
    def pull(self, key: str, timeout: float = 5.0) -> bytes: ...

    def close(self) -> None:
        pass

    def handshake_metadata(self) -> dict:
        """What a remote peer needs to reach us."""
        return {}

    def set_remote_handshake(self, meta: dict) -> None:
        """Register a remote peer's handshake metadata."""


class InProcTransport(Transport):
    """In-process shared dict (connector/transport.py:63-77)."""

    def __init__(self):
        self._store = {}
        self._lock = threading.Lock()

    def push(self, key, buf):
        with self._lock:
            self._store[key] = buf

    def pull(self, key, timeout=5.0):
        t0 = time.time()
        while True:
            with self._lock:
                if key in self._store:
                    return self._store[key]
            if time.time() - t0 > timeout:
                raise TimeoutError(f"pull timeout: {key}")
            time.sleep(0.001)

    def close(self):
        self._store.clear()


class ShmTransport(Transport):
    """/dev/shm file-backed store, cross-process on one host (connector/transport.py:80-101).
    Same file naming and atomic write-tmp-then-rename publish as the reference."""

    def __init__(self, root="/dev/shm/rngd_kv"):
        self.root = root
        os.makedirs(root, exist_ok=True)

    def _path(self, key):
        return os.path.join(self.root, key.replace("/", "__"))

    def push(self, key, buf):
        p = self._path(key)
        tmp = p + f".tmp.{os.getpid()}"
        with open(tmp, "wb") as f:
            f.write(buf)
            f.flush()
            os.fsync(f.fileno())
        os.rename(tmp, p)

    def pull(self, key, timeout=5.0):
        p = self._path(key)
        t0 = time.time()
        while not os.path.exists(p):
            if time.time() - t0 > timeout:
                raise TimeoutError(f"pull timeout: {key}")
            time.sleep(0.001)
        with open(p, "rb") as f:
            return f.read()


def _relay_endpoint(remote, serve_port):
    """(own relay or None, (host, port) or None, TcpKVClient or None) for a transport that talks
    to a TcpKVServer: remote, else $AIRM_KV_TCP_ADDR, else the relay started on serve_port."""
    from rngd_pd.connector.tcpkv import TcpKVClient, TcpKVServer, parse_addr
    server = None
    if serve_port is not None:
        server = TcpKVServer(serve_port)
        server.start()
        serve_port = server.wait_ready()
    if remote is None:
        env = os.environ.get("AIRM_KV_TCP_ADDR")
        if env:
            remote = parse_addr(env)
        elif serve_port is not None:
            remote = ("127.0.0.1", serve_port)
    remote = (remote[0], int(remote[1])) if remote else None
    return server, remote, (TcpKVClient(*remote) if remote else None)


def _audit_line(tag, op, key, buf, t0):
    import hashlib
    import sys
    line = (f"[{tag}] {op} {key} {memoryview(buf).nbytes} {hashlib.sha256(buf).hexdigest()[:16]} "
            f"{(time.perf_counter() - t0) * 1e3:.2f}ms\n")
    sys.stdout.write(line)      # one write per line: several threads may log
    sys.stdout.flush()


class TcpTransport(Transport):
    """Cross-node KV through one TcpKVServer relay (connector/transport.py:104-154).

    remote=(host, port) names the relay, default $AIRM_KV_TCP_ADDR ("host:port"); serve_port=
    also runs a relay in this process (0 = any free port), which is then the default remote.
    Prefill and decode name the same relay, beside the decode worker or on a third node.  The
    client pools persistent connections and every blob carries a CRC-32 checked by the relay and
    the taker, so a pull returns the pushed bytes or raises.  select_transport("tcp") gives one
    instance per process (`shared`).  AIRM_KV_TCP_LOG=1 prints one line per blob (key, bytes,
    sha256 prefix, ms) for byte-exact audits."""
    shared = True

    def __init__(self, remote=None, serve_port=None):
        self.server, self.remote, self._client = _relay_endpoint(remote, serve_port)

    def _relay(self):
        if self._client is None:
            raise ValueError("tcp transport needs remote=(host, port) or AIRM_KV_TCP_ADDR=host:port")
        return self._client

    def push(self, key, buf):
        t0 = time.perf_counter()
        self._relay().push(key, buf)
        self._audit("push", key, buf, t0)

    def pull(self, key, timeout=5.0):
        t0 = time.perf_counter()
        buf = self._relay().take(key, timeout=timeout)     # the relay waits for the key: no polling
        self._audit("pull", key, buf, t0)
        return buf

    @staticmethod
    def _audit(op, key, buf, t0):
        if os.environ.get("AIRM_KV_TCP_LOG", "0") not in ("0", ""):
            _audit_line("kv-tcp", op, key, buf, t0)

    def handshake_metadata(self):
        return {"tcp": "%s:%d" % self.remote} if self.remote else {}

    def close(self):
        if self._client is not None:
            self._client.close()
        if self.server is not None:
            self.server.stop()


class NixlUcxTransport(Transport):
    """Cross-node KV through NIXL's UCX backend (connector/transport.py:157-211; the store is
    rngd_pd.connector.ucxkv): push() stages the blob in this process's NIXL-registered arena
    and publishes a descriptor in the TcpKVServer at remote=(host, port) or $AIRM_KV_TCP_ADDR
    (descriptors only); pull() takes the descriptor and READs the bytes from the pushing
    process over UCX, so the pusher must stay up until the reader has read.  UCX_TLS picks the
    wire (tcp, or rc/ud verbs with an RDMA NIC).  CRC-32 per blob end to end; AIRM_KV_UCX_LOG=1
    prints size and SHA-256 per blob.  One shared instance per process (select_transport), so
    the agent, its registered arenas and the UCX endpoints outlive a request.  No NIXL raises."""
    shared = True

    def __init__(self, remote=None, serve_port=None, agent=None, pool_bytes=None):
        from rngd_pd.connector.ucxkv import UcxKVStore
        self.server, self.remote, self._client = _relay_endpoint(remote, serve_port)
        self.store = UcxKVStore(self._client, agent=agent, pool_bytes=pool_bytes)

    def _ready(self):
        if self._client is None:
            raise ValueError("nixl-ucx transport needs remote=(host, port) or AIRM_KV_TCP_ADDR=host:port "
                             "(a TcpKVServer for the descriptors)")
        return self.store

    def push(self, key, buf):
        t0 = time.perf_counter()
        self._ready().push(key, buf)
        self._audit("push", key, buf, t0)

    def pull(self, key, timeout=5.0):
        t0 = time.perf_counter()
        buf = self._ready().pull(key, timeout=timeout)
        self._audit("pull", key, buf, t0)
        return buf

    @staticmethod
    def _audit(op, key, buf, t0):
        if os.environ.get("AIRM_KV_UCX_LOG", "0") not in ("0", ""):
            _audit_line("kv-ucx", op, key, buf, t0)

    def handshake_metadata(self):
        out = dict(self.store.describe())
        if self.remote:
            out["tcp"] = "%s:%d" % self.remote
        return out

    def close(self):
        self.store.close()
        if self._client is not None:
            self._client.close()
        if self.server is not None:
            self.server.stop()


class FencedTransport(Transport):
    """Connector Transport over an rm-core tier-to-tier KVTransport (connector/transport.py:238-289):
    push() plans and submits one transfer per key; pull() waits on that transfer's completion
    fence and only then returns the bytes; a failed or missing fence raises."""

    def __init__(self, impl, src=None, dst=None):
        from rngd_pd.airm import KVLayout, MemoryTier
        self.impl = impl
        self.name = impl.name
        self.src = src or MemoryTier("prefill", "host-dram", 1 << 40)
        self.dst = dst or MemoryTier("decode", "host-dram", 1 << 40)
        self._layout = KVLayout(num_layers=1, num_kv_heads=1, head_dim=1, dtype="int8")
        self._pending = {}
        self._lock = threading.Lock()

    def push(self, key, buf):
        n = len(buf)
        plan = self.impl.plan(key, self.src, self.dst, self._layout, self._layout, (0, max(1, (n + 1) // 2)))
        with self._lock:
            if key in self._pending:
                raise ValueError(f"{self.name}: {key} pushed twice before it was pulled")
            self._pending[key] = None
        handle = self.impl.submit(plan)
        with self._lock:
            self._pending[key] = (handle, buf)

    def pull(self, key, timeout=5.0):
        from rngd_pd.airm import TransportError
        t0 = time.time()
        while True:
            with self._lock:
                entry = self._pending.get(key)
            if entry is not None:
                break
            if time.time() - t0 > timeout:
                raise TimeoutError(f"pull timeout: {key}")
            time.sleep(0.001)
        handle, buf = entry
        try:
            res = self.impl.wait(handle, timeout_s=max(0.0, timeout - (time.time() - t0)))
        finally:
            with self._lock:
                self._pending.pop(key, None)
        if not res.ok:
            raise TransportError(f"{self.name}: transfer {key} failed: {res.error}")
        return buf

    def close(self):
        with _LOCK:
            for k in [k for k, v in _FENCED.items() if v is self]:
                del _FENCED[k]
        self.impl.close()


# This package's own adapters, used when rm-core's registry is not installed or does not
# know the name.  The reference's rm-core `nixl` transport (rngd_pd.kv_nixl, an RDMA plugin
# absent here) resolves only through rm-core's registry when installed.
_OWN = {"shm": "rngd_pd.airm:ShmTransport", "tcp": "rngd_pd.airm:TcpTransport",
        "nixl-ucx": "rngd_pd.airm:NixlUcxTransport", "nvlink": "rngd_pd.airm:NvlinkTransport",
        "inproc": "rngd_pd.connector.transport:InProcTransport"}
_CLASSES = {}
_FENCED = {}
_SHARED = {}
_LOCK = threading.Lock()


def _own(name, kw):
    import importlib
    mod, obj = _OWN[name].split(":")
    cls = getattr(importlib.import_module(mod), obj)
    _CLASSES[name] = cls
    if name == "shm" and "root" not in kw:
        kw = dict(kw, root=os.environ.get("PD_SHM_ROOT") or None)
    return cls(**kw)


def _resolve(name, kw):
    """An instance of the implementation registered as `name` (connector/transport.py:302-327)."""
    if name in _CLASSES:
        return _own(name, kw) if name in _OWN else _CLASSES[name](**kw)
    try:
        from rm_core import registry
    except ImportError:
        if name in _OWN:
            return _own(name, kw)
        raise KeyError(f"AIRM_KV_TRANSPORT={name!r}: no transport of that name "
                       f"(this build provides {sorted(_OWN)}; others need rm-core installed)")
    try:
        impl = registry.load("airm.kv_transports", name, **kw)
    except KeyError:
        if name not in _OWN:
            raise
        impl = _own(name, kw)
    _CLASSES[name] = type(impl)
    return impl


def select_transport(name=None, **kw) -> Transport:
    """The connector's KV path chosen by name (connector/transport.py:330-350): name falls back
    to $AIRM_KV_TRANSPORT, then "shm".  A tier-to-tier KVTransport is wrapped in FencedTransport;
    instances marked `shared` are one per process.  Unknown names raise KeyError."""
    name = name or os.environ.get("AIRM_KV_TRANSPORT") or "shm"
    with _LOCK:
        if not kw and name in _FENCED:
            return _FENCED[name]
        if not kw and name in _SHARED:
            return _SHARED[name]
        impl = _resolve(name, kw)
        if isinstance(impl, Transport):
            if not kw and getattr(impl, "shared", False):
                _SHARED[name] = impl
            return impl
        t = FencedTransport(impl)
        if not kw:
            _FENCED[name] = t
        return t


def make_transport(backend="shm", **kw) -> Transport:
    """Factory (connector/transport.py:353-361): backend in {inproc, shm, tcp, nixl-ucx, nvlink}."""
    b = backend.lower()
    if b == "inproc":
        return InProcTransport()
    if b == "shm":
        return ShmTransport(**kw)
    if b == "tcp":
        return TcpTransport(**kw)
    if b == "nixl-ucx":
        return NixlUcxTransport(**kw)
    if b == "nvlink":
        from rngd_pd.nvlink import NvlinkTransport
        return NvlinkTransport(**kw)
    raise ValueError(f"unknown transport backend: {backend}")
