"""KV transport abstraction for the connector (API of src/rngd_pd/connector/transport.py).

One interface, swappable backends, chosen by name:

  Transport (ABC): push(key, buf) / pull(key, timeout) / close()
    + the NIXL-parity handshake hooks handshake_metadata() / set_remote_handshake()
    ├─ InProcTransport   in-process dict (tests, single process)
    ├─ ShmTransport      /dev/shm files, atomic publish (cross-process, same host)
    └─ NvlinkTransport   GPU -> GPU peer-to-peer stores over NVLink (rngd_pd.nvlink),
                         registered as `nvlink`; moves device KV with push_device()

`ser` / `deser` are byte-compatible with the reference's wire (fp16 default, `bf16` =
fp32 bits >> 16), so pods on the reference's code and on this build interoperate over
the same shm directory.  `select_transport(name)` resolves a name through rm-core's
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
# know the name.  The reference's tcp / nixl / nixl-ucx transports are host-staging paths
# outside this build; they resolve only through rm-core's registry when installed.
_OWN = {"shm": "rngd_pd.airm:ShmTransport", "nvlink": "rngd_pd.airm:NvlinkTransport",
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
    """Factory (connector/transport.py:353-361): backend in {inproc, shm, nvlink}."""
    b = backend.lower()
    if b == "inproc":
        return InProcTransport()
    if b == "shm":
        return ShmTransport(**kw)
    if b == "nvlink":
        from rngd_pd.nvlink import NvlinkTransport
        return NvlinkTransport(**kw)
    raise ValueError(f"unknown transport backend: {backend}")
