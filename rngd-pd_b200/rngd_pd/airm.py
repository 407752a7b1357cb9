"""ai-rm protocol v0.1 adapters for this build's KV paths (API of src/rngd_pd/airm.py:52-221).

  ShmTransport     the connector's /dev/shm path as an rm-core KVTransport (entry point
                   `airm.kv_transports` name `shm`): host-dram -> host-dram on one machine,
                   bf16/fp16 wire, plan / submit / wait / take (airm.py:137-221).
  TcpTransport     the cross-node relay path (name `tcp`, airm.py:224-271): host-dram ->
                   host-dram on any two machines through a TcpKVServer, CRC-checked.
  NvlinkTransport  the new GPU -> GPU path (name `nvlink`): device-hbm -> device-hbm tiers,
                   payload moved by peer-to-peer stores into the decode cache (rngd_pd.nvlink).

rm-core's protocol types come from `rm_core` when it is installed, else from
rngd_pd._rmcore (a restatement of the same names).  The workload runner and the Prometheus
metrics of the reference module are outside this build; both transports record rm-core's
`kv_transfer_ms` (and nvlink also `kv_transfer_gbps`) measurements.
"""
import collections
import os
import threading
import time
import uuid

import numpy as np

try:  # pragma: no cover - depends on the host
    from rm_core import (ContractError, KVLayout, Measurement, MemoryTier, TransferHandle, TransferPlan,
                         TransferResult, TransportError)
except ImportError:
    from rngd_pd._rmcore import (ContractError, KVLayout, Measurement, MemoryTier, TransferHandle, TransferPlan,
                                 TransferResult, TransportError)

from rngd_pd import nvlink as _nv
from rngd_pd.connector import transport as _kv

COMPONENT = "rngd-pd"
WIRE_DTYPES = ("bf16", "fp16")
SHM_ROOT = "/dev/shm/rngd_kv_cluster"


class _KeyedKV:
    """rm-core KVTransport methods over a key -> bytes Transport (airm.py:57-134)."""

    def _init_kv(self):
        self._pending = {}
        self._delivered = {}
        self._lock = threading.Lock()
        self.measurements = collections.deque(maxlen=1024)

    def _sent(self, key):
        pass

    def plan(self, request_id, src, dst, src_layout, dst_layout, tokens):
        if not self.supports(src, dst):
            raise TransportError(f"{self.name}: {self.SCOPE}, not {src.kind}:{src.name} -> {dst.kind}:{dst.name}")
        src_layout.validate()
        dst_layout.validate()
        if src_layout != dst_layout:
            raise TransportError(f"{self.name}: src and dst layouts differ; convert in the model adapter")
        if src_layout.dtype not in WIRE_DTYPES:
            raise TransportError(f"{self.name}: wire carries {WIRE_DTYPES}, not {src_layout.dtype}")
        start, end = tokens
        if not 0 <= start < end:
            raise TransportError(f"{self.name}: bad token range {tokens}")
        return TransferPlan(request_id, src.validate(), dst.validate(), src_layout, dst_layout, (start, end),
                            (end - start) * src_layout.bytes_per_token(),
                            detail=dict(self._detail(), wire=src_layout.dtype))

    def submit(self, plan, kv=None):
        n = plan.nbytes // 2
        if kv is None:
            kv = np.zeros(n, np.float32)
        elif np.asarray(kv).size != n:
            raise ContractError(f"{self.name}: kv has {np.asarray(kv).size} elements, plan needs {n}")
        token = uuid.uuid4().hex
        key = f"{plan.request_id}/{plan.dst.name}/{plan.tokens[0]}-{plan.tokens[1]}.{token[:8]}"
        started = time.perf_counter()
        self.push(key, _kv.ser(np.asarray(kv, np.float32), wire=plan.detail.get("wire", "bf16")))
        with self._lock:
            self._pending[token] = (plan, key, started)
        self._sent(key)
        return TransferHandle(plan.request_id, self.name, token)

    def wait(self, handle, timeout_s):
        with self._lock:
            entry = self._pending.pop(handle.token, None)
        if entry is None:
            raise TransportError(f"{self.name}: unknown or already-waited handle {handle.token}")
        plan, key, started = entry
        try:
            got = _kv.deser(self._fetch(key, timeout_s)).size * 2
        except TimeoutError as e:
            return TransferResult(plan.request_id, False, 0, time.perf_counter() - started, str(e))
        seconds = time.perf_counter() - started
        if got != plan.nbytes:
            return TransferResult(plan.request_id, False, got, seconds,
                                  f"segment holds {got} bytes, plan moved {plan.nbytes}")
        self.measurements.append(Measurement("kv_transfer_ms", seconds * 1e3,
                                             {"component": COMPONENT, "kv_transport": self.name}).validate())
        with self._lock:
            self._delivered[(plan.request_id, plan.tokens)] = key
        return TransferResult(plan.request_id, True, plan.nbytes, seconds)

    def take(self, plan):
        with self._lock:
            key = self._delivered.pop((plan.request_id, plan.tokens), None)
        if key is None:
            raise TransportError(f"{self.name}: nothing delivered for {plan.request_id} {plan.tokens}")
        return _kv.deser(self._consume(key))


class ShmTransport(_KeyedKV, _kv.ShmTransport):
    """KV between two host-memory tiers on one machine through /dev/shm (airm.py:137-221).
    root defaults to $PD_SHM_ROOT, else /dev/shm/rngd_kv_cluster; created on first write."""

    name = "shm"
    SCOPE = "only host-dram -> host-dram on one machine"

    def __init__(self, root=None):
        self.root = str(root or os.environ.get("PD_SHM_ROOT") or SHM_ROOT)
        self._written = set()
        self._init_kv()

    def push(self, key, buf):
        os.makedirs(self.root, exist_ok=True)
        super().push(key, buf)

    def supports(self, src, dst):
        return src.kind == "host-dram" and dst.kind == "host-dram" and src.name != dst.name

    def _detail(self):
        return {"root": self.root}

    def _sent(self, key):
        with self._lock:
            self._written.add(key)

    def _fetch(self, key, timeout):
        return self.pull(key, timeout=timeout)

    def _consume(self, key):
        buf = self.pull(key, timeout=0)
        self._unlink(key)
        return buf

    def _unlink(self, key):
        try:
            os.unlink(self._path(key))
        except FileNotFoundError:
            pass
        with self._lock:
            self._written.discard(key)

    def close(self):
        with self._lock:
            keys, self._written = self._written, set()
            self._pending.clear()
            self._delivered.clear()
        for key in keys:
            self._unlink(key)


class TcpTransport(_KeyedKV, _kv.TcpTransport):
    """KV between two host-memory tiers on any two machines over TCP (airm.py:224-271).

    remote=(host, port) is the relay both sides use (default $AIRM_KV_TCP_ADDR); serve_port=
    also runs one in this process.  A host-staging path: KV leaves the card, crosses host memory
    and the network, and is uploaded on the other side.  The relay hands a blob out once, so
    wait() keeps the bytes it fetched (CRC-checked) for take()."""

    name = "tcp"
    SCOPE = "only host-dram -> host-dram"

    def __init__(self, remote=None, serve_port=None):
        _kv.TcpTransport.__init__(self, remote=remote, serve_port=serve_port)
        self._held = {}
        self._init_kv()

    def supports(self, src, dst):
        return src.kind == "host-dram" and dst.kind == "host-dram" and src.name != dst.name

    def _detail(self):
        return {"server": "%s:%d" % self.remote if self.remote else None}

    def _fetch(self, key, timeout):
        buf = self.pull(key, timeout=timeout)
        with self._lock:
            self._held[key] = buf
        return buf

    def _consume(self, key):
        with self._lock:
            return self._held.pop(key)

    def close(self):
        with self._lock:
            self._pending.clear()
            self._delivered.clear()
            self._held.clear()
        _kv.TcpTransport.close(self)

    def conformance_case(self):
        """Two host tiers and, when no relay is named, one on a free loopback port in this process."""
        if self.remote is None:
            _kv.TcpTransport.__init__(self, serve_port=0)
        return (MemoryTier("tcp-prefill", "host-dram", 1 << 30), MemoryTier("tcp-decode", "host-dram", 1 << 30),
                KVLayout(num_layers=2, num_kv_heads=2, head_dim=8, dtype="bf16"))


class NvlinkTransport(_nv.NvlinkTransport):
    """KV between two device-HBM tiers over NVLink: the rm-core protocol (plan / submit / wait /
    take) on top of everything rngd_pd.nvlink.NvlinkTransport offers."""

    SCOPE = "only device-hbm -> device-hbm (NVLink peer-to-peer)"

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self._handles = {}
        self._delivered_plans = {}

    def supports(self, src, dst):
        return src.kind == "device-hbm" and dst.kind == "device-hbm"

    def plan(self, request_id, src, dst, src_layout, dst_layout, tokens):
        if not self.supports(src, dst):
            raise TransportError(f"{self.name}: {self.SCOPE}, not {src.kind}:{src.name} -> {dst.kind}:{dst.name}")
        src_layout.validate()
        dst_layout.validate()
        if src_layout != dst_layout:
            raise TransportError(f"{self.name}: src and dst layouts differ")
        if src_layout.dtype != "bf16":
            raise TransportError(f"{self.name}: moves bf16 KV, not {src_layout.dtype}")
        start, end = tokens
        if not 0 <= start < end:
            raise TransportError(f"{self.name}: bad token range {tokens}")
        return TransferPlan(request_id, src.validate(), dst.validate(), src_layout, dst_layout, (start, end),
                            (end - start) * src_layout.bytes_per_token(), detail={"device": self.device.index})

    def submit(self, plan, kv=None):
        """kv: the request's device cache in the prefill layout [L][2][NKV][S][HD]."""
        import torch
        if kv is None or not torch.is_tensor(kv) or not kv.is_cuda:
            raise ContractError(f"{self.name}: submit needs the request's device KV tensor")
        s = torch.cuda.current_stream(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        moved = self.push_device(plan.request_id, kv, stream=s)
        e1.record(s)
        token = uuid.uuid4().hex
        with self._lock:
            self._handles[token] = (plan, e0, e1, moved)
        return TransferHandle(plan.request_id, self.name, token)

    def wait(self, handle, timeout_s=5.0, layer0=0, layer1=None, timeout=None):
        """rm-core form wait(handle, timeout_s) -> TransferResult; the receiver form
        wait(req_id, layer0, layer1, timeout) of the base class is kept for request ids."""
        if not isinstance(handle, TransferHandle):
            return super().wait(handle, layer0, layer1, timeout if timeout is not None else timeout_s)
        with self._lock:
            entry = self._handles.pop(handle.token, None)
        if entry is None:
            raise TransportError(f"{self.name}: unknown or already-waited handle {handle.token}")
        plan, e0, e1, moved = entry
        t0 = time.perf_counter()
        try:
            super().wait(plan.request_id, timeout=timeout_s)
        except TimeoutError as e:
            return TransferResult(plan.request_id, False, 0, time.perf_counter() - t0, str(e))
        e1.synchronize()
        seconds = e0.elapsed_time(e1) / 1e3
        self.record(seconds, moved)
        with self._lock:
            self._delivered_plans[(plan.request_id, plan.tokens)] = plan
        return TransferResult(plan.request_id, True, moved, seconds)

    def take(self, plan):
        with self._lock:
            p = self._delivered_plans.pop((plan.request_id, plan.tokens), None)
        if p is None:
            raise TransportError(f"{self.name}: nothing delivered for {plan.request_id} {plan.tokens}")
        return self.lane_views(plan.request_id)


def summarize_transfers(measurements):
    """Median kv_transfer_ms / kv_transfer_gbps of a transport's recorded measurements."""
    out = {}
    for name in ("kv_transfer_ms", "kv_transfer_gbps"):
        vals = [m.value for m in measurements if m.name == name]
        if vals:
            out[name] = float(np.median(vals))
    return out
