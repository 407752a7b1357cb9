"""ai-rm protocol v0.1 adapters for this build's KV paths (API of src/rngd_pd/airm.py:52-221).

  ShmTransport     the connector's /dev/shm path as an rm-core KVTransport (entry point
                   `airm.kv_transports` name `shm`): host-dram -> host-dram on one machine,
                   bf16/fp16 wire, plan / submit / wait / take (airm.py:137-221).
  TcpTransport     the cross-node relay path (name `tcp`, airm.py:224-271): host-dram ->
                   host-dram on any two machines through a TcpKVServer, CRC-checked.
  NixlUcxTransport cross-node through NIXL's UCX backend (name `nixl-ucx`, airm.py:274-318):
                   one-sided READ between registered host arenas, descriptors via the relay.
  NvlinkTransport  the new GPU -> GPU path (name `nvlink`): device-hbm -> device-hbm tiers,
                   payload moved by peer-to-peer stores into the decode cache (rngd_pd.nvlink).

rm-core's protocol types come from `rm_core` when it is installed, else from
rngd_pd._rmcore (a restatement of the same names).  The transports record rm-core's
`kv_transfer_ms` (nvlink also `kv_transfer_gbps`) measurements.  The serving metrics of the
reference module (airm.py:393-507) are here too: `summarize` turns per-request records into
rm-core-named figures (ttft_p90_ms, tpot_p90_ms, tok_s, kv_transfer_ms), `Window` keeps the
last requests a gateway served, and `serve_metrics` exposes them as airm_* gauges over HTTP.
The workload runner (airm.py:223-391, process launch) is outside this build.
"""
import collections
import os
import threading
import time
import uuid

import numpy as np

try:  # pragma: no cover - depends on the host
    from rm_core import (ContractError, KVLayout, Measurement, MemoryTier, TransferHandle, TransferPlan,
                         TransferResult, TransportError, prometheus_name)
    from rm_core.metrics import METRICS
except ImportError:
    from rngd_pd._rmcore import (METRICS, ContractError, KVLayout, Measurement, MemoryTier, TransferHandle,
                                 TransferPlan, TransferResult, TransportError, prometheus_name)

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


class NixlUcxTransport(_KeyedKV, _kv.NixlUcxTransport):
    """KV between two host-memory tiers on any two machines through NIXL's UCX backend
    (airm.py:274-318).  remote=(host, port) is the relay for the descriptors (default
    $AIRM_KV_TCP_ADDR), serve_port= also runs one here, agent= a NIXL agent (tests pass a fake),
    pool_bytes= the arena per side.  wait() READs the blob (CRC-checked) and keeps it for take()."""

    name = "nixl-ucx"
    SCOPE = "only host-dram -> host-dram"

    def __init__(self, remote=None, serve_port=None, agent=None, pool_bytes=None):
        _kv.NixlUcxTransport.__init__(self, remote=remote, serve_port=serve_port, agent=agent, pool_bytes=pool_bytes)
        self._held = {}
        self._init_kv()

    def supports(self, src, dst):
        return src.kind == "host-dram" and dst.kind == "host-dram" and src.name != dst.name

    def _detail(self):
        return {"server": "%s:%d" % self.remote if self.remote else None, "agent": self.store.name}

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
        _kv.NixlUcxTransport.close(self)


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


# ------------------------------------------------------------------ serving metrics
def _pct(vals, q):
    vals = [float(v) for v in vals if v is not None]
    return round(float(np.percentile(vals, q)), 1) if vals else None


def summarize(records, wall_s=None):
    """rm-core-named summary of per-request records (airm.py:400-422).

    A record holds ttft_ms, tpot_ms, out_tokens and, when the KV crossed between cards,
    kv_save_ms / kv_load_ms.  Records with an "error" are left out.  tok_s divides the
    generated tokens by wall_s, else by the span from the first start (t0) to the last end
    (t1); kv_transfer_ms is the median per-request handoff (save + load).  Figures without
    data are omitted."""
    recs = [r for r in records if r and "error" not in r]
    if not recs:
        return {}
    if wall_s is None and all("t0" in r and "t1" in r for r in recs):
        wall_s = max(r["t1"] for r in recs) - min(r["t0"] for r in recs)
    xfer = [(r.get("kv_save_ms") or 0.0) + (r.get("kv_load_ms") or 0.0) for r in recs
            if r.get("kv_save_ms") is not None or r.get("kv_load_ms") is not None]
    tokens = sum(r.get("out_tokens") or 0 for r in recs)
    out = {"ttft_p90_ms": _pct([r.get("ttft_ms") for r in recs], 90),
           "tpot_p90_ms": _pct([r.get("tpot_ms") for r in recs], 90),
           "tok_s": round(tokens / wall_s, 1) if wall_s else None,
           "kv_transfer_ms": _pct(xfer, 50)}
    return {k: v for k, v in out.items() if v is not None}


def measurements(summary, **tags):
    """Validated rm-core Measurements of a summarize() result (airm.py:425-432); the
    kv_transport tag stays on kv_transfer_ms only."""
    base = dict({"component": COMPONENT}, **tags)
    out = []
    for name, value in summary.items():
        t = dict(base)
        if name != "kv_transfer_ms":
            t.pop("kv_transport", None)
        out.append(Measurement(name, float(value), t).validate())
    return out


def prometheus_text(ms):
    """Prometheus exposition of measurements as gauges (airm.py:435-445)."""
    lines, typed = [], set()
    for m in ms:
        series = prometheus_name(m.name)
        if series not in typed:
            lines.append(f"# HELP {series} {METRICS[m.name][2]} ({m.unit})")
            lines.append(f"# TYPE {series} gauge")
            typed.add(series)
        labels = ",".join(f'{k}="{v}"' for k, v in sorted(m.tags.items()))
        lines.append(f"{series}{{{labels}}} {m.value:g}")
    return "\n".join(lines) + "\n"


class Window:
    """The last `size` requests a gateway served, as airm_* gauges (airm.py:448-485).

    TPOT is what a client sees, (wall - TTFT) / (tokens - 1), not the decode loop's median
    step: the wait for a lane and admission stalls count, so the gauge rises when the decode
    side saturates."""

    def __init__(self, size=512):
        self.recs = collections.deque(maxlen=size)
        self.lock = threading.Lock()

    def record(self, t0, t1, resp):
        pd = resp.get("pd", {}) if isinstance(resp, dict) else {}
        n = (resp.get("usage") or {}).get("completion_tokens", 0) if isinstance(resp, dict) else 0
        ttft = pd.get("ttft_ms")
        wall = (t1 - t0) * 1e3
        if isinstance(ttft, (int, float)) and n and n > 1:
            tpot = max(0.0, wall - ttft) / (n - 1)
        else:
            tpot = pd.get("tpot_ms")
        rec = {"t0": t0, "t1": t1, "ttft_ms": ttft, "tpot_ms": tpot, "out_tokens": n}
        if pd.get("mode") == "disaggregated-kv-transfer":
            rec.update(kv_save_ms=pd.get("kv_save_ms"), kv_load_ms=pd.get("kv_load_ms"))
        with self.lock:
            self.recs.append(rec)

    def observe(self, fn):
        """Wrap a route so every completed request is recorded."""
        def wrapped(body):
            t0 = time.perf_counter()
            resp = fn(body)
            self.record(t0, time.perf_counter(), resp)
            return resp
        return wrapped

    def summary(self):
        with self.lock:
            recs = list(self.recs)
        return summarize(recs)

    def text(self, kv_transport=None):
        kv = kv_transport or os.environ.get("AIRM_KV_TRANSPORT") or "shm"
        return prometheus_text(measurements(self.summary(), kv_transport=kv))


def serve_metrics(window, port, host="0.0.0.0"):
    """airm_* gauges of `window` on http://host:port/metrics from a daemon thread
    (airm.py:488-507); returns the server (server_address has the bound port)."""
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

    class _Metrics(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_GET(self):
            if self.path.rstrip("/") != "/metrics":
                self.send_response(404)
                self.end_headers()
                return
            body = window.text().encode()
            self.send_response(200)
            self.send_header("Content-Type", "text/plain; version=0.0.4")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

    srv = ThreadingHTTPServer((host, port), _Metrics)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv
