"""ai-rm protocol v0.1 adapters for this build's KV paths, and the serving metrics (the names of
the reference's src/rngd_pd/airm.py: ShmTransport, TcpTransport, NixlUcxTransport, summarize,
measurements, prometheus_text, Window, serve_metrics; plus NvlinkTransport).

Each adapter is at once a connector Transport (push / pull by key; select_transport() hands it
to the serving workers) and an rm-core KVTransport between two memory tiers (plan / submit /
wait / take), registered under `airm.kv_transports`:

  shm        host-dram -> host-dram on one machine, /dev/shm files published atomically
  tcp        host-dram -> host-dram on any two machines, through a TcpKVServer relay
  nixl-ucx   host-dram -> host-dram on any two machines, one-sided NIXL READ over UCX
  nvlink     device-hbm -> device-hbm, peer-to-peer stores into the decode cache (rngd_pd.nvlink)

How the host-staged adapters are built: `_HostStagedKV` holds the rm-core methods once, over a
`_TransferBook` (one lock; tickets by handle while submitted, then by (request, token range)
once delivered).  A transport supplies three hooks: `_publish(key, bytes)`, `_collect(key,
timeout)` (the delivered bytes, or TimeoutError / OSError) and `_discard(key)` (drop what the
transfer left behind, e.g. the shm file).  wait() keeps the collected bytes on the ticket, so
take() decodes them without a second read and every transport hands a blob out once.  Any
failure to collect is an ok=False result, never data and never a silent fallback.

rm-core's types come from `rm_core` when it is installed, else from rngd_pd._rmcore.  The
workload runner of the reference module (process launch) is outside this build.
"""
import collections
import os
import threading
import time
import uuid
from dataclasses import dataclass

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
WIRE_DTYPES = ("bf16", "fp16")          # the host wire moves 2-byte elements
SHM_ROOT = "/dev/shm/rngd_kv_cluster"


def _checked_plan(transport, request_id, src, dst, src_layout, dst_layout, tokens, dtypes, detail):
    """A TransferPlan for `tokens` of KV between two tiers, or TransportError naming what the
    transport cannot do."""
    who = transport.name
    if not transport.supports(src, dst):
        raise TransportError(f"{who} moves {transport.SCOPE}; asked for "
                             f"{src.kind}:{src.name} -> {dst.kind}:{dst.name}")
    for layout in (src_layout, dst_layout):
        layout.validate()
    if src_layout != dst_layout:
        raise TransportError(f"{who}: the two layouts differ ({src_layout} vs {dst_layout}); "
                             "the model adapter converts, the transport does not")
    if src_layout.dtype not in dtypes:
        raise TransportError(f"{who}: carries {'/'.join(dtypes)} KV, not {src_layout.dtype}")
    first, last = tokens
    if first < 0 or last <= first:
        raise TransportError(f"{who}: token range {tokens} is empty or negative")
    nbytes = (last - first) * src_layout.bytes_per_token()
    return TransferPlan(request_id, src.validate(), dst.validate(), src_layout, dst_layout, (first, last),
                        nbytes, detail=detail)


def _host_tiers(a, b):
    return a.kind == "host-dram" and b.kind == "host-dram" and a.name != b.name


@dataclass
class _Ticket:
    plan: object
    key: str
    started: float
    payload: object = None


class _TransferBook:
    """Tickets of one transport: by handle token until waited, then by (request id, token range)
    until taken."""

    def __init__(self):
        self.lock = threading.Lock()
        self.open = {}
        self.done = {}

    def add(self, ticket):
        token = uuid.uuid4().hex
        with self.lock:
            self.open[token] = ticket
        return token

    def close(self, token, name):
        with self.lock:
            ticket = self.open.pop(token, None)
        if ticket is None:
            raise TransportError(f"{name}: handle {token} is unknown or was waited already")
        return ticket

    def deliver(self, ticket):
        with self.lock:
            self.done[(ticket.plan.request_id, tuple(ticket.plan.tokens))] = ticket

    def claim(self, plan, name):
        with self.lock:
            ticket = self.done.pop((plan.request_id, tuple(plan.tokens)), None)
        if ticket is None:
            raise TransportError(f"{name}: no delivered transfer for {plan.request_id} tokens {plan.tokens}")
        return ticket

    def drain(self):
        with self.lock:
            tickets = list(self.open.values()) + list(self.done.values())
            self.open.clear()
            self.done.clear()
        return tickets


class _HostStagedKV:
    """rm-core KVTransport methods for a host-staged connector Transport (see the module
    docstring for the hooks a subclass supplies)."""

    SCOPE = "host-dram -> host-dram"

    def _init_rm(self):
        self.book = _TransferBook()
        self.measurements = collections.deque(maxlen=1024)

    def supports(self, src, dst):
        return _host_tiers(src, dst)

    def _detail(self):
        return {}

    def plan(self, request_id, src, dst, src_layout, dst_layout, tokens):
        return _checked_plan(self, request_id, src, dst, src_layout, dst_layout, tokens, WIRE_DTYPES,
                             dict(self._detail(), wire=src_layout.dtype))

    def submit(self, plan, kv=None):
        """Publish the plan's KV: an array of nbytes / 2 elements (zeros when omitted), sent on
        the plan's wire (bf16 or fp16)."""
        count = plan.nbytes // 2
        values = np.zeros(count, np.float32) if kv is None else np.asarray(kv, np.float32)
        if values.size != count:
            raise ContractError(f"{self.name}: the plan moves {count} elements, kv has {values.size}")
        stamp = uuid.uuid4().hex[:12]
        key = f"{plan.request_id}/{plan.dst.name}/t{plan.tokens[0]}-{plan.tokens[1]}/{stamp}"
        ticket = _Ticket(plan, key, time.perf_counter())
        self._publish(key, _kv.ser(values, wire=plan.detail.get("wire", "bf16")))
        return TransferHandle(plan.request_id, self.name, self.book.add(ticket))

    def wait(self, handle, timeout_s):
        ticket = self.book.close(handle.token, self.name)
        plan = ticket.plan
        try:
            blob = self._collect(ticket.key, timeout_s)
            values = _kv.deser(blob)
        except (TimeoutError, OSError, RuntimeError, ValueError) as e:
            self._discard(ticket.key)
            return TransferResult(plan.request_id, False, 0, time.perf_counter() - ticket.started, str(e))
        elapsed = time.perf_counter() - ticket.started
        moved = values.size * 2
        if moved != plan.nbytes:
            self._discard(ticket.key)
            return TransferResult(plan.request_id, False, moved, elapsed,
                                  f"{self.name}: the segment holds {moved} bytes, the plan {plan.nbytes}")
        ticket.payload = values
        self.book.deliver(ticket)
        self.measurements.append(Measurement("kv_transfer_ms", elapsed * 1e3,
                                             {"component": COMPONENT, "kv_transport": self.name}).validate())
        return TransferResult(plan.request_id, True, plan.nbytes, elapsed)

    def take(self, plan):
        """The delivered KV of `plan` as float32 values; it is gone afterwards."""
        ticket = self.book.claim(plan, self.name)
        self._discard(ticket.key)
        return ticket.payload

    def _forget_all(self):
        for ticket in self.book.drain():
            self._discard(ticket.key)

    def _discard(self, key):
        """Nothing is left behind once a relay or a READ has handed a blob out."""


class ShmTransport(_HostStagedKV, _kv.ShmTransport):
    """KV between two host tiers of one machine through files under `root` ($PD_SHM_ROOT, else
    /dev/shm/rngd_kv_cluster).  The directory is made on the first write, so constructing one
    touches nothing.  Prefill and decode must see the same directory (in k8s a hostPath
    /dev/shm on both pods)."""

    name = "shm"
    SCOPE = "host-dram -> host-dram on one machine"

    def __init__(self, root=None):
        self.root = str(root or os.environ.get("PD_SHM_ROOT") or SHM_ROOT)
        self._init_rm()

    def push(self, key, buf):
        os.makedirs(self.root, exist_ok=True)
        _kv.ShmTransport.push(self, key, buf)

    def _detail(self):
        return {"root": self.root}

    def _publish(self, key, blob):
        self.push(key, blob)

    def _collect(self, key, timeout):
        return self.pull(key, timeout=timeout)

    def _discard(self, key):
        try:
            os.unlink(self._path(key))
        except FileNotFoundError:
            pass

    def close(self):
        self._forget_all()

    def conformance_case(self):
        """Two host tiers in a private directory beside the serving root, so a conformance run
        never writes where live workers read."""
        parent = os.path.dirname(self.root.rstrip("/")) or "/dev/shm"
        self.root = os.path.join(parent, f"rngd_kv_conformance.{os.getuid()}.{os.getpid()}")
        os.makedirs(self.root, exist_ok=True)
        return (MemoryTier("shm-prefill", "host-dram", 1 << 30), MemoryTier("shm-decode", "host-dram", 1 << 30),
                KVLayout(num_layers=2, num_kv_heads=2, head_dim=8, dtype="bf16"))


class TcpTransport(_HostStagedKV, _kv.TcpTransport):
    """KV between two host tiers on any two machines through a TcpKVServer relay.

    remote=(host, port) is the relay both sides name (default $AIRM_KV_TCP_ADDR); serve_port=
    also runs one in this process.  Every blob carries a CRC-32 checked by the relay and by the
    taker, so wait() is ok only for the bytes submit() sent."""

    name = "tcp"

    def __init__(self, remote=None, serve_port=None):
        _kv.TcpTransport.__init__(self, remote=remote, serve_port=serve_port)
        self._init_rm()

    def _detail(self):
        return {"server": "%s:%d" % self.remote if self.remote else None}

    def _publish(self, key, blob):
        self.push(key, blob)

    def _collect(self, key, timeout):
        return self.pull(key, timeout=timeout)

    def close(self):
        self._forget_all()
        _kv.TcpTransport.close(self)

    def conformance_case(self):
        """Two host tiers, and a relay on a free loopback port here when none is named."""
        if self.remote is None:
            _kv.TcpTransport.__init__(self, serve_port=0)
        return (MemoryTier("tcp-prefill", "host-dram", 1 << 30), MemoryTier("tcp-decode", "host-dram", 1 << 30),
                KVLayout(num_layers=2, num_kv_heads=2, head_dim=8, dtype="bf16"))


class NixlUcxTransport(_HostStagedKV, _kv.NixlUcxTransport):
    """KV between two host tiers on any two machines through NIXL's UCX backend.

    remote=(host, port) is the relay for the descriptors (default $AIRM_KV_TCP_ADDR),
    serve_port= also runs one here, agent= a NIXL agent (tests pass a fake), pool_bytes= the
    registered pool per side.  A READ that fails, a CRC mismatch or a missing NIXL is ok=False."""

    name = "nixl-ucx"

    def __init__(self, remote=None, serve_port=None, agent=None, pool_bytes=None):
        _kv.NixlUcxTransport.__init__(self, remote=remote, serve_port=serve_port, agent=agent, pool_bytes=pool_bytes)
        self._init_rm()

    def _detail(self):
        return dict(self.store.describe(), server="%s:%d" % self.remote if self.remote else None)

    def _publish(self, key, blob):
        self.push(key, blob)

    def _collect(self, key, timeout):
        return self.pull(key, timeout=timeout)

    def close(self):
        self._forget_all()
        _kv.NixlUcxTransport.close(self)


class NvlinkTransport(_nv.NvlinkTransport):
    """KV between two device-HBM tiers over NVLink: the rm-core methods (plan / submit / wait /
    take) on top of everything rngd_pd.nvlink.NvlinkTransport offers."""

    SCOPE = "device-hbm -> device-hbm (NVLink peer-to-peer)"

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.book = _TransferBook()

    def supports(self, src, dst):
        return src.kind == "device-hbm" and dst.kind == "device-hbm"

    def plan(self, request_id, src, dst, src_layout, dst_layout, tokens):
        return _checked_plan(self, request_id, src, dst, src_layout, dst_layout, tokens, ("bf16",),
                             {"device": self.device.index})

    def submit(self, plan, kv=None):
        """kv: the request's device cache in the prefill layout [L][2][NKV][S][HD]."""
        import torch
        if kv is None or not torch.is_tensor(kv) or not kv.is_cuda:
            raise ContractError(f"{self.name}: submit needs the request's KV as a device tensor")
        stream = torch.cuda.current_stream(self.device)
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record(stream)
        moved = self.push_device(plan.request_id, kv, stream=stream)
        end.record(stream)
        return TransferHandle(plan.request_id, self.name,
                              self.book.add(_Ticket(plan, plan.request_id, 0.0, (begin, end, moved))))

    def wait(self, handle, timeout_s=5.0, layer0=0, layer1=None, timeout=None):
        """rm-core form wait(handle, timeout_s) -> TransferResult.  Given a request id instead of
        a handle it is the receiver's wait(req_id, layer0, layer1, timeout) of the base class."""
        if not isinstance(handle, TransferHandle):
            return super().wait(handle, layer0, layer1, timeout if timeout is not None else timeout_s)
        ticket = self.book.close(handle.token, self.name)
        begin, end, moved = ticket.payload
        t0 = time.perf_counter()
        try:
            super().wait(ticket.plan.request_id, timeout=timeout_s)
        except TimeoutError as e:
            return TransferResult(ticket.plan.request_id, False, 0, time.perf_counter() - t0, str(e))
        end.synchronize()
        seconds = begin.elapsed_time(end) / 1e3
        self.record(seconds, moved)
        self.book.deliver(ticket)
        return TransferResult(ticket.plan.request_id, True, moved, seconds)

    def take(self, plan):
        """The decode lane the transfer landed in, as (K, V) views."""
        self.book.claim(plan, self.name)
        return self.lane_views(plan.request_id)


def summarize_transfers(measurements):
    """Median kv_transfer_ms / kv_transfer_gbps of a transport's recorded measurements."""
    by_name = collections.defaultdict(list)
    for m in measurements:
        by_name[m.name].append(m.value)
    return {n: float(np.median(by_name[n])) for n in ("kv_transfer_ms", "kv_transfer_gbps") if by_name[n]}


# ------------------------------------------------------------------ serving metrics
def _quantile(values, q):
    """The q-th percentile of the non-missing values, to 0.1; None when there are none."""
    xs = np.asarray([v for v in values if v is not None], dtype=np.float64)
    return round(float(np.percentile(xs, q)), 1) if xs.size else None


def summarize(records, wall_s=None):
    """rm-core figures of finished requests: ttft_p90_ms, tpot_p90_ms, tok_s, kv_transfer_ms.

    A record holds ttft_ms, tpot_ms and out_tokens, t0 / t1 (start and end), and kv_save_ms /
    kv_load_ms when its KV crossed between cards.  Records with an "error" do not count.  tok_s
    is generated tokens over wall_s, or over first start -> last end when wall_s is not given;
    kv_transfer_ms is the median of save + load per request.  Figures without data are left out."""
    good = [r for r in records if r and "error" not in r]
    if not good:
        return {}
    if wall_s is None and all("t0" in r and "t1" in r for r in good):
        wall_s = max(r["t1"] for r in good) - min(r["t0"] for r in good)
    moved = [(r.get("kv_save_ms") or 0.0) + (r.get("kv_load_ms") or 0.0)
             for r in good if r.get("kv_save_ms") is not None or r.get("kv_load_ms") is not None]
    tokens = sum(r.get("out_tokens") or 0 for r in good)
    figures = {
        "ttft_p90_ms": _quantile((r.get("ttft_ms") for r in good), 90),
        "tpot_p90_ms": _quantile((r.get("tpot_ms") for r in good), 90),
        "tok_s": round(tokens / wall_s, 1) if wall_s else None,
        "kv_transfer_ms": _quantile(moved, 50),
    }
    return {name: v for name, v in figures.items() if v is not None}


def measurements(summary, **tags):
    """A summarize() result as validated rm-core Measurements.  The kv_transport tag belongs to
    kv_transfer_ms only."""
    common = {"component": COMPONENT, **tags}
    shared = {k: v for k, v in common.items() if k != "kv_transport"}
    return [Measurement(name, float(value), dict(common if name == "kv_transfer_ms" else shared)).validate()
            for name, value in summary.items()]


def prometheus_text(ms):
    """Measurements as Prometheus gauges: one HELP / TYPE header per series, then its samples."""
    series = collections.OrderedDict()
    for m in ms:
        series.setdefault(m.name, []).append(m)
    out = []
    for name, group in series.items():
        metric = prometheus_name(name)
        out += [f"# HELP {metric} {METRICS[name][2]} ({group[0].unit})", f"# TYPE {metric} gauge"]
        for m in group:
            labels = ",".join('%s="%s"' % kv for kv in sorted(m.tags.items()))
            out.append(f"{metric}{{{labels}}} {m.value:g}")
    return "\n".join(out) + "\n"


class Window:
    """The last `size` requests a gateway answered, kept as summarize() records.

    Its TPOT is the one a client sees, (wall time - TTFT) / (tokens - 1), not the decode loop's
    median step: waiting for a lane and admission stalls are in it, so it rises when the decode
    side saturates (a rebalancer reads this gauge)."""

    def __init__(self, size=512):
        self.recs = collections.deque(maxlen=size)
        self.lock = threading.Lock()

    def record(self, t0, t1, resp):
        resp = resp if isinstance(resp, dict) else {}
        pd = resp.get("pd") or {}
        n = (resp.get("usage") or {}).get("completion_tokens") or 0
        ttft = pd.get("ttft_ms")
        rec = {"t0": t0, "t1": t1, "ttft_ms": ttft, "out_tokens": n, "tpot_ms": pd.get("tpot_ms")}
        if n > 1 and isinstance(ttft, (int, float)):
            rec["tpot_ms"] = max(0.0, (t1 - t0) * 1e3 - ttft) / (n - 1)
        if pd.get("mode") == "disaggregated-kv-transfer":
            rec["kv_save_ms"], rec["kv_load_ms"] = pd.get("kv_save_ms"), pd.get("kv_load_ms")
        with self.lock:
            self.recs.append(rec)

    def observe(self, route):
        """`route` wrapped so that every request it answers is recorded."""
        def recorded(body):
            start = time.perf_counter()
            answer = route(body)
            self.record(start, time.perf_counter(), answer)
            return answer
        return recorded

    def summary(self):
        with self.lock:
            snapshot = list(self.recs)
        return summarize(snapshot)

    def text(self, kv_transport=None):
        transport = kv_transport or os.environ.get("AIRM_KV_TRANSPORT") or "shm"
        return prometheus_text(measurements(self.summary(), kv_transport=transport))


def serve_metrics(window, port, host="0.0.0.0"):
    """Serve `window` as airm_* gauges at http://host:port/metrics from a daemon thread; returns
    the server (its server_address carries the bound port; shutdown() stops it)."""
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

    class MetricsPage(BaseHTTPRequestHandler):
        def log_message(self, *args):
            pass

        def do_GET(self):
            found = self.path.split("?")[0].rstrip("/") == "/metrics"
            body = window.text().encode() if found else b"not found\n"
            self.send_response(200 if found else 404)
            self.send_header("Content-Type", "text/plain; version=0.0.4")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

    server = ThreadingHTTPServer((host, port), MetricsPage)
    server.daemon_threads = True
    threading.Thread(target=server.serve_forever, daemon=True, name="airm-metrics").start()
    return server
