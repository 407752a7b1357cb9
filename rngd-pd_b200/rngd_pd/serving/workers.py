"""The worker glue around the connector for host-staged KV paths (shm, tcp, nixl-ucx): the
prefill side's per-group save and the decode side's load and prefetch
(the reference's FullPrefillWorker.run, serving/cluster.py:180-218, and DecodeWorkerBase,
serving/cluster.py:350-467), without the HTTP workers around them.

PrefillSaver.run(req_id, tokens) prefills the prompt one layer group at a time and hands each
group's layers to one ordered writer thread, which saves them through RngdKVConnector while
the next group computes.  On B200 the group stays on the device: K is turned into the
connector's layout [NKV, HD, S] on the engine's stream, an event orders the writer after it,
and the connector stages each bf16 layer as raw bits (2 bytes per element cross PCIe, no fp32
pass on the host).

KVLoader loads a request into one contiguous zeroed K [L, NKV, HD, S] / V [L, NKV, S, HD]
pair handed to the connector as per-layer views: float32 host arrays as in the reference, or
bf16 device tensors (device=...) that the connector fills in place from the wire bits, ready
for BatchDecodeEngine.adopt_kv_device / write_slot_kv.  The consumed shm files of the request
are removed.  prefetch(req_id) starts that load in the background as soon as the request is
announced (the reference's /prefetch), so decode finds it done; the map of prefetches is
bounded (PD_PREFETCH_CAP, 8) and entries older than PD_PREFETCH_TTL_S (900 s) are reclaimed.
"""
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector


class PrefillSaver:
    def __init__(self, engine, transport):
        """engine: a FullPrefillEngine (or anything with prefill_stream_device); transport: the
        connector's transport, or a callable returning one per request."""
        self.eng, self._transport = engine, transport
        self.nl, self.NG = engine.cfg.n_layers, engine.NG

    def _conn(self, req_id):
        t = self._transport() if callable(self._transport) else self._transport
        return RngdKVConnector(KVConnectorRole.WORKER, req_id=req_id, transport=t, n_layers=self.nl)

    def run(self, req_id, tokens):
        """Prefill `tokens`, saving every layer as its group finishes.  Returns the reference's
        record: next token, pos, layers, kv_mb (bf16), prefill_ms, bucket_C, save_ms, ms_per_token."""
        import torch
        conn = self._conn(req_id)
        stream = getattr(self.eng, "stream", None)
        writer = ThreadPoolExecutor(max_workers=1)            # one writer: saves stay in order
        pending, nbytes = [], [0]

        def save(g, k_t, v, ready):
            if ready is not None:
                ready.synchronize()
            for j in range(k_t.shape[0]):
                conn.save_kv_layer(f"layer.{g * self.NG + j}", (k_t[j], v[j]))

        def sink(g, kv_group):
            ready = None
            if stream is not None:
                with torch.cuda.stream(stream):
                    k_t = kv_group[:, 0].transpose(-1, -2).contiguous()     # [NG, NKV, HD, S]
                    v = kv_group[:, 1]
                    ready = torch.cuda.Event()
                    ready.record(stream)
            else:
                k_t, v = kv_group[:, 0].transpose(-1, -2).contiguous(), kv_group[:, 1]
            nbytes[0] += 2 * k_t.numel() * k_t.element_size()
            pending.append(writer.submit(save, g, k_t, v, ready))

        t0 = time.perf_counter()
        try:
            nxt = self.eng.prefill_stream_device(tokens, sink)
            prefill_ms = (time.perf_counter() - t0) * 1e3
            for f in pending:
                f.result()
            conn.wait_for_save()
        finally:
            writer.shutdown(wait=True)
        save_ms = max((time.perf_counter() - t0) * 1e3 - prefill_ms, 0.0)
        return {"next": int(nxt), "pos": len(tokens), "layers": self.nl, "kv_mb": round(nbytes[0] / 1e6, 1),
                "prefill_ms": round(prefill_ms, 1), "bucket_C": getattr(self.eng, "last_C", None),
                "save_ms": round(save_ms, 1), "ms_per_token": round(prefill_ms / max(len(tokens), 1), 3)}


class KVLoader:
    def __init__(self, transport, n_layers, n_kv, head_dim, S, device=None, shm_root=None):
        """transport: the connector's transport, or a callable returning one per request;
        device: None for float32 host arrays, else bf16 tensors on that CUDA device;
        shm_root: the shm directory whose files for a request are removed once it is loaded
        (default: the transport's `root`, when it has one)."""
        self._transport = transport
        self.nl, self.NKV, self.HD, self.S = n_layers, n_kv, head_dim, S
        self.device = device
        self.shm_root = shm_root
        self.cap = int(os.environ.get("PD_PREFETCH_CAP", "8"))
        self.ttl_s = float(os.environ.get("PD_PREFETCH_TTL_S", "900"))
        self._prefetch = {}                      # req_id -> (future, started)
        self._lock = threading.Lock()
        # one worker per prefetch the map can hold: a prefetch whose KV never arrives blocks its
        # own worker until the connector's pull timeout, never a later request's load
        self._pool = ThreadPoolExecutor(max_workers=max(1, self.cap), thread_name_prefix="kv-prefetch")

    def _buffers(self):
        kshape, vshape = (self.nl, self.NKV, self.HD, self.S), (self.nl, self.NKV, self.S, self.HD)
        if self.device is None:
            return np.zeros(kshape, np.float32), np.zeros(vshape, np.float32)
        import torch
        return (torch.zeros(kshape, dtype=torch.bfloat16, device=self.device),
                torch.zeros(vshape, dtype=torch.bfloat16, device=self.device))

    def load_now(self, req_id):
        """(K, V, load_ms): every layer of `req_id` pulled through the connector into zeroed
        buffers (a prompt shorter than S leaves the tail zero).  The wait per layer is the
        connector's ($PD_KV_PULL_TIMEOUT)."""
        t = self._transport() if callable(self._transport) else self._transport
        K, V = self._buffers()
        conn = RngdKVConnector(KVConnectorRole.WORKER, req_id=req_id, transport=t, n_layers=self.nl)
        conn.register_kv_caches(([K[i] for i in range(self.nl)], [V[i] for i in range(self.nl)]))
        conn.bind_connector_metadata(conn.build_connector_meta(None))
        t0 = time.perf_counter()
        conn.start_load_kv()
        for i in range(self.nl):
            conn.wait_for_layer_load(f"layer.{i}")
        load_ms = (time.perf_counter() - t0) * 1e3
        self._cleanup(req_id, t)
        return K, V, load_ms

    def _cleanup(self, req_id, transport):
        root = self.shm_root or getattr(transport, "root", None)
        if not root or not os.path.isdir(root):
            return
        prefix = req_id + "__"
        for f in os.listdir(root):
            if f.startswith(prefix):
                try:
                    os.unlink(os.path.join(root, f))
                except OSError:
                    pass

    def prefetch(self, req_id):
        """Start loading `req_id` in the background; a status dict as the reference's /prefetch."""
        with self._lock:
            if req_id in self._prefetch:
                return {"prefetch": "already running"}
            now = time.perf_counter()
            for old in [k for k, (_f, t0) in self._prefetch.items() if now - t0 > self.ttl_s]:
                # a queued load is cancelled; one already running cannot be stopped and ends
                # by itself (its result is dropped)
                self._prefetch.pop(old)[0].cancel()
            if len(self._prefetch) >= self.cap:
                return {"prefetch": "skipped (full)", "req_id": req_id}
            self._prefetch[req_id] = (self._pool.submit(self.load_now, req_id), now)
        return {"prefetch": "started", "req_id": req_id}

    def load(self, req_id, stream=None):
        """(K, V, load_ms, lead_ms): the prefetched load when one was started (lead_ms = how long
        before this call it began), else a load now (lead_ms = -1).

        Device buffers are filled on the loading thread, complete when this returns, and come
        from that thread's stream's memory pool.  Pass the stream that will read them (the decode
        engine's, for write_slot_kv / adopt_kv_device) as `stream`: they are then recorded on it,
        so dropping K and V right after queuing the copy cannot hand their memory to another
        load while the copy still reads it.  Without `stream`, keep K and V alive until that
        stream has consumed them."""
        with self._lock:
            entry = self._prefetch.pop(req_id, None)
        if entry is None:
            K, V, ms = self.load_now(req_id)
            lead = -1.0
        else:
            fut, t0 = entry
            K, V, ms = fut.result()
            lead = (time.perf_counter() - t0) * 1e3
        if stream is not None and self.device is not None and getattr(K, "is_cuda", False):
            K.record_stream(stream)
            V.record_stream(stream)
        return K, V, ms, lead

    def close(self):
        self._pool.shutdown(wait=False, cancel_futures=True)


__all__ = ["PrefillSaver", "KVLoader"]
