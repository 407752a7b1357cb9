"""Cross-node KV relay over TCP (API and wire protocol of src/rngd_pd/connector/tcpkv.py).

Where NVLink does not reach (prefill and decode on different nodes) the KV cache is staged
through host memory and a relay: the prefill side pushes each layer's wire bytes to a
TcpKVServer, the decode side takes them, and neither has to reach the other directly.  The
relay holds a blob in host memory until one take hands it out (or its time-to-live passes).

    python -m rngd_pd.connector.tcpkv --port 5577     # a relay process, standard library only

Wire (little-endian; one connection carries any number of requests).  It is byte-for-byte the
reference's, so prefill and decode pods of either build share one relay:

    push   b"P" klen:i32 key  n:i64 crc:u32 data   -> b"OK" | b"ER" (crc mismatch, blob dropped)
    take   b"W" klen:i32 key  wait_ms:i32          -> n:i64 crc:u32 data   (n = -1: absent after wait_ms)
    stats  b"S"                                    -> n:i64 json

crc is zlib.crc32 of the data, computed by the pusher and checked by the relay on arrival and
by the taker on delivery (0 = unchecked; AIRM_KV_TCP_CRC=0 stops computing it), so a take
returns the pushed bytes or raises.
"""
import argparse
import json
import os
import queue
import socket
import socketserver
import struct
import threading
import time
import zlib

DEFAULT_PORT = 5577
_BLOB = struct.Struct("<qI")      # n, crc
_I32 = struct.Struct("<i")
_I64 = struct.Struct("<q")


def crc_enabled():
    return os.environ.get("AIRM_KV_TCP_CRC", "1") not in ("0", "false", "no")


def recv_exact(sock, n):
    """Exactly n bytes from sock into one bytearray, or ConnectionError if the peer closes."""
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = sock.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError(f"peer closed after {got} of {n} bytes")
        got += k
    return buf


def _nbytes(data):
    return memoryview(data).nbytes


class _Handler(socketserver.BaseRequestHandler):
    """One client connection: requests in order until the client closes or sends garbage."""

    def setup(self):
        self.request.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)

    def handle(self):
        relay, s = self.server.relay, self.request
        try:
            while True:
                op = s.recv(1)
                if not op:
                    return
                if op == b"S":
                    s.sendall(relay._stats_reply())
                    continue
                if op not in (b"P", b"W"):
                    return                                  # unknown request: drop the connection
                (klen,) = _I32.unpack(recv_exact(s, 4))
                if klen < 0:
                    return
                key = recv_exact(s, klen).decode()
                if op == b"P":
                    n, crc = _BLOB.unpack(recv_exact(s, _BLOB.size))
                    if n < 0:
                        return
                    s.sendall(b"OK" if relay._put(key, recv_exact(s, n), crc) else b"ER")
                else:
                    (wait_ms,) = _I32.unpack(recv_exact(s, 4))
                    entry = relay._take(key, max(0, wait_ms) / 1e3)
                    if entry is None:
                        s.sendall(_BLOB.pack(-1, 0))
                    else:
                        s.sendall(_BLOB.pack(len(entry[0]), entry[1]))
                        s.sendall(entry[0])
        except (ConnectionError, OSError):
            return


class _ThreadedServer(socketserver.ThreadingMixIn, socketserver.TCPServer):
    daemon_threads = True
    allow_reuse_address = True
    request_queue_size = 64

    def __init__(self, addr, relay):
        self.relay = relay
        super().__init__(addr, _Handler)

    def service_actions(self):          # once per poll of the accept loop
        self.relay._expire()


class TcpKVServer(threading.Thread):
    """In-memory key -> bytes relay behind a TCP port (tcpkv.py:50-152): start(), wait_ready()
    (returns the bound port; port 0 picks a free one), stop().  A blob nobody takes within
    ttl_s seconds ($AIRM_KV_TCP_TTL_S, default 900) is dropped, so a request that died between
    prefill and decode does not hold its cache forever.  `stats` counts pushed / taken /
    expired blobs, crc errors and bytes in and out."""

    def __init__(self, port, host="0.0.0.0", ttl_s=None):
        super().__init__(daemon=True, name=f"tcpkv:{port}")
        self.port, self.host = int(port), host
        self.ttl_s = float(ttl_s if ttl_s is not None else os.environ.get("AIRM_KV_TCP_TTL_S", "900"))
        self.store = {}                                     # key -> (data, crc, arrival time)
        self.cv = threading.Condition()
        self.stats = {"pushed": 0, "taken": 0, "expired": 0, "crc_errors": 0, "bytes_in": 0, "bytes_out": 0}
        self._srv = None
        self._error = None
        self._ready = threading.Event()

    def run(self):
        try:
            self._srv = _ThreadedServer((self.host, self.port), self)
        except OSError as e:
            self._error = e
            self._ready.set()
            return
        self.port = self._srv.server_address[1]
        self._ready.set()
        try:
            self._srv.serve_forever(poll_interval=0.25)
        finally:
            self._srv.server_close()

    def wait_ready(self, timeout=5.0):
        if not self._ready.wait(timeout) or self._error is not None:
            raise RuntimeError(f"TcpKVServer did not start on {self.host}:{self.port}: {self._error}")
        return self.port

    def stop(self):
        """Stop accepting and close the listening socket (open connections finish on their own)."""
        if self._srv is not None and self.is_alive():
            self._srv.shutdown()

    # -- the store, shared by the connection threads ------------------------------------------
    def _put(self, key, data, crc):
        if crc and zlib.crc32(data) != crc:
            with self.cv:
                self.stats["crc_errors"] += 1
            return False
        with self.cv:
            self.store[key] = (data, crc, time.monotonic())
            self.stats["pushed"] += 1
            self.stats["bytes_in"] += len(data)
            self.cv.notify_all()
        return True

    def _take(self, key, wait_s):
        deadline = time.monotonic() + wait_s
        with self.cv:
            while key not in self.store:
                left = deadline - time.monotonic()
                if left <= 0:
                    break
                self.cv.wait(left)
            entry = self.store.pop(key, None)
            if entry is not None:
                self.stats["taken"] += 1
                self.stats["bytes_out"] += len(entry[0])
        return entry

    def _expire(self):
        now = time.monotonic()
        with self.cv:
            old = [k for k, (_d, _c, t) in self.store.items() if now - t > self.ttl_s]
            for k in old:
                del self.store[k]
            self.stats["expired"] += len(old)

    def _stats_reply(self):
        with self.cv:
            snap = dict(self.stats, keys=len(self.store), bytes_held=sum(len(e[0]) for e in self.store.values()))
        body = json.dumps(snap).encode()
        return _I64.pack(len(body)) + body


class TcpKVClient:
    """push / take / stats against one TcpKVServer over a pool of persistent connections
    (tcpkv.py:155-230): a fresh connection per 1 MB layer would restart TCP slow start each
    time.  Thread-safe: every call borrows a connection of its own and returns it when done;
    a connection whose state is unknown after an error is closed, never reused."""

    def __init__(self, host, port, connect_timeout=10.0):
        self.addr = (host, int(port))
        self.connect_timeout = connect_timeout
        self._idle = queue.LifoQueue()

    def _checkout(self):
        try:
            return self._idle.get_nowait()
        except queue.Empty:
            s = socket.create_connection(self.addr, timeout=self.connect_timeout)
            s.settimeout(None)
            s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            return s

    def _call(self, fn):
        s = self._checkout()
        try:
            out = fn(s)
        except BaseException:
            s.close()
            raise
        self._idle.put(s)
        return out

    def push(self, key, data):
        """Store `data` (any contiguous buffer: bytes, bytearray, memoryview, numpy array) under
        `key`; IOError if the relay rejects it (crc mismatch in transit)."""
        kb = key.encode()
        n = _nbytes(data)
        crc = zlib.crc32(data) if crc_enabled() else 0

        def go(s):
            s.sendall(b"P" + _I32.pack(len(kb)) + kb + _BLOB.pack(n, crc))
            s.sendall(data)
            ack = bytes(recv_exact(s, 2))
            if ack != b"OK":
                raise IOError(f"tcpkv push {key}: relay rejected the blob ({ack!r}: crc mismatch)")
        self._call(go)

    def take(self, key, timeout=5.0):
        """The blob pushed under `key` (a bytearray), waiting up to `timeout` s for it, and removed
        from the relay; TimeoutError if it never came, IOError on a crc mismatch."""
        kb = key.encode()
        wait_ms = max(0, int(timeout * 1e3))

        def go(s):
            s.sendall(b"W" + _I32.pack(len(kb)) + kb + _I32.pack(wait_ms))
            n, crc = _BLOB.unpack(recv_exact(s, _BLOB.size))
            if n < 0:
                return None
            data = recv_exact(s, n)
            if crc and crc_enabled() and zlib.crc32(data) != crc:
                raise IOError(f"tcpkv take {key}: crc mismatch on delivery")
            return data
        data = self._call(go)
        if data is None:
            raise TimeoutError(f"pull timeout: {key}")
        return data

    def stats(self):
        def go(s):
            s.sendall(b"S")
            (n,) = _I64.unpack(recv_exact(s, 8))
            return json.loads(bytes(recv_exact(s, n)))
        return self._call(go)

    def close(self):
        while True:
            try:
                self._idle.get_nowait().close()
            except queue.Empty:
                return


def parse_addr(text, default_port=DEFAULT_PORT):
    """'host:port' or 'host' -> (host, port)."""
    text = text.strip()
    if ":" not in text:
        return text, int(default_port)
    host, _, port = text.rpartition(":")
    return host, int(port or default_port)


def main(argv=None):
    ap = argparse.ArgumentParser(description="KV relay: holds pushed KV blobs until one take hands each out")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=int(os.environ.get("AIRM_KV_TCP_PORT", str(DEFAULT_PORT))))
    ap.add_argument("--stats-every", type=float, default=60.0, help="print the counters every N s (0: never)")
    a = ap.parse_args(argv)
    srv = TcpKVServer(a.port, a.host)
    srv.start()
    print(f"[tcpkv] relay on {a.host}:{srv.wait_ready()}", flush=True)
    last = None
    try:
        while srv.is_alive():
            time.sleep(a.stats_every or 3600)
            if a.stats_every:
                with srv.cv:
                    snap = dict(srv.stats, keys=len(srv.store))
                if snap != last:
                    print(f"[tcpkv] {json.dumps(snap)}", flush=True)
                    last = snap
    except KeyboardInterrupt:
        srv.stop()


if __name__ == "__main__":
    main()
