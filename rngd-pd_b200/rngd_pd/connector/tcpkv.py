"""Cross-node KV relay over TCP (the public names and wire protocol of the reference's
src/rngd_pd/connector/tcpkv.py: TcpKVServer, TcpKVClient, parse_addr, the relay CLI).

Where NVLink does not reach (prefill and decode on different nodes), each layer's wire bytes
are pushed to a relay, and the decode side takes them from it; neither side has to reach the
other directly.  The relay keeps a blob in host memory until one take hands it out or its
time to live passes.

    python -m rngd_pd.connector.tcpkv --port 5577     # a relay; standard library only

Wire (little-endian).  One connection carries any number of requests, one after another:

    push   b"P" klen:i32 key  n:i64 crc:u32 data   -> b"OK" | b"ER" (crc mismatch, blob dropped)
    take   b"W" klen:i32 key  wait_ms:i32          -> n:i64 crc:u32 data   (n = -1: absent after wait_ms)
    stats  b"S"                                    -> n:i64 json

crc is zlib.crc32 of the data.  The pusher computes it, the relay checks it on arrival and the
taker on delivery (0 = unchecked; AIRM_KV_TCP_CRC=0 stops computing it).  The protocol and the
stats JSON (its keys and their order) are shared with the reference's relay, so pods of either
build use one relay.

How this module is built: the relay keeps one mailbox per key (the blob, an event, the number
of takers waiting), so a push wakes only the takes of its own key, and a sweeper thread drops
blobs past their time to live.  Each connection has a thread of its own with blocking reads into
one preallocated buffer per blob; socket reads and zlib's CRC release the GIL, so several
connections move and check their blobs at once.  Requests are dispatched by their op byte
through a table, and an unknown op drops only its own connection.  The client keeps a
small bounded set of persistent connections, each with its own lock; a call takes whichever
connection is idle, opens another while fewer than `max_connections` exist, and otherwise
waits for one.  A request goes out as one scatter-gather send of header and payload, without
joining them in memory.
"""
import argparse
import json
import os
import socket
import struct
import threading
import time
import zlib

DEFAULT_PORT = 5577
_SIZE_CRC = struct.Struct("<qI")
_I32 = struct.Struct("<i")
_I64 = struct.Struct("<q")
_SOCK_BUF = 4 << 20
_STAT_KEYS = ("pushed", "taken", "expired", "crc_errors", "bytes_in", "bytes_out")


def crc_enabled():
    return os.environ.get("AIRM_KV_TCP_CRC", "1").strip().lower() not in ("0", "false", "no")


def _tune(sock):
    """No Nagle delay, and socket buffers large enough that a 1 MiB layer moves in few reads."""
    sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    for opt in (socket.SO_RCVBUF, socket.SO_SNDBUF):
        try:
            sock.setsockopt(socket.SOL_SOCKET, opt, _SOCK_BUF)
        except OSError:
            pass


# --------------------------------------------------------------------------------- relay
class _Mailbox:
    """One key's slot in the relay: the blob once pushed, an event its takers wait on, and how
    many takers are waiting."""
    __slots__ = ("entry", "filled", "takers")

    def __init__(self):
        self.entry = None                   # (data, crc, stored at)
        self.filled = threading.Event()
        self.takers = 0


class TcpKVServer(threading.Thread):
    """The relay: start(), wait_ready() -> bound port (port 0 picks a free one), stop().

    A blob nobody takes within ttl_s seconds ($AIRM_KV_TCP_TTL_S, default 900) is dropped, so a
    request that died between prefill and decode does not hold its cache.  `stats` counts
    pushed / taken / expired blobs, CRC errors and the bytes in and out."""

    SWEEP_S = 0.25

    def __init__(self, port, host="0.0.0.0", ttl_s=None):
        super().__init__(daemon=True, name=f"tcpkv-relay:{port}")
        self.host, self.port = host, int(port)
        self.ttl_s = float(ttl_s if ttl_s is not None else os.environ.get("AIRM_KV_TCP_TTL_S", "900"))
        self.stats = dict.fromkeys(_STAT_KEYS, 0)
        self._boxes = {}                    # key -> _Mailbox
        self._mu = threading.Lock()         # the mailbox table and the counters
        self._listener = None
        self._failure = None
        self._up = threading.Event()
        self._down = threading.Event()
        self._ops = {b"P": self._op_push, b"W": self._op_take, b"S": self._op_stats}

    # -- lifecycle ------------------------------------------------------------------------------
    def run(self):
        try:
            self._listener = socket.create_server((self.host, self.port), backlog=64)
        except OSError as e:
            self._failure = e
            self._up.set()
            return
        self.port = self._listener.getsockname()[1]
        self._up.set()
        threading.Thread(target=self._sweep, daemon=True, name="tcpkv-sweep").start()
        while not self._down.is_set():
            try:
                conn, _ = self._listener.accept()
            except OSError:
                break                       # stop() shut the listener down
            _tune(conn)
            threading.Thread(target=self._serve, args=(conn,), daemon=True, name="tcpkv-conn").start()

    def wait_ready(self, timeout=5.0):
        if not self._up.wait(timeout) or self._failure is not None:
            raise RuntimeError(f"TcpKVServer could not listen on {self.host}:{self.port}: {self._failure}")
        return self.port

    def stop(self):
        """Stop accepting; connections already open end when their clients close them."""
        self._down.set()
        if self._listener is not None:
            try:
                self._listener.shutdown(socket.SHUT_RDWR)
            except OSError:
                pass
            self._listener.close()

    def snapshot(self):
        """The stats reply's fields: counters, keys held and the bytes they hold."""
        with self._mu:
            held = [b.entry[0] for b in self._boxes.values() if b.entry is not None]
            return dict(self.stats, keys=len(held), bytes_held=sum(len(d) for d in held))

    # -- the store ------------------------------------------------------------------------------
    def _sweep(self):
        while not self._down.wait(self.SWEEP_S):
            cutoff = time.monotonic() - self.ttl_s
            with self._mu:
                for key, box in list(self._boxes.items()):
                    if box.entry is not None and box.entry[2] <= cutoff:
                        box.entry = None
                        box.filled.clear()
                        self.stats["expired"] += 1
                        if not box.takers:
                            del self._boxes[key]

    def _store(self, key, data, crc):
        with self._mu:
            box = self._boxes.get(key)
            if box is None:
                box = self._boxes[key] = _Mailbox()
            box.entry = (data, crc, time.monotonic())
            self.stats["pushed"] += 1
            self.stats["bytes_in"] += len(data)
            box.filled.set()

    def _claim(self, key, wait_s):
        """The blob under `key`, removed; waits up to wait_s for a push.  None if none came."""
        deadline = time.monotonic() + wait_s
        with self._mu:
            box = self._boxes.get(key)
            if box is None:
                box = self._boxes[key] = _Mailbox()
            box.takers += 1
        entry = None
        try:
            while True:
                with self._mu:
                    if box.entry is not None:
                        entry, box.entry = box.entry, None
                        box.filled.clear()
                        self.stats["taken"] += 1
                        self.stats["bytes_out"] += len(entry[0])
                        return entry
                left = deadline - time.monotonic()
                if left <= 0 or not box.filled.wait(left):
                    return None
        finally:
            with self._mu:
                box.takers -= 1
                if not box.takers and box.entry is None and self._boxes.get(key) is box:
                    del self._boxes[key]

    # -- one connection -------------------------------------------------------------------------
    def _op_push(self, conn):
        key = _recv_into_new(conn, _I32.unpack(_recv_into_new(conn, 4))[0]).decode()
        n, crc = _SIZE_CRC.unpack(_recv_into_new(conn, _SIZE_CRC.size))
        if n < 0:
            return False
        data = _recv_into_new(conn, n)
        if crc and zlib.crc32(data) != crc:
            with self._mu:
                self.stats["crc_errors"] += 1
            conn.sendall(b"ER")
        else:
            self._store(key, data, crc)
            conn.sendall(b"OK")
        return True

    def _op_take(self, conn):
        key = _recv_into_new(conn, _I32.unpack(_recv_into_new(conn, 4))[0]).decode()
        (wait_ms,) = _I32.unpack(_recv_into_new(conn, 4))
        entry = self._claim(key, max(0, wait_ms) / 1e3)
        if entry is None:
            conn.sendall(_SIZE_CRC.pack(-1, 0))
        else:
            _send_parts(conn, (_SIZE_CRC.pack(len(entry[0]), entry[1]), entry[0]))
        return True

    def _op_stats(self, conn):
        body = json.dumps(self.snapshot()).encode()
        _send_parts(conn, (_I64.pack(len(body)), body))
        return True

    def _serve(self, conn):
        try:
            while True:
                op = conn.recv(1)
                handler = self._ops.get(op)
                if handler is None or not handler(conn):
                    return                  # closed, or a request this relay does not know
        except (ConnectionError, OSError, ValueError, struct.error):
            return
        finally:
            conn.close()


# --------------------------------------------------------------------------------- client
def _send_parts(sock, parts):
    """Send every byte of `parts` (buffers) with scatter-gather sends."""
    views = [memoryview(p).cast("B") for p in parts if memoryview(p).nbytes]
    while views:
        sent = sock.sendmsg(views)
        while views and sent >= views[0].nbytes:
            sent -= views[0].nbytes
            views.pop(0)
        if sent:
            views[0] = views[0][sent:]


def _recv_into_new(sock, n):
    """Exactly n bytes from sock as a bytearray; ConnectionError if the peer closes first."""
    buf = bytearray(n)
    view, got = memoryview(buf), 0
    while got < n:
        k = sock.recv_into(view[got:])
        if not k:
            raise ConnectionError(f"relay closed the connection after {got} of {n} bytes")
        got += k
    return buf


class _Link:
    """One persistent connection to the relay and the lock that serialises its requests."""

    def __init__(self):
        self.lock = threading.Lock()
        self.sock = None


class TcpKVClient:
    """push / take / stats against one relay, thread-safe.

    Connections persist across calls (a fresh one per 1 MB layer would restart TCP slow start
    every time).  A call uses an idle connection, opens a new one while fewer than
    `max_connections` are open, else waits for the next to come free.  A connection whose
    state is unknown after an error is closed and reopened by its next user."""

    def __init__(self, host, port, connect_timeout=10.0, max_connections=8):
        self.addr = (host, int(port))
        self.connect_timeout = float(connect_timeout)
        self.max_connections = max(1, int(max_connections))
        self._links = []
        self._grow = threading.Lock()
        self._turn = 0

    def _acquire(self):
        for link in list(self._links):
            if link.lock.acquire(blocking=False):
                return link
        with self._grow:
            if len(self._links) < self.max_connections:
                link = _Link()
                link.lock.acquire()
                self._links.append(link)
                return link
            self._turn = (self._turn + 1) % len(self._links)
            link = self._links[self._turn]
        link.lock.acquire()
        return link

    def _exchange(self, request):
        link = self._acquire()
        try:
            if link.sock is None:
                s = socket.create_connection(self.addr, timeout=self.connect_timeout)
                s.settimeout(None)
                _tune(s)
                link.sock = s
            try:
                return request(link.sock)
            except BaseException:
                link.sock.close()
                link.sock = None
                raise
        finally:
            link.lock.release()

    def connections(self):
        """How many connections to the relay are open."""
        return sum(1 for link in list(self._links) if link.sock is not None)

    def push(self, key, data):
        """Store `data` (any contiguous buffer: bytes, bytearray, memoryview, numpy array)
        under `key`; IOError if the relay rejects it (its CRC did not match in transit)."""
        payload = memoryview(data).cast("B")
        kb = key.encode()
        crc = zlib.crc32(payload) if crc_enabled() else 0
        head = b"".join((b"P", _I32.pack(len(kb)), kb, _SIZE_CRC.pack(payload.nbytes, crc)))

        def request(sock):
            _send_parts(sock, (head, payload))
            reply = bytes(_recv_into_new(sock, 2))
            if reply != b"OK":
                raise IOError(f"tcpkv push {key}: the relay rejected the blob ({reply!r}: crc mismatch)")
        self._exchange(request)

    def take(self, key, timeout=5.0):
        """The blob pushed under `key` (a bytearray), waited for up to `timeout` s and removed
        from the relay.  TimeoutError if it never came, IOError if its CRC does not match."""
        kb = key.encode()
        head = b"".join((b"W", _I32.pack(len(kb)), kb, _I32.pack(max(0, int(timeout * 1e3)))))

        def request(sock):
            _send_parts(sock, (head,))
            n, crc = _SIZE_CRC.unpack(_recv_into_new(sock, _SIZE_CRC.size))
            return (None, 0) if n < 0 else (_recv_into_new(sock, n), crc)
        data, crc = self._exchange(request)
        if data is None:
            raise TimeoutError(f"pull timeout: {key}")
        if crc and crc_enabled() and zlib.crc32(data) != crc:
            raise IOError(f"tcpkv take {key}: crc mismatch on delivery")
        return data

    def stats(self):
        def request(sock):
            _send_parts(sock, (b"S",))
            (n,) = _I64.unpack(_recv_into_new(sock, _I64.size))
            return json.loads(bytes(_recv_into_new(sock, n)))
        return self._exchange(request)

    def close(self):
        for link in list(self._links):
            with link.lock:
                if link.sock is not None:
                    link.sock.close()
                    link.sock = None


def parse_addr(text, default_port=DEFAULT_PORT):
    """'host:port', 'host', '[v6 address]:port' or '[v6 address]' -> (host, port)."""
    text = text.strip()
    if text.startswith("["):
        host, _, rest = text[1:].partition("]")
        port = rest[1:] if rest.startswith(":") else ""
    elif text.count(":") == 1:
        host, port = text.split(":")
    else:
        host, port = text, ""
    return host, int(port) if port else int(default_port)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m rngd_pd.connector.tcpkv",
                                 description="KV relay: keeps each pushed blob until one take hands it out")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=int(os.environ.get("AIRM_KV_TCP_PORT", DEFAULT_PORT)))
    ap.add_argument("--ttl", type=float, default=None, help="seconds an untaken blob is kept (AIRM_KV_TCP_TTL_S)")
    ap.add_argument("--stats-every", type=float, default=60.0,
                    help="print the counters every N s when they changed (0: never)")
    opts = ap.parse_args(argv)
    relay = TcpKVServer(opts.port, opts.host, ttl_s=opts.ttl)
    relay.start()
    print(f"[tcpkv] relay on {opts.host}:{relay.wait_ready()}", flush=True)
    shown = None
    try:
        while relay.is_alive():
            relay.join(opts.stats_every or None)
            now = relay.snapshot()
            if opts.stats_every and now != shown:
                print(f"[tcpkv] {json.dumps(now)}", flush=True)
                shown = now
    except KeyboardInterrupt:
        relay.stop()


if __name__ == "__main__":
    main()
