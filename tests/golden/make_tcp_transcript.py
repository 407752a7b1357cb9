"""Record the reference's TCP KV relay protocol as a byte transcript (run in the build container).

Imports the reference's own relay module (src/rngd_pd/connector/tcpkv.py: TcpKVServer and
TcpKVClient; nothing is copied into this repository), starts its server on a loopback port,
and drives its client through a recording proxy over one connection:

    push  r1/layer.0/k  (bf16 wire bytes of a seeded [2, 4, 8] array, ser from
                         src/rngd_pd/connector/transport.py)
    push  r1/layer.0/v  (seeded random bytes)
    take  r1/layer.0/k  timeout 1 s
    take  missing       timeout 0.05 s   (absent: n = -1)
    stats
    take  r1/layer.0/v  timeout 1 s
    stats

then, on a second raw connection, a push whose crc does not match (rejected with b"ER") and
stats.  The fixture holds both byte streams of each connection and the two blobs; the tests
replay the client streams against this build's relay and compare the replies, and compare the
bytes this build's client sends for the same calls.

    python tests/golden/make_tcp_transcript.py --reference <reference checkout>   (or $RNGD_REFERENCE)
"""
import argparse
import os
import socket
import struct
import sys
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class Recorder:
    """A one-connection TCP proxy that keeps every byte in both directions."""

    def __init__(self, target):
        self.target = target
        self.c2s, self.s2c = bytearray(), bytearray()
        self.lsock = socket.socket()
        self.lsock.bind(("127.0.0.1", 0))
        self.lsock.listen(1)
        self.port = self.lsock.getsockname()[1]
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _pump(self, a, b, log):
        while True:
            d = a.recv(1 << 16)
            if not d:
                b.shutdown(socket.SHUT_WR)
                return
            log += d
            b.sendall(d)

    def _run(self):
        c, _ = self.lsock.accept()
        s = socket.create_connection(self.target)
        t = threading.Thread(target=self._pump, args=(s, c, self.s2c), daemon=True)
        t.start()
        self._pump(c, s, self.c2s)
        t.join(10)
        c.close()
        s.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RNGD_REFERENCE"),
                    help="the reference project checkout (default $RNGD_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference <reference checkout> or set RNGD_REFERENCE")
    sys.path.insert(0, os.path.join(a.reference, "src"))
    from rngd_pd.connector import tcpkv
    from rngd_pd.connector.transport import ser
    assert os.path.abspath(tcpkv.__file__).startswith(os.path.abspath(a.reference)), tcpkv.__file__
    os.environ["AIRM_KV_TCP_CRC"] = "1"

    rng = np.random.default_rng(11)
    blob_k = ser(rng.standard_normal((2, 4, 8)).astype(np.float32), wire="bf16")
    blob_v = rng.integers(0, 256, 5000, dtype=np.uint8).tobytes()

    srv = tcpkv.TcpKVServer(0, "127.0.0.1")
    srv.start()
    port = srv.wait_ready()

    rec = Recorder(("127.0.0.1", port))
    c = tcpkv.TcpKVClient("127.0.0.1", rec.port)
    c.push("r1/layer.0/k", blob_k)
    c.push("r1/layer.0/v", blob_v)
    assert bytes(c.take("r1/layer.0/k", timeout=1)) == blob_k
    try:
        c.take("missing", timeout=0.05)
        raise AssertionError("take of a missing key returned")
    except TimeoutError:
        pass
    c.stats()
    assert bytes(c.take("r1/layer.0/v", timeout=1)) == blob_v
    c.stats()
    c.close()
    rec.thread.join(10)

    rec2 = Recorder(("127.0.0.1", port))
    s = socket.create_connection(("127.0.0.1", rec2.port))
    data = b"payload"
    s.sendall(b"P" + struct.pack("<i", 1) + b"k" + struct.pack("<qI", len(data), 12345) + data)
    assert s.recv(2) == b"ER"
    s.sendall(b"S")
    n = struct.unpack("<q", s.recv(8))[0]
    got = b""
    while len(got) < n:
        got += s.recv(n - len(got))
    s.close()
    rec2.thread.join(10)
    srv.stop()

    out = os.path.join(HERE, "tcp_transcript.npz")
    u8 = lambda b: np.frombuffer(bytes(b), np.uint8)  # noqa: E731
    np.savez_compressed(out, c2s=u8(rec.c2s), s2c=u8(rec.s2c), c2s_raw=u8(rec2.c2s), s2c_raw=u8(rec2.s2c),
                        blob_k=u8(blob_k), blob_v=u8(blob_v))
    print(f"wrote {out}: {len(rec.c2s)} + {len(rec.s2c)} bytes, raw {len(rec2.c2s)} + {len(rec2.s2c)}")


if __name__ == "__main__":
    main()
