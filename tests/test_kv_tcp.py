"""The cross-node `tcp` KV transport on the host (no GPU): the relay and its pooled client, the
reference's wire protocol byte for byte (a transcript recorded from the reference's own client
and server), the key -> bytes transport and its rm-core adapter, the registry, the connector's
tensor staging, and a two-process handoff.  Mirrors the reference's tests/test_kv_tcp.py and
tests/test_connector_tcp.py."""
import multiprocessing as mp
import os
import socket
import struct
import sys
import threading
import time
import unittest
from unittest import mock

import numpy as np
import pytest
import torch

from rngd_pd.connector import tcpkv
from rngd_pd.connector import transport as kv

from tests.test_connector import HD, NKV, NL, S, _handoff, _kv, bf16_trunc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tcp_transcript.npz")


def _server():
    srv = tcpkv.TcpKVServer(0, "127.0.0.1")
    srv.start()
    return srv, srv.wait_ready()


def _recv_n(s, n, timeout=10):
    s.settimeout(timeout)
    out = bytearray()
    while len(out) < n:
        d = s.recv(n - len(out))
        if not d:
            break
        out += d
    return bytes(out)


class RelayTests(unittest.TestCase):
    def setUp(self):
        self.srv, self.port = _server()
        self.c = tcpkv.TcpKVClient("127.0.0.1", self.port)

    def tearDown(self):
        self.c.close()
        self.srv.stop()

    def test_round_trip_is_byte_exact_and_taken_once(self):
        blob = np.random.default_rng(0).bytes(3 << 20)
        self.c.push("r/layer.0/k", blob)
        self.assertEqual(bytes(self.c.take("r/layer.0/k", timeout=1)), blob)
        with self.assertRaises(TimeoutError):
            self.c.take("r/layer.0/k", timeout=0.05)

    def test_push_accepts_any_contiguous_buffer(self):
        arr = np.arange(1000, dtype=np.uint16)
        self.c.push("arr", arr)                               # 2000 bytes, not 1000
        self.assertEqual(bytes(self.c.take("arr")), arr.tobytes())
        self.c.push("mv", memoryview(b"abc"))
        self.assertEqual(bytes(self.c.take("mv")), b"abc")

    def test_take_waits_for_a_later_push(self):
        got = {}
        t = threading.Thread(target=lambda: got.update(v=bytes(self.c.take("late", timeout=5))))
        t.start()
        time.sleep(0.2)
        other = tcpkv.TcpKVClient("127.0.0.1", self.port)
        other.push("late", b"xyz")
        other.close()
        t.join(5)
        self.assertEqual(got.get("v"), b"xyz")

    def test_connections_are_reused(self):
        for i in range(20):
            self.c.push(f"k{i}", b"a" * 1000)
            self.c.take(f"k{i}")
        self.assertEqual(self.c.connections(), 1)

    def test_concurrent_clients(self):
        blobs = {f"q{i}/layer.{j}/k": os.urandom(50_000) for i in range(8) for j in range(4)}
        errs = []

        def worker(keys):
            try:
                for k in keys:
                    self.c.push(k, blobs[k])
                for k in keys:
                    if bytes(self.c.take(k, timeout=5)) != blobs[k]:
                        errs.append(k)
            except Exception as e:                            # noqa: BLE001 - reported below
                errs.append(repr(e))
        keys = sorted(blobs)
        ts = [threading.Thread(target=worker, args=(keys[i::8],)) for i in range(8)]
        [t.start() for t in ts]
        [t.join(30) for t in ts]
        self.assertEqual(errs, [])
        st = self.c.stats()
        self.assertEqual((st["pushed"], st["taken"], st["keys"], st["crc_errors"]), (32, 32, 0, 0))

    def test_corrupt_push_is_rejected(self):
        s = socket.create_connection(("127.0.0.1", self.port))
        data = b"payload"
        s.sendall(b"P" + struct.pack("<i", 1) + b"k" + struct.pack("<qI", len(data), 12345) + data)
        self.assertEqual(_recv_n(s, 2), b"ER")
        s.close()
        self.assertEqual(self.c.stats()["crc_errors"], 1)
        with self.assertRaises(TimeoutError):
            self.c.take("k", timeout=0.05)

    def test_crc_off_is_unchecked(self):
        with mock.patch.dict(os.environ, {"AIRM_KV_TCP_CRC": "0"}):
            self.c.push("nocrc", b"data")
            self.assertEqual(bytes(self.c.take("nocrc")), b"data")

    def test_unknown_request_drops_only_that_connection(self):
        s = socket.create_connection(("127.0.0.1", self.port))
        s.sendall(b"Z")
        self.assertEqual(_recv_n(s, 1), b"")                  # closed by the relay
        s.close()
        self.c.push("still", b"up")
        self.assertEqual(bytes(self.c.take("still")), b"up")

    def test_expired_blobs_are_dropped(self):
        self.srv.ttl_s = 0.0
        self.c.push("old", b"x")
        time.sleep(1.2)                                       # the relay sweeps every 0.25 s
        self.assertEqual(self.c.stats()["expired"], 1)

    def test_port_in_use_fails_loud(self):
        srv = tcpkv.TcpKVServer(self.port, "127.0.0.1")
        srv.start()
        with self.assertRaises(RuntimeError):
            srv.wait_ready()

    def test_parse_addr(self):
        self.assertEqual(tcpkv.parse_addr("relay.ns.svc:6000"), ("relay.ns.svc", 6000))
        self.assertEqual(tcpkv.parse_addr("relay"), ("relay", 5577))
        self.assertEqual(tcpkv.parse_addr(" [::1]:7000 "), ("::1", 7000))
        self.assertEqual(tcpkv.parse_addr("[fe80::2]"), ("fe80::2", 5577))

    def test_connections_are_bounded_and_shared(self):
        c = tcpkv.TcpKVClient("127.0.0.1", self.port, max_connections=2)
        errs = []

        def worker(i):
            try:
                for j in range(10):
                    c.push(f"b{i}.{j}", bytes([i]) * 5000)
                    if bytes(c.take(f"b{i}.{j}")) != bytes([i]) * 5000:
                        errs.append((i, j))
            except Exception as e:                            # noqa: BLE001 - reported below
                errs.append(repr(e))
        ts = [threading.Thread(target=worker, args=(i,)) for i in range(6)]
        [t.start() for t in ts]
        [t.join(30) for t in ts]
        self.assertEqual(errs, [])
        self.assertLessEqual(c.connections(), 2)
        c.close()
        self.assertEqual(c.connections(), 0)

    def test_take_parked_before_the_push_gets_it_directly(self):
        results = []
        t = threading.Thread(target=lambda: results.append(bytes(self.c.take("direct", timeout=5))))
        t.start()
        time.sleep(0.2)
        other = tcpkv.TcpKVClient("127.0.0.1", self.port)
        other.push("direct", b"handed over")
        other.close()
        t.join(5)
        self.assertEqual(results, [b"handed over"])
        st = self.c.stats()
        self.assertEqual((st["pushed"], st["taken"], st["keys"]), (1, 1, 0))


class WireTranscript(unittest.TestCase):
    """The reference's relay protocol, pinned by bytes recorded from its own client and server
    (tests/golden/make_tcp_transcript.py)."""

    @classmethod
    def setUpClass(cls):
        z = np.load(GOLDEN)
        cls.g = {k: z[k].tobytes() for k in z.files}

    def setUp(self):
        self.srv, self.port = _server()

    def tearDown(self):
        self.srv.stop()

    def test_relay_replies_as_the_reference(self):
        for c2s, s2c in (("c2s", "s2c"), ("c2s_raw", "s2c_raw")):
            s = socket.create_connection(("127.0.0.1", self.port))
            s.sendall(self.g[c2s])
            got = _recv_n(s, len(self.g[s2c]))
            s.close()
            self.assertEqual(got, self.g[s2c], c2s)

    def test_client_sends_what_the_reference_sends(self):
        rec = _Recorder(("127.0.0.1", self.port))
        c = tcpkv.TcpKVClient("127.0.0.1", rec.port)
        with mock.patch.dict(os.environ, {"AIRM_KV_TCP_CRC": "1"}):
            c.push("r1/layer.0/k", self.g["blob_k"])
            c.push("r1/layer.0/v", self.g["blob_v"])
            self.assertEqual(bytes(c.take("r1/layer.0/k", timeout=1)), self.g["blob_k"])
            with self.assertRaises(TimeoutError):
                c.take("missing", timeout=0.05)
            c.stats()
            self.assertEqual(bytes(c.take("r1/layer.0/v", timeout=1)), self.g["blob_v"])
            c.stats()
        c.close()
        rec.done.wait(10)
        self.assertEqual(bytes(rec.c2s), self.g["c2s"])
        self.assertEqual(bytes(rec.s2c), self.g["s2c"])


class _Recorder:
    """A one-connection proxy that keeps the bytes of both directions."""

    def __init__(self, target):
        self.c2s, self.s2c = bytearray(), bytearray()
        self.done = threading.Event()
        self.lsock = socket.socket()
        self.lsock.bind(("127.0.0.1", 0))
        self.lsock.listen(1)
        self.port = self.lsock.getsockname()[1]
        threading.Thread(target=self._run, args=(target,), daemon=True).start()

    @staticmethod
    def _pump(a, b, log):
        while True:
            d = a.recv(1 << 16)
            if not d:
                b.shutdown(socket.SHUT_WR)
                return
            log += d
            b.sendall(d)

    def _run(self, target):
        c, _ = self.lsock.accept()
        s = socket.create_connection(target)
        t = threading.Thread(target=self._pump, args=(s, c, self.s2c), daemon=True)
        t.start()
        self._pump(c, s, self.c2s)
        t.join(10)
        c.close()
        s.close()
        self.lsock.close()
        self.done.set()


class TensorWire(unittest.TestCase):
    """ser_tensor / deser_into give the reference's wire bytes straight from torch tensors."""

    def _vals(self, shape=(NKV, S, HD)):
        v = np.random.default_rng(3).standard_normal(shape).astype(np.float32) * 4
        v.flat[:6] = [0.0, -0.0, 1e-30, 7e4, -3e38, np.inf]    # subnormal, fp16 overflow, large
        return bf16_trunc(v)

    def test_bf16_tensor_gives_the_same_bytes(self):
        v = self._vals()
        t = torch.from_numpy(v).to(torch.bfloat16)
        with np.errstate(over="ignore"):                      # 7e4 and 3e38 overflow fp16, as in ser()
            for wire in ("bf16", "fp16"):
                self.assertEqual(kv.ser_tensor(t, wire=wire), kv.ser(v, wire=wire), wire)

    def test_float32_tensor_gives_the_same_bytes(self):
        v = np.random.default_rng(4).standard_normal((3, 5, 7)).astype(np.float32)
        t = torch.from_numpy(v)
        for wire in ("bf16", "fp16"):
            self.assertEqual(kv.ser_tensor(t, wire=wire), kv.ser(v, wire=wire), wire)

    def test_module_wire_default_is_followed(self):
        v = self._vals((2, 3))
        t = torch.from_numpy(v).to(torch.bfloat16)
        with mock.patch.object(kv, "WIRE", "bf16"):
            self.assertEqual(kv.ser_tensor(t), kv.ser(v, wire="bf16"))
        self.assertEqual(kv.ser_tensor(t), kv.ser(v, wire="fp16"))

    def test_deser_into_matches_deser(self):
        v = self._vals()
        for wire in ("bf16", "fp16"):
            with np.errstate(over="ignore"):
                buf = kv.ser(v, wire=wire)
            ref = kv.deser(buf)
            for dt in (torch.bfloat16, torch.float32):
                dst = torch.zeros(v.shape, dtype=dt)
                kv.deser_into(buf, dst)
                np.testing.assert_array_equal(dst.float().numpy(), torch.from_numpy(ref).to(dt).float().numpy())
        with self.assertRaises(ValueError):
            kv.deser_into(kv.ser(v, wire="bf16"), torch.zeros(3, dtype=torch.bfloat16))


class _Env:
    def setUp(self):
        self.srv, self.port = _server()
        self.wire = kv.WIRE
        kv.WIRE = "bf16"
        kv._FENCED.clear()
        kv._CLASSES.clear()
        kv._SHARED.clear()
        self.env = mock.patch.dict(os.environ, {"AIRM_KV_TCP_ADDR": f"127.0.0.1:{self.port}"})
        self.env.start()
        os.environ.pop("AIRM_KV_TRANSPORT", None)

    def tearDown(self):
        self.env.stop()
        kv.WIRE = self.wire
        for t in list(kv._SHARED.values()):
            t.close()
        kv._FENCED.clear()
        kv._CLASSES.clear()
        kv._SHARED.clear()
        self.srv.stop()


class Selection(_Env, unittest.TestCase):
    def test_tcp_by_name_is_one_shared_instance(self):
        from rngd_pd import airm
        os.environ["AIRM_KV_TRANSPORT"] = "tcp"
        a, b = kv.select_transport(), kv.select_transport()
        self.assertIsInstance(a, airm.TcpTransport)
        self.assertIs(a, b)
        self.assertEqual(a.remote, ("127.0.0.1", self.port))
        self.assertEqual(a.handshake_metadata(), {"tcp": f"127.0.0.1:{self.port}"})

    def test_tcp_without_rm_core(self):
        with mock.patch.dict(sys.modules, {"rm_core": None}):
            self.assertIsInstance(kv.select_transport("tcp"), kv.TcpTransport)
        self.assertIsInstance(kv.make_transport("tcp"), kv.TcpTransport)

    def test_needs_an_address(self):
        os.environ.pop("AIRM_KV_TCP_ADDR")
        t = kv.TcpTransport()
        with self.assertRaises(ValueError):
            t.push("k", b"x")

    def test_serve_port_runs_a_relay_in_process(self):
        os.environ.pop("AIRM_KV_TCP_ADDR")
        t = kv.TcpTransport(serve_port=0)
        try:
            t.push("a", b"123")
            self.assertEqual(bytes(t.pull("a", timeout=1)), b"123")
            with self.assertRaises(TimeoutError):
                t.pull("a", timeout=0.05)
        finally:
            t.close()

    def test_connector_handoff_bit_exact(self):
        """prefill save -> relay -> decode load through the real connector, bf16 wire."""
        os.environ["AIRM_KV_TRANSPORT"] = "tcp"
        dk, dv = _handoff(kv.select_transport(), kv.select_transport())
        ck, cv = _kv(0)
        np.testing.assert_array_equal(dk, bf16_trunc(np.stack(ck)))
        np.testing.assert_array_equal(dv, bf16_trunc(np.stack(cv)))

    def test_connector_stages_tensors_as_raw_bf16(self):
        """Torch bf16 layers in, torch bf16 buffers out: the bits arrive unchanged."""
        from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
        t = kv.select_transport("tcp")
        ck, cv = _kv(5)
        tk = [torch.from_numpy(a).to(torch.bfloat16) for a in ck]
        tv = [torch.from_numpy(a).to(torch.bfloat16) for a in cv]
        pf = RngdKVConnector(KVConnectorRole.WORKER, req_id="rt", transport=t, n_layers=NL)
        for i in range(NL):
            pf.save_kv_layer(f"layer.{i}", (tk[i], tv[i]))
        dk = torch.zeros((NL, NKV, S, HD), dtype=torch.bfloat16)
        dv = torch.zeros_like(dk)
        dc = RngdKVConnector(KVConnectorRole.WORKER, req_id="rt", transport=t, n_layers=NL)
        dc.register_kv_caches((dk, dv))
        dc.start_load_kv()
        for i in range(NL):
            k, v = dc.wait_for_layer_load(f"layer.{i}")
            self.assertEqual(k.data_ptr(), dk[i].data_ptr())
        self.assertTrue(torch.equal(dk.view(torch.int16), torch.stack(tk).view(torch.int16)))
        self.assertTrue(torch.equal(dv.view(torch.int16), torch.stack(tv).view(torch.int16)))


class Adapter(_Env, unittest.TestCase):
    def test_payload_round_trip(self):
        from rngd_pd import airm
        t = airm.TcpTransport()
        src, dst, layout = t.conformance_case()
        kv_in = np.random.default_rng(1).standard_normal((2, 2, 4, 2, 8)).astype(np.float32)
        plan = t.plan("q", src, dst, layout, layout, (0, 4))
        self.assertEqual(plan.detail["server"], f"127.0.0.1:{self.port}")
        res = t.wait(t.submit(plan, kv=kv_in), timeout_s=5)
        self.assertTrue(res.ok)
        got = t.take(plan).reshape(kv_in.shape)
        np.testing.assert_array_equal(got.view(np.uint32), kv_in.view(np.uint32) >> 16 << 16)
        self.assertEqual(t.measurements[-1].tags["kv_transport"], "tcp")
        t.close()

    def test_own_relay_when_none_is_named(self):
        from rngd_pd import airm
        os.environ.pop("AIRM_KV_TCP_ADDR")
        t = airm.TcpTransport()
        src, dst, layout = t.conformance_case()
        self.assertIsNotNone(t.server)
        plan = t.plan("q2", src, dst, layout, layout, (0, 2))
        self.assertTrue(t.wait(t.submit(plan), timeout_s=5).ok)
        t.close()

    def test_rejects_device_tiers_and_timeouts_are_results(self):
        from rngd_pd import airm
        t = airm.TcpTransport()
        src, dst, layout = t.conformance_case()
        with self.assertRaises(airm.TransportError):
            t.plan("bad", airm.MemoryTier("gpu0", "device-hbm", 1 << 30), dst, layout, layout, (0, 4))
        plan = t.plan("q3", src, dst, layout, layout, (0, 4))
        h = t.submit(plan)
        t._relay().take(t.book.open[h.token].key, timeout=1)      # someone else took it
        res = t.wait(h, timeout_s=0.1)
        self.assertFalse(res.ok)
        t.close()


def _prefill_proc(port, q):
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rngd-pd_b200")]
    from rngd_pd.connector import transport as tr
    tr.WIRE = "bf16"
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    ck, cv = _kv(9)
    c = RngdKVConnector(KVConnectorRole.WORKER, req_id="xt", transport=tr.TcpTransport(remote=("127.0.0.1", port)),
                        n_layers=NL)
    for i in range(NL):
        c.save_kv_layer(f"layer.{i}", (ck[i], cv[i]))
    q.put("saved")


def test_two_process_tcp_handoff():
    """Prefill and decode as separate OS processes through a relay owned by the decode side,
    bit-exact on the bf16 wire (the reference's tests/test_connector_tcp.py)."""
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    srv, port = _server()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_prefill_proc, args=(port, q))
    p.start()
    try:
        dk = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
        dv = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
        dc = RngdKVConnector(KVConnectorRole.WORKER, req_id="xt",
                             transport=kv.TcpTransport(remote=("127.0.0.1", port)), n_layers=NL)
        dc.register_kv_caches((dk, dv))
        dc.start_load_kv()
        with mock.patch.dict(os.environ, {"PD_KV_PULL_TIMEOUT": "120"}):
            for i in range(NL):
                dc.wait_for_layer_load(f"layer.{i}")
        assert q.get(timeout=120) == "saved"
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
        srv.stop()
    ck, cv = _kv(9)
    np.testing.assert_array_equal(np.stack(dk), bf16_trunc(np.stack(ck)))
    np.testing.assert_array_equal(np.stack(dv), bf16_trunc(np.stack(cv)))


@pytest.mark.gpu
def test_device_tensors_stage_the_reference_wire_bytes():
    """A bf16 cache layer on the GPU gives the reference's wire bytes (raw bits on the bf16
    wire, the device's fp16 conversion on the fp16 wire), and wire bytes land in a device bf16
    buffer bit for bit."""
    v = np.random.default_rng(6).standard_normal((NKV, 512, HD)).astype(np.float32) * 3
    v.flat[:5] = [0.0, -0.0, 1e-30, 7e4, -3e38]
    v = bf16_trunc(v)
    t = torch.from_numpy(v).to(torch.bfloat16).cuda()
    with np.errstate(over="ignore"):
        for wire in ("bf16", "fp16"):
            assert kv.ser_tensor(t, wire=wire) == kv.ser(v, wire=wire), wire
    dst = torch.zeros_like(t)
    kv.deser_into(kv.ser(v, wire="bf16"), dst)
    assert torch.equal(dst.view(torch.int16), t.view(torch.int16))
