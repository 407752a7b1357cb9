"""The cross-node `nixl-ucx` KV transport on the host (no GPU, no NIXL): the arena, the
reference's descriptor bytes (fixture made by the reference's own pack_desc), the store over a
fake NIXL fabric (READ between registered regions, a notification frees the sender's slot), the
transport and its rm-core adapter, and the connector handoff.  Mirrors the reference's
tests/test_kv_ucx.py."""
import ctypes
import json
import os
import sys
import threading
import time
import unittest
from unittest import mock

import numpy as np

from rngd_pd.connector import tcpkv, ucxkv
from rngd_pd.connector import transport as kv

from tests.test_connector import _handoff, _kv, bf16_trunc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ucx_desc.npz")


class Fabric:
    """Agents of one process; a READ copies bytes between their registered regions."""

    def __init__(self):
        self.agents = {}

    def agent(self, name, **kw):
        a = FakeAgent(self, name, **kw)
        self.agents[name] = a
        return a


class FakeXfer:
    def __init__(self, run, polls):
        self.run, self.polls, self.released = run, polls, False

    def release(self):
        self.released = True


class FakeAgent:
    def __init__(self, fabric, name, polls=1, final="DONE"):
        self.fabric, self.name, self.polls, self.final = fabric, name, polls, final
        self.regions, self.remotes, self.inbox = {}, set(), {}
        self.lock = threading.Lock()
        self.deregistered = 0

    def register_memory(self, descs, mem, backends):
        assert mem == "DRAM" and backends == ["UCX"]
        token = object()
        self.regions[token] = [(a, n) for a, n, _dev, _x in descs]
        return token

    def deregister_memory(self, reg, backends):
        del self.regions[reg]
        self.deregistered += 1

    def get_agent_metadata(self):
        return json.dumps({"name": self.name, "regions": len(self.regions)}).encode()

    def add_remote_agent(self, md):
        name = json.loads(bytes(md))["name"]
        self.remotes.add(name)
        return name.encode()

    def remove_remote_agent(self, name):
        self.remotes.discard(name)

    def get_xfer_descs(self, descs, mem):
        return list(descs)

    def _inside(self, a, n):
        return any(r <= a and a + n <= r + rn for regs in self.regions.values() for r, rn in regs)

    def initialize_xfer(self, op, local, remote, name, notif, backends):
        assert op == "READ" and len(local) == len(remote) == 1
        peer = self.fabric.agents[name]
        assert name == self.name or name in self.remotes, "READ from an agent never added"
        (la, n, _), (ra, rn, _) = local[0], remote[0]
        assert n == rn and self._inside(la, n) and peer._inside(ra, n), "READ outside registered memory"

        def run():
            if self.final == "DONE":
                ctypes.memmove(la, ra, n)
                with peer.lock:
                    peer.inbox.setdefault(self.name, []).append(bytes(notif))
            return self.final
        return FakeXfer(run, self.polls)

    def transfer(self, h):
        return "PROC"

    def check_xfer_state(self, h):
        h.polls -= 1
        return h.run() if h.polls <= 0 else "PROC"

    def get_new_notifs(self):
        with self.lock:
            out, self.inbox = self.inbox, {}
        return out


def _relay():
    srv = tcpkv.TcpKVServer(0, "127.0.0.1")
    srv.start()
    return srv, srv.wait_ready()


def _until(cond, t=5.0):
    end = time.monotonic() + t
    while time.monotonic() < end:
        if cond():
            return True
        time.sleep(0.01)
    return False


class PoolAndDescriptor(unittest.TestCase):
    def test_pages_in_ring_order(self):
        p = ucxkv.HostPool(8 * 4096)
        assert p.address % 4096 == 0
        a = p.take(100)                     # one page
        b = p.take(4097)                    # two pages
        self.assertEqual((a, b), ((0, 1), (4096, 2)))
        p.give(*a)
        self.assertEqual(p.take(1), (3 * 4096, 1))        # the cursor moves on, not back to page 0
        self.assertEqual(p.take(4 * 4096), (4 * 4096, 4))  # up to the end of the pool
        self.assertEqual(p.take(1), (0, 1))               # then round to the first free page
        self.assertEqual(p.free_bytes(), 0)
        with self.assertRaises(ValueError):
            p.take(9 * 4096)

    def test_freed_run_is_found_when_the_cursor_has_no_room(self):
        p = ucxkv.HostPool(4 * 4096)
        slots = [p.take(4096) for _ in range(4)]
        p.give(*slots[1])
        p.give(*slots[2])
        self.assertEqual(p.take(2 * 4096), (4096, 2))
        self.assertEqual(p.free_bytes(), 0)

    def test_take_waits_then_times_out(self):
        p = ucxkv.HostPool(4096)
        slot = p.take(4096)
        threading.Timer(0.1, lambda: p.give(*slot)).start()
        self.assertEqual(p.take(512, timeout=2.0), (0, 1))
        with self.assertRaises(TimeoutError):
            p.take(1024, timeout=0.05)

    def test_bytes_land_where_the_address_says(self):
        p = ucxkv.HostPool(2 * 4096)
        off, _ = p.take(10)
        p.view(off, 10)[:] = np.arange(10, dtype=np.uint8)
        raw = (ctypes.c_uint8 * 10).from_address(p.address + off)
        self.assertEqual(list(raw), list(range(10)))

    def test_descriptors_equal_the_reference(self):
        z = np.load(GOLDEN)
        for i in range(3):
            name, md_hex, addr, n, crc = json.loads(z[f"args{i}"].tobytes())
            md = bytes.fromhex(md_hex)
            self.assertEqual(ucxkv.pack_desc(name, md, addr, n, crc), z[f"desc{i}"].tobytes())
            self.assertEqual(ucxkv.unpack_desc(z[f"desc{i}"].tobytes()), (name, md, addr, n, crc))
        for bad in (b"", b"XXXX" + bytes(28), z["desc0"].tobytes()[:-1]):
            with self.assertRaises(IOError):
                ucxkv.unpack_desc(bad)


class Store(unittest.TestCase):
    def setUp(self):
        self.srv, self.port = _relay()
        self.fab = Fabric()
        self.ctl = tcpkv.TcpKVClient("127.0.0.1", self.port)
        self.tx = ucxkv.UcxKVStore(self.ctl, agent=self.fab.agent("prefill"), pool_bytes=1 << 20)
        self.rx = ucxkv.UcxKVStore(self.ctl, agent=self.fab.agent("decode", polls=3), pool_bytes=1 << 20)

    def tearDown(self):
        self.tx.close()
        self.rx.close()
        self.ctl.close()
        self.srv.stop()

    def test_round_trip_frees_the_source_slot(self):
        blob = os.urandom(300_000)
        self.tx.push("r/layer.0/k", blob)
        self.assertEqual(self.tx.pending(), ["r/layer.0/k"])
        self.assertEqual(bytes(self.rx.pull("r/layer.0/k", timeout=2)), blob)
        self.assertTrue(_until(lambda: not self.tx.pending()))
        self.assertEqual(self.tx.stats["freed"], 1)
        self.assertEqual(self.tx.outbox.pool.free_bytes(), 1 << 20)
        self.assertEqual(self.fab.agents["decode"].remotes, {"prefill"})
        with self.assertRaises(TimeoutError):
            self.rx.pull("r/layer.0/k", timeout=0.05)     # the descriptor was taken once

    def test_slots_in_flight_stay_intact(self):
        a, b = os.urandom(5000), os.urandom(7000)
        self.tx.push("a", a)
        self.tx.push("b", b)
        self.assertEqual(bytes(self.rx.pull("b")), b)
        self.assertEqual(bytes(self.rx.pull("a")), a)

    def test_concurrent_requests(self):
        blobs = {f"q{i}/layer.{j}/v": os.urandom(20_000 + 37 * i) for i in range(6) for j in range(4)}
        errs = []

        def worker(keys):
            try:
                for k in keys:
                    self.tx.push(k, blobs[k])
                for k in keys:
                    if bytes(self.rx.pull(k, timeout=5)) != blobs[k]:
                        errs.append(k)
            except Exception as e:   # noqa: BLE001 - reported below
                errs.append(repr(e))
        keys = sorted(blobs)
        ts = [threading.Thread(target=worker, args=(keys[i::6],)) for i in range(6)]
        [t.start() for t in ts]
        [t.join(30) for t in ts]
        self.assertEqual(errs, [])
        self.assertTrue(_until(lambda: not self.tx.pending()))

    def test_full_arena_waits_for_reads(self):
        small = ucxkv.UcxKVStore(self.ctl, agent=self.fab.agent("tiny"), pool_bytes=4096, xfer_timeout_s=5)
        try:
            small.push("one", b"1" * 3000)
            done = threading.Event()
            threading.Thread(target=lambda: (small.push("two", b"2" * 3000), done.set()), daemon=True).start()
            self.assertFalse(done.wait(0.2))                 # no room until "one" is read
            self.assertEqual(bytes(self.rx.pull("one")), b"1" * 3000)
            self.assertTrue(done.wait(5))
            self.assertEqual(bytes(self.rx.pull("two")), b"2" * 3000)
        finally:
            small.close()

    def test_failed_read_raises(self):
        bad = ucxkv.UcxKVStore(self.ctl, agent=self.fab.agent("broken", final="ERR"), pool_bytes=1 << 16)
        try:
            self.tx.push("x", b"abc")
            with self.assertRaises(IOError):
                bad.pull("x")
        finally:
            bad.close()

    def test_overwritten_source_fails_the_crc(self):
        self.tx.push("c", b"clean bytes")
        self.tx.outbox.pool.buf[0:5] = np.frombuffer(b"dirty", np.uint8)
        with self.assertRaises(IOError):
            self.rx.pull("c")

    def test_ttl_frees_unread_slots(self):
        self.tx.ttl_s = 0.0
        self.tx.push("old", b"x" * 100)
        self.assertTrue(_until(lambda: not self.tx.pending()))
        self.assertEqual(self.tx.stats["expired"], 1)

    def test_close_deregisters(self):
        self.tx.push("k", b"1")
        self.rx.pull("k")
        self.tx.close()
        self.rx.close()
        self.assertEqual(self.fab.agents["prefill"].deregistered, 1)
        self.assertEqual(self.fab.agents["decode"].deregistered, 1)
        self.assertEqual(self.fab.agents["decode"].remotes, set())


class _Env:
    def setUp(self):
        self.srv, self.port = _relay()
        self.fab = Fabric()
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
    def test_by_name_is_one_shared_instance(self):
        from rngd_pd import airm
        os.environ["AIRM_KV_TRANSPORT"] = "nixl-ucx"
        a, b = kv.select_transport(), kv.select_transport()
        self.assertIsInstance(a, airm.NixlUcxTransport)
        self.assertIs(a, b)
        self.assertEqual(a.handshake_metadata()["tcp"], f"127.0.0.1:{self.port}")

    def test_without_rm_core(self):
        with mock.patch.dict(sys.modules, {"rm_core": None}):
            t = kv.select_transport("nixl-ucx")
            self.assertIsInstance(t, kv.NixlUcxTransport)
        t2 = kv.make_transport("nixl-ucx")
        self.assertIsInstance(t2, kv.NixlUcxTransport)
        t2.close()

    def test_needs_an_address(self):
        os.environ.pop("AIRM_KV_TCP_ADDR")
        t = kv.NixlUcxTransport(agent=self.fab.agent("a"))
        with self.assertRaises(ValueError):
            t.push("k", b"x")
        t.close()

    def test_no_nixl_raises_never_falls_back(self):
        def boom(name):
            raise ImportError("no module named nixl")
        t = kv.NixlUcxTransport()
        try:
            with mock.patch.object(ucxkv, "make_agent", boom), self.assertRaises(RuntimeError):
                t.push("k", b"x")
        finally:
            t.close()

    def test_connector_handoff_bit_exact(self):
        pt = kv.NixlUcxTransport(agent=self.fab.agent("prefill"), pool_bytes=8 << 20)
        dt = kv.NixlUcxTransport(agent=self.fab.agent("decode"), pool_bytes=8 << 20)
        try:
            dk, dv = _handoff(pt, dt)
        finally:
            pt.close()
            dt.close()
        ck, cv = _kv(0)
        np.testing.assert_array_equal(dk, bf16_trunc(np.stack(ck)))
        np.testing.assert_array_equal(dv, bf16_trunc(np.stack(cv)))


class Adapter(_Env, unittest.TestCase):
    def test_payload_round_trip(self):
        from rngd_pd import airm
        t = airm.NixlUcxTransport(agent=self.fab.agent("solo"), pool_bytes=1 << 20)
        src = airm.MemoryTier("ucx-prefill", "host-dram", 1 << 30)
        dst = airm.MemoryTier("ucx-decode", "host-dram", 1 << 30)
        layout = airm.KVLayout(num_layers=2, num_kv_heads=2, head_dim=8, dtype="bf16")
        kv_in = np.random.default_rng(2).standard_normal((2, 2, 4, 2, 8)).astype(np.float32)
        plan = t.plan("q", src, dst, layout, layout, (0, 4))
        self.assertEqual(plan.detail["agent"], "solo")
        res = t.wait(t.submit(plan, kv=kv_in), timeout_s=5)
        self.assertTrue(res.ok)
        got = t.take(plan).reshape(kv_in.shape)
        np.testing.assert_array_equal(got.view(np.uint32), kv_in.view(np.uint32) >> 16 << 16)
        self.assertEqual(t.measurements[-1].tags["kv_transport"], "nixl-ucx")
        with self.assertRaises(airm.TransportError):
            t.plan("bad", airm.MemoryTier("gpu0", "device-hbm", 1 << 30), dst, layout, layout, (0, 4))
        t.close()
