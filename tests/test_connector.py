"""The KV connector and its transports on the host (no GPU): the reference's wire bytes,
the vLLM connector contract, the transport registry, the rm-core shm adapter, fenced
transports, and a two-process handoff.  Mirrors the reference's tests/test_airm.py and
tests/test_connector_tcp.py with shm in place of the absent rm-core / TCP relay."""
import multiprocessing as mp
import os
import tempfile
import unittest
from unittest import mock

import numpy as np
import pytest

NL, NKV, S, HD = 4, 8, 16, 128


def _kv(seed):
    rng = np.random.default_rng(seed)
    return ([rng.standard_normal((NKV, S, HD)).astype(np.float32) for _ in range(NL)],
            [rng.standard_normal((NKV, S, HD)).astype(np.float32) for _ in range(NL)])


def _handoff(pt, dt, req_id="r1"):
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    ck, cv = _kv(0)
    pf = RngdKVConnector(KVConnectorRole.WORKER, req_id=req_id, transport=pt, n_layers=NL)
    for i in range(NL):
        pf.save_kv_layer(f"layer.{i}", (ck[i], cv[i]))
    dk = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
    dv = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
    dc = RngdKVConnector(KVConnectorRole.WORKER, req_id=req_id, transport=dt, n_layers=NL)
    dc.register_kv_caches((dk, dv))
    dc.bind_connector_metadata(dc.build_connector_meta(None))
    dc.start_load_kv()
    for i in range(NL):
        dc.wait_for_layer_load(f"layer.{i}")
    return np.stack(dk), np.stack(dv)


bf16_trunc = lambda a: (a.view(np.uint32) >> 16 << 16).view(np.float32)


def test_wire_bytes_equal_the_reference(golden):
    from rngd_pd.connector import transport as tr
    arr = golden["wire/input"]
    for wire in ("bf16", "fp16"):
        buf = tr.ser(arr, wire=wire)
        assert buf == golden[f"wire/{wire}/bytes"].tobytes()
        np.testing.assert_array_equal(tr.deser(buf), golden[f"wire/{wire}/deser"])


def test_real_vllm_connector():
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    assert issubclass(RngdKVConnector, KVConnectorBase_V1)
    assert len(RngdKVConnector.__abstractmethods__) == 0
    c = RngdKVConnector(KVConnectorRole.WORKER, "rX", None, 3)
    assert isinstance(c, KVConnectorBase_V1) and c.req_id == "rX" and c.n_layers == 3
    meta = c.build_connector_meta(None)
    assert meta.load_layers == ["layer.0", "layer.1", "layer.2"] and meta.save_layers == meta.load_layers


class _Env:
    def setUp(self):
        from rngd_pd.connector import transport as tr
        self.tr = tr
        self.tmp = tempfile.TemporaryDirectory(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
        self.wire = tr.WIRE
        tr.WIRE = "bf16"
        tr._FENCED.clear(); tr._CLASSES.clear(); tr._SHARED.clear()
        self.env = mock.patch.dict(os.environ, {"PD_SHM_ROOT": self.tmp.name})
        self.env.start()
        os.environ.pop("AIRM_KV_TRANSPORT", None)

    def tearDown(self):
        self.env.stop()
        self.tr.WIRE = self.wire
        self.tr._FENCED.clear(); self.tr._CLASSES.clear(); self.tr._SHARED.clear()
        self.tmp.cleanup()


class Selection(_Env, unittest.TestCase):
    def test_inproc_handoff_bit_exact_under_bf16_wire(self):
        t = self.tr.InProcTransport()
        dk, dv = _handoff(t, t)
        ck, cv = _kv(0)
        np.testing.assert_array_equal(dk, bf16_trunc(np.stack(ck)))
        np.testing.assert_array_equal(dv, bf16_trunc(np.stack(cv)))

    def test_shm_is_default_and_reads_env_root(self):
        from rngd_pd import airm
        t = self.tr.select_transport()
        self.assertIsInstance(t, airm.ShmTransport)
        self.assertIsInstance(t, self.tr.ShmTransport)
        self.assertEqual(t.root, self.tmp.name)

    def test_env_selected_shm_gives_the_same_bytes(self):
        before = _handoff(self.tr.ShmTransport(self.tmp.name + "/legacy"), self.tr.ShmTransport(self.tmp.name + "/legacy"))
        os.environ["AIRM_KV_TRANSPORT"] = "shm"
        after = _handoff(None, None, req_id="r2")
        for a, b in zip(before, after):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        self.assertTrue(np.any(after[0]))

    def test_shm_files_readable_by_reference_naming(self):
        """The shm files use the reference's names (key with '/' -> '__') and raw wire bytes."""
        t = self.tr.select_transport("shm")
        t.push("req/layer.0/k", b"abc")
        with open(os.path.join(self.tmp.name, "req__layer.0__k"), "rb") as f:
            self.assertEqual(f.read(), b"abc")
        old = self.tr.ShmTransport(self.tmp.name)
        old.push("req/layer.0/v", b"xyz")
        self.assertEqual(t.pull("req/layer.0/v", timeout=1), b"xyz")

    def test_unknown_name_fails_loud(self):
        os.environ["AIRM_KV_TRANSPORT"] = "no-such-path"
        with self.assertRaises(KeyError):
            self.tr.select_transport()

    def test_nvlink_is_registered(self):
        self.assertIn("nvlink", self.tr._OWN)
        self.assertEqual(self.tr._OWN["nvlink"], "rngd_pd.airm:NvlinkTransport")

    def test_fenced_duplicate_push_and_failure(self):
        from rngd_pd import airm

        class Loop:
            name = "loopback"

            def __init__(self, fail=()):
                self.fail, self.n = set(fail), 0

            def plan(self, rid, src, dst, sl, dl, tokens):
                return airm.TransferPlan(rid, src, dst, sl, dl, tokens, 0)

            def submit(self, plan):
                return airm.TransferHandle(plan.request_id, self.name, plan.request_id)

            def wait(self, h, timeout_s):
                ok = h.request_id not in self.fail
                return airm.TransferResult(h.request_id, ok, 0, 0.0, None if ok else "injected failure")

            def close(self):
                pass

        t = self.tr.FencedTransport(Loop())
        t.push("k", b"ab")
        with self.assertRaises(ValueError):
            t.push("k", b"cd")
        self.assertEqual(t.pull("k", timeout=1), b"ab")
        f = self.tr.FencedTransport(Loop(fail=["req/layer.0/k"]))
        f.push("req/layer.0/k", b"abcd")
        with self.assertRaises(airm.TransportError):
            f.pull("req/layer.0/k", timeout=1)

    def test_pull_timeout(self):
        t = self.tr.InProcTransport()
        with self.assertRaises(TimeoutError):
            t.pull("nothing", timeout=0.05)


class AirmShm(_Env, unittest.TestCase):
    def _case(self):
        from rngd_pd import airm
        return (airm.MemoryTier("shm-prefill", "host-dram", 1 << 30), airm.MemoryTier("shm-decode", "host-dram", 1 << 30),
                airm.KVLayout(num_layers=2, num_kv_heads=2, head_dim=8, dtype="bf16"))

    def test_payload_round_trip(self):
        from rngd_pd import airm
        t = airm.ShmTransport()
        src, dst, layout = self._case()
        kv_in = np.random.default_rng(1).standard_normal((2, 2, 4, 2, 8)).astype(np.float32)
        plan = t.plan("q", src, dst, layout, layout, (0, 4))
        res = t.wait(t.submit(plan, kv=kv_in), timeout_s=5)
        self.assertTrue(res.ok)
        got = t.take(plan).reshape(kv_in.shape)
        np.testing.assert_array_equal(got.view(np.uint32), kv_in.view(np.uint32) >> 16 << 16)
        self.assertEqual(t.measurements[-1].tags["kv_transport"], "shm")
        t.close()

    def test_rejects_unsupported(self):
        from rngd_pd import airm
        t = airm.ShmTransport()
        src, dst, layout = self._case()
        dev = airm.MemoryTier("gpu0", "device-hbm", 1 << 30)
        for args in [(dev, dst, layout, layout, (0, 4)),
                     (src, dst, layout, airm.KVLayout(2, 2, 16, "bf16"), (0, 4)),
                     (src, dst, airm.KVLayout(2, 2, 8, "fp8"), airm.KVLayout(2, 2, 8, "fp8"), (0, 4)),
                     (src, dst, layout, layout, (3, 3))]:
            with self.assertRaises(airm.TransportError):
                t.plan("bad", *args)
        t.close()


def _prefill_proc(root, q):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rngd-pd_b200")]
    from rngd_pd.connector import transport as tr
    tr.WIRE = "bf16"
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    ck, cv = _kv(7)
    c = RngdKVConnector(KVConnectorRole.WORKER, req_id="xp", transport=tr.ShmTransport(root), n_layers=NL)
    for i in range(NL):
        c.save_kv_layer(f"layer.{i}", (ck[i], cv[i]))
    q.put("saved")


def test_two_process_shm_handoff(tmp_path):
    """Prefill and decode as separate OS processes (spawn), the bytes bit-exact (bf16 wire)."""
    from rngd_pd.connector import transport as tr
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_prefill_proc, args=(str(tmp_path), q))
    p.start()
    try:
        dk = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
        dv = [np.zeros((NKV, S, HD), np.float32) for _ in range(NL)]
        dc = RngdKVConnector(KVConnectorRole.WORKER, req_id="xp", transport=tr.ShmTransport(str(tmp_path)), n_layers=NL)
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
    ck, cv = _kv(7)
    np.testing.assert_array_equal(np.stack(dk), bf16_trunc(np.stack(ck)))
    np.testing.assert_array_equal(np.stack(dv), bf16_trunc(np.stack(cv)))
