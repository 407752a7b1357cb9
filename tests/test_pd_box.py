"""Prefill/decode splits in one process (serving/pd.py build_pd, PrefillPool and the pooled
NvlinkProducer) on the host: fake engines and a fake transport that writes the pushed cache
into the leased lane.  Every request gets its solo tokens whichever prefill and decode GPU
served it; a prefill engine never runs two prompts at once; 2P:6D shares the prefill GPUs,
P = D pairs them."""
import threading
import time

import pytest

from rngd_pd.serving.pd import build_pd, parse_split
from rngd_pd.serving.scheduler import PrefillPool
from tests.test_scheduler import GROUPS, S, FakeDecode, _alone, _prefill, _requests


class Dev:
    def __init__(self, index):
        self.index = index


class FakePrefill:
    def __init__(self, gpu):
        self.dev, self.stream = Dev(gpu), None
        self.busy, self.overlaps, self.calls = False, 0, 0

    def prefill_kv_device(self, tokens):
        if self.busy:
            self.overlaps += 1
        self.busy = True
        self.calls += 1
        time.sleep(0.002)
        K, V, first = _prefill(tokens)
        self.busy = False
        return (K, V), first


class FakeDecodeGPU(FakeDecode):
    def __init__(self, B, gpu):
        super().__init__(B)
        self.dev = Dev(gpu)

    def full_kv(self, Kd, Vd):
        return Kd, Vd


class FakeLink:
    """Receiver and sender in one class: a push writes rows [0, S - 1) of the leased lane."""

    def __init__(self, dev):
        self.dev, self.cache, self.leases, self.arrived, self.sent = dev, None, {}, set(), {}
        self.lock = threading.Lock()

    def bind_cache(self, Kd, Vd):
        self.cache = (Kd, Vd)

    def handshake_metadata(self):
        return {"rx": self}

    def set_remote_handshake(self, meta):
        return meta["rx"]

    def reserve(self, req, lane, sender_device=None):
        with self.lock:
            assert lane not in self.leases.values(), "lane leased twice"
            self.leases[req] = lane
        return {"req": req, "lane": lane}

    def add_lease(self, peer, ticket):
        self.sent[ticket["req"]] = (peer, ticket["lane"])

    def push_device(self, req, kv, stream=None, tokens=None):
        peer, lane = self.sent.pop(req)
        (K, V), (Kd, Vd) = kv, peer.cache
        for g in range(GROUPS):
            Kd[g][:, lane, :S - 1] = K[g][:, :S - 1]
            Vd[g][:, lane, :S - 1] = V[g][:, :S - 1]
        with peer.lock:
            peer.arrived.add(req)
        return 1000

    def wait(self, req, timeout=5.0):
        with self.lock:
            assert req in self.arrived
            self.arrived.discard(req)

    def release(self, req):
        with self.lock:
            self.leases.pop(req, None)

    def close(self):
        pass


def test_pool_holds_an_engine_exclusively_and_spreads_prompts():
    engines = [FakePrefill(0), FakePrefill(1)]
    pool = PrefillPool(engines)
    used = []

    def job():
        with pool.take() as e:
            used.append(e.dev.index)
            e.prefill_kv_device([1, 2, 3])
    ts = [threading.Thread(target=job) for _ in range(12)]
    [t.start() for t in ts]
    [t.join(10) for t in ts]
    assert sorted(set(used)) == [0, 1]
    assert all(e.overlaps == 0 for e in engines)
    assert sum(e.calls for e in engines) == 12
    with pytest.raises(ValueError):
        PrefillPool([])


@pytest.mark.parametrize("split", [(2, 6), (2, 2), (1, 3)])
def test_split_serves_solo_tokens(split):
    made = {}

    def mk_pre(g):
        made[g] = FakePrefill(g)
        return made[g]
    box = build_pd(None, split=split, B=4, S=S, make_prefill=mk_pre,
                   make_decode=lambda g: FakeDecodeGPU(4, g), transport=FakeLink)
    try:
        if split[0] == split[1]:
            assert [p.pool.engines for p in box.producers] == [[e] for e in box.prefill_engines]
        else:
            assert all(p.pool is box.producers[0].pool for p in box.producers)
        reqs = _requests(36, seed=7)
        out = [None] * len(reqs)

        def client(i, r):
            time.sleep(r["delay"])
            try:
                out[i] = box.gateway.complete({"tokens": r["tokens"], "max_tokens": r["max_new"]})
            except Exception as e:   # noqa: BLE001 - inspected below
                out[i] = e
        ts = [threading.Thread(target=client, args=(i, r)) for i, r in enumerate(reqs)]
        [t.start() for t in ts]
        [t.join(60) for t in ts]
        for r, res in zip(reqs, out):
            assert not isinstance(res, Exception), res
            assert res["choices"][0]["tokens"] == _alone(r["tokens"], r["max_new"])
            assert res["pd"]["mode"] == "disaggregated-kv-transfer" and "kv_load_ms" in res["pd"]
        assert all(e.overlaps == 0 for e in box.prefill_engines)
        assert all(e.calls > 0 for e in box.prefill_engines)
        assert all(d.steps > 0 for d in box.decode_engines)
        assert set(box.gateway.window.summary()) >= {"ttft_p90_ms", "tok_s", "kv_transfer_ms"}
    finally:
        box.close()


def test_split_parsing_and_gpu_count():
    assert parse_split("2P:6D") == (2, 6) and parse_split("1p:1d") == (1, 1)
    with pytest.raises(ValueError):
        parse_split("2:6")
    with pytest.raises(ValueError, match="needs 8 GPUs"):
        build_pd(None, split=(2, 6), gpus=[0, 1, 2], make_prefill=FakePrefill,
                 make_decode=lambda g: FakeDecodeGPU(4, g), transport=FakeLink)
