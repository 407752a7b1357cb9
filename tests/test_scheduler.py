"""ContinuousScheduler (serving/scheduler.py, the reference's _ContinuousScheduler,
serving/cluster.py:832-1134) on the host with fake engines: every request gets the tokens it
gets alone, whatever it is batched with and whenever it arrives; admission staged between
decode steps; TieredDecode underneath; a failing step ends its own streams only."""
import random
import threading
import time

import pytest
import torch

from rngd_pd.engines.tiers import TieredDecode
from rngd_pd.serving.scheduler import ContinuousScheduler

S, GROUPS, LAYERS, VOCAB = 64, 2, 2, 997


class FakeDecode:
    """Lane caches [layers, B, S] on the CPU; a lane's next token depends on its own cache only."""

    def __init__(self, B, fail_at=None):
        self.B, self.steps, self.fail_at = B, 0, fail_at

    def blank_kv(self):
        z = lambda: [torch.zeros((LAYERS, self.B, S), dtype=torch.float64) for _ in range(GROUPS)]
        return z(), z()

    def write_slot_kv(self, Kd, Vd, idx, K, V):
        for g in range(GROUPS):
            Kd[g][:, idx] = K[g]
            Vd[g][:, idx] = V[g]
        return Kd, Vd

    def step(self, toks, pos, Kd, Vd):
        self.steps += 1
        if self.fail_at is not None and self.steps == self.fail_at:
            raise RuntimeError("injected step failure")
        out = []
        for b in range(self.B):
            for g in range(GROUPS):
                Kd[g][:, b, pos[b] % S] += toks[b] + 1
                Vd[g][:, b, pos[b] % S] += 2 * toks[b] + 1
            out.append(int(sum(float(Kd[g][:, b, :S - 1].sum() + Vd[g][:, b, :S - 1].sum())
                               for g in range(GROUPS))) % VOCAB)
        return out, Kd, Vd


def _prefill(tokens):
    """A fake prefill: a cache and a first token that depend on the whole prompt."""
    h = sum((i + 1) * t for i, t in enumerate(tokens))
    K = [torch.full((LAYERS, S), float(h % 101 + g), dtype=torch.float64) for g in range(GROUPS)]
    V = [torch.full((LAYERS, S), float(h % 89 + 2 * g), dtype=torch.float64) for g in range(GROUPS)]
    return K, V, h % VOCAB


class Producer:
    def __init__(self, stage_groups=3):
        self.calls, self.staged, self.stage_groups = 0, 0, stage_groups

    def produce(self, item):
        self.calls += 1
        K, V, first = _prefill(item["tokens"])
        return K, V, first, len(item["tokens"]), 0.0

    def begin_produce(self, item):
        self.staged += 1
        outer, left = self, [self.stage_groups]

        class _Stage:
            def advance(self, n=1):
                left[0] -= n
                return left[0] <= 0

            def result(self):
                return outer.produce(item)
        return _Stage()


def _alone(tokens, max_new):
    """The request on a fresh engine, lane 0, nothing else running."""
    eng = FakeDecode(1)
    Kd, Vd = eng.blank_kv()
    K, V, first = _prefill(tokens)
    Kd, Vd = eng.write_slot_kv(Kd, Vd, 0, K, V)
    out, cur, pos = [first], first, len(tokens)
    while len(out) < max_new:
        nxt, Kd, Vd = eng.step([cur], [pos], Kd, Vd)
        out.append(nxt[0])
        cur, pos = nxt[0], pos + 1
    return out


def _requests(n, seed):
    rnd = random.Random(seed)
    return [{"tokens": [rnd.randrange(VOCAB) for _ in range(rnd.randrange(1, 20))],
             "max_new": rnd.randrange(1, 24), "delay": rnd.random() * 0.02} for _ in range(n)]


def _serve(sched, reqs):
    results, streamed = [None] * len(reqs), [[] for _ in reqs]

    def client(i, r):
        time.sleep(r["delay"])
        item = {"tokens": r["tokens"], "max_new": r["max_new"], "on_token": streamed[i].append}
        try:
            results[i] = sched.submit(item)
        except Exception as e:   # noqa: BLE001 - the test inspects it
            results[i] = e
    threads = [threading.Thread(target=client, args=(i, r)) for i, r in enumerate(reqs)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    return results, streamed


@pytest.mark.parametrize("stage", [False, True])
def test_every_request_gets_its_solo_tokens(stage):
    reqs = _requests(40, seed=1)
    prod = Producer()
    sched = ContinuousScheduler(8, FakeDecode(8), prod.produce, produce_owner=prod, stage_groups=2,
                                stage_admission=stage)
    try:
        results, streamed = _serve(sched, reqs)
    finally:
        sched.close()
    for r, res, st in zip(reqs, results, streamed):
        want = _alone(r["tokens"], r["max_new"])
        assert res["tokens"] == want
        assert st == want                                   # streamed in order as produced
        assert res["pos"] == len(r["tokens"])
    assert 0 < sched.occupancy() <= 1
    if stage:
        assert prod.staged > 0                              # some prompts were staged between steps


def test_tiered_engine_underneath():
    reqs = _requests(24, seed=2)
    prod = Producer()
    tiers = TieredDecode([FakeDecode(2), FakeDecode(4), FakeDecode(8)])
    sched = ContinuousScheduler(8, tiers, prod.produce, produce_owner=prod)
    try:
        results, _ = _serve(sched, reqs)
    finally:
        sched.close()
    for r, res in zip(reqs, results):
        assert res["tokens"] == _alone(r["tokens"], r["max_new"])
    assert sum(tiers.steps_at.values()) == sched.steps


def test_failing_step_ends_its_streams_and_the_loop_goes_on():
    prod = Producer()
    eng = FakeDecode(4, fail_at=3)
    sched = ContinuousScheduler(4, eng, prod.produce)
    try:
        first, _ = _serve(sched, [{"tokens": [1, 2, 3], "max_new": 10, "delay": 0.0}])
        assert isinstance(first[0], RuntimeError)
        later, _ = _serve(sched, [{"tokens": [4, 5], "max_new": 5, "delay": 0.0}])
        assert later[0]["tokens"] == _alone([4, 5], 5)
    finally:
        sched.close()


def test_admit_min_holds_lanes_while_streams_run():
    prod = Producer()
    sched = ContinuousScheduler(4, FakeDecode(4), prod.produce, admit_min=2)
    try:
        reqs = [{"tokens": [i + 1], "max_new": 6, "delay": 0.004 * i} for i in range(6)]
        results, _ = _serve(sched, reqs)
    finally:
        sched.close()
    for r, res in zip(reqs, results):
        assert res["tokens"] == _alone(r["tokens"], r["max_new"])
    assert sched.held_lane_steps + sched.starved_lane_steps > 0


class LaneFiller:
    """A producer that fills the lane itself from another thread, like a prefill on another GPU
    pushing into the leased lane: rows [0, S - 1) only, while the other lanes keep stepping."""

    def __init__(self, kv, fail_every=None):
        from concurrent.futures import ThreadPoolExecutor
        self.Kd, self.Vd = kv
        self.pool = ThreadPoolExecutor(max_workers=2)
        self.fail_every, self.n = fail_every, 0

    def start_lane(self, item, lane):
        self.n += 1
        fail = self.fail_every is not None and self.n % self.fail_every == 0

        def fill():
            time.sleep(0.002)
            if fail:
                raise RuntimeError("injected fill failure")
            K, V, first = _prefill(item["tokens"])
            for g in range(GROUPS):
                self.Kd[g][:, lane, :S - 1] = K[g][:, :S - 1]
                self.Vd[g][:, lane, :S - 1] = V[g][:, :S - 1]
            return None, None, first, len(item["tokens"]), 0.0
        return self.pool.submit(fill)


def test_lanes_filled_elsewhere_overlap_the_steps():
    reqs = _requests(30, seed=3)
    eng = FakeDecode(6)
    kv = eng.blank_kv()
    filler = LaneFiller(kv, fail_every=7)
    sched = ContinuousScheduler(6, eng, None, produce_owner=filler, idle_pos=S - 1, kv=kv)
    try:
        results, _ = _serve(sched, reqs)
    finally:
        sched.close()
    failed = 0
    for r, res in zip(reqs, results):
        if isinstance(res, RuntimeError):
            failed += 1                                  # its own fill failed, nobody else's
            continue
        assert res["tokens"] == _alone(r["tokens"], r["max_new"])
    assert failed == len(reqs) // 7
