"""ContinuousScheduler over the real engines on one B200 (small model): every request's
tokens under continuous batching equal the tokens it gets decoded alone (the decode step is
batch-invariant by design), with staged and with block admission."""
import threading

import pytest

from oracle import ref_np as R

pytestmark = pytest.mark.gpu

SMALL = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
S = 256


def _cfg(d):
    from rngd_pd.engines.model import ModelConfig
    return ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)


@pytest.fixture(scope="module")
def engines():
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(SMALL)
    dec = BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=4, S=S, group=1, chip=0)
    pre = FullPrefillEngine(cfg, dec.w, C=128, group=1, S=S)
    return dec, pre


def _alone(dec, pre, tokens, max_new):
    K, V, first = pre.prefill_device(tokens)
    Kd, Vd = dec.blank_kv()
    Kd, Vd = dec.write_slot_kv(Kd, Vd, 0, K, V)
    out, cur, pos = [first], first, len(tokens)
    while len(out) < max_new:
        nxt, Kd, Vd = dec.step([cur, 0, 0, 0], [pos, 0, 0, 0], Kd, Vd)
        out.append(nxt[0])
        cur, pos = nxt[0], pos + 1
    return out


@pytest.mark.parametrize("stage", [True, False])
def test_scheduled_tokens_equal_solo_tokens(engines, stage):
    from rngd_pd import _lib
    from rngd_pd.serving.scheduler import ContinuousScheduler, OneCardProducer
    dec, pre = engines
    reqs = [([(13 * i + 7 * j) % SMALL.V for j in range(5 + 9 * i)], 3 + (i % 5)) for i in range(10)]
    want = [_alone(dec, pre, t, n) for t, n in reqs]
    prod = OneCardProducer(pre)
    sched = ContinuousScheduler(4, dec, prod.produce, produce_owner=prod, stage_groups=1, stage_admission=stage)
    got = [None] * len(reqs)

    def client(i):
        got[i] = sched.submit({"tokens": reqs[i][0], "max_new": reqs[i][1]})["tokens"]
    threads = [threading.Thread(target=client, args=(i,)) for i in range(len(reqs))]
    try:
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=120)
    finally:
        sched.close()
    assert got == want
    assert _lib.device_status() == 0
