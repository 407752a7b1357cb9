"""TieredDecode (engines/tiers.py): every stream gets the same tokens whether one wide engine
or several widths serve it, including when the width changes while streams are live.
Host logic with fake engines (after the reference's tests/test_decode_tiers.py), plus a
GPU check with real engines sharing one set of weights."""
import numpy as np
import pytest
import torch

from rngd_pd.engines.tiers import TieredDecode

S, GROUPS, LAYERS = 32, 2, 2


class FakeEngine:
    """Per-lane cache [layers, B, S] on the CPU; the next token depends on the lane's whole cache."""

    def __init__(self, B):
        self.B, self.steps = B, 0

    def blank_kv(self):
        return ([torch.zeros((LAYERS, self.B, S), dtype=torch.float64) for _ in range(GROUPS)],
                [torch.zeros((LAYERS, self.B, S), dtype=torch.float64) for _ in range(GROUPS)])

    def write_slot_kv(self, Kd, Vd, idx, K, V):
        for g in range(GROUPS):
            Kd[g][:, idx] = K[g]
            Vd[g][:, idx] = V[g]
        return Kd, Vd

    def step(self, toks, pos, Kd, Vd):
        assert len(toks) == self.B
        self.steps += 1
        out = []
        for b in range(self.B):
            for g in range(GROUPS):
                Kd[g][:, b, pos[b] % S] += toks[b] + 1
                Vd[g][:, b, pos[b] % S] += 2 * toks[b] + 1
            out.append(int(sum(float(Kd[g][:, b].sum() + Vd[g][:, b].sum()) for g in range(GROUPS))) % 997)
        return out, Kd, Vd


def _kv(seed):
    K = [torch.full((LAYERS, S), float(seed + g), dtype=torch.float64) for g in range(GROUPS)]
    V = [torch.full((LAYERS, S), float(2 * seed + g), dtype=torch.float64) for g in range(GROUPS)]
    return K, V


def _run(engine, plan, B):
    """plan: per step, lanes admitted before it and lanes retired after it."""
    Kd, Vd = engine.blank_kv()
    live, toks, pos, out = [], [0] * B, [0] * B, []
    for admit, retire in plan:
        for lane in admit:
            K, V = _kv(lane + 1)
            if hasattr(engine, "set_live"):
                engine.set_live(live)
            Kd, Vd = engine.write_slot_kv(Kd, Vd, lane, K, V)
            live.append(lane)
            toks[lane], pos[lane] = lane % 7, 3
        if hasattr(engine, "set_live"):
            engine.set_live(live)
        nxt, Kd, Vd = engine.step(toks, pos, Kd, Vd)
        out.append({lane: nxt[lane] for lane in live})
        for lane in live:
            toks[lane], pos[lane] = nxt[lane], pos[lane] + 1
        live = [lane for lane in live if lane not in retire]
    return out


PLAN = [([0], []), ([], []), ([1, 2], []), ([], []), ([5], []), ([], []), ([11], []), ([], [11]), ([], [5]),
        ([], []), ([], [1, 2]), ([], []), ([3], []), ([], [])]


def test_tiers_match_one_wide_engine():
    wide = _run(FakeEngine(16), PLAN, 16)
    engines = [FakeEngine(4), FakeEngine(8), FakeEngine(16)]
    tiers = TieredDecode(engines)
    got = _run(tiers, PLAN, 16)
    assert got == wide
    assert tiers.switches >= 3                     # widened to 8 and 16, narrowed back
    assert tiers.steps_at[4] > 0 and tiers.steps_at[8] > 0 and tiers.steps_at[16] > 0


def test_tiers_reject_bad_setups():
    with pytest.raises(ValueError):
        TieredDecode([])
    with pytest.raises(ValueError):
        TieredDecode([FakeEngine(4), FakeEngine(4)])
    t = TieredDecode([FakeEngine(4), FakeEngine(8)])
    with pytest.raises(ValueError):
        t.set_live([8])


@pytest.mark.gpu
def test_tiers_real_engines_match_wide_engine():
    """Widths 2 / 4 sharing weights, streams admitted mid-run: the same greedy tokens as one
    B=4 engine, bit for bit."""
    from oracle import ref_np as R
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.synth import SyntheticState, request_kv
    d = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
    cfg = ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)
    wide = BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=4, S=256, group=1)
    narrow = BatchDecodeEngine(cfg, None, B=2, S=256, group=1, share=wide)
    tiers = TieredDecode([narrow, BatchDecodeEngine(cfg, None, B=4, S=256, group=1, share=wide)])
    kvs = [request_kv(cfg, 256, 100 + i, 40 + 10 * i) for i in range(4)]

    def run(engine, tiered):
        Kd, Vd = engine.blank_kv()
        live, toks, pos, out = [], [0] * 4, [0] * 4, []
        for step in range(8):
            if step in (0, 3):   # lanes 0-1 first, lanes 2-3 from step 3 (forces a widening)
                for lane in ((0, 1) if step == 0 else (2, 3)):
                    if tiered:
                        engine.set_live(live)
                    Kd, Vd = engine.write_slot_kv(Kd, Vd, lane, kvs[lane][0], kvs[lane][1])
                    live.append(lane)
                    toks[lane], pos[lane] = 7 * lane + 1, 40 + 10 * lane
            if tiered:
                engine.set_live(live)
            nxt, Kd, Vd = engine.step(toks, pos, Kd, Vd)
            out.append([nxt[lane] for lane in live])
            for lane in live:
                toks[lane], pos[lane] = nxt[lane], pos[lane] + 1
        return out

    assert run(tiers, True) == run(wide, False)
    assert tiers.switches == 1
