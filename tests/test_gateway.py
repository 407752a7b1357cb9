"""The in-process Gateway (serving/gateway.py, the reference's Gateway,
serving/cluster.py:1457-1598) and the airm serving metrics (airm.py:393-507) on the host with
fake engines: routing by model name with round-robin, the completion record and its pd
fields, tokens equal to a solo run under concurrency, and the Window's airm_* gauges."""
import threading
import urllib.error
import urllib.request

import numpy as np
import pytest

from rngd_pd import airm
from rngd_pd.serving.gateway import Gateway
from rngd_pd.serving.scheduler import ContinuousScheduler
from tests.test_scheduler import S, FakeDecode, LaneFiller, Producer, _alone, _requests


class XferFiller(LaneFiller):
    """A lane filler that reports a transfer record, as NvlinkProducer does."""

    def start_lane(self, item, lane):
        fut = super().start_lane(item, lane)
        item["_xfer"] = {"prefill_ms": 1.5, "kv_save_ms": 0.01, "kv_load_ms": 0.2, "kv_mb": 3.0}
        return fut


def _one_card(B=4):
    prod = Producer()
    return ContinuousScheduler(B, FakeDecode(B), prod.produce, produce_owner=prod, stage_admission=False)


def _split(B=4):
    eng = FakeDecode(B)
    kv = eng.blank_kv()
    return ContinuousScheduler(B, eng, None, produce_owner=XferFiller(kv), idle_pos=S - 1, kv=kv)


@pytest.fixture
def gw():
    a, b, c = _one_card(), _split(), _split()
    g = Gateway({"solo": a, "pd": [b, c]}, S=S)
    yield g, (a, b, c)
    for s in (a, b, c):
        s.close()


def test_record_and_tokens(gw):
    g, _ = gw
    for model, mode in (("solo", "single-card"), ("pd", "disaggregated-kv-transfer")):
        streamed = []
        r = g.complete({"model": model, "tokens": [5, 6, 7], "max_tokens": 9}, on_token=streamed.append)
        want = _alone([5, 6, 7], 9)
        assert r["choices"][0]["tokens"] == want == streamed
        assert r["usage"] == {"prompt_tokens": 3, "completion_tokens": 9, "total_tokens": 12}
        pd = r["pd"]
        assert pd["mode"] == mode and pd["config"] == model
        assert 0 <= pd["ttft_ms"] <= pd["wall_ms"]
        assert pd["sched"] == "continuous" and pd["batch_width"] == 4
        if mode == "disaggregated-kv-transfer":
            assert (pd["kv_save_ms"], pd["kv_load_ms"], pd["kv_mb"]) == (0.01, 0.2, 3.0)
        else:
            assert pd["kv_mb"] == 0.0
    assert len(g.window.recs) == 2


def test_routing(gw):
    g, (_a, b, c) = gw
    for _ in range(4):
        g.complete({"model": "pd", "tokens": [1, 2], "max_tokens": 3})
    assert b.steps > 0 and c.steps > 0                       # round-robin over the pairings
    with pytest.raises(ValueError, match="unknown model"):
        g.complete({"model": "nope", "tokens": [1], "max_tokens": 2})
    with pytest.raises(ValueError, match="unknown model"):   # several pairings: a name is needed
        g.complete({"tokens": [1], "max_tokens": 2})
    with pytest.raises(ValueError, match="tokenizer"):
        g.complete({"model": "solo", "prompt": "hello", "max_tokens": 2})
    with pytest.raises(ValueError, match="empty prompt"):
        g.complete({"model": "solo", "tokens": [], "max_tokens": 2})


def test_single_pairing_is_the_default_and_prompts_are_cut_to_fit():
    s = _one_card()
    try:
        g = Gateway({"only": s}, S=S)
        long = list(range(1, 200))
        r = g.complete({"prompt": long, "max_tokens": 4})
        kept = long[:S - 4 - 1]
        assert r["usage"]["prompt_tokens"] == len(kept)
        assert r["choices"][0]["tokens"] == _alone(kept, 4)
    finally:
        s.close()


def test_text_prompts_with_a_tokenizer():
    class Tok:
        def encode(self, text, add_special_tokens=False):
            return [ord(ch) % 97 + 1 for ch in text]

        def decode(self, ids):
            return " ".join(map(str, ids))
    s = _one_card()
    try:
        g = Gateway({"m": s}, S=S, tokenizer=Tok())
        r = g.complete({"messages": [{"content": "hi"}, {"content": "there"}], "max_tokens": 3})
        toks = Tok().encode("hi\nthere")
        assert r["choices"][0]["tokens"] == _alone(toks, 3)
        assert r["choices"][0]["text"] == " ".join(map(str, _alone(toks, 3)))
    finally:
        s.close()


def test_concurrent_requests_get_their_solo_tokens(gw):
    g, _ = gw
    reqs = _requests(30, seed=5)
    out = [None] * len(reqs)

    def client(i, r):
        try:
            out[i] = g.complete({"model": ("solo", "pd")[i % 2], "tokens": r["tokens"], "max_tokens": r["max_new"]})
        except Exception as e:   # noqa: BLE001 - inspected below
            out[i] = e
    ts = [threading.Thread(target=client, args=(i, r)) for i, r in enumerate(reqs)]
    [t.start() for t in ts]
    [t.join(60) for t in ts]
    for r, res in zip(reqs, out):
        assert not isinstance(res, Exception), res
        assert res["choices"][0]["tokens"] == _alone(r["tokens"], r["max_new"])
    s = g.window.summary()
    assert set(s) == {"ttft_p90_ms", "tpot_p90_ms", "tok_s", "kv_transfer_ms"}
    assert s["tok_s"] > 0


def test_summarize_by_hand():
    recs = [{"t0": 0.0, "t1": 2.0, "ttft_ms": 100.0, "tpot_ms": 4.0, "out_tokens": 64,
             "kv_save_ms": 1.0, "kv_load_ms": 2.0},
            {"t0": 0.5, "t1": 4.0, "ttft_ms": 300.0, "tpot_ms": 6.0, "out_tokens": 36},
            {"error": "boom", "t0": 0.0, "t1": 9.0}]
    s = airm.summarize(recs)
    assert s == {"ttft_p90_ms": round(float(np.percentile([100, 300], 90)), 1),
                 "tpot_p90_ms": round(float(np.percentile([4, 6], 90)), 1),
                 "tok_s": 25.0, "kv_transfer_ms": 3.0}
    assert airm.summarize(recs, wall_s=10.0)["tok_s"] == 10.0
    assert airm.summarize([{"error": "x"}]) == {}


def test_window_tpot_is_what_the_client_sees():
    w = airm.Window(size=2)
    resp = {"usage": {"completion_tokens": 11}, "pd": {"mode": "single-card", "ttft_ms": 50.0, "tpot_ms": 1.0}}
    w.record(0.0, 0.25, resp)                      # (250 - 50) / 10 = 20 ms, not the loop's 1 ms
    assert w.recs[-1]["tpot_ms"] == pytest.approx(20.0)
    assert "kv_save_ms" not in w.recs[-1]
    w.record(0.0, 1.0, {"usage": {"completion_tokens": 1}, "pd": {"mode": "disaggregated-kv-transfer",
                                                                  "ttft_ms": 9.0, "tpot_ms": 2.0,
                                                                  "kv_save_ms": 0.1, "kv_load_ms": 0.4}})
    assert w.recs[-1]["tpot_ms"] == 2.0 and w.recs[-1]["kv_load_ms"] == 0.4
    w.record(0.0, 1.0, resp)
    assert len(w.recs) == 2                         # the last `size` requests


def test_metrics_endpoint():
    w = airm.Window()
    wrapped = w.observe(lambda body: {"usage": {"completion_tokens": 5},
                                      "pd": {"mode": "disaggregated-kv-transfer", "ttft_ms": 10.0,
                                             "kv_save_ms": 0.5, "kv_load_ms": 1.5}})
    wrapped({})
    srv = airm.serve_metrics(w, 0, host="127.0.0.1")
    try:
        port = srv.server_address[1]
        text = urllib.request.urlopen(f"http://127.0.0.1:{port}/metrics", timeout=5).read().decode()
        assert "# TYPE airm_ttft_p90_ms gauge" in text
        assert 'airm_ttft_p90_ms{component="rngd-pd"} 10' in text
        assert 'kv_transport=' in text.split("airm_kv_transfer_ms{")[1].split("}")[0]
        assert 'airm_tok_s{component="rngd-pd"}' in text
        with pytest.raises(urllib.error.HTTPError):
            urllib.request.urlopen(f"http://127.0.0.1:{port}/other", timeout=5)
    finally:
        srv.shutdown()
