"""The worker glue (serving/workers.py: the reference's FullPrefillWorker.run save path and
DecodeWorkerBase load / prefetch, serving/cluster.py:180-218, 350-467) on the host with a fake
streaming prefill engine: every layer arrives bit-exact in the decode layouts over shm and tcp,
into float32 host arrays or bf16 tensors; consumed shm files are removed; prefetch overlaps
the save and is bounded."""
import os
import threading
import time
from types import SimpleNamespace
from unittest import mock

import numpy as np
import pytest
import torch

from rngd_pd.connector import tcpkv
from rngd_pd.connector import transport as kv
from rngd_pd.serving.workers import KVLoader, PrefillSaver

L, NG, NKV, S, HD = 4, 2, 2, 16, 8


class StreamEngine:
    """prefill_stream_device as FullPrefillEngine's: groups of [NG, 2, NKV, S, HD] bf16, the
    prompt's positions filled from its tokens, the tail zero."""

    def __init__(self, delay=0.0):
        self.cfg, self.NG, self.stream, self.last_C, self.delay = SimpleNamespace(n_layers=L), NG, None, 64, delay
        self.kv = None

    def prefill_stream_device(self, tokens, sink):
        P = len(tokens)
        g = torch.Generator().manual_seed(sum(tokens))
        kvb = torch.zeros((L, 2, NKV, S, HD), dtype=torch.bfloat16)
        kvb[:, :, :, :P] = torch.randn((L, 2, NKV, P, HD), generator=g).to(torch.bfloat16)
        self.kv = kvb
        for i in range(L // NG):
            threading.Event().wait(self.delay)
            sink(i, kvb[i * NG:(i + 1) * NG])
        return sum(tokens) % 1000


@pytest.fixture(autouse=True)
def bf16_wire():
    with mock.patch.object(kv, "WIRE", "bf16"):
        yield


def _expect(eng):
    return eng.kv[:, 0].transpose(-1, -2).float().numpy(), eng.kv[:, 1].float().numpy()


def test_save_then_load_over_shm_bit_exact_and_cleaned(tmp_path):
    t = kv.ShmTransport(str(tmp_path))
    eng = StreamEngine()
    rec = PrefillSaver(eng, t).run("rq1", [5, 6, 7])
    assert rec["next"] == 18 and rec["pos"] == 3 and rec["layers"] == L and rec["bucket_C"] == 64
    assert rec["kv_mb"] == round(2 * L * NKV * S * HD * 2 / 1e6, 1)
    assert len(os.listdir(tmp_path)) == 2 * L
    K, V, ms = KVLoader(t, L, NKV, HD, S).load_now("rq1")
    ek, ev = _expect(eng)
    np.testing.assert_array_equal(K, ek)
    np.testing.assert_array_equal(V, ev)
    assert K.dtype == np.float32 and K.shape == (L, NKV, HD, S) and ms >= 0
    assert not np.any(K[..., 3:]) and not np.any(V[:, :, 3:])      # the tail stays zero
    assert os.listdir(tmp_path) == []                                 # consumed files removed


def test_load_into_bf16_tensors_over_tcp():
    srv = tcpkv.TcpKVServer(0, "127.0.0.1")
    srv.start()
    port = srv.wait_ready()
    t = kv.TcpTransport(remote=("127.0.0.1", port))
    try:
        eng = StreamEngine()
        PrefillSaver(eng, t).run("rq2", list(range(1, 12)))
        K, V, _ = KVLoader(lambda: t, L, NKV, HD, S, device="cpu").load_now("rq2")
        assert K.dtype == torch.bfloat16 and tuple(V.shape) == (L, NKV, S, HD)
        assert torch.equal(K.view(torch.int16), eng.kv[:, 0].transpose(-1, -2).contiguous().view(torch.int16))
        assert torch.equal(V.view(torch.int16), eng.kv[:, 1].contiguous().view(torch.int16))
    finally:
        t.close()
        srv.stop()


def test_prefetch_overlaps_the_save(tmp_path):
    t = kv.ShmTransport(str(tmp_path))
    loader = KVLoader(t, L, NKV, HD, S)
    try:
        assert loader.prefetch("rq3") == {"prefetch": "started", "req_id": "rq3"}
        assert loader.prefetch("rq3") == {"prefetch": "already running"}
        eng = StreamEngine(delay=0.05)                   # groups arrive while the load waits
        PrefillSaver(eng, t).run("rq3", [9, 9])
        K, V, ms, lead = loader.load("rq3")
        ek, ev = _expect(eng)
        np.testing.assert_array_equal(K, ek)
        np.testing.assert_array_equal(V, ev)
        assert lead >= ms >= 0
        PrefillSaver(StreamEngine(), t).run("rq4", [1])
        K4, _, _, lead4 = loader.load("rq4")             # no prefetch: loaded now
        assert lead4 == -1.0 and K4.shape == (L, NKV, HD, S)
    finally:
        loader.close()


def test_prefetch_map_is_bounded(tmp_path):
    t = kv.ShmTransport(str(tmp_path))
    with mock.patch.dict(os.environ, {"PD_PREFETCH_CAP": "1", "PD_KV_PULL_TIMEOUT": "0.2"}):
        loader = KVLoader(t, L, NKV, HD, S)
    try:
        assert loader.prefetch("a")["prefetch"] == "started"
        assert loader.prefetch("b") == {"prefetch": "skipped (full)", "req_id": "b"}
        loader.ttl_s = 0.0
        assert loader.prefetch("b")["prefetch"] == "started"     # the stale entry is reclaimed
    finally:
        loader.close()


def test_a_failed_save_raises():
    class Broken(kv.InProcTransport):
        def push(self, key, buf):
            raise ConnectionError("link down")
    with pytest.raises(ConnectionError, match="link down"):
        PrefillSaver(StreamEngine(), Broken()).run("rq5", [1, 2])


def test_a_stuck_prefetch_does_not_delay_another_load(tmp_path):
    """Two prefetches whose KV never arrives hold their own workers until the pull timeout; a
    third request whose KV has landed still loads at once."""
    t = kv.ShmTransport(str(tmp_path))
    with mock.patch.dict(os.environ, {"PD_PREFETCH_CAP": "3", "PD_KV_PULL_TIMEOUT": "3"}):
        loader = KVLoader(t, L, NKV, HD, S)
        try:
            assert loader.prefetch("ghost1")["prefetch"] == "started"
            assert loader.prefetch("ghost2")["prefetch"] == "started"
            eng = StreamEngine()
            PrefillSaver(eng, t).run("real", [4, 5])
            assert loader.prefetch("real")["prefetch"] == "started"
            t0 = time.perf_counter()
            K, V, _ms, _lead = loader.load("real")
            assert time.perf_counter() - t0 < 1.5
            ek, ev = _expect(eng)
            np.testing.assert_array_equal(K, ek)
            np.testing.assert_array_equal(V, ev)
        finally:
            loader.close()


def test_reclaimed_prefetch_that_has_not_started_is_cancelled(tmp_path):
    t = kv.ShmTransport(str(tmp_path))
    with mock.patch.dict(os.environ, {"PD_PREFETCH_CAP": "1", "PD_KV_PULL_TIMEOUT": "0.5"}):
        loader = KVLoader(t, L, NKV, HD, S)
    gate = threading.Event()
    try:
        loader._pool.submit(gate.wait)                     # the only worker is busy
        loader.prefetch("queued")
        fut = loader._prefetch["queued"][0]
        loader.ttl_s = 0.0
        loader.prefetch("next")
        assert fut.cancelled() and "queued" not in loader._prefetch
    finally:
        gate.set()
        loader.close()


@pytest.mark.gpu
def test_device_save_and_load_bit_exact_on_the_gpu(tmp_path):
    """The device half: PrefillSaver over a real FullPrefillEngine (2 layers of the Llama-3.1-8B
    shape) transposes K on the engine's stream and stages bf16 bits; KVLoader(device='cuda')
    fills bf16 device buffers from the wire.  Both equal prefill_device's cache bit for bit."""
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = ModelConfig.from_dims(L=2)
    eng = FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=128, group=1, S=256)
    toks = [(13 * i + 7) % cfg.vocab for i in range(100)]
    Kref, Vref, nref = eng.prefill_device(toks)
    t = kv.ShmTransport(str(tmp_path))
    rec = PrefillSaver(eng, t).run("gpu1", toks)
    assert rec["next"] == nref
    loader = KVLoader(t, cfg.n_layers, cfg.n_kv, cfg.head_dim, eng.S, device="cuda")
    try:
        s = torch.cuda.Stream()
        K, V, _ms, _lead = loader.load("gpu1", stream=s)
    finally:
        loader.close()
    assert K.is_cuda and K.dtype == torch.bfloat16
    assert torch.equal(K.view(torch.int16), Kref.contiguous().view(torch.int16))     # both [L, NKV, HD, S]
    assert torch.equal(V.view(torch.int16), Vref.contiguous().view(torch.int16))
    assert os.listdir(tmp_path) == []
