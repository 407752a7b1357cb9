"""The `nvlink` KV transport between two B200s: GPU 0 prefills and pushes, GPU 1 decodes.

  * one process driving both GPUs (peer access, direct pointers), receiver ordering its
    stream with the bounded device wait (rngd_kv_wait) on the sender's flags;
  * two processes (spawned), the receiver's cache and flags exported by CUDA IPC handles
    carried in the handshake metadata;
  * the full path: prefill on GPU 0 -> handoff -> decode on GPU 1 equals prefill and decode
    both on GPU 1 (bit-exact logits).
Skipped on a box with fewer than two GPUs."""
import multiprocessing as mp
import os
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

L, BCAP, NKV, S, HD = 4, 3, 8, 512, 128
BF = torch.bfloat16
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _kv(seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((L, 2, NKV, S, HD), generator=g).to(BF).to(device)


def _bits(t):
    return t.contiguous().view(torch.int16)


def test_peer_handoff_one_process_with_device_wait():
    from rngd_pd.nvlink import NvlinkTransport
    rx, tx = NvlinkTransport(1), NvlinkTransport(0)
    K = torch.zeros((L, BCAP, NKV, S, HD), dtype=BF, device="cuda:1")
    V = torch.zeros_like(K)
    rx.bind_cache(K, V)
    rx.reserve("r", 2, sender_device=0)
    tx.set_remote_handshake(rx.handshake_metadata())
    s1 = torch.cuda.Stream(device="cuda:1")
    outcome = rx.wait_stream("r", s1, timeout=5.0)
    kv = _kv(11, "cuda:0")
    s0 = torch.cuda.Stream(device="cuda:0")
    s0.wait_stream(torch.cuda.current_stream("cuda:0"))
    tx.push_device("r", kv, stream=s0)
    assert outcome(block=True) is True
    with torch.cuda.stream(s1):
        landed_k, landed_v = K[:, 2].clone(), V[:, 2].clone()
    s1.synchronize()
    assert torch.equal(_bits(landed_k).cpu(), _bits(kv[:, 0]).cpu())
    assert torch.equal(_bits(landed_v).cpu(), _bits(kv[:, 1]).cpu())
    assert not K[:, 0].any() and not K[:, 1].any()
    tx.close()
    rx.close()


def _receiver(q_out, q_in):
    sys.path[:0] = [REPO, os.path.join(REPO, "rngd-pd_b200")]
    import torch
    from rngd_pd.nvlink import NvlinkTransport, ipc_empty
    try:
        torch.cuda.set_device(1)
        rx = NvlinkTransport(1)
        K = ipc_empty((L, BCAP, NKV, S, HD), BF, "cuda:1")
        V = ipc_empty((L, BCAP, NKV, S, HD), BF, "cuda:1")
        rx.bind_cache(K, V)
        rx.reserve("xp", 1, sender_device=0)
        q_out.put(("meta", rx.handshake_metadata()))
        s = torch.cuda.Stream(device="cuda:1")
        ok = rx.wait_stream("xp", s, timeout=8.0)(block=True)
        want = _kv(12, "cuda:1")
        with torch.cuda.stream(s):
            same = bool(torch.equal(_bits(K[:, 1]), _bits(want[:, 0])) and torch.equal(_bits(V[:, 1]), _bits(want[:, 1])))
            untouched = not bool(K[:, 0].any() or K[:, 2].any())
        s.synchronize()
        q_out.put(("result", ok, same, untouched))
        q_in.get(timeout=60)          # the sender has closed its mapping
        rx.close()
    except Exception as e:            # reported to the test, never swallowed
        q_out.put(("error", repr(e)))


def test_cross_process_ipc_handoff():
    from rngd_pd.nvlink import NvlinkTransport
    ctx = mp.get_context("spawn")
    q_out, q_in = ctx.Queue(), ctx.Queue()
    p = ctx.Process(target=_receiver, args=(q_out, q_in))
    p.start()
    tx = None
    try:
        msg = q_out.get(timeout=180)
        assert msg[0] == "meta", msg
        meta = msg[1]
        assert meta["pid"] != os.getpid() and all(meta["handles"].values())
        tx = NvlinkTransport(0)
        tx.set_remote_handshake(meta)
        tx.push_device("xp", _kv(12, "cuda:0"))
        torch.cuda.synchronize(0)
        res = q_out.get(timeout=60)
        assert res == ("result", True, True, True), res
    finally:
        if tx is not None:
            tx.close()
        q_in.put("closed")
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert p.exitcode == 0


def test_prefill_on_gpu0_decode_on_gpu1_equals_one_card():
    from oracle import ref_np as R
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.nvlink import NvlinkTransport
    from rngd_pd.synth import SyntheticState
    d = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
    cfg = ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)
    pf0 = FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=256, group=1, S=256, chip=0)
    dec1 = BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=2, S=256, group=1, chip=1)
    prompts = [[(3 * i + 1) % d.V for i in range(40)], [(5 * i + 2) % d.V for i in range(130)]]
    Kd, Vd = dec1.blank_kv()
    rx, tx = NvlinkTransport(1), NvlinkTransport(0)
    rx.bind_cache(*dec1.full_kv(Kd, Vd))
    for b in range(2):
        rx.reserve(f"p{b}", b, sender_device=0)
    tx.set_remote_handshake(rx.handshake_metadata())
    nxt = []
    for b, p in enumerate(prompts):
        kv, n = pf0.prefill_kv_device(p)
        tx.push_device(f"p{b}", kv, stream=pf0.stream, tokens=len(p))
        nxt.append(n)
    for b in range(2):
        rx.wait_stream(f"p{b}", dec1.stream, timeout=5.0)(block=True)
    pos = [len(p) for p in prompts]
    dec1.step(nxt, pos, Kd, Vd)
    got = dec1.logits_bv().cpu()

    pf1 = FullPrefillEngine(cfg, dec1.w, C=256, group=1, S=256, chip=1)
    Ks, Vs, ns = [], [], []
    for p in prompts:
        K, V, n = pf1.prefill_device(p)
        Ks.append(K)
        Vs.append(V)
        ns.append(n)
    assert ns == nxt
    Ka, Va = dec1.adopt_kv_device(Ks, Vs)
    dec1.step(nxt, pos, Ka, Va)
    assert torch.equal(got, dec1.logits_bv().cpu())
    tx.close()
    rx.close()


def test_continuous_batching_with_prefill_on_another_gpu_equals_one_card():
    """ContinuousScheduler + NvlinkProducer: prompts prefilled on GPU 0 are pushed into the
    decode lanes leased on GPU 1 while GPU 1 keeps stepping; every request's tokens equal the
    tokens of prefill and decode both on GPU 1 (the decode step is batch-invariant)."""
    import threading
    from oracle import ref_np as R
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.serving.scheduler import ContinuousScheduler, NvlinkProducer
    from rngd_pd.synth import SyntheticState
    d = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
    cfg = ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)
    Sd = 256
    pf0 = FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=128, group=1, S=Sd, chip=0)
    dec1 = BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=4, S=Sd, group=1, chip=1)
    pf1 = FullPrefillEngine(cfg, dec1.w, C=128, group=1, S=Sd)
    reqs = [([(11 * i + 3 * j) % d.V for j in range(4 + 11 * i)], 3 + i % 4) for i in range(9)]

    def alone(tokens, n):
        K, V, first = pf1.prefill_device(tokens)
        Kd, Vd = dec1.blank_kv()
        Kd, Vd = dec1.write_slot_kv(Kd, Vd, 0, K, V)
        out, cur, pos = [first], first, len(tokens)
        while len(out) < n:
            nxt, Kd, Vd = dec1.step([cur, 0, 0, 0], [pos, 0, 0, 0], Kd, Vd)
            out.append(nxt[0])
            cur, pos = nxt[0], pos + 1
        return out
    want = [alone(t, n) for t, n in reqs]
    kv = dec1.blank_kv()
    prod = NvlinkProducer(pf0, dec1, kv)
    sched = ContinuousScheduler(4, dec1, None, produce_owner=prod, idle_pos=Sd - 1, kv=kv)
    got = [None] * len(reqs)

    def client(i):
        try:
            got[i] = sched.submit({"tokens": reqs[i][0], "max_new": reqs[i][1]})["tokens"]
        except Exception as e:   # noqa: BLE001 - compared below
            got[i] = repr(e)
    threads = [threading.Thread(target=client, args=(i,)) for i in range(len(reqs))]
    try:
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=120)
    finally:
        sched.close()
        prod.close()
    assert got == want
