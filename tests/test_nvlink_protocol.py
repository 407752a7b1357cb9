"""The NVLink handoff's lease / handshake protocol across two processes on the host (no GPU).

The receiver is the real NvlinkTransport (reserve, release, handshake_metadata, arrived, wait,
arrived_all, wait_all, lane_views and the rm-core wait that turns a timeout into a failed
TransferResult) with its cache and per-lane flags in shared host memory instead of HBM: only
the flag read is swapped for a read of that memory.  The sender is a spawned process that learns leases through the
real SenderLeases (from the receiver's handshake metadata, or from a ticket forwarded with a
request) and stores a request's bytes into its leased lane, then publishes the lease's
sequence number in each layer's flag -- the order the handoff kernel keeps (data, fence,
flags).  Checked: arrival is seen only after the flags are published; a lane's stale flags
never satisfy its next lease; layers arrive in ranges; a push for a request without a lease
is refused by the sender; a wait that runs out is TimeoutError, and a failed TransferResult
through the rm-core adapter.
"""
import multiprocessing as mp
import os
import sys
import time
from multiprocessing import shared_memory

import numpy as np
import pytest
import torch

L, BCAP, NKV, S, HD = 4, 3, 2, 128, 128
PER_LAYER = 256                                 # payload bytes per layer in the fake lane memory
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _sender(flags_name, lanes_name, q_in, q_out):
    sys.path[:0] = [REPO, os.path.join(REPO, "rngd-pd_b200")]
    from rngd_pd.nvlink import SenderLeases
    fs = shared_memory.SharedMemory(name=flags_name)
    ls = shared_memory.SharedMemory(name=lanes_name)
    flags = np.ndarray((BCAP, L), np.int64, buffer=fs.buf)
    lanes = np.ndarray((BCAP, L, PER_LAYER), np.uint8, buffer=ls.buf)
    known = SenderLeases()
    try:
        while True:
            msg = q_in.get(timeout=60)
            if msg[0] == "handshake":
                known.learn(msg[1], msg[2])
            elif msg[0] == "ticket":
                known.add(msg[1], msg[2])
            elif msg[0] == "push":
                _, req, layer0, layer1, fill = msg
                target = known.find(req)
                if target is None:
                    q_out.put(("unknown", req))
                    continue
                _key, lane, seq = target
                lanes[lane, layer0:layer1] = fill                  # the request's bytes first
                for l in range(layer0, layer1):                     # then each layer's flag
                    flags[lane, l] = seq
                q_out.put(("pushed", req, lane, seq))
            elif msg[0] == "stop":
                return
    finally:
        del flags, lanes
        fs.close()
        ls.close()


def _host_receiver(flags):
    """A real NvlinkTransport whose bound cache and flags are host memory (construction makes
    no CUDA call; only the flag read is replaced)."""
    from rngd_pd import airm
    from rngd_pd.nvlink import LaneLeases
    t = airm.NvlinkTransport(device=torch.device("cuda", 0))
    K = torch.zeros((L, BCAP, NKV, S, HD), dtype=torch.bfloat16)
    t._cache = (K, torch.zeros_like(K), torch.from_numpy(flags))
    t.leases = LaneLeases(BCAP)
    for b in range(BCAP):
        t.leases.start_after(b, int(flags[b].max()))
    t._read_all_flags = lambda: flags.copy()
    return t


@pytest.fixture()
def pair():
    ctx = mp.get_context("spawn")
    fs = shared_memory.SharedMemory(create=True, size=BCAP * L * 8)
    ls = shared_memory.SharedMemory(create=True, size=BCAP * L * PER_LAYER)
    flags = np.ndarray((BCAP, L), np.int64, buffer=fs.buf)
    lanes = np.ndarray((BCAP, L, PER_LAYER), np.uint8, buffer=ls.buf)
    flags[:] = 0
    lanes[:] = 0
    q_in, q_out = ctx.Queue(), ctx.Queue()
    proc = ctx.Process(target=_sender, args=(fs.name, ls.name, q_in, q_out), daemon=True)
    proc.start()
    try:
        yield flags, lanes, q_in, q_out
    finally:
        q_in.put(("stop",))
        proc.join(30)
        if proc.is_alive():
            proc.kill()
        del flags, lanes
        fs.close()
        fs.unlink()
        ls.close()
        ls.unlink()


def _push(q_in, q_out, req, layer0, layer1, fill):
    q_in.put(("push", req, layer0, layer1, fill))
    return q_out.get(timeout=30)


def test_lease_handshake_push_and_stale_flags_across_processes(pair):
    flags, lanes, q_in, q_out = pair
    rx = _host_receiver(flags)
    t1 = rx.reserve("r1", 2)
    assert t1 == {"req": "r1", "lane": 2, "seq": 1}
    meta = rx.handshake_metadata()
    assert meta["leases"] == {"r1": [2, 1]} and meta["shape"] == [L, BCAP, NKV, S, HD]
    key = [meta["host"], meta["pid"], meta["device"], meta["ptrs"]["k"]]
    q_in.put(("handshake", key, meta["leases"]))

    assert not rx.arrived("r1")
    with pytest.raises(TimeoutError):
        rx.wait("r1", timeout=0.05)
    assert _push(q_in, q_out, "r1", 0, L, 7) == ("pushed", "r1", 2, 1)
    assert rx.wait("r1", timeout=5) < 5
    assert (lanes[2] == 7).all() and (flags[2] == 1).all() and not lanes[:2].any()

    # the lane's next lease: the flags still hold 1, which must not satisfy seq 2
    rx.release("r1")
    t2 = rx.reserve("r2", 2)
    assert t2["seq"] == 2
    assert not rx.arrived("r2")
    with pytest.raises(TimeoutError):
        rx.wait("r2", timeout=0.1)
    q_in.put(("ticket", key, t2))                                  # forwarded with the request
    assert _push(q_in, q_out, "r2", 0, L // 2, 9)[0] == "pushed"
    assert rx.arrived("r2", 0, L // 2) and not rx.arrived("r2")
    _push(q_in, q_out, "r2", L // 2, L, 9)
    assert rx.wait("r2", timeout=5) < 5 and (lanes[2] == 9).all()

    # several requests waited at once: one flag read per poll, complete only when both landed
    rx.release("r2")
    ta, tb = rx.reserve("ra", 0), rx.reserve("rb", 1)
    q_in.put(("ticket", key, ta))
    q_in.put(("ticket", key, tb))
    _push(q_in, q_out, "ra", 0, L, 3)
    assert not rx.arrived_all(["ra", "rb"]) and rx.arrived_all(["ra"])
    with pytest.raises(TimeoutError):
        rx.wait_all(["ra", "rb"], timeout=0.05)
    _push(q_in, q_out, "rb", 0, L, 4)
    assert rx.wait_all(["ra", "rb"], timeout=5) < 5
    assert (lanes[0] == 3).all() and (lanes[1] == 4).all()

    # a request the sender holds no lease for is refused, and nothing is written
    before = lanes.copy()
    assert _push(q_in, q_out, "nobody", 0, L, 1) == ("unknown", "nobody")
    assert np.array_equal(lanes, before)


def test_timeout_is_a_failed_transfer_result(pair):
    from rngd_pd import airm
    flags, _lanes, _q_in, _q_out = pair
    rx = _host_receiver(flags)
    tier = lambda n: airm.MemoryTier(n, "device-hbm", 1 << 34)
    layout = airm.KVLayout(num_layers=L, num_kv_heads=NKV, head_dim=HD, dtype="bf16")
    plan = rx.plan("r3", tier("gpu0"), tier("gpu1"), layout, layout, (0, S))
    rx.reserve("r3", 1)
    handle = airm.TransferHandle("r3", "nvlink", rx.book.add(airm._Ticket(plan, "r3", 0.0, (None, None, 0))))
    t0 = time.perf_counter()
    res = rx.wait(handle, timeout_s=0.1)
    assert not res.ok and res.nbytes == 0 and "did not arrive" in res.error
    assert time.perf_counter() - t0 < 5
    with pytest.raises(airm.TransportError):
        rx.wait(handle, timeout_s=0.1)                             # a handle is waited once


def test_lease_rules():
    from rngd_pd.nvlink import LaneLeases
    book = LaneLeases(2)
    book.start_after(1, 5)                                         # flags already at 5
    assert book.reserve("a", 1)["seq"] == 6
    with pytest.raises(ValueError):
        book.reserve("b", 1)                                       # one request per lane
    with pytest.raises(ValueError):
        book.reserve("a", 0)                                       # one lane per request
    with pytest.raises(IndexError):
        book.reserve("c", 2)
    with pytest.raises(KeyError):
        book.lookup("zzz")
    book.release("a")
    assert book.reserve("b", 1)["seq"] == 7
    assert LaneLeases.landed([7, 7, 6], 7, 0, 2) and not LaneLeases.landed([7, 7, 6], 7, 0, 3)
