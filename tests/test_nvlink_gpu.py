"""The `nvlink` KV transport on one B200: the fused handoff kernel moves a request's
prefill-layout cache [L][2][NKV][S][HD] into a leased lane of the decode cache
[L][Bcap][NKV][S][HD] byte for byte, publishes per-layer flags under the lease's sequence
number, and the connector / rm-core entry points built on it.  Sender and receiver share
one GPU here, so arrival is observed by host polling; the device-side wait runs only on a
flag already set (arrival) or on one nothing sets (its bounded timeout).  Cross-GPU and
cross-process handoffs are in test_nvlink_multi_gpu.py."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

L, BCAP, NKV, S, HD = 4, 3, 2, 256, 128
BF = torch.bfloat16


def _kv(seed, layers=L):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((layers, 2, NKV, S, HD), generator=g).to(BF).cuda()


def _bits(t):
    return t.contiguous().view(torch.int16)


@pytest.fixture()
def rx():
    from rngd_pd.nvlink import NvlinkTransport
    t = NvlinkTransport(0)
    K = torch.zeros((L, BCAP, NKV, S, HD), dtype=BF, device="cuda")
    V = torch.zeros_like(K)
    t.bind_cache(K, V)
    yield t, K, V
    t.close()


def test_push_device_lands_byte_exact_in_the_leased_lane(rx):
    t, K, V = rx
    tk = t.reserve("r1", 1)
    kv = _kv(1)
    assert t.push_device("r1", kv) == kv.numel() * 2
    t.wait("r1", timeout=5)
    assert torch.equal(_bits(K[:, 1]), _bits(kv[:, 0])) and torch.equal(_bits(V[:, 1]), _bits(kv[:, 1]))
    assert not K[:, 0].any() and not K[:, 2].any() and not V[:, 0].any() and not V[:, 2].any()
    flags = t._cache[2].cpu()
    assert flags[1].tolist() == [tk["seq"]] * L and not flags[0].any() and not flags[2].any()


@pytest.mark.parametrize("tokens", [1, 77, 200])
def test_prompt_positions_only(rx, tokens):
    """tokens=P moves positions [0, P) of every head; the rest of the lane keeps what it held."""
    t, K, V = rx
    K[:, 0].fill_(3.0)
    V[:, 0].fill_(-3.0)
    t.reserve("p", 0)
    kv = _kv(10 + tokens)
    assert t.push_device("p", kv, tokens=tokens) == L * 2 * NKV * tokens * HD * 2
    t.wait("p", timeout=5)
    assert torch.equal(_bits(K[:, 0, :, :tokens]), _bits(kv[:, 0, :, :tokens]))
    assert torch.equal(_bits(V[:, 0, :, :tokens]), _bits(kv[:, 1, :, :tokens]))
    assert (K[:, 0, :, tokens:] == 3.0).all() and (V[:, 0, :, tokens:] == -3.0).all()
    assert not K[:, 1:].any()


def test_push_many_one_launch_per_sixteen_requests():
    """push_many: 20 requests with different prompt lengths into 20 lanes (two launches of the
    batched kernel); every lane byte-exact, every lease's flags published."""
    from rngd_pd.nvlink import NvlinkTransport
    Lb, Bb, Sb = 2, 20, 128
    t = NvlinkTransport(0)
    K = torch.zeros((Lb, Bb, NKV, Sb, HD), dtype=BF, device="cuda")
    V = torch.zeros_like(K)
    t.bind_cache(K, V)
    g = torch.Generator().manual_seed(99)
    kvs = [torch.randn((Lb, 2, NKV, Sb, HD), generator=g).to(BF).cuda() for _ in range(Bb)]
    toks = [1 + (17 * b) % Sb for b in range(Bb)]
    items = []
    for b in range(Bb):
        t.reserve(f"q{b}", Bb - 1 - b)
        items.append((f"q{b}", kvs[b], toks[b]))
    moved = t.push_many(items)
    assert moved == sum(Lb * 2 * NKV * n * HD * 2 for n in toks)
    for b in range(Bb):
        t.wait(f"q{b}", timeout=5)
        lane, n = Bb - 1 - b, toks[b]
        assert torch.equal(_bits(K[:, lane, :, :n]), _bits(kvs[b][:, 0, :, :n]))
        assert torch.equal(_bits(V[:, lane, :, :n]), _bits(kvs[b][:, 1, :, :n]))
        assert not K[:, lane, :, n:].any() and not V[:, lane, :, n:].any()
    t.close()


def test_batched_entry_point_rejects_bad_batches(rx):
    from rngd_pd import _lib
    t, K, V = rx
    kv = _kv(21)
    done = torch.zeros(16, dtype=torch.int32, device="cuda")
    st = _lib.stream_handle(torch.cuda.current_stream())

    def call(items, n=None):
        arr = (_lib.KvItem * max(len(items), 1))(*items)
        return _lib.call("rngd_kv_handoff_batch", arr, len(items) if n is None else n, 2 * NKV * S * HD,
                         _lib.ptr(K), _lib.ptr(V), L, NKV, S, HD, BCAP, 0, L, _lib.ptr(done),
                         _lib.ptr(t._cache[2]), st)

    it = lambda lane, tokens=S: _lib.KvItem(kv.data_ptr(), kv[:, 1].data_ptr(), lane, tokens, 1)
    for bad in ([], [it(0), it(0)], [it(0, 0)], [it(0, S + 1)], [it(BCAP)]):
        with pytest.raises(_lib.RngdError):
            call(bad)
    with pytest.raises(_lib.RngdError):
        call([it(0)] * 17, n=17)
    torch.cuda.synchronize()
    assert not K.any() and not t._cache[2].any()   # nothing was launched


def test_layer_blocks_single_layers_and_partial_wait(rx):
    t, K, V = rx
    t.reserve("r", 0)
    kv = _kv(2)
    t.push_device("r", kv[0:2].contiguous(), layer0=0, layer1=2)
    t.wait("r", 0, 2, timeout=5)
    assert not t.arrived("r", 2, 4)
    with pytest.raises(TimeoutError):
        t.wait("r", 2, 4, timeout=0.2)
    for l in (2, 3):
        t.push_layer("r", l, kv[l, 0].contiguous(), kv[l, 1].contiguous())
    t.wait("r", timeout=5)
    assert torch.equal(_bits(K[:, 0]), _bits(kv[:, 0])) and torch.equal(_bits(V[:, 0]), _bits(kv[:, 1]))


def test_a_stale_flag_never_satisfies_a_new_lease(rx):
    t, K, V = rx
    t.reserve("old", 2)
    t.push_device("old", _kv(3))
    t.wait("old", timeout=5)
    t.release("old")
    t.reserve("new", 2)
    with pytest.raises(TimeoutError):
        t.wait("new", timeout=0.2)
    kv = _kv(4)
    t.push_device("new", kv)
    t.wait("new", timeout=5)
    assert torch.equal(_bits(K[:, 2]), _bits(kv[:, 0]))
    with pytest.raises(ValueError):
        t.reserve("again", 2)


def test_device_wait_reports_arrival_and_bounded_timeout(rx):
    """rngd_kv_wait: a flag already published -> status 0; a flag nothing sets -> its bounded
    wait gives up and reports a timeout through host-mapped memory; the context stays usable."""
    t, K, V = rx
    remote = 1 if t.device.index != 1 else 0     # declared sender GPU (not this one)
    t.reserve("a", 0, sender_device=remote)
    kv = _kv(5)
    t.push_device("a", kv)
    t.wait("a", timeout=5)
    s = torch.cuda.Stream()
    assert t.wait_stream("a", s, timeout=1.0)(block=True) is True
    t.reserve("b", 1, sender_device=remote)
    outcome = t.wait_stream("b", s, timeout=0.3)
    with pytest.raises(TimeoutError):
        outcome(block=True)
    s.synchronize()
    kv2 = _kv(6)
    t.push_device("b", kv2)
    t.wait("b", timeout=5)
    assert torch.equal(_bits(K[:, 1]), _bits(kv2[:, 0]))


def test_connector_device_path_per_layer(rx):
    from rngd_pd.connector.rngd_kv import KVConnectorRole, RngdKVConnector
    t, K, V = rx
    dec = RngdKVConnector(KVConnectorRole.WORKER, req_id="q", transport=t, n_layers=L)
    dec.register_kv_caches((K, V))
    t.reserve("q", 2)
    pf = RngdKVConnector(KVConnectorRole.WORKER, req_id="q", transport=t, n_layers=L)
    kv = _kv(7)
    for i in range(L):
        pf.save_kv_layer(f"layer.{i}", (kv[i, 0], kv[i, 1]))
    pf.wait_for_save()
    dec.start_load_kv()
    for i in range(L):
        k, v = dec.wait_for_layer_load(f"layer.{i}")
        assert torch.equal(_bits(k), _bits(kv[i, 0])) and torch.equal(_bits(v), _bits(kv[i, 1]))


def test_registry_resolves_nvlink_to_one_shared_instance():
    from rngd_pd import airm
    from rngd_pd.connector import transport as tr
    tr._SHARED.pop("nvlink", None)
    a, b = tr.select_transport("nvlink"), tr.select_transport("nvlink")
    assert a is b and isinstance(a, airm.NvlinkTransport) and isinstance(a, tr.Transport)
    with pytest.raises(airm.TransportError):
        a.push("k", b"bytes")
    with pytest.raises(airm.TransportError):
        a.pull("k", timeout=0)
    tr._SHARED.pop("nvlink", None)
    a.close()


def test_rm_core_plan_submit_wait_take():
    from rngd_pd import airm
    t = airm.NvlinkTransport(0)
    K = torch.zeros((L, BCAP, NKV, S, HD), dtype=BF, device="cuda")
    V = torch.zeros_like(K)
    t.bind_cache(K, V)
    t.reserve("a", 0)
    src = airm.MemoryTier("gpu0-prefill", "device-hbm", 1 << 34)
    dst = airm.MemoryTier("gpu0-decode", "device-hbm", 1 << 34)
    layout = airm.KVLayout(num_layers=L, num_kv_heads=NKV, head_dim=HD, dtype="bf16")
    plan = t.plan("a", src, dst, layout, layout, (0, S))
    kv = _kv(8)
    assert plan.nbytes == kv.numel() * 2
    res = t.wait(t.submit(plan, kv), timeout_s=5)
    assert res.ok and res.nbytes == plan.nbytes and res.seconds > 0
    Kl, Vl = t.take(plan)
    assert torch.equal(_bits(Kl), _bits(kv[:, 0])) and torch.equal(_bits(Vl), _bits(kv[:, 1]))
    summ = airm.summarize_transfers(t.measurements)
    assert summ["kv_transfer_gbps"] > 0 and summ["kv_transfer_ms"] > 0
    host = airm.MemoryTier("host", "host-dram", 1 << 34)
    with pytest.raises(airm.TransportError):
        t.plan("a", host, dst, layout, layout, (0, S))
    with pytest.raises(airm.TransportError):
        t.plan("a", src, dst, airm.KVLayout(L, NKV, HD, "fp16"), airm.KVLayout(L, NKV, HD, "fp16"), (0, S))
    with pytest.raises(airm.ContractError):
        t.submit(plan, None)
    with pytest.raises(airm.TransportError):
        t.take(plan)
    t.close()


def test_bad_arguments_fail_loudly(rx):
    from rngd_pd import _lib
    t, K, V = rx
    with pytest.raises(IndexError):
        t.reserve("x", BCAP)
    with pytest.raises(KeyError):
        t.push_device("nobody", _kv(9))
    t.reserve("x", 0)
    with pytest.raises(ValueError):
        t.push_device("x", _kv(9)[:, :, :, :128].contiguous())
    with pytest.raises(ValueError):
        t.push_device("x", _kv(9).float())
    with pytest.raises(ValueError):
        t.wait("x", 0, L + 1, timeout=0.1)
    with pytest.raises(ValueError):
        t.bind_cache(K[:, :2], V)
    kv = _kv(9)
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.RngdError):   # lane outside the cache: refused on the host, nothing launched
        _lib.call("rngd_kv_handoff", _lib.ptr(kv), _lib.ptr(kv[:, 1]), 2 * NKV * S * HD, _lib.ptr(K), _lib.ptr(V),
                  L, NKV, S, HD, S, BCAP, BCAP, 0, L, _lib.ptr(done), _lib.ptr(t._cache[2]), 1,
                  _lib.stream_handle(torch.cuda.current_stream()))
    with pytest.raises(_lib.RngdError):   # more tokens than the cache holds
        _lib.call("rngd_kv_handoff", _lib.ptr(kv), _lib.ptr(kv[:, 1]), 2 * NKV * S * HD, _lib.ptr(K), _lib.ptr(V),
                  L, NKV, S, HD, S + 1, 0, BCAP, 0, L, _lib.ptr(done), _lib.ptr(t._cache[2]), 1,
                  _lib.stream_handle(torch.cuda.current_stream()))
    with pytest.raises(_lib.RngdError):   # layer range outside [0, L)
        _lib.call("rngd_kv_handoff", _lib.ptr(kv), _lib.ptr(kv[:, 1]), 2 * NKV * S * HD, _lib.ptr(K), _lib.ptr(V),
                  L, NKV, S, HD, S, 0, BCAP, 2, L + 1, _lib.ptr(done), _lib.ptr(t._cache[2]), 1,
                  _lib.stream_handle(torch.cuda.current_stream()))


SMALL = dict(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)


def test_prefill_handoff_then_decode_equals_local_adoption():
    """prefill_kv_device -> nvlink push of the prompt positions into decode lanes -> decode step
    gives the same lanes and the same logits, bit for bit, as handing the same prompts' caches over
    with adopt_kv_device (whose tail past the prompt is zero, like a blank lane's)."""
    from oracle import ref_np as R
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.nvlink import NvlinkTransport
    from rngd_pd.synth import SyntheticState
    d = R.Dims(**SMALL)
    cfg = ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)
    pf = FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=256, group=1, S=256)
    dec = BatchDecodeEngine(cfg, pf.w, B=2, S=256, group=1)
    p1 = [(3 * i + 1) % d.V for i in range(40)]
    p2 = [(5 * i + 2) % d.V for i in range(130)]

    Kd, Vd = dec.blank_kv()
    t = NvlinkTransport(0)
    t.bind_cache(*dec.full_kv(Kd, Vd))
    nxt = []
    for b, p in enumerate((p1, p2)):
        t.reserve(f"p{b}", b)
        kv, n = pf.prefill_kv_device(p)
        t.push_device(f"p{b}", kv, stream=pf.stream, tokens=len(p))
        nxt.append(n)
    for b in range(2):
        t.wait(f"p{b}", timeout=5)
    toks, pos = nxt, [len(p1), len(p2)]
    dec.step(toks, pos, Kd, Vd)
    got = dec.logits_bv().clone()

    K1, V1, n1 = pf.prefill_device(p1)
    K2, V2, n2 = pf.prefill_device(p2)
    assert [n1, n2] == nxt
    Ka, Va = dec.adopt_kv_device([K1, K2], [V1, V2])
    dec.step(toks, pos, Ka, Va)            # also writes the new token's K/V at `pos`, as it did in Kd
    assert torch.equal(got, dec.logits_bv())
    for g in range(len(Kd)):
        assert torch.equal(_bits(Kd[g]), _bits(Ka[g])) and torch.equal(_bits(Vd[g]), _bits(Va[g]))
    t.close()


def test_ipc_cache_allocation_is_usable_by_the_engine():
    """blank_kv(ipc=True): the resident cache lives in IPC-exportable memory, and the
    transport publishes its handles for a prefill process to map."""
    from oracle import ref_np as R
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.nvlink import NvlinkTransport
    from rngd_pd.synth import SyntheticState
    d = R.Dims(**SMALL)
    cfg = ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)
    dec = BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=2, S=256, group=1)
    Kd, Vd = dec.blank_kv(ipc=True)
    assert not any(k.any() for k in Kd)
    t = NvlinkTransport(0)
    t.bind_cache(*dec.full_kv(Kd, Vd))
    meta = t.handshake_metadata()
    assert all(meta["handles"][n] for n in ("k", "v", "flags"))
    dec.step([1, 2], [0, 5], Kd, Vd)
    assert torch.isfinite(dec.logits_bv()).all()
    t.close()


def test_push_many_with_a_layer_block_and_wait_all(rx):
    """push_many of three requests in one launch -- a whole cache, another whole cache, and a
    layer block [1, 3) of a third -- lands byte-exact; wait_all sees all three with one flag
    read per poll, and a request whose layers have not all landed is not reported as arrived."""
    t, K, V = rx
    kv = [_kv(20 + i) for i in range(3)]
    for i in range(3):
        t.reserve(f"m{i}", i)
    blk = kv[2][1:3].contiguous()
    t.push_many([("m0", kv[0], None), ("m1", kv[1], None)])
    t.push_many([("m2", blk, None)], layer0=1, layer1=3)
    t.wait_all(["m0", "m1"], timeout=5)
    t.wait_all(["m2"], layer0=1, layer1=3, timeout=5)
    assert not t.arrived_all(["m0", "m2"])             # m2's layers 0 and 3 were never pushed
    for i in range(2):
        assert torch.equal(_bits(K[:, i]), _bits(kv[i][:, 0])) and torch.equal(_bits(V[:, i]), _bits(kv[i][:, 1]))
    assert torch.equal(_bits(K[1:3, 2]), _bits(blk[:, 0])) and not K[0, 2].any() and not K[3, 2].any()
    with pytest.raises(TimeoutError):
        t.wait_all(["m2"], timeout=0.05)
