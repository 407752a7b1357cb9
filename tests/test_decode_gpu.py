"""Decode parity on the B200 through the C ABI (BatchDecodeEngine and kernel-level ops).

Checks: device synthetic generator == oracle generator bit for bit; GEMV,
rmsnorm and attention kernels vs numpy fp32; a small-dimension model's logits
and greedy tokens vs the numpy restatement; BASELINE config 1 at full
Llama-3.1-8B size vs the C restatement (logits within 2e-2 max-abs, 64 greedy
steps identical); a lane's result independent of the batch it rides in.
"""
import numpy as np
import pytest
import torch

from oracle import ref_np as R
from oracle import synth_np as sy

pytestmark = pytest.mark.gpu

SMALL = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)


def _cfg(d):
    from rngd_pd.engines.model import ModelConfig
    return ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps,
                                 theta=d.theta)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_synth_bits_match_oracle():
    from rngd_pd import synth
    for seed, tid, start, n, sigma in [(0, 5, 0, 100_000, 0.02), (9, 0x7001, 2**33 + 7, 4099, 1.0)]:
        t = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        synth.fill_gauss(t, seed, tid, sigma, start)
        np.testing.assert_array_equal(_bits(t), sy.gauss_bf16_bits(seed, tid, n, sigma, start))
    ids = synth.uniform_i32(1000, 2, synth.T_TOKENS, 128256).cpu().numpy()
    np.testing.assert_array_equal(ids, sy.uniform_ints(2, sy.T_TOKENS, 1000, 128256))


@pytest.mark.parametrize("B,N,K", [(1, 37, 264), (3, 300, 512), (5, 129, 1024), (16, 64, 4096)])
def test_gemv_matches_fp32(B, N, K):
    from rngd_pd import _lib
    g = torch.Generator().manual_seed(N * K + B)
    W = torch.randn(N, K, generator=g).to(torch.bfloat16)
    X = torch.randn(B, K, generator=g)
    Y0 = torch.randn(B, N, generator=g)
    ref = (W.float() @ X.T).T
    Wd, Xd = W.cuda(), X.cuda()
    for acc in (0, 1):
        Yd = Y0.clone().cuda()
        _lib.call("rngd_gemv_bf16", _lib.ptr(Wd), N, K, _lib.ptr(Xd), K, B, _lib.ptr(Yd), N, acc,
                  _lib.stream_handle())
        torch.cuda.synchronize()
        want = ref + (Y0 if acc else 0)
        np.testing.assert_allclose(Yd.cpu().numpy(), want.numpy(), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("B,N,K", [(1, 128, 64), (4, 256, 512), (16, 384, 4096), (16, 4096, 14336),
                                   (3, 28672, 4096)])
def test_tc_gemv_matches_fp32(B, N, K):
    """tcgen05 GEMV (hi/lo bf16 operand, TMEM fp32 accumulation, split-K) vs fp32 matmul."""
    import ctypes
    from rngd_pd import _lib
    g = torch.Generator().manual_seed(N + K + B)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(B, K, generator=g)
    Y0 = torch.randn(B, N, generator=g)
    pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _lib.call("rngd_tc_gemv_workspace", N, K, ctypes.byref(pf), ctypes.byref(ct))
    act = torch.zeros(32, K, dtype=torch.bfloat16, device="cuda")
    part = torch.zeros(max(pf.value, 1), device="cuda")
    cnt = torch.zeros(max(ct.value, 1), dtype=torch.int32, device="cuda")
    Wd = W.cuda()
    # each run has other inputs, so a split-tile piece left by the previous run (older epoch)
    # that were taken for this run's would show up as an error
    for rep in range(3):
        Xr = X * (1.0 - 1.5 * rep) + 0.25 * rep
        want = (W.double() @ Xr.double().T).T + Y0.double()
        Yd, Xd = Y0.clone().cuda(), Xr.cuda()
        _lib.call("rngd_tc_gemv", _lib.ptr(Wd), N, K, _lib.ptr(Xd), K, B, _lib.ptr(Yd), N, _lib.ptr(act),
                  _lib.ptr(part), _lib.ptr(cnt), 1, _lib.stream_handle())
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        got = Yd.cpu().double()
        scale = (W.double().abs() @ Xr.double().abs().T).T.max().item()
        err = (got - want).abs().max().item()
        assert err <= 2e-6 * scale + 1e-6, f"max err {err} (scale {scale})"
        # split tiles advanced their epoch once per run; whole tiles never touch theirs
        assert set(cnt.cpu().tolist()) <= {0, rep + 1}


def test_rmsnorm_matches_reference_formula():
    from rngd_pd import _lib
    x = torch.randn(5, 4096) * 3
    w = torch.rand(4096) + 0.5
    xd, wd, od = x.cuda(), w.cuda(), torch.empty(5, 4096, device="cuda")
    _lib.call("rngd_rmsnorm_f32", _lib.ptr(xd), 5, 4096, _lib.ptr(wd), 1e-5, _lib.ptr(od), _lib.stream_handle())
    torch.cuda.synchronize()
    ref = R.rms(x.numpy(), w.numpy(), 1e-5)
    np.testing.assert_allclose(od.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("S,positions", [(256, [0, 5, 127, 128, 255]), (512, [300, 511, 1])])
def test_attention_matches_numpy(S, positions):
    from rngd_pd import _lib
    B, NKV, NH, HD = len(positions), 2, 8, 128
    g = torch.Generator().manual_seed(S)
    q = torch.randn(B, NH * HD, generator=g)
    K = torch.randn(B, NKV, S, HD, generator=g).to(torch.bfloat16)
    V = torch.randn(B, NKV, S, HD, generator=g).to(torch.bfloat16)
    pos = torch.tensor(positions, dtype=torch.int32)
    part = torch.empty(B, NH, S // 128, HD + 2, device="cuda")
    ao = torch.empty(B, NH * HD, device="cuda")
    qd, Kd, Vd, pd = q.cuda(), K.cuda(), V.cuda(), pos.cuda()
    _lib.call("rngd_attn_decode", _lib.ptr(qd), _lib.ptr(Kd), _lib.ptr(Vd), _lib.ptr(pd), B, B, NH, NKV, HD, S,
              _lib.ptr(part), _lib.ptr(ao), _lib.stream_handle())
    torch.cuda.synchronize()
    Kf, Vf, qn = K.float().numpy(), V.float().numpy(), q.numpy().reshape(B, NKV, NH // NKV, HD)
    for b, p in enumerate(positions):
        sc = np.einsum("kgh,ksh->kgs", qn[b], Kf[b][:, :p + 1]) / np.sqrt(HD)
        sc -= sc.max(-1, keepdims=True)
        pr = np.exp(sc)
        pr /= pr.sum(-1, keepdims=True)
        want = np.einsum("kgs,ksh->kgh", pr, Vf[b][:, :p + 1]).reshape(-1)
        np.testing.assert_allclose(ao[b].cpu().numpy(), want, rtol=1e-4, atol=1e-5)


def _small_engine(B, S, share=None):
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(SMALL)
    return BatchDecodeEngine(cfg, SyntheticState(cfg, seed=0), B=B, S=S, group=1, chip=0, share=share)


def test_small_model_steps_match_numpy_oracle():
    from rngd_pd import synth
    d, B, S = SMALL, 3, 256
    eng = _small_engine(B, S)
    lens = [10, 130, 255 - 8]
    Ks_dev, Vs_dev, Ks, Vs = [], [], [], []
    for b in range(B):
        K, V = synth.request_kv(eng.cfg, S, 100 + b, lens[b])
        Ks_dev.append(K)
        Vs_dev.append(V)
    Kd, Vd = eng.adopt_kv_device(Ks_dev, Vs_dev)
    m = R.SynthModel(d, seed=0)
    Kn = [np.zeros((B, d.NKV, d.HD, S), np.float32) for _ in range(d.L)]
    Vn = [np.zeros((B, d.NKV, S, d.HD), np.float32) for _ in range(d.L)]
    for b in range(B):
        K, V = R.synth_kv(d, S, 100 + b, lens[b])
        for l in range(d.L):
            Kn[l][b], Vn[l][b] = K[l], V[l]
    toks, pos = [1, 999, 500], list(lens)
    for step in range(8):
        lg_dev, Kd, Vd = eng.step_logits(toks, pos, Kd, Vd)
        lg = eng.logits_bv().cpu().numpy()
        lg_ref = R.decode_step(m, toks, pos, Kn, Vn, S, kv_bf16=True)
        np.testing.assert_allclose(lg, lg_ref, rtol=1e-3, atol=2e-3)
        nxt = [int(i) for i in lg.argmax(-1)]
        assert nxt == R.greedy(lg_ref), f"step {step}"
        toks, pos = nxt, [p + 1 for p in pos]
    # the device cache, read back in the reference layout, equals the oracle's
    Kh, Vh = eng.download_kv(Kd, Vd)
    np.testing.assert_allclose(Kh, np.stack(Kn), rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(Vh, np.stack(Vn), rtol=2e-2, atol=2e-2)


def test_step_api_tokens_and_graph_replay():
    """step() (CUDA-graph replay) and step_logits() (same graph) agree; greedy_tokens works."""
    from rngd_pd.engines.decode_batch import greedy_tokens
    eng = _small_engine(2, 128)
    Kd, Vd = eng.blank_kv()
    lg, Kd, Vd = eng.step_logits([3, 4], [0, 0], Kd, Vd)
    want = greedy_tokens(lg, eng.Vp, eng.V, eng.B)
    Kd2, Vd2 = eng.blank_kv()
    got, _, _ = eng.step([3, 4], [0, 0], Kd2, Vd2)
    assert got == want


def test_lane_result_independent_of_batch():
    """A stream's logits are bit-identical whether it runs alone or among 4 (batch invariance)."""
    from rngd_pd import synth
    e4 = _small_engine(4, 256)
    e1 = _small_engine(1, 256, share=e4)
    K, V = synth.request_kv(e4.cfg, 256, 77, 40)
    others = [synth.request_kv(e4.cfg, 256, 78 + i, 90 + 30 * i) for i in range(3)]
    Kd4, Vd4 = e4.adopt_kv_device([K] + [o[0] for o in others], [V] + [o[1] for o in others])
    Kd1, Vd1 = e1.adopt_kv_device([K], [V])
    t4, p4, t1, p1 = [11, 12, 13, 14], [40, 90, 120, 150], [11], [40]
    for _ in range(4):
        t4, Kd4, Vd4 = e4.step(t4, p4, Kd4, Vd4)
        l4 = e4.logits_bv()[0].clone()
        t1, Kd1, Vd1 = e1.step(t1, p1, Kd1, Vd1)
        assert torch.equal(l4, e1.logits_bv()[0])
        assert t4[0] == t1[0]
        p4, p1 = [p + 1 for p in p4], [p1[0] + 1]


def test_bad_inputs_raise():
    eng = _small_engine(2, 128)
    Kd, Vd = eng.blank_kv()
    with pytest.raises(ValueError):
        eng.step([1, 2], [0, 128], Kd, Vd)          # position outside the cache
    with pytest.raises(ValueError):
        eng.step([1, 5000], [0, 0], Kd, Vd)         # token outside the vocabulary
    with pytest.raises(IndexError):
        eng.write_slot_kv(Kd, Vd, 2, np.zeros((2, 2, 128, 128)), np.zeros((2, 2, 128, 128)))


# ---------------------------------------------------------------- full size
def _engine_with(cfg, w, B, S):
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    return BatchDecodeEngine(cfg, w, B=B, S=S, group=8)


@pytest.mark.slow
def test_config1_full_llama_logits_and_64_greedy_steps(full_llama):
    """B=4, 256 past tokens of seeded bf16 KV ~N(0,1) each, token ids U[0,V)
    (seed 2); logits within 2e-2 max-abs, then 64 greedy steps identical to the CPU fp32 oracle."""
    from rngd_pd import synth
    cfg, w, cm = full_llama
    B, S, past = 4, 512, 256
    eng = _engine_with(cfg, w, B, S)
    Ks, Vs = zip(*[synth.request_kv(cfg, S, 100 + b, past) for b in range(B)])
    Kd, Vd = eng.adopt_kv_device(list(Ks), list(Vs))
    Kc, Vc = cm.new_cache(B, S)
    for b in range(B):
        cm.fill_lane(Kc, Vc, b, 100 + b, past)
    toks = synth.tokens(B, seed=2)
    pos = [past] * B
    lg_dev, Kd, Vd = eng.step_logits(toks, pos, Kd, Vd)
    nxt_ref, lg_ref, _ = cm.decode_step(toks, pos, Kc, Vc)
    lg = eng.logits_bv().cpu().numpy()
    err = float(np.abs(lg - lg_ref).max())
    assert err < 2e-2, f"logits max-abs {err}"
    dev_tokens, ref_tokens = [], []
    cur_d, cur_r = [int(i) for i in lg.argmax(-1)], [int(i) for i in nxt_ref]
    assert cur_d == cur_r
    for step in range(63):
        pos = [p + 1 for p in pos]
        cur_d, Kd, Vd = eng.step(cur_d, pos, Kd, Vd)
        cur_r = [int(i) for i in cm.decode_step(cur_r, pos, Kc, Vc, want_logits=False)[0]]
        dev_tokens.append(cur_d)
        ref_tokens.append(cur_r)
        assert cur_d == cur_r, f"greedy tokens diverge at step {step + 1}"


@pytest.mark.slow
def test_config4_B16_128_greedy_steps(full_llama):
    """B=16 streams, past lengths U[64, 384] (seed 3) so that 128 more steps
    fit in S=512, seeded bf16 KV ~N(0,1), token ids U[0, V) (seed 2), 128 greedy steps against
    the CPU fp32 oracle, teacher-forced as the reference's own check is (both sides consume the
    oracle's token each step, bench/teacher_forced.py), through the public step() API.

    With random-init weights the top two of 128256 logits are often very close, so over 2048
    argmax decisions fp32-level differences (summation order) are expected to flip a few near
    ties.  Checked: the first step's logits within 2e-2 max-abs (the config-1 bar); every
    step's within 0.1 (bf16 K/V entries that round one ulp apart accumulate in both caches, so
    the difference grows with the steps); each device choice is the oracle's argmax or a token
    the oracle scores within twice that row's logit difference of its maximum (a genuine near
    tie); and such flips are at most 1% of the decisions."""
    from rngd_pd import synth
    cfg, w, cm = full_llama
    B, S, steps = 16, 512, 128
    lens = synth.context_lengths(B)
    assert min(lens) >= 64 and max(lens) + steps <= S
    eng = _engine_with(cfg, w, B, S)
    Ks, Vs = zip(*[synth.request_kv(cfg, S, 100 + b, lens[b]) for b in range(B)])
    Kd, Vd = eng.adopt_kv_device(list(Ks), list(Vs))
    del Ks, Vs
    Kc, Vc = cm.new_cache(B, S)
    for b in range(B):
        cm.fill_lane(Kc, Vc, b, 100 + b, lens[b])
    cur, pos = synth.tokens(B, seed=2), list(lens)
    ties, errs = [], []
    for step in range(steps):
        nxt_ref, lg_ref, _ = cm.decode_step(cur, pos, Kc, Vc)
        nxt_dev, Kd, Vd = eng.step(cur, pos, Kd, Vd)
        diff = np.abs(eng.logits_bv().cpu().numpy() - lg_ref)
        errs.append(float(diff.max()))
        for b in range(B):
            r, d = int(nxt_ref[b]), int(nxt_dev[b])
            if r == d:
                continue
            gap = float(lg_ref[b][r] - lg_ref[b][d])
            row = float(diff[b].max())
            assert gap <= 2 * row, f"step {step} stream {b}: device {d} vs oracle {r}, gap {gap} > 2 x {row}"
            ties.append((step, b, round(gap, 5)))
        cur, pos = [int(t) for t in nxt_ref], [p + 1 for p in pos]
    assert errs[0] < 2e-2, f"first-step logits max-abs {errs[0]}"
    assert max(errs) < 0.1, f"logits max-abs {max(errs)} at step {int(np.argmax(errs))}"
    assert len(ties) <= 0.01 * steps * B, f"{len(ties)} near-tie flips in {steps * B} decisions: {ties}"
