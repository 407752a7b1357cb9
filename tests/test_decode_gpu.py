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


@pytest.mark.parametrize("S,positions", [(256, [0, 5, 127, 128, 255]), (512, [300, 511, 1]),
                                         (1024, [700, 1023, 0, 129])])
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


def test_host_kv_intake_round_trips_and_pads_by_repeating_the_last():
    """The host-KV intake of the reference's decode worker (engines/decode_batch.py:305-351):
    load_kv = upload_prepared_kv(prepare_kv(...)) places request b in lane b and fills the
    lanes past the last request with copies of it; download_kv / upload_kv round-trip the
    resident cache bit for bit; stage_host_kv casts float32 host arrays to bf16; write_slot_kv
    replaces one lane."""
    from rngd_pd import synth
    eng = _small_engine(3, 128)
    cfg = eng.cfg
    reqs = [synth.request_kv(cfg, 128, 300 + i, 20 + 30 * i) for i in range(2)]
    host = [(k.float().cpu().numpy(), v.float().cpu().numpy()) for k, v in reqs]   # [nl, NKV, HD|S, S|HD]
    Kd, Vd = eng.load_kv([h[0] for h in host], [h[1] for h in host])
    K, V = eng.download_kv(Kd, Vd)                        # [nl, B, NKV, HD, S] / [nl, B, NKV, S, HD]
    for lane, src in ((0, 0), (1, 1), (2, 1)):            # lane 2: the last request repeated
        np.testing.assert_array_equal(K[:, lane], host[src][0])
        np.testing.assert_array_equal(V[:, lane], host[src][1])
    prepared = eng.prepare_kv([h[0] for h in host], [h[1] for h in host])
    Kd2, Vd2 = eng.upload_prepared_kv(prepared)
    for a, b in zip(Kd + Vd, Kd2 + Vd2):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    Kd3, Vd3 = eng.upload_kv(K, V)
    for a, b in zip(Kd + Vd, Kd3 + Vd3):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    Ks, Vs = eng.stage_host_kv(K, V)
    assert Ks.dtype == torch.bfloat16 and not Ks.is_cuda
    np.testing.assert_array_equal(Ks.float().numpy(), K)
    new_k, new_v = synth.request_kv(cfg, 128, 999, 50)
    eng.write_slot_kv(Kd, Vd, 1, new_k, new_v)
    K4, V4 = eng.download_kv(Kd, Vd)
    np.testing.assert_array_equal(K4[:, 1], new_k.float().cpu().numpy())
    np.testing.assert_array_equal(V4[:, 0], host[0][1])


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


def _parity_log(name, record):
    """Write a parity record as JSON into $RNGD_PARITY_LOG (a directory) when it is set."""
    import json
    import os
    out = os.environ.get("RNGD_PARITY_LOG")
    if out:
        os.makedirs(out, exist_ok=True)
        with open(os.path.join(out, name), "w") as f:
            json.dump(record, f, indent=1)


def _device_rows(Kd, Vd, pos):
    """The K/V rows a device step just wrote (position pos[b] of lane b, every layer and kv
    head) as bf16 bits [L][B][NKV][HD], the layout of the C oracle's cache rows."""
    B = len(pos)
    lanes = torch.arange(B, device=Kd[0].device)
    at = torch.tensor(pos, device=Kd[0].device)
    rk = [kg[:, lanes, :, at, :].transpose(0, 1) for kg in Kd]          # each [NG, B, NKV, HD]
    rv = [vg[:, lanes, :, at, :].transpose(0, 1) for vg in Vd]
    bits = lambda rows: torch.cat(rows, 0).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return bits(rk), bits(rv)


def _bf16_rows_close(a, b):
    """K/V rows [L][B][NKV][HD] as bf16 bits: (all elements close, max |a - b| / rms of the row).

    Two fp32 computations of the same row (different summation orders over K = 4096..14336
    terms, 32 layers deep) differ by a small fraction of the row's scale, and rounding each to
    bf16 then differs by at most one unit in the last place -- except for elements near zero,
    where that same absolute difference spans more units.  Close: |a - b| <= one bf16 ulp of
    the larger magnitude (2^-7 relative bounds it) + 2^-9 of the row's rms."""
    fa = (a.astype(np.uint32) << 16).view(np.float32)
    fb = (b.astype(np.uint32) << 16).view(np.float32)
    rms = np.sqrt(np.mean(fb.astype(np.float64) ** 2, axis=-1, keepdims=True)).astype(np.float32)
    d = np.abs(fa - fb)
    ok = d <= np.maximum(np.abs(fa), np.abs(fb)) * 2.0 ** -7 + rms * 2.0 ** -9
    return bool(ok.all()), float((d / np.maximum(rms, 1e-30)).max())


@pytest.mark.slow
def test_config4_B16_128_steps_per_step_parity(full_llama):
    """B=16 streams, past lengths U[64, 384] (seed 3) so that 128 more steps
    fit in S=512, seeded bf16 KV ~N(0,1), token ids U[0, V) (seed 2), 128 steps through the
    public step() API against the CPU fp32 oracle, teacher-forced as the reference's own check
    is (bench/teacher_forced.py: both sides consume the oracle's token each step).

    Each step is checked on its own: the device steps first, the K/V rows it wrote are put into
    the oracle's cache, and the oracle steps over that cache keeping those rows and reporting
    the rows it computes itself.  So both sides read identical bits at every cache position,
    and two things are measured per step: (a) the device's new K/V rows against the oracle's,
    each element within one bf16 ulp plus 2^-9 of its row's rms (_bf16_rows_close); (b) the
    logits within 2e-2 max-abs (north_star's per-step bound).  A greedy choice may still differ where the oracle's top two are closer than that
    bound can separate: with both logit vectors within e = 2e-2, the device can prefer the
    oracle's runner-up only if the oracle's gap is at most 2e = 4e-2; each such flip is checked
    against that fixed bound and recorded."""
    from rngd_pd import synth
    cfg, w, cm = full_llama
    B, S, steps, tol = 16, 512, 128, 2e-2
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
    errs, flips, row_same, row_close, row_dev = [], [], [], [], []
    for step in range(steps):
        nxt_dev, Kd, Vd = eng.step(cur, pos, Kd, Vd)
        lg_dev = eng.logits_bv().cpu().numpy()
        dk, dv = _device_rows(Kd, Vd, pos)
        for b in range(B):
            Kc[:, b, :, pos[b]] = dk[:, b]
            Vc[:, b, :, pos[b]] = dv[:, b]
        nxt_ref, lg_ref, ok_, ov_ = cm.decode_step_given_rows(cur, pos, Kc, Vc)
        row_same.append(float(np.mean(np.concatenate([(dk == ok_).ravel(), (dv == ov_).ravel()]))))
        (ck, dk_rel), (cv, dv_rel) = _bf16_rows_close(dk, ok_), _bf16_rows_close(dv, ov_)
        row_close.append(ck and cv)
        row_dev.append(max(dk_rel, dv_rel))
        diff = np.abs(lg_dev - lg_ref)
        errs.append(float(diff.max()))
        for b in range(B):
            r, d = int(nxt_ref[b]), int(nxt_dev[b])
            if r != d:
                flips.append({"step": step, "stream": b, "oracle": r, "device": d,
                              "gap": float(lg_ref[b][r] - lg_ref[b][d]), "row_err": float(diff[b].max())})
        cur, pos = [int(t) for t in nxt_ref], [p + 1 for p in pos]
    _parity_log("config4_teacher_forced.json",
                {"steps": steps, "streams": B, "tol": tol, "max_err": max(errs), "mean_err": float(np.mean(errs)),
                 "per_step_max_err": [round(e, 6) for e in errs], "kv_rows_bit_identical": float(np.mean(row_same)),
                 "kv_rows_min_identical_step": min(row_same), "kv_rows_close_all_steps": all(row_close),
                 "kv_rows_max_dev_over_rms": max(row_dev),
                 "decisions": steps * B, "flips": flips})
    assert all(row_close), f"K/V rows not close at steps {[i for i, c in enumerate(row_close) if not c]}"
    worst = int(np.argmax(errs))
    assert errs[worst] < tol, f"step {worst}: logits max-abs {errs[worst]} >= {tol}"
    for f in flips:
        assert f["gap"] <= 2 * tol, f"not a near tie: {f}"


@pytest.mark.slow
def test_config4_free_running_first_divergence(full_llama):
    """Config 4 free-running, as the reference's bench/teacher_forced.py reports it: device and
    oracle each feed back their own greedy tokens and keep their own caches for 128 steps; the
    first step where a stream's tokens differ is recorded with the oracle's gap between its
    choice and the device's.  Random-init logits are 128256 draws of similar size, so their
    top two often lie within fp32 summation-order noise; a divergence must be such a near tie
    (the device's token is the oracle's runner-up, less than 0.1 below its maximum, against a
    typical top-two spacing of ~0.3 here)."""
    from rngd_pd import synth
    cfg, w, cm = full_llama
    B, S, steps = 16, 512, 128
    lens = synth.context_lengths(B)
    eng = _engine_with(cfg, w, B, S)
    Ks, Vs = zip(*[synth.request_kv(cfg, S, 100 + b, lens[b]) for b in range(B)])
    Kd, Vd = eng.adopt_kv_device(list(Ks), list(Vs))
    del Ks, Vs
    Kc, Vc = cm.new_cache(B, S)
    for b in range(B):
        cm.fill_lane(Kc, Vc, b, 100 + b, lens[b])
    dev_tok = ref_tok = synth.tokens(B, seed=2)
    pos = list(lens)
    first = None
    agree_steps = 0
    for step in range(steps):
        nxt_ref, lg_ref, _ = cm.decode_step(ref_tok, pos, Kc, Vc)
        nxt_dev, Kd, Vd = eng.step(dev_tok, pos, Kd, Vd)
        nxt_ref = [int(t) for t in nxt_ref]
        if first is None:
            bad = [b for b in range(B) if nxt_ref[b] != nxt_dev[b]]
            if bad:
                b = bad[0]
                order = np.argsort(-lg_ref[b])
                first = {"step": step, "stream": b, "oracle": nxt_ref[b], "device": nxt_dev[b],
                         "gap": float(lg_ref[b][nxt_ref[b]] - lg_ref[b][nxt_dev[b]]),
                         "device_rank_in_oracle": int(np.where(order == nxt_dev[b])[0][0]),
                         "streams_diverging": len(bad)}
            else:
                agree_steps += 1
        dev_tok, ref_tok, pos = nxt_dev, nxt_ref, [p + 1 for p in pos]
    _parity_log("config4_free_running.json", {"steps": steps, "streams": B, "identical_steps": agree_steps,
                                               "first_divergence": first})
    if first is not None:
        assert first["device_rank_in_oracle"] == 1 and first["gap"] < 0.1, f"divergence is not a near tie: {first}"

