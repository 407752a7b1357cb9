"""prefill_full parity on the B200 through the C ABI (FullPrefillEngine).

Small-dimension prompts across buckets against the numpy restatement of the
reference's cpu_layer_p (KV cache and last-token logits), the staged / streamed /
device entry points against each other, prefill -> decode on one card, and
BASELINE config 2 at full Llama-3.1-8B size against the C restatement (last-token
logits within 2e-2 max-abs, same next token, layer-0 KV within one bf16 ulp, every
layer's KV within 0.05 max-abs and 5e-3 mean-abs).
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
    return ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)


def _engine(C=128, S=256, group=1):
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(SMALL)
    return FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=C, group=group, S=S)


@pytest.fixture(scope="module")
def small():
    eng = _engine()
    eng.add_bucket(256)
    return eng, R.SynthModel(SMALL, seed=0)


@pytest.mark.parametrize("P", [1, 100, 128, 200, 256])
def test_small_prefill_matches_numpy_oracle(small, P):
    eng, m = small
    toks = [(7 * i + 3) % SMALL.V for i in range(P)]
    K, V, nxt = eng.prefill(toks)
    Kr, Vr, lgr = R.prefill(m, toks, eng.S, kv_bf16=True)
    np.testing.assert_allclose(K, Kr, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(V, Vr, rtol=1e-2, atol=1e-2)
    assert not K[..., P:].any() and not V[:, :, P:].any()          # zero past the prompt
    lg = eng.logits().cpu().numpy()
    np.testing.assert_allclose(lg, lgr, rtol=1e-3, atol=2e-3)
    assert nxt == int(np.argmax(lgr))
    assert eng.last_C == (128 if P <= 128 else 256)


WIDE = R.Dims(H=512, M=4864, NH=8, NKV=2, HD=128, L=2, V=1000)


@pytest.fixture(scope="module")
def wide():
    """A 512-token bucket over a model whose gate/up GEMM has 76 weight tiles: at C=512 it takes
    two weight tiles per work unit (the MT=2 epilogue) and every other GEMM one, the
    attention's last query tiles read four key chunks, and the O and down GEMMs (16 units over
    148 CTAs) cut units into up to ten pieces."""
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(WIDE)
    return FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=512, group=1, S=512), R.SynthModel(WIDE, seed=0)


@pytest.mark.parametrize("P", [300, 512])
def test_wide_512_token_bucket_matches_numpy_oracle(wide, P):
    eng, m = wide
    toks = [(13 * i + 7) % WIDE.V for i in range(P)]
    K, V, nxt = eng.prefill(toks)
    Kr, Vr, lgr = R.prefill(m, toks, eng.S, kv_bf16=True)
    np.testing.assert_allclose(K, Kr, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(V, Vr, rtol=1e-2, atol=1e-2)
    assert not K[..., P:].any() and not V[:, :, P:].any()
    lg = eng.logits().cpu().numpy()
    np.testing.assert_allclose(lg, lgr, rtol=1e-3, atol=2e-3)
    assert nxt == int(np.argmax(lgr))
    assert eng.last_C == 512


def test_stage_stream_and_device_paths_agree(small):
    eng, _ = small
    toks = [(11 * i + 5) % SMALL.V for i in range(150)]
    K, V, nxt = eng.prefill(toks)
    st = eng.begin_device_prefill(toks)
    while not st.advance(1):
        pass
    K2, V2, nxt2 = st.result()
    got = {}
    nxt3 = eng.prefill_stream(toks, lambda g, kh, vh: got.__setitem__(g, (kh, vh)))
    K3 = np.concatenate([got[g][0] for g in sorted(got)])
    V3 = np.concatenate([got[g][1] for g in sorted(got)])
    kv, nxt4 = eng.prefill_kv_device(toks)
    np.testing.assert_array_equal(K, K2.float().cpu().numpy())
    np.testing.assert_array_equal(V, V2.float().cpu().numpy())
    np.testing.assert_array_equal(K, K3)
    np.testing.assert_array_equal(V, V3)
    np.testing.assert_array_equal(K, kv[:, 0].transpose(-1, -2).float().cpu().numpy())
    assert nxt == nxt2 == nxt3 == nxt4


def test_prefill_then_decode_on_one_card(small):
    """prefill_device -> adopt_kv_device -> decode step equals the oracle's decode after its prefill."""
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    eng, m = small
    dec = BatchDecodeEngine(eng.cfg, eng.w, B=2, S=eng.S, group=1)
    p1 = [(3 * i + 1) % SMALL.V for i in range(40)]
    p2 = [(5 * i + 2) % SMALL.V for i in range(130)]
    K1, V1, n1 = eng.prefill_device(p1)
    K2, V2, n2 = eng.prefill_device(p2)
    Kd, Vd = dec.adopt_kv_device([K1, K2], [V1, V2])
    toks, pos = [n1, n2], [len(p1), len(p2)]
    dec.step(toks, pos, Kd, Vd)
    lg = dec.logits_bv().cpu().numpy()
    S = eng.S
    Ks = [np.zeros((2, SMALL.NKV, SMALL.HD, S), np.float32) for _ in range(SMALL.L)]
    Vs = [np.zeros((2, SMALL.NKV, S, SMALL.HD), np.float32) for _ in range(SMALL.L)]
    for b, p in enumerate((p1, p2)):
        Kr, Vr, lgr = R.prefill(m, p, S, kv_bf16=True)
        assert int(np.argmax(lgr)) == (n1, n2)[b]
        for l in range(SMALL.L):
            Ks[l][b], Vs[l][b] = Kr[l], Vr[l]
    ref = R.decode_step(m, toks, pos, Ks, Vs, S, kv_bf16=True)
    np.testing.assert_allclose(lg, ref, rtol=1e-3, atol=2e-3)


@pytest.mark.parametrize("C,N,K", [(128, 256, 512), (256, 384, 4096), (512, 128, 14336)])
def test_tc_gemm_tokens_matches_fp32(C, N, K):
    """The prefill tcgen05 GEMM (token tiles, hi/lo operand rows, stream-K) vs an fp64 matmul."""
    import ctypes
    from rngd_pd import _lib
    g = torch.Generator().manual_seed(C + N + K)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(C, K, generator=g)
    Y0 = torch.randn(C, N, generator=g)
    pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _lib.call("rngd_tc_gemm_tokens_workspace", N, K, C, ctypes.byref(pf), ctypes.byref(ct))
    act = torch.zeros(2 * C, K, dtype=torch.bfloat16, device="cuda")
    part = torch.zeros(max(pf.value, 1), device="cuda")
    cnt = torch.zeros(max(ct.value, 1), dtype=torch.int32, device="cuda")
    Wd = W.cuda()
    # each run has other inputs, so a piece of a split unit left by the previous run (older
    # epoch) that were taken for this run's would show up as an error
    for rep in range(3):
        Xr = X * (1.0 - 1.5 * rep) + 0.25 * rep
        want = Xr.double() @ W.double().T + Y0.double()
        Yd, Xd = Y0.clone().cuda(), Xr.cuda()
        _lib.call("rngd_tc_gemm_tokens", _lib.ptr(Wd), N, K, _lib.ptr(Xd), C, _lib.ptr(Yd), _lib.ptr(act),
                  _lib.ptr(part), _lib.ptr(cnt), 1, _lib.stream_handle())
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        scale = (Xr.double().abs() @ W.double().abs().T).max().item()
        err = (Yd.cpu().double() - want).abs().max().item()
        assert err <= 2e-6 * scale + 1e-6, f"max err {err} (scale {scale})"
        # split units advanced their epoch once per run and published their later pieces
        # under (tag 5, epoch); everything else is untouched
        assert set(cnt.cpu().tolist()) <= {0, rep + 1, (5 << 28) | (rep + 1)}


def test_prefill_rejects_bad_prompts(small):
    eng, _ = small
    with pytest.raises(ValueError):
        eng.prefill([1] * 300)                  # over the widest bucket (256)
    with pytest.raises(ValueError):
        eng.prefill([SMALL.V])                  # token outside the vocabulary


@pytest.mark.slow
def test_config2_full_prefill_C256(full_llama):
    """one 256-token prompt (ids U[0, V), seed 4) at full Llama-3.1-8B size."""
    from rngd_pd import synth
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    cfg, w, cm = full_llama
    eng = FullPrefillEngine(cfg, w, C=256, group=2, S=256)
    toks = synth.tokens(256, seed=4)
    kv, nxt = eng.prefill_kv_device(toks)
    lg = eng.logits().cpu().numpy()
    Kr, Vr, lgr, nxt_ref, _ = cm.prefill(toks, 256)
    err = float(np.abs(lg - lgr).max())
    assert err < 2e-2, f"last-token logits max-abs {err}"
    assert nxt == nxt_ref
    # KV: both sides round to bf16.  Layer 0 sees only one GEMM's summation-order noise, so its
    # values agree to the last bf16 bit but for rounding-boundary cases; each later layer feeds
    # the previous differences through 32 random-weight layers, which grow them steadily
    # (measured: mean |dKV| 1e-6 at layer 0, 2.3e-3 at layer 31, values of rms 1.27; max 0.031)
    Kd = kv[:, 0].transpose(-1, -2).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    Vd = kv[:, 1].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    for dev_bits, ref_bits in ((Kd, Kr), (Vd, Vr)):
        ulps0 = np.abs(_ordered(dev_bits[0]) - _ordered(ref_bits[0]))
        assert (ulps0 <= 1).mean() > 0.999, f"layer 0: {(ulps0 <= 1).mean():.5f} of KV values within one bf16 ulp"
        for l in range(cfg.n_layers):
            d = np.abs(sy.bf16_bits_to_f32(dev_bits[l]) - sy.bf16_bits_to_f32(ref_bits[l]))
            assert d.max() < 0.05, f"layer {l}: KV max-abs difference {d.max()}"
            assert d.mean() < 5e-3, f"layer {l}: KV mean-abs difference {d.mean()}"


def _ordered(bits):
    """bf16 bit patterns -> integers whose differences count ulps across zero."""
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def test_prefill_kv_fills_a_lane_like_the_reference_layout_copy(small):
    """write_slot_kv of a PrefillKV (the prefill-layout cache, moved by the handoff kernel on the
    engine's stream) writes the prompt's positions of the lane bit for bit as the reference-layout
    lane copy does, and leaves the lane's later positions and every other lane untouched."""
    from rngd_pd.engines.decode_batch import BatchDecodeEngine, PrefillKV
    eng, _ = small
    dec = BatchDecodeEngine(eng.cfg, eng.w, B=3, S=eng.S, group=1)
    P = 150
    toks = [(17 * i + 3) % SMALL.V for i in range(P)]
    kv, _nxt = eng.prefill_kv_device(toks)
    K, V = eng.reference_layout(kv)
    Ka, Va = dec.blank_kv()
    Kb, Vb = dec.blank_kv()
    for t in Ka + Va + Kb + Vb:
        t.fill_(7.0)                                   # what an earlier request left behind
    dec.write_slot_kv(Ka, Va, 1, K, V)
    dec.write_slot_kv(Kb, Vb, 1, PrefillKV(kv, P), None)
    torch.cuda.synchronize()
    bits = lambda t: t.contiguous().view(torch.int16)
    for ga, gb in zip(Ka + Va, Kb + Vb):
        assert torch.equal(bits(ga[:, 1, :, :P]), bits(gb[:, 1, :, :P]))
        assert bool((gb[:, 1, :, P:] == 7.0).all())
        assert bool((gb[:, 0] == 7.0).all()) and bool((gb[:, 2] == 7.0).all())
    with pytest.raises(ValueError):
        dec.write_slot_kv(Kb, Vb, 0, PrefillKV(kv[:1].contiguous(), P), None)   # wrong shape
