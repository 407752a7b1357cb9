"""The reference's kernel-module names (src/rngd_pd/kernels/decode_batch.py, prefill_full.py,
prefill_chunk.py) over the B200 C ABI: DecodeModel, PrefillModel and ChunkModel called with
the reference's graph inputs (transposed projections, q pre-scaled by 1/sqrt(HD), norms tiled
and scaled by sqrt(H), eps*H and nh = -0.5, rotation / mask / one-hot rows), checked against
the oracle's restatement of the reference's cpu_layer / cpu_layer_p / chunked cpu_layer on
the same weights.  The CPU part checks names, tables and argument validation."""
import math

import numpy as np
import pytest
import torch

from oracle import ref_np as R

SMALL = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
BF = torch.bfloat16


# ------------------------------------------------------------------ CPU: names, tables, checks
def test_names_and_constants():
    from rngd_pd.kernels import decode_batch as D, prefill_chunk as C, prefill_full as P
    for mod in (D, P, C):
        assert (mod.H, mod.M, mod.NH, mod.NKV, mod.HD, mod.G) == (4096, 14336, 32, 8, 128, 4)
        assert mod.BF is torch.bfloat16
    assert isinstance(D.HINT, str) and D.MAX_SHAPES == {}
    assert issubclass(D.DecodeModel, torch.nn.Module) and issubclass(P.PrefillModel, torch.nn.Module)
    assert issubclass(C.ChunkModel, torch.nn.Module)


def test_rotation_tables_equal_the_reference_restatement():
    from rngd_pd.kernels import decode_batch as D, prefill_chunk as C, prefill_full as P
    inv = R.inv_freq(R.LLAMA8B)
    pos = [0, 1, 77, 300, 511]
    np.testing.assert_array_equal(D.rot_batch(inv, pos), R.rot_batch(inv, pos))
    np.testing.assert_array_equal(P.rot_matrices(inv, 9), R.rot_batch(inv, np.arange(9)))
    np.testing.assert_array_equal(C.rot_matrices(inv, 40, 8), R.rot_batch(inv, np.arange(40, 48, dtype=np.float32)))


def test_constructor_limits():
    from rngd_pd.kernels.decode_batch import DecodeModel
    from rngd_pd.kernels.prefill_chunk import ChunkModel
    from rngd_pd.kernels.prefill_full import PrefillModel
    with pytest.raises(ValueError):
        DecodeModel(17, 512, 2)
    with pytest.raises(ValueError):
        DecodeModel(4, 500, 2)
    with pytest.raises(ValueError):
        PrefillModel(100, 2)
    with pytest.raises(ValueError):
        ChunkModel(32, 512, 2)


def test_host_tensors_are_refused():
    from rngd_pd.kernels.decode_batch import DecodeModel
    m = DecodeModel(2, 128, 1)
    with pytest.raises(ValueError, match="CUDA"):
        m(torch.zeros(2, 512, dtype=BF), *([None] * 16))


# ------------------------------------------------------------------ GPU parity
def _reference_inputs(m, layers, rows, dev):
    """The reference engines' graph inputs for `layers` of the synthetic model, and the
    weights those inputs stand for in the oracle's [out, in] form (q un-scaled and the norms
    un-tiled the way the kernels read them back)."""
    d = m.d
    sh, shd = math.sqrt(d.H), math.sqrt(d.HD)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))
    an1, aq, ak, av, ao, an2, awg, awu, awd, ws = [], [], [], [], [], [], [], [], [], []
    for i in layers:
        n1, wq, wk, wv, wo, n2, wgu, wd = m.layer(i)
        q_in = t(wq.T / shd).to(BF)
        an1.append(t(np.tile(n1 * sh, (rows, 1))).to(BF))
        an2.append(t(np.tile(n2 * sh, (rows, 1))).to(BF))
        aq.append(q_in)
        ak.append(t(wk.T).to(BF))
        av.append(t(wv.T).to(BF))
        ao.append(t(wo.T).to(BF))
        awg.append(t(wgu[:d.M].T).to(BF))
        awu.append(t(wgu[d.M:].T).to(BF))
        awd.append(t(wd.T).to(BF))
        n_eff = lambda a: (a[0].float() / sh).numpy()
        wq_eff = (q_in.float() * shd).to(BF).float().numpy().T
        ws.append((n_eff(an1[-1]), wq_eff, wk, wv, wo, n_eff(an2[-1]), wgu, wd))
    stack = lambda xs: torch.stack(xs).to(dev)
    eps = torch.full((rows, d.H), d.eps * d.H, dtype=torch.float32, device=dev)
    nh = torch.full((rows, d.H), -0.5, dtype=torch.float32, device=dev)
    args = (eps, nh, stack(an1), stack(aq), stack(ak), stack(av), stack(ao), stack(an2), stack(awg), stack(awu),
            stack(awd))
    return args, ws


def _close(got, want, tol):
    got = got.float().cpu().numpy() if torch.is_tensor(got) else got
    err = np.abs(got - want).max() / max(1.0, np.abs(want).max())
    assert err < tol, f"max scaled error {err:.3e} >= {tol}"


@pytest.mark.gpu
def test_decode_model_matches_cpu_layer():
    from rngd_pd.kernels.decode_batch import DecodeModel, rot_batch
    d, dev = SMALL, torch.device("cuda", 0)
    m = R.SynthModel(d, seed=0)
    B, S, nl = 3, 256, 2
    pos = [17, 130, 255]
    args, ws = _reference_inputs(m, range(nl), B, dev)
    x = m.embed()[[5, 77, 901]].astype(np.float32)
    Kp = np.zeros((nl, B, d.NKV, d.HD, S), np.float32)
    Vp = np.zeros((nl, B, d.NKV, S, d.HD), np.float32)
    for b in range(B):
        K, V = R.synth_kv(d, S, 100 + b, pos[b])
        Kp[:, b], Vp[:, b] = K, V
    inv = R.inv_freq(d)
    rot = torch.from_numpy(rot_batch(inv, pos)).to(BF).to(dev)
    mask = torch.full((B, S), -1e4, dtype=torch.float32)
    oh = torch.zeros((B, S), dtype=torch.float32)
    for b, p in enumerate(pos):
        mask[b, :p + 1] = 0.0
        oh[b, p] = 1.0
    model = DecodeModel(B, S, nl)
    xd = torch.from_numpy(x).to(BF).to(dev)
    out, Kf, Vf = model(xd, *args, torch.from_numpy(Kp).to(BF).to(dev), torch.from_numpy(Vp).to(BF).to(dev),
                        rot, mask.to(BF).to(dev), oh.to(BF).to(dev))
    torch.cuda.synchronize()
    xr, Kr, Vr = torch.from_numpy(x).to(BF).float().numpy(), Kp.copy(), Vp.copy()
    for l in range(nl):
        xr, Kr[l], Vr[l] = R.cpu_layer(xr, ws[l], Kr[l], Vr[l], inv, pos, S, d.eps, d, kv_bf16=True)
    assert out.dtype == BF and tuple(out.shape) == (B, d.H)
    _close(out, xr, 2e-2)
    _close(Kf, Kr, 2e-2)
    _close(Vf, Vr, 2e-2)
    # the step writes only each stream's own slot: everything else is the input cache
    for b, p in enumerate(pos):
        keep = np.ones(S, bool)
        keep[p] = False
        np.testing.assert_array_equal(Kf[:, b][..., keep].float().cpu().numpy(), Kp[:, b][..., keep])
    # a second call with the same weights reuses the packed group
    model(xd, *args, torch.from_numpy(Kp).to(BF).to(dev), torch.from_numpy(Vp).to(BF).to(dev), rot,
          mask.to(BF).to(dev), oh.to(BF).to(dev))
    assert len(model._packs._groups) == 1


@pytest.mark.gpu
def test_decode_model_refuses_inputs_outside_the_decode_step():
    from rngd_pd.kernels.decode_batch import DecodeModel, rot_batch
    d, dev = SMALL, torch.device("cuda", 0)
    m = R.SynthModel(d, seed=0)
    B, S, nl = 2, 128, 1
    args, _ = _reference_inputs(m, range(nl), B, dev)
    pos = [3, 9]
    rot = torch.from_numpy(rot_batch(R.inv_freq(d), pos)).to(BF).to(dev)
    mask = torch.full((B, S), -1e4, device=dev)
    oh = torch.zeros((B, S), device=dev)
    for b, p in enumerate(pos):
        mask[b, :p + 1] = 0
        oh[b, p] = 1
    K = torch.zeros((nl, B, d.NKV, d.HD, S), dtype=BF, device=dev)
    V = torch.zeros((nl, B, d.NKV, S, d.HD), dtype=BF, device=dev)
    x = torch.zeros((B, d.H), dtype=BF, device=dev)
    model = DecodeModel(B, S, nl)
    model(x, *args, K, V, rot, mask, oh)                      # the contract: accepted
    bad_oh = oh.clone()
    bad_oh[0, 4] = 1
    with pytest.raises(ValueError, match="one-hot"):
        model(x, *args, K, V, rot, mask, bad_oh)
    with pytest.raises(ValueError, match="rotation"):
        model(x, *args, K, V, torch.from_numpy(rot_batch(R.inv_freq(d), [4, 9])).to(BF).to(dev), mask, oh)
    full = K.clone()
    full[0, 1, 0, 0, 9] = 1.0
    with pytest.raises(ValueError, match="empty K slot"):
        model(x, *args, full, V, rot, mask, oh)


@pytest.mark.gpu
def test_prefill_model_matches_cpu_layer_p():
    from rngd_pd.kernels.prefill_full import PrefillModel, rot_matrices
    d, dev = SMALL, torch.device("cuda", 0)
    m = R.SynthModel(d, seed=0)
    C, nl = 128, 2
    args, ws = _reference_inputs(m, range(nl), C, dev)
    toks = [(7 * i + 3) % d.V for i in range(C)]
    x = torch.from_numpy(m.embed()[toks].astype(np.float32)).to(BF)
    inv = R.inv_freq(d)
    causal = np.triu(np.full((C, C), -1e4, np.float32), 1)
    mask = torch.from_numpy(np.tile(causal, (d.G, 1)).reshape(1, d.G * C, C)).to(BF).to(dev)
    rot = torch.from_numpy(rot_matrices(inv, C)).to(BF).to(dev)
    out, kT, vT = PrefillModel(C, nl)(x.to(dev), *args, rot, mask)
    torch.cuda.synchronize()
    xr = x.float().numpy()
    for l in range(nl):
        xr, kr, vr = R.cpu_layer_p(xr, ws[l], inv, C, d.eps, d, kv_bf16=True)
        _close(kT[l], kr, 2e-2)
        _close(vT[l], vr, 2e-2)
    assert tuple(kT.shape) == (nl, d.NKV, d.HD, C) and tuple(vT.shape) == (nl, d.NKV, C, d.HD)
    _close(out, xr, 2e-2)


@pytest.mark.gpu
def test_chunk_model_matches_chunked_cpu_layer():
    from rngd_pd.kernels.prefill_chunk import ChunkModel, rot_matrices
    d, dev = SMALL, torch.device("cuda", 0)
    m = R.SynthModel(d, seed=0)
    C, S, nl, base = 8, 256, 2, 40
    args, ws = _reference_inputs(m, range(nl), C, dev)
    K, V = R.synth_kv(d, S, 7, base)                  # earlier chunks' positions 0..base-1
    toks = [(11 * i + 5) % d.V for i in range(C)]
    x = torch.from_numpy(m.embed()[toks].astype(np.float32)).to(BF)
    inv = R.inv_freq(d)
    ohK = np.zeros((C, S), np.float32)
    mk = np.full((C, S), -1e4, np.float32)
    for c in range(C):
        ohK[c, base + c] = 1.0
        mk[c, :base + c + 1] = 0.0
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(BF).to(dev)
    out, Kf, Vf = ChunkModel(C, S, nl)(x.to(dev), *args, dv(K[:nl]), dv(V[:nl]),
                                       dv(rot_matrices(inv, base, C)), dv(ohK), dv(ohK.T),
                                       dv(np.tile(mk, (d.G, 1)).reshape(1, d.G * C, S)))
    torch.cuda.synchronize()
    xr, Kr, Vr = x.float().numpy(), K[:nl].copy(), V[:nl].copy()
    for l in range(nl):
        xr, Kr[l], Vr[l] = R.cpu_layer_chunk(xr, ws[l], Kr[l], Vr[l], inv, base, C, S, d.eps, d, kv_bf16=True)
    _close(out, xr, 2e-2)
    _close(Kf, Kr, 2e-2)
    _close(Vf, Vr, 2e-2)
