"""The oracle restatement against the reference's own CPU functions (golden fixtures).

Fixtures come from tests/golden/make_golden.py, which runs the reference's
cpu_layer / cpu_layer_p / chunked cpu_layer / rot_batch / GenericRuntime /
ser on the same seeded inputs rebuilt here.
"""
import numpy as np
import pytest

from oracle import ref_np as R
from oracle import synth_np as sy
from tests.golden import make_golden as MG


def _close(a, b, rtol=2e-6, atol=2e-6):
    np.testing.assert_allclose(a, b, rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", ["decode_small", "decode_full"])
def test_decode_layer_matches_reference(golden, name):
    d, B, S, pos, seed = MG.DECODE_CASES[name]
    w = MG.layer_weights(d, seed, 0.05)
    x, K, V = MG.decode_inputs(d, B, S, pos, seed)
    x2, K2, V2 = R.cpu_layer(x, w, K, V, R.inv_freq(d), list(pos), S, d.eps, d)
    _close(x2, golden[name + "/x"])
    _close(np.stack([K2[b, :, :, p] for b, p in enumerate(pos)]), golden[name + "/kcol"])
    _close(np.stack([V2[b, :, p, :] for b, p in enumerate(pos)]), golden[name + "/vrow"])
    _close(R.rot_batch(R.inv_freq(d), np.asarray(pos), d.HD), golden[name + "/rot"], 0, 0)


@pytest.mark.parametrize("name", ["prefill_small", "prefill_full"])
def test_prefill_layer_matches_reference(golden, name):
    d, C, seed = MG.PREFILL_CASES[name]
    w = MG.layer_weights(d, seed, 0.05)
    x = MG.prefill_inputs(d, C, seed)
    x2, kT, vT = R.cpu_layer_p(x, w, R.inv_freq(d), C, d.eps, d)
    _close(x2, golden[name + "/x"])
    _close(kT, golden[name + "/kT"])
    _close(vT, golden[name + "/vT"])


def test_chunk_layer_matches_reference(golden):
    d, C, S, base, seed = MG.CHUNK_CASES["chunk_small"]
    w = MG.layer_weights(d, seed, 0.05)
    x, K, V = MG.chunk_inputs(d, C, S, base, seed)
    x2, Kf, Vf = R.cpu_layer_chunk(x, w, K, V, R.inv_freq(d), base, C, S, d.eps, d)
    _close(x2, golden["chunk_small/x"])
    _close(Kf, golden["chunk_small/K"])
    _close(Vf, golden["chunk_small/V"])


def test_bf16_kv_rounding_is_small(golden):
    """kv_bf16 (what the device stores) moves the layer output by bf16-rounding noise only."""
    d, B, S, pos, seed = MG.DECODE_CASES["decode_small"]
    w = MG.layer_weights(d, seed, 0.05)
    x, K, V = MG.decode_inputs(d, B, S, pos, seed)
    x2, K2, _ = R.cpu_layer(x, w, K, V, R.inv_freq(d), list(pos), S, d.eps, d, kv_bf16=True)
    ref = golden["decode_small/x"]
    assert np.abs(x2 - ref).max() < 2e-2 * np.abs(ref).max()
    col = np.stack([K2[b, :, :, p] for b, p in enumerate(pos)])
    np.testing.assert_array_equal(col, sy.bf16_round(col))


def test_generic_runtime_greedy(golden):
    """B=1 greedy generation through the batched decode restatement equals GenericRuntime."""
    g = MG.GENERIC
    d = g["dims"]
    m = R.SynthModel(d, seed=g["seed"])
    np.testing.assert_array_equal(R.inv_freq(d), golden["generic/inv"])
    S = 32
    Ks = [np.zeros((1, d.NKV, d.HD, S), np.float32) for _ in range(d.L)]
    Vs = [np.zeros((1, d.NKV, S, d.HD), np.float32) for _ in range(d.L)]
    tf, gen, tok = [], [], None
    for p, t in enumerate(g["prompt"]):
        lg = R.decode_step(m, [t], [p], Ks, Vs, S, kv_bf16=False)
        tf.append(R.greedy(lg)[0])
    tok, p = tf[-1], len(g["prompt"])
    gen.append(tok)
    for _ in range(g["n_new"] - 1):
        tok = R.greedy(R.decode_step(m, [tok], [p], Ks, Vs, S, kv_bf16=False))[0]
        gen.append(tok)
        p += 1
    assert tf == list(golden["generic/tf"])
    assert gen == list(golden["generic/gen"])


def test_prefill_then_decode_equals_token_by_token():
    """The prefill restatement's cache equals feeding the prompt one decode step at a time."""
    d = MG.SMALL
    m = R.SynthModel(d, seed=5)
    S, toks = 16, [7, 3, 250, 11, 42]
    K, V, lg = R.prefill(m, toks, S, kv_bf16=True)
    Ks = [np.zeros((1, d.NKV, d.HD, S), np.float32) for _ in range(d.L)]
    Vs = [np.zeros((1, d.NKV, S, d.HD), np.float32) for _ in range(d.L)]
    for p, t in enumerate(toks):
        lg2 = R.decode_step(m, [t], [p], Ks, Vs, S, kv_bf16=True)
    np.testing.assert_allclose(np.stack([k[0] for k in Ks]), K, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(lg2[0], lg, rtol=1e-4, atol=1e-4)
