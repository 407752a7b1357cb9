"""The C restatement (full-size oracle) against the numpy restatement at small dims."""
import numpy as np
import pytest

from oracle import corc
from oracle import ref_np as R
from oracle import synth_np as sy

SMALL = R.Dims(H=256, M=384, NH=8, NKV=2, HD=32, L=2, V=300)


@pytest.mark.parametrize("seed,tid,start,n,sigma", [(0, 0, 0, 1000, 0.02), (7, 0x7001, 12345, 777, 1.0),
                                                     (2**40 + 3, 31 * 16 + 6, 2**33, 64, 0.02)])
def test_gauss_bits_c_equals_numpy(seed, tid, start, n, sigma):
    a = corc.gauss_bf16_bits(seed, tid, n, sigma, start)
    b = sy.gauss_bf16_bits(seed, tid, n, sigma, start)
    np.testing.assert_array_equal(a, b)


def test_gauss_distribution():
    x = sy.bf16_bits_to_f32(sy.gauss_bf16_bits(3, 9, 200000, 0.02))
    assert abs(x.mean()) < 2e-4 and abs(x.std() - 0.02) < 2e-4


def _np_lane_cache(d, S, B, seeds, lens):
    Ks = [np.zeros((B, d.NKV, d.HD, S), np.float32) for _ in range(d.L)]
    Vs = [np.zeros((B, d.NKV, S, d.HD), np.float32) for _ in range(d.L)]
    for b in range(B):
        K, V = R.synth_kv(d, S, seeds[b], lens[b])
        for l in range(d.L):
            Ks[l][b], Vs[l][b] = K[l], V[l]
    return Ks, Vs


def test_decode_steps_c_equals_numpy():
    d, S, B = SMALL, 16, 3
    seeds, lens = [101, 102, 103], [4, 9, 1]
    m = R.SynthModel(d, seed=0)
    cm = corc.CModel(d, seed=0)
    Kc, Vc = cm.new_cache(B, S)
    for b in range(B):
        cm.fill_lane(Kc, Vc, b, seeds[b], lens[b])
    Ks, Vs = _np_lane_cache(d, S, B, seeds, lens)
    np.testing.assert_array_equal(sy.bf16_bits_to_f32(Kc).transpose(0, 1, 2, 4, 3), np.stack(Ks))
    toks, pos = [5, 299, 17], list(lens)
    for _ in range(3):
        nxt, lg, _ = cm.decode_step(toks, pos, Kc, Vc)
        lg_ref = R.decode_step(m, toks, pos, Ks, Vs, S, kv_bf16=True)
        np.testing.assert_allclose(lg, lg_ref, rtol=1e-4, atol=1e-4)
        assert list(nxt) == R.greedy(lg_ref)
        toks, pos = list(nxt), [p + 1 for p in pos]
    Kn = sy.bf16_bits_to_f32(Kc).transpose(0, 1, 2, 4, 3)
    np.testing.assert_allclose(Kn, np.stack(Ks), rtol=1e-2, atol=1e-2)
    cm.close()


def test_prefill_c_equals_numpy():
    d, S = SMALL, 16
    toks = [7, 3, 250, 11, 42, 0, 299]
    m = R.SynthModel(d, seed=4)
    cm = corc.CModel(d, seed=4)
    K, V, lg, nxt, _ = cm.prefill(toks, S)
    Kr, Vr, lgr = R.prefill(m, toks, S, kv_bf16=True)
    np.testing.assert_allclose(sy.bf16_bits_to_f32(K), Kr, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(sy.bf16_bits_to_f32(V), Vr, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(lg, lgr, rtol=1e-4, atol=1e-4)
    assert nxt == int(np.argmax(lgr))
    cm.close()


def test_chunked_prefill_driver_matches_whole_prompt_prefill():
    """The restated chunked engine loop (engines/prefill_chunk.py:108-142) gives the same cache
    and logits as the whole-prompt prefill for one chunk and for several."""
    import numpy as np
    from oracle import ref_np as R
    d = R.Dims(H=256, M=512, NH=4, NKV=1, HD=128, L=2, V=300)
    m = R.SynthModel(d, seed=0)
    toks = [(7 * i + 3) % d.V for i in range(24)]
    K1, V1, l1 = R.prefill(m, toks, 32, kv_bf16=True)
    for C in (24, 8):
        K2, V2, l2 = R.prefill_chunked(m, toks, 32, C, kv_bf16=True)
        np.testing.assert_allclose(K2, K1, rtol=1e-2, atol=2e-3)
        np.testing.assert_allclose(V2, V1, rtol=1e-2, atol=2e-3)
        np.testing.assert_allclose(l2, l1, rtol=1e-4, atol=1e-4)


def test_given_rows_step_equals_the_plain_step_on_its_own_rows():
    """orc_decode_step_rows with the rows decode_step itself writes reproduces decode_step bit for
    bit, reports those rows, and leaves the caller's rows in place."""
    d, S, B = SMALL, 16, 2
    cm = corc.CModel(d, seed=0)
    Ka, Va = cm.new_cache(B, S)
    for b in range(B):
        cm.fill_lane(Ka, Va, b, 200 + b, 5 + b)
    Kb, Vb = Ka.copy(), Va.copy()
    toks, pos = [3, 77], [5, 6]
    nxt_a, lg_a, _ = cm.decode_step(toks, pos, Ka, Va)
    for b in range(B):                                   # the rows step A wrote, put in by hand
        Kb[:, b, :, pos[b]] = Ka[:, b, :, pos[b]]
        Vb[:, b, :, pos[b]] = Va[:, b, :, pos[b]]
    nxt_b, lg_b, own_k, own_v = cm.decode_step_given_rows(toks, pos, Kb, Vb)
    np.testing.assert_array_equal(lg_a, lg_b)
    assert list(nxt_a) == list(nxt_b)
    for b in range(B):
        np.testing.assert_array_equal(own_k[:, b], Ka[:, b, :, pos[b]])
        np.testing.assert_array_equal(own_v[:, b], Va[:, b, :, pos[b]])
    Kc, Vc = Kb.copy(), Vb.copy()
    Kc[:, 0, :, pos[0]] = 0                              # different rows are used as given
    _, lg_c, own_c, _ = cm.decode_step_given_rows(toks, pos, Kc, Vc)
    assert not (Kc[:, 0, :, pos[0]]).any() and not np.array_equal(lg_c, lg_a)
    np.testing.assert_array_equal(own_c[:, 1], own_k[:, 1])
    cm.close()
