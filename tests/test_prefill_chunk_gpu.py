"""Chunked prefill against a live cache on the B200 (ChunkPrefillEngine, the reference's
engines/prefill_chunk.py:36-142): one decode step of C streams sharing one cache lane per
chunk, checked against the numpy restatement of the reference's chunked layer
(kernels/prefill_chunk.py:198-232) driven the way its engine drives it.
"""
import numpy as np
import pytest

from oracle import ref_np as R

pytestmark = pytest.mark.gpu

SMALL = R.Dims(H=512, M=1024, NH=8, NKV=2, HD=128, L=2, V=1000)
S = 256


def _cfg(d):
    from rngd_pd.engines.model import ModelConfig
    return ModelConfig.from_dims(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=d.L, V=d.V, eps=d.eps, theta=d.theta)


@pytest.fixture(scope="module")
def model():
    return R.SynthModel(SMALL, seed=0)


def _engine(C, group=1):
    from rngd_pd.engines.prefill_chunk import ChunkPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(SMALL)
    return ChunkPrefillEngine(cfg, SyntheticState(cfg, seed=0), S=S, C=C, group=group, chip=0)


@pytest.mark.parametrize("C,P", [(16, 1), (16, 16), (16, 37), (16, 100), (8, 61), (1, 5)])
def test_chunk_prefill_matches_numpy_oracle(model, C, P):
    from rngd_pd import _lib
    eng = _engine(C)
    toks = [(7 * i + 3) % SMALL.V for i in range(P)]
    K, V, nxt = eng.prefill(toks)
    assert _lib.device_status() == 0
    Kr, Vr, lgr = R.prefill_chunked(model, toks, S, C, kv_bf16=True)
    np.testing.assert_allclose(K, Kr, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(V, Vr, rtol=1e-2, atol=1e-2)
    end = P + (-P) % C                     # the pad positions are written too, nothing past them
    assert not K[..., end:].any() and not V[:, :, end:].any()
    assert nxt == int(np.argmax(lgr))


def test_chunk_prefill_equals_whole_prompt_prefill(model):
    """Chunks of 16 and one whole-prompt pass build the same cache (the two reference engines
    compute the same function of the prompt)."""
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.synth import SyntheticState
    cfg = _cfg(SMALL)
    full = FullPrefillEngine(cfg, SyntheticState(cfg, seed=0), C=128, group=1, S=S)
    toks = [(5 * i + 1) % SMALL.V for i in range(96)]   # a whole number of chunks: no pad rows
    Kc, Vc, nc = _engine(16).prefill(toks)
    Kf, Vf, nf = full.prefill(toks)
    np.testing.assert_allclose(Kc, Kf, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(Vc, Vf, rtol=1e-2, atol=1e-2)
    assert nc == nf


def test_chunk_prefill_rejects_bad_prompts():
    eng = _engine(16)
    with pytest.raises(ValueError):
        eng.prefill([1] * (S + 1))
    with pytest.raises(ValueError):
        eng.prefill([])
    with pytest.raises(ValueError):
        _engine(17)
