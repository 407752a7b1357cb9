import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "rngd-pd_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: full-size case that runs for more than a few seconds")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "reference_golden.npz"))


@pytest.fixture(scope="session")
def full_llama():
    """Llama-3.1-8B-shaped synthetic model (seed 0): device weights + the C oracle's copy."""
    import torch
    from oracle import corc
    from oracle import ref_np as R
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.weights import DeviceWeights
    from rngd_pd.synth import SyntheticState
    cfg = ModelConfig.llama31_8b()
    w = DeviceWeights(cfg, SyntheticState(cfg, seed=0), torch.device("cuda", 0))
    cm = corc.CModel(R.LLAMA8B, seed=0)
    yield cfg, w, cm
    cm.close()
