import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def tiny_cfg():
    from witchcraft_b200.synth import T5Config
    return T5Config(vocab_size=512, d_model=256, d_ff=512, num_heads=4, num_layers=2)


@pytest.fixture(scope="session")
def tiny_model(tiny_cfg):
    from witchcraft_b200.synth import make_synthetic_model
    g = np.load(os.path.join(GOLDEN, "t5_tiny_golden.npz"))
    return make_synthetic_model(tiny_cfg, seed=int(g["seed"]))


@pytest.fixture(scope="session")
def xtr_model():
    """Full XTR-base shape (12 x 768, d_ff 2048, vocab 32128), seed 0."""
    from witchcraft_b200.synth import make_synthetic_model
    return make_synthetic_model(seed=0)


@pytest.fixture(scope="session")
def cuda_lib():
    from witchcraft_b200._lib import lib
    return lib()
