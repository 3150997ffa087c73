import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libthvm_sm100.so")


@pytest.fixture(scope="session")
def golden_ops():
    return dict(np.load(GOLDEN / "ops.npz"))


@pytest.fixture(scope="session")
def golden_gpt2():
    return dict(np.load(GOLDEN / "gpt2.npz"))


@pytest.fixture(scope="session")
def gpt2_small_weights():
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_weights
    return gpt2_weights(GPT2_SMALL, seed=0)


@pytest.fixture(scope="session")
def device():
    """The sm_100a device; GPU tests fail (not skip) when it is unusable."""
    from thvm_b200.device import Device
    return Device.get()
