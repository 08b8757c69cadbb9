import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "lucebox-hub_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


@pytest.fixture(scope="session")
def full_weights_cpu():
    """Seeded random-init Qwen3.5-0.8B-architecture weights (bf16, CPU), built once."""
    from qwen35_b200.config import QWEN35_0P8B
    from qwen35_b200.weights import make_random_weights
    return make_random_weights(1234, QWEN35_0P8B)
