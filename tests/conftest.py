import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")
for p in (os.path.join(ROOT, "oracle"), PKG, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)

os.environ.setdefault("ADAPTIVE_LOG_LEVEL", "ERROR")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


def golden(name):
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", name), allow_pickle=False)
