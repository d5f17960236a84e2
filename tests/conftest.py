import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libwfk.so")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        if name.endswith(".npz"):
            return np.load(os.path.join(GOLDEN, name))
        import json

        with open(os.path.join(GOLDEN, name)) as f:
            return json.load(f)

    return load


def bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)
