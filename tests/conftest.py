import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def golden_calls(data):
    """Iterate the recorded attention calls of a golden file in order."""
    for i in range(int(data["calln"])):
        p = f"call{i}_"
        layer, start, lq, key_len = (int(x) for x in data[p + "meta"])
        rec = {"layer": layer, "start": start, "lq": lq, "key_len": key_len}
        for name in ("q_proj", "k_proj", "v_proj", "cos", "sin", "q", "k_new", "v_new", "out", "full_k", "full_v"):
            if p + name in data:
                rec[name] = data[p + name]
        yield rec


@pytest.fixture(scope="session")
def tiny_ref():
    return load_golden("tiny_ref.npz")


@pytest.fixture(scope="session")
def small_d128():
    return load_golden("small_d128.npz")
