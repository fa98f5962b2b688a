import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libomcuda.so)")


@pytest.fixture(scope="session")
def gpu():
    """Initialise the backend on device 0 for the calling thread; fail loudly otherwise."""
    from omnimatchdeeplearningtool_b200 import backend
    backend.init(0)
    yield backend
    assert backend.kernel_error() == 0, "a bounded in-kernel wait gave up"


def rel_err(a, b):
    """max |a-b| / max |b|: the normalised error used for 16-bit paths."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_err_floor(a, b):
    """max |a-b| / max(|b|, 1e-3 * max|b|): element-wise relative error with an absolute
    floor for near-zero outputs, the fp32-path metric (tolerance 1e-4)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    floor = 1e-3 * max(np.abs(b).max(), 1e-30)
    return float((np.abs(a - b) / np.maximum(np.abs(b), floor)).max())
