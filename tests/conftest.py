import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


GOLDEN = os.path.join(ROOT, "tests", "golden")


def golden(name):
    import numpy as np

    return dict(np.load(os.path.join(GOLDEN, name)))


def rel_err(a, ref):
    """max|a - ref| / max|ref|: the parity metric for every float path."""
    import numpy as np

    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = max(float(np.max(np.abs(ref))), 1e-30)
    return float(np.max(np.abs(a - ref))) / denom
