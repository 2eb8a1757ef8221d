import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "poly-attention_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture
def golden():
    import numpy as np

    def load(name):
        with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
            return {k: z[k] for k in z.files}
    return load
