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


@pytest.fixture(autouse=True)
def _no_device_timeouts(request):
    """After every GPU test: no kernel's bounded wait may have given up."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from poly_attention_b200 import _lib
    torch.cuda.synchronize()
    err = _lib.device_error(reset=True)
    assert err == 0, f"a kernel wait gave up: device error word {err:#x} (site {err >> 8})"
