"""The opt-in two-tile pipelined backward (POLY_BWD_TWO_TILE=1) against the
oracle, in a child process (the switch is read once per process): causal and
not, ragged tails, GQA, the key bias with its gradient, bf16 and fp16."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_tile_backward_parity():
    env = dict(os.environ, POLY_BWD_TWO_TILE="1")
    cmd = [sys.executable, "-m", "pytest", os.path.join(ROOT, "tests", "test_parity_gpu.py"), "-q", "-x",
           "-m", "gpu", "-k", "backward or order2 or ragged or dbias or flash"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
