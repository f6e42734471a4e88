"""GPU: the tensor-core single-token GEMV (k_tmv, opt-in with KQ_TMV=1) against the CPU oracle.

The switch is read once per device when the library initialises it, so the GEMV parity tests
(test_gpu_quant.py: every matvec shape, partial row tiles, edge activations, NaN propagation) and
the decode tests (test_gpu_decode.py: greedy tokens identical to the oracle, logits / hidden / K/V
within 1e-3 relative L2, on the graph path whose q/k/v, o, gate/up and down GEMVs then run on
k_tmv) are run again in a child process with the switch set."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tensor_core_gemv_parity():
    env = dict(os.environ, KQ_TMV="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        "tests/test_gpu_quant.py", "tests/test_gpu_decode.py"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout
