import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    # Build the native libraries if a fresh checkout lacks them (nvcc cross-compiles without a GPU).
    lib = os.path.join(ROOT, "low_latency_inference_gpu_b200", "_lib", "libll_b200.so")
    olib = os.path.join(ROOT, "oracle", "liboracle.so")
    if not (os.path.exists(lib) and os.path.exists(olib)):
        subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.build()"], cwd=ROOT, check=True)


@pytest.fixture(scope="session")
def golden():
    import json

    with open(os.path.join(TESTS, "golden", "golden.json")) as f:
        return json.load(f)


def rel_err(y, ref):
    """max |y - ref| / max |ref| (norm-wise relative error; documented tolerance metric)."""
    import numpy as np

    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(float(np.max(np.abs(ref))), 1e-30)
    return float(np.max(np.abs(y - ref))) / den


def close(y, ref, tol):
    """Both tolerance checks: norm-wise rel_err <= tol, and element-wise
    |y - ref| <= tol * |ref| + (tol / 5) * max|ref| (relative per element, with an
    absolute floor a fifth of the norm-wise bound for outputs near zero)."""
    import numpy as np

    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(float(np.max(np.abs(ref))), 1e-30)
    elem = np.abs(y - ref) <= tol * np.abs(ref) + (tol / 5.0) * scale
    return rel_err(y, ref) <= tol and bool(np.all(elem))
