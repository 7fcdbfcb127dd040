"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on the CPU."""
import os
import sys
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402

MODEL_CACHE = os.environ.get("QWC_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "qwc_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: full-size model checks")


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import bindings
    if not os.path.exists(bindings.ORACLE_SO):
        bindings.build()
    return bindings


def model_dir(pkg, shape_name, seed=0):
    shape = pkg.synth.SHAPES[shape_name]
    return pkg.synth.write_model(shape, os.path.join(MODEL_CACHE, f"{shape_name}-s{seed}"), seed=seed)


def rel_l2(a, b):
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
