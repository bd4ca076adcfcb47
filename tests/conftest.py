"""Shared fixtures.  Tests marked `gpu` need a CUDA GPU (a B200); everything
else runs on the CPU: the oracle against the golden vectors, the host-side
logic, and the C-ABI library's exports (no compute calls without a GPU)."""
import importlib.util
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen600-rocm-inference_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_qb():
    spec = importlib.util.spec_from_file_location("qwen_b200", os.path.join(PKG, "qwen_b200.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def qb():
    return load_qb()


@pytest.fixture(scope="session")
def O():
    import oracle_py
    return oracle_py


@pytest.fixture(scope="session")
def checkpoint(qb):
    return qb.default_checkpoint(0)


@pytest.fixture(scope="session")
def engine(qb, checkpoint):
    e = qb.Engine(checkpoint, 0)
    yield e
    e.close()


def rel_rms(a, b):
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2) / np.mean(b ** 2)))
