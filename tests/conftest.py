import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


@pytest.fixture(scope="session")
def oracle():
    lib = os.path.join(ROOT, "oracle", "_build", "liboracle.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True,
                       capture_output=True)
    from oracle.binding import Oracle
    return Oracle()


def _load(name):
    path = os.path.join(GOLDEN, name + ".npz")
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name}.npz missing")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_ops():
    return _load("ops")


@pytest.fixture(scope="session")
def golden_tiny():
    return _load("model_tiny")


@pytest.fixture(scope="session")
def golden_llama():
    return _load("model_llama2_l2")


@pytest.fixture(scope="session")
def golden_qwen2():
    return _load("model_qwen2")


@pytest.fixture(scope="session")
def mlb():
    """The product library (C-ABI) through its Python binding."""
    from mini_llama_b200 import capi
    return capi.load()


@pytest.fixture(scope="session")
def gpu(mlb):
    count = mlb.device_count()
    if count < 1:
        pytest.fail("no CUDA device visible to the product library")
    return 0
