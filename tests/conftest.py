"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and are skipped when no
CUDA device is visible; the CPU suite pins the oracle and the C ABI."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size configuration checks")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Restated()


@pytest.fixture(scope="session")
def ref():
    import oracle
    try:
        return oracle.Reference()
    except FileNotFoundError as e:
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def jb():
    import jules_b200
    jules_b200.lib()  # raises if the library was not built
    return jules_b200


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


# Tolerances stated by the north star: bf16/fp16 vs the fp32 oracle
# max-abs <= 2e-2 and rel-L2 <= 5e-3; fp32 rel-L2 <= 1e-5.
BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 5e-3
F32_REL_L2 = 1e-5
