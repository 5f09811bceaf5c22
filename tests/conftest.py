import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (str(REPO), str(REPO / "swllm.cpp_b200"), str(REPO / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libswq.so")


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# matmul tolerance: relative L2 against the reference's fp32 result
REL_L2_TOL = 1e-3


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(GOLDEN / f"golden_{name}.npz"))
    return load


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.oracle_lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    """torch on a B200; GPU tests fail loudly (never skip to a CPU path)."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "libswq targets sm_100a (B200)"
    import swq
    swq.lib()
    return torch
