import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "openflowlm-next_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = ROOT / "tests" / "golden"
    return {n: np.load(d / f"{n}.npz") for n in ("q4_1", "router", "moe", "expert_pool", "q4nx", "gemm_q4")}
