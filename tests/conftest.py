import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); the parity tests proper")


@pytest.fixture(scope="session")
def orc():
    """The parity checker (oracle/): built on first use."""
    import oracle

    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    d = os.path.join(ROOT, "tests", "golden")
    return {f[:-4]: np.load(os.path.join(d, f)) for f in os.listdir(d) if f.endswith(".npz")}


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import breadv2_b200 as bb

    bb.lib()  # fails loudly when the CUDA library is missing
    return torch.device("cuda:0")
