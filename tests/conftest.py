import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU oracle case")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "kern_golden.npz")))


@pytest.fixture(scope="session")
def ora():
    import oracle

    oracle.build()
    oracle.set_threads(min(8, os.cpu_count() or 1))
    return oracle


@pytest.fixture(scope="session")
def gsv():
    """The product package (directory gpt-sovits-native_b200/)."""
    import __graft_entry__

    return __graft_entry__.package()


@pytest.fixture(scope="session")
def dev(gsv):
    """Initialised CUDA device 0 through the C-ABI; skips without a GPU."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    gsv.device_init(0)
    return gsv
