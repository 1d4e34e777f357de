import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C ABI")


GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="session")
def golden_dequant():
    import numpy as np
    return np.load(os.path.join(GOLDEN, "golden_dequant.npz"))


@pytest.fixture(scope="session")
def golden_linear():
    import numpy as np
    return np.load(os.path.join(GOLDEN, "golden_linear.npz"))


@pytest.fixture(scope="session")
def golden_moe():
    import numpy as np
    return np.load(os.path.join(GOLDEN, "golden_moe.npz"))
