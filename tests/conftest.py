import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "inferencer-jetson_b200"), os.path.join(REPO, "oracle"),
          os.path.join(REPO, "tests", "golden"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "ref_kernels.npz"))


@pytest.fixture(scope="session")
def golden_inputs():
    import make_ref_golden
    return make_ref_golden.inputs()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ijb200 import lib
    lib.load()  # fails loudly when the library is missing
    return torch.device("cuda:0")
