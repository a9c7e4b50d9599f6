import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA extension")


@pytest.fixture(scope="session")
def golden():
    data = np.load(GOLDEN)
    return {k: data[k] for k in data.files}


def golden_cases(golden):
    """Names of the quantiser cases stored in golden.npz."""
    return sorted({k.split("/")[0] for k in golden if k.endswith("/packed") and not k.startswith("gemm")})


@pytest.fixture(scope="session")
def cuda_ext():
    """The built extension on a GPU box; GPU tests fail (not skip) when it is missing."""
    import torch

    from gemm3_b200 import build

    build.build()
    import gemm3_b200

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    assert gemm3_b200.supported(), "device is not sm_100 or libgemm3_b200.so failed to load"
    return gemm3_b200
