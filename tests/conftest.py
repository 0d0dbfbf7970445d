import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ecc-kv-cache_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def compress_golden():
    return dict(np.load(os.path.join(GOLDEN, "compress_golden.npz")))


@pytest.fixture(scope="session")
def decode_golden():
    return dict(np.load(os.path.join(GOLDEN, "decode_golden.npz")))


@pytest.fixture(scope="session")
def oracle():
    import ecc_oracle
    ecc_oracle.build()
    return ecc_oracle


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
