import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "vram-compression_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_case(path):
    z = np.load(path)
    codes = z["codes"].astype(np.int64)
    enc = dict(words=z["words"], offs=z["offs"], table=z["table"], R=int(z["R"]), C=int(z["C"]),
               shape=codes.shape)
    return codes, enc, z["step"], z["x"], z["y"], z["bits"]


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
