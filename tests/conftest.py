import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libod_b200.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (no silent skip) when selected with -m gpu on a machine without CUDA
    pass


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(GOLDEN, "ops.npz")))


def from_bits(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """Inverse of make_golden.bits: raw 16-bit patterns back to a bf16/fp16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a)).view(dtype)


def digest(*ts: torch.Tensor) -> np.ndarray:
    import hashlib
    h = hashlib.sha256()
    for t in ts:
        if t.dtype in (torch.bfloat16, torch.float16):
            b = t.contiguous().view(torch.int16).numpy()
        else:
            b = t.contiguous().numpy()
        h.update(b.tobytes())
    return np.frombuffer(h.digest()[:8], dtype=np.uint8).copy()


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    from opendecider_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)
