import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_vectors.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def built_lib():
    """Path of libmserve_kv.so, building it (nvcc, sm_100a) if it is missing or stale."""
    from mserve_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_numpy_bits(t: torch.Tensor) -> np.ndarray:
    """Raw element bits of any tensor as an unsigned-integer numpy array (bitwise compare)."""
    t = t.detach().cpu().contiguous()
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.view(view).numpy()


def from_bits(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """Inverse of the fixture encoding: uint16 bits -> bfloat16, other arrays as-is."""
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)
