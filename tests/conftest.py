import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "fast-moss-tokenizer_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def same_bits(a, b):
    """Bitwise float32 equality that treats every NaN as equal to every NaN."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    nan_a, nan_b = np.isnan(a), np.isnan(b)
    if not np.array_equal(nan_a, nan_b):
        return False
    return np.array_equal(a[~nan_a].view(np.uint32), b[~nan_b].view(np.uint32))


def bf16_ulp_diff(a, b):
    """Max distance in bf16 units in the last place between bf16-valued arrays
    (NaN must match NaN; +-inf must match exactly)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan_a, nan_b = np.isnan(a), np.isnan(b)
    assert np.array_equal(nan_a, nan_b), "NaN positions differ"
    ia = (a[~nan_a].view(np.uint32) >> 16).astype(np.int64)
    ib = (b[~nan_b].view(np.uint32) >> 16).astype(np.int64)
    # map sign-magnitude to a monotonic integer line
    ia = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    ib = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    return int(np.max(np.abs(ia - ib))) if ia.size else 0


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def moss(cuda_device):
    """The product package with its native library loaded (fails loudly if
    the library is missing)."""
    import fast_moss_b200
    from fast_moss_b200 import _lib

    _lib.load()
    return fast_moss_b200
