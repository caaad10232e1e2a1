"""Test set-up: the package directory on sys.path, the `gpu` marker, shared helpers."""
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "mlx-heimr-sparse-down_b200")
for p in (PKG_ROOT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and libhsd.so")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail (not skip) when none is present, because on the GPU
    box a missing device or library is an error, not a reason to pass."""
    assert torch.cuda.is_available(), "this test needs a CUDA device"
    import hsd_b200._lib as L
    L.lib()
    return torch.device("cuda", 0)


def words_np(t):
    """Packed int32 / uint32 tensor -> numpy uint32 (same bits)."""
    return t.detach().cpu().contiguous().view(torch.int32).numpy().view(np.uint32)


def bits16_np(t):
    """bf16 / f16 tensor -> numpy uint16 bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32_np(t):
    return t.detach().cpu().float().numpy()


def rel_err(a, b):
    """max |a - b| / max |b| -- the reference's error metric (tests/test_layout_decode.py:176)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
