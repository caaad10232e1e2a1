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


# ---- fixtures produced by the reference's own code (tests/golden/make_reference_golden.py)

REF_HASHED_SHAPES = ((2688, 232), (1856, 336), (3712, 336), (3, 2688, 232))


def reference_words(shape):
    """The seeded words whose reference transpose is pinned by sha256 in reference_layout.npz
    (the same rule as the generator: default_rng(prod(shape) mod 2^31))."""
    rng = np.random.default_rng(int(np.prod(shape)) % (2**31))
    return rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32)


def sha256_np(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def reference_tile_cases():
    """(name, sel, E, tt, tile_e, tile_slot) of every case in reference_tiles.npz."""
    g = np.load(os.path.join(GOLDEN, "reference_tiles.npz"))
    names = sorted(k[:-len("_dims")] for k in g.files if k.endswith("_dims"))
    out = []
    for n in names:
        T, topk, E, tt = (int(v) for v in g[n + "_dims"])
        out.append((n, g[n + "_sel"], E, tt, g[n + "_tile_e"], g[n + "_tile_slot"]))
    return out


def reference_down_case():
    """reference_down.npz: (dims dict, arrays) -- y from the reference test's reference()."""
    g = np.load(os.path.join(GOLDEN, "reference_down.npz"))
    D, F, FS, E, topk, B = (int(x) for x in g["dims"])
    return dict(D=D, F=F, FS=FS, E=E, topk=topk, B=B), g
