"""The numpy stand-in of mlx.core that tests/golden/make_reference_golden.py runs the
reference's own functions on: each call it provides behaves as the fixtures assume (no GPU,
and nothing of the reference is needed here)."""
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.quant import dequantize


def _gen():
    spec = importlib.util.spec_from_file_location("make_reference_golden",
                                                  os.path.join(GOLDEN, "make_reference_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture
def standin():
    """The generator module with its mlx.core stand-in installed, removed again afterwards."""
    saved = {k: sys.modules[k] for k in ("mlx", "mlx.core", "mlx.nn") if k in sys.modules}
    g = _gen()
    g.install_standin()
    yield g
    for k in ("mlx", "mlx.core", "mlx.nn"):
        sys.modules.pop(k, None)
    sys.modules.update(saved)


def test_bf16_round_is_round_to_nearest_even():
    g = _gen()
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 1, 4096), rng.normal(0, 1e-3, 1024), rng.normal(0, 1e4, 1024)]).astype(np.float32)
    ties = (np.arange(1, 513, dtype=np.uint32) << 16 | 0x8000).view(np.float32)   # exactly halfway
    x = np.concatenate([x, ties, -ties])
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(g.bf16_round(x), want)


def test_scatter_add_accumulates_duplicates_and_copies(standin):
    mx = sys.modules["mlx.core"]
    a = mx.zeros((5,), dtype=mx.int32)
    b = a.at[mx.array([1, 3, 1, 1], dtype=mx.int32)].add(1)
    assert b.tolist() == [0, 3, 0, 1, 0] and a.tolist() == [0] * 5
    o = mx.full((4,), -1, dtype=mx.int32).at[mx.array([2, 0])].add(mx.array([7, 5]))
    assert o.tolist() == [4, -1, 6, -1]


def test_argsort_is_stable(standin):
    mx = sys.modules["mlx.core"]
    x = mx.array([3, 1, 3, 0, 1, 3], dtype=mx.int32)
    assert mx.argsort(x).tolist() == [3, 1, 4, 0, 2, 5]


def test_dequantize_is_the_affine_format_rounded_to_bf16():
    g = _gen()
    rng = np.random.default_rng(1)
    w = rng.integers(0, 2**32, size=(3, 16, 8), dtype=np.uint64).astype(np.uint32)
    s = g.bf16_round(rng.normal(0, 0.02, (3, 16, 1)).astype(np.float32))
    b = g.bf16_round(rng.normal(0, 0.01, (3, 16, 1)).astype(np.float32))
    out = np.asarray(g._dequantize(w, s, b, group_size=64, bits=4))
    assert out.shape == (3, 16, 64)
    assert np.array_equal(out, g.bf16_round(dequantize(w, s, b)))
