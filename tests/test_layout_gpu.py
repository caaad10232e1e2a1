"""nibble_transpose / to_neuron_major on the GPU against the oracle: bit-exact and
self-inverse over the reference test's shapes (tests/test_layout_decode.py:55-83)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, REF_HASHED_SHAPES, bits16_np, reference_words, sha256_np, words_np
from oracle import layout as ol

import hsd_b200

REF_SHAPES = ((5, 24, 9), (2688, 232), (1856, 336), (3712, 336), (3, 2688, 232))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", REF_SHAPES + ((1, 8, 1), (2, 520, 33), (7, 264, 70)))
def test_nibble_transpose_exact_and_self_inverse(cuda, shape):
    rng = np.random.default_rng(0)
    w = rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32)
    wt = torch.from_numpy(w.view(np.int32)).to(cuda)
    t = hsd_b200.nibble_transpose(wt)
    assert tuple(t.shape) == (*shape[:-2], shape[-1] * 8, shape[-2] // 8)
    assert np.array_equal(words_np(t), ol.nibble_transpose(w))
    back = hsd_b200.nibble_transpose(t)
    assert torch.equal(back, wt)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["nibble_transpose_5x24x9.npz", "nibble_transpose_2x16x4.npz"])
def test_nibble_transpose_golden(cuda, name):
    g = np.load(os.path.join(GOLDEN, name))
    t = hsd_b200.nibble_transpose(torch.from_numpy(g["w"].view(np.int32)).to(cuda))
    assert np.array_equal(words_np(t), g["t"])


@pytest.mark.gpu
def test_uint32_words_accepted(cuda):
    w = torch.randint(-2**31, 2**31 - 1, (16, 3), dtype=torch.int32, device=cuda)
    t32 = hsd_b200.nibble_transpose(w.view(torch.uint32))
    assert t32.dtype == torch.uint32
    assert torch.equal(t32.view(torch.int32), hsd_b200.nibble_transpose(w))


@pytest.mark.gpu
def test_to_neuron_major_full_expert_stack(cuda):
    """The reference's routed shapes: w [128, 2688, 232], s / b [128, 2688, 29]."""
    from hsd_b200 import synth
    gen = torch.Generator(device=cuda).manual_seed(5)
    w, s, b = synth.quantized_weights((128, 2688, 1856), gen, cuda)
    pw, ps, pb = hsd_b200.to_neuron_major(w, s, b)
    assert tuple(pw.shape) == (128, 1856, 336) and tuple(ps.shape) == (128, 29, 2688)
    assert torch.equal(ps, s.transpose(-1, -2).contiguous())
    assert torch.equal(pb, b.transpose(-1, -2).contiguous())
    for e in (0, 77, 127):                         # three experts through the numpy oracle
        assert np.array_equal(words_np(pw[e]), ol.nibble_transpose(words_np(w[e])))
    assert torch.equal(hsd_b200.nibble_transpose(pw), w)


@pytest.mark.gpu
def test_swap_last2_f16_and_odd_sizes(cuda):
    x = torch.randn((3, 37, 45), device=cuda).half()
    y = hsd_b200.swap_last2(x)
    assert torch.equal(y, x.transpose(-1, -2).contiguous())
    assert np.array_equal(bits16_np(y), np.swapaxes(bits16_np(x), -1, -2))


def _u16(a, dev):
    return torch.from_numpy(a.view(np.int16)).to(dev).view(torch.bfloat16)


@pytest.mark.gpu
def test_layout_matches_reference_code(cuda):
    """The CUDA permutation against outputs of the reference's own hsd/layout.py:34-74 (run
    through a numpy stand-in of mlx.core): two small shapes, a 20-expert stack (more than the
    16-expert chunk) and a 2-D shared expert, words and bf16 scale / bias bits bit-exact."""
    g = np.load(os.path.join(GOLDEN, "reference_layout.npz"))
    for key in ("5x24x9", "2x16x4"):
        t = hsd_b200.nibble_transpose(torch.from_numpy(g["nt_w_" + key].view(np.int32)).to(cuda))
        assert np.array_equal(words_np(t), g["nt_t_" + key])
    for pre in ("ntm_", "ntm_s"):
        w = torch.from_numpy(g[pre + "w"].view(np.int32)).to(cuda)
        pw, ps, pb = hsd_b200.to_neuron_major(w, _u16(g[pre + "s"], cuda), _u16(g[pre + "b"], cuda))
        assert np.array_equal(words_np(pw), g[pre + "pw"])
        assert np.array_equal(bits16_np(ps), g[pre + "ps"]) and np.array_equal(bits16_np(pb), g[pre + "pb"])


@pytest.mark.gpu
@pytest.mark.parametrize("shape", REF_HASHED_SHAPES)
def test_nibble_transpose_reference_hash(cuda, shape):
    """The reference test's larger shapes: sha256 of the CUDA transpose of the seeded words ==
    sha256 of the reference code's own transpose of the same words."""
    g = np.load(os.path.join(GOLDEN, "reference_layout.npz"))
    t = hsd_b200.nibble_transpose(torch.from_numpy(reference_words(shape).view(np.int32)).to(cuda))
    assert sha256_np(words_np(t)) == str(g["nt_sha_" + "x".join(map(str, shape))])
