"""Prefill on the GPU against the oracle (the reference's tests/test_prefill_kernel.py
bound: max|out - ref| / max|ref| < 5e-3 at the bf16/fp16 level), and the tile order and
live unions bit-exact (hsd/prefill.py:247-291)."""
import numpy as np
import pytest
import torch

from conftest import bits16_np, f32_np, reference_down_case, reference_tile_cases, rel_err, words_np
from oracle import cport
from oracle import prefill as op

import hsd_b200
from hsd_b200 import prefill as hp
from hsd_b200 import synth

TOL = 5e-3        # the reference's prefill bound (tests/test_prefill_kernel.py:20)


def layouts(c):
    return hsd_b200.to_neuron_major(c["w"], c["s"], c["b"]) + hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])


def oracle_rows(c, rows):
    """fp32 dequantised reference for a subset of tokens (C oracle, dense path)."""
    h = f32_np(c["h"])[rows]
    return cport.dense_down(h, c["sel"].cpu().numpy()[rows], c["gains"].cpu().numpy()[rows], words_np(c["w"]),
                            bits16_np(c["s"]), bits16_np(c["b"]), words_np(c["sw"]), bits16_np(c["ss"]),
                            bits16_np(c["sb"]), F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"])


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,topk,tt", [(100, 16, 6, 32), (512, 128, 6, 128), (2048, 128, 6, 64), (1, 8, 2, 128),
                                         (300, 4, 2, 128)])
def test_build_tiles_bit_exact(cuda, T, E, topk, tt):
    gen = torch.Generator(device=cuda).manual_seed(T + E)
    sel, _ = synth.route_zipf(T, E, topk, gen, cuda)
    te, ts = hp.build_tiles(sel, E, tt)
    ote, ots = op.build_tiles(sel.cpu().numpy(), E, tt)
    assert np.array_equal(te.cpu().numpy(), ote)
    assert np.array_equal(ts.cpu().numpy(), ots)


@pytest.mark.gpu
@pytest.mark.parametrize("case", reference_tile_cases(), ids=lambda c: c[0])
def test_build_tiles_matches_reference_code(cuda, case):
    """The CUDA tile order against outputs of the reference's own hsd/prefill.py:247-278 (run
    through a numpy stand-in of mlx.core), same tile count, bit-exact."""
    name, sel, E, tt, te_ref, ts_ref = case
    te, ts = hp.build_tiles(torch.from_numpy(sel).to(cuda), E, tt)
    assert np.array_equal(te.cpu().numpy(), te_ref)
    assert np.array_equal(ts.cpu().numpy(), ts_ref)


@pytest.mark.gpu
def test_prefill_matches_reference_code_fp32_reference(cuda):
    """The prefill path against y of the reference test's own fp32 reference
    (tests/test_layout_decode.py:128-142, run unmodified on a numpy stand-in of mlx.core),
    within the reference's prefill bound."""
    dims, g = reference_down_case()
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(cuda)  # noqa: E731
    bf = lambda a: t(a, np.int16).view(torch.bfloat16)  # noqa: E731
    lay = hsd_b200.to_neuron_major(t(g["w"], np.int32), bf(g["s"]), bf(g["b"])) + \
        hsd_b200.to_neuron_major(t(g["sw"], np.int32), bf(g["ss"]), bf(g["sb"]))
    y = hsd_b200.sparse_down_prefill(bf(g["h"]), t(g["sel"], np.int32), t(g["gains"], np.float32), *lay,
                                     F=dims["F"], FS=dims["FS"], D=dims["D"], topk=dims["topk"], E=dims["E"],
                                     out_dtype=torch.float32)
    assert rel_err(f32_np(y), g["y"]) < TOL
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("z", [0.5, 0.9, 0.99])
def test_build_union_bit_exact(cuda, z):
    T, E, topk, F, FS, tt = 96, 8, 2, 128, 256, 32
    gen = torch.Generator(device=cuda).manual_seed(7)
    sel, _ = synth.route_zipf(T, E, topk, gen, cuda)
    h = synth.relu2_activations((T, topk * F + FS), z, gen, cuda)
    te, ts = hp.build_tiles(sel, E, tt)
    ul, uc = hp.build_union(h, te, ts, F=F, FS=FS, topk=topk, E=E, tt=tt)
    oul, ouc = op.build_union(f32_np(h), te.cpu().numpy(), ts.cpu().numpy(), F=F, FS=FS, topk=topk, E=E, tt=tt,
                              umax=ul.shape[1])
    assert np.array_equal(uc.cpu().numpy(), ouc)
    assert np.array_equal(ul.cpu().numpy(), oul)


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [
    dict(T=100, D=384, F=128, FS=256, E=8, topk=2),
    dict(T=1, D=192, F=64, FS=64, E=3, topk=1),
    dict(T=257, D=576, F=192, FS=128, E=16, topk=4),
])
def test_prefill_small_shapes(cuda, dims):
    T = dims.pop("T")
    c = synth.decode_case(seed=21, B=T, zero_frac=0.9, device=cuda, routing="zipf", **dims)
    y = hp.sparse_down_prefill(c["h"], c["sel"], c["gains"], *layouts(c), F=c["F"], FS=c["FS"], D=c["D"],
                               topk=c["topk"], E=c["E"], out_dtype=torch.float32)
    ref = oracle_rows(c, np.arange(T))
    assert rel_err(f32_np(y), ref) < TOL
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("T", [512, 2048])
def test_prefill_reference_shapes_zipf(cuda, T):
    """Config 2: reference shapes, Zipf(1.1) routing, 90 % zeros; 96 tokens checked against
    the oracle, all tokens against the decode kernel on the same inputs."""
    c = synth.decode_case(seed=31, B=T, zero_frac=0.9, device=cuda, routing="zipf")
    lay = layouts(c)
    kw = dict(F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"])
    y = hp.sparse_down_prefill(c["h"], c["sel"], c["gains"], *lay, E=c["E"], out_dtype=torch.float32, **kw)
    rows = np.random.default_rng(0).choice(T, 96, replace=False)
    assert rel_err(f32_np(y)[rows], oracle_rows(c, rows)) < TOL
    yd = hsd_b200.sparse_down(c["h"], c["sel"], c["gains"], *lay, out_dtype=torch.float32, **kw)
    assert rel_err(f32_np(y), f32_np(yd)) < TOL
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
def test_prefill_resid_dtype_and_given_tiles(cuda):
    c = synth.decode_case(seed=41, B=200, D=384, F=128, FS=256, E=8, topk=2, zero_frac=0.8, device=cuda)
    lay = layouts(c)
    kw = dict(F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"], E=c["E"])
    tiles = hp.build_tiles(c["sel"], c["E"], 128)
    resid = torch.randn((200, c["D"]), device=cuda).to(torch.bfloat16)
    y = hp.sparse_down_prefill(c["h"], c["sel"], c["gains"], *lay, tiles=tiles, resid=resid, **kw)
    assert y.dtype == torch.bfloat16
    y32 = hp.sparse_down_prefill(c["h"], c["sel"], c["gains"], *lay, out_dtype=torch.float32, **kw)
    assert rel_err(f32_np(y), f32_np(resid.float() + y32)) < 1e-2   # bf16 rounding of resid + y
    # deterministic: the same bits twice
    assert torch.equal(y32, hp.sparse_down_prefill(c["h"], c["sel"], c["gains"], *lay, out_dtype=torch.float32, **kw))


@pytest.mark.gpu
def test_prefill_skips_dead_k_tiles_exactly(cuda):
    """Correlated zeros (a trained model's dead neuron groups): every third 64-group of every
    slot is zero for all tokens, and one rarely chosen expert's slots are zero throughout, so
    its tiles have no live K-tile at all. The GEMM skips those K-tiles (the gather's masks);
    the result still matches the oracle, the decode kernel, and the same call with the dead
    groups holding an exact zero everywhere -- the skipped work only ever added zeros."""
    T = 512
    c = synth.decode_case(seed=61, B=T, zero_frac=0.9, device=cuda, routing="zipf")
    F, FS, topk = c["F"], c["FS"], c["topk"]
    h = c["h"].clone()
    cols = torch.arange(topk * F + FS, device=cuda)
    grp = torch.where(cols < topk * F, (cols % F) // 64, (cols - topk * F) // 64)
    h[:, grp % 3 == 0] = 0
    rare = int(torch.bincount(c["sel"].reshape(-1).long(), minlength=c["E"]).argmin())
    for k in range(topk):
        h[c["sel"][:, k] == rare, k * F:(k + 1) * F] = 0
    lay = layouts(c)
    kw = dict(F=F, FS=FS, D=c["D"], topk=topk)
    y = hp.sparse_down_prefill(h, c["sel"], c["gains"], *lay, E=c["E"], out_dtype=torch.float32, **kw)
    c2 = dict(c, h=h)
    rows = np.random.default_rng(1).choice(T, 64, replace=False)
    assert rel_err(f32_np(y)[rows], oracle_rows(c2, rows)) < TOL
    yd = hsd_b200.sparse_down(h, c["sel"], c["gains"], *lay, out_dtype=torch.float32, **kw)
    assert rel_err(f32_np(y), f32_np(yd)) < TOL
    assert torch.equal(y, hp.sparse_down_prefill(h, c["sel"], c["gains"], *lay, E=c["E"], out_dtype=torch.float32,
                                                 **kw))
    assert hsd_b200.device_status() == 0
