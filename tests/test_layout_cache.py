"""The on-disk cache of the neuron-major layout (hsd_b200.layout_cache): the tensors come
back bit for bit, a cache written for other weights is refused, and the load-or-build helper
builds once and loads afterwards. The GPU test runs the sparse kernel on the loaded layout."""
import os

import pytest
import torch

from hsd_b200 import layout_cache as lc


def _fake_layer(seed, E=3, F=128, D=64, FS=64):
    g = torch.Generator().manual_seed(seed)
    w = lambda *s: torch.randint(-2**31, 2**31 - 1, s, generator=g, dtype=torch.int64).to(torch.int32)  # noqa: E731
    h = lambda *s: torch.randn(s, generator=g).to(torch.bfloat16)  # noqa: E731
    return (w(E, F, D // 8), h(E, F // 64, D), h(E, F // 64, D), w(FS, D // 8).to(torch.uint32),
            h(FS // 64, D), h(FS // 64, D))


def _same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_round_trip_bit_exact(tmp_path):
    layers = [_fake_layer(s) for s in range(3)]
    p = str(tmp_path / "layout.safetensors")
    lc.save_layout_cache(p, layers, key="synthetic seed 0")
    assert not os.path.exists(p + ".tmp")
    back = lc.load_layout_cache(p, key="synthetic seed 0", device="cpu")
    assert len(back) == 3
    for a, b in zip(layers, back):
        for x, y in zip(a, b):
            assert _same(x, y)


def test_other_key_or_format_is_refused(tmp_path):
    p = str(tmp_path / "layout.safetensors")
    lc.save_layout_cache(p, [_fake_layer(1)], key="checkpoint A")
    with pytest.raises(lc.LayoutCacheMismatch):
        lc.load_layout_cache(p, key="checkpoint B", device="cpu")
    from safetensors.torch import save_file
    save_file({"x": torch.zeros(1)}, p, metadata={"format": "something else", "key": "checkpoint A"})
    with pytest.raises(lc.LayoutCacheMismatch):
        lc.load_layout_cache(p, key="checkpoint A", device="cpu")


def test_load_or_build_builds_once(tmp_path):
    p = str(tmp_path / "layout.safetensors")
    calls = []

    def build():
        calls.append(1)
        return [_fake_layer(7), _fake_layer(8)]

    first, cached = lc.neuron_major_layers(p, "k", build, device="cpu")
    assert not cached and len(calls) == 1
    second, cached = lc.neuron_major_layers(p, "k", build, device="cpu")
    assert cached and len(calls) == 1
    for a, b in zip(first, second):
        for x, y in zip(a, b):
            assert _same(x, y)
    _, cached = lc.neuron_major_layers(p, "other weights", build, device="cpu")   # stale: rebuilt
    assert not cached and len(calls) == 2


@pytest.mark.gpu
def test_loaded_layout_feeds_the_sparse_kernel(cuda, tmp_path):
    import hsd_b200
    from hsd_b200 import synth
    c = synth.decode_case(seed=61, B=2, zero_frac=0.9, device=cuda, D=512, F=256, FS=512, E=8, topk=2)
    lay = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"]) + hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
    p = str(tmp_path / "layout.safetensors")
    lc.save_layout_cache(p, [lay], key="decode case 61")
    (back,) = lc.load_layout_cache(p, key="decode case 61", device=cuda)
    for x, y in zip(lay, back):
        assert y.is_cuda and _same(x.cpu(), y.cpu())
    kw = dict(F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"], out_dtype=torch.float32)
    y0 = hsd_b200.sparse_down(c["h"], c["sel"], c["gains"], *lay, **kw)
    y1 = hsd_b200.sparse_down(c["h"], c["sel"], c["gains"], *back, **kw)
    assert torch.equal(y0, y1)
