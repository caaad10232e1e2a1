"""The allocation-free prefill entry point (hsd_sparse_down_prefill_noalloc), for callers
that cannot call cudaMalloc -- code under CUDA graph capture without a memory pool, or a
runtime that owns all device memory. It keeps its scratch in a fixed device array inside
libhsd.so, so it must give what the workspace-taking hsd_sparse_down_prefill gives, call
after call, and refuse a chunk whose scratch would not fit. This file is named to be
collected last, so that a run stopping at the first failure has run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import f32_np, rel_err

import hsd_b200
import hsd_b200._lib as L
from hsd_b200 import prefill as hp
from hsd_b200 import synth

TOL = 5e-3        # the prefill tolerance of tests/test_prefill_gpu.py
REF = dict(D=2688, F=1856, FS=3712, topk=6, E=128)   # the reference model's MoE shapes


def scratch_bytes(T, D, F, FS, topk, E, tt=hp.GEMM_TT):
    """The scratch a call needs, as the library lays it out: the compacted tile order (at most
    every full tile of slots + one partial tile per expert with slots + the shared expert's
    tiles), their live-K-tile masks, the fp16 A rows of those tiles and the fp32 partial rows."""
    nr, ns = hp.num_tiles(T, topk, E, tt)
    slots = T * topk
    nc = min(nr, slots // tt + min(E, slots)) + ns
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    mask_row = (max(F, FS) // 64 + 7) // 8 * 8                 # a mask byte per K-tile, rows of 8
    hc_off = up(up(up(4 * nc) + 4 * nc * tt) + nc * mask_row)
    part_off = up(hc_off + nc * tt * max(F, FS) * 2)
    return part_off + T * (topk + 1) * D * 4


def largest_chunk(cap, **shape):
    T = 1
    while scratch_bytes(T + 1, **shape) <= cap:
        T += 1
    return T


def _args(c, lay, tiles, y):
    te, ts = tiles
    return [L.ptr(c["h"]), L.dtype_code(c["h"], "h"), L.ptr(c["gains"]), L.ptr(te), L.ptr(ts), te.shape[0],
            L.ptr(lay[0]), L.ptr(lay[1]), L.ptr(lay[2]), L.dtype_code(lay[1], "s"), L.ptr(lay[3]), L.ptr(lay[4]),
            L.ptr(lay[5]), None, L.ptr(y), L.dtype_code(y, "y"), c["h"].shape[0], c["D"], c["F"], c["FS"],
            c["topk"], c["E"]]


def _existing(c, lay, tiles):
    """The workspace-taking entry point, through the C ABI."""
    y = torch.empty((c["h"].shape[0], c["D"]), dtype=torch.float32, device=c["h"].device)
    n = hp.workspace_bytes(c["h"].shape[0], c["D"], c["F"], c["FS"], c["topk"], c["E"])
    ws = torch.empty(n, dtype=torch.uint8, device=c["h"].device)
    L.call("hsd_sparse_down_prefill", *_args(c, lay, tiles, y), L.ptr(ws), n, L.stream_of(c["h"]))
    return y


def _noalloc(c, lay, tiles):
    y = torch.empty((c["h"].shape[0], c["D"]), dtype=torch.float32, device=c["h"].device)
    L.call("hsd_sparse_down_prefill_noalloc", *_args(c, lay, tiles, y), L.stream_of(c["h"]))
    return y


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_two_calls(cuda):
    """Two calls in a row (the reference shapes with 8 tokens, then a narrower layer with 200
    tokens, which reuses the same scratch) each equal the workspace entry point's output."""
    cases = [dict(seed=51, B=8, zero_frac=0.9, routing="zipf"),
             dict(seed=52, B=200, D=384, F=128, FS=256, E=8, topk=2, zero_frac=0.8, routing="zipf")]
    for kw in cases:
        c = synth.decode_case(device=cuda, **kw)
        lay = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"]) + hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
        tiles = hp.build_tiles(c["sel"], c["E"], hp.GEMM_TT)
        y_ref = _existing(c, lay, tiles)
        y = _noalloc(c, lay, tiles)
        torch.cuda.synchronize()
        assert rel_err(f32_np(y), f32_np(y_ref)) < TOL
        assert hsd_b200.device_status() == 0


@pytest.mark.gpu
def test_noalloc_largest_chunk_that_fits(cuda):
    """The largest chunk the fixed scratch admits at the reference shapes (its scratch reaches
    the array's last tenth) equals the workspace entry point; one token more is refused."""
    cap = ctypes.c_size_t(0)
    L.call("hsd_prefill_noalloc_max_bytes", ctypes.byref(cap))
    T = largest_chunk(cap.value, **REF)
    assert scratch_bytes(T, **REF) > 0.9 * cap.value            # the array's last tenth is in use
    assert scratch_bytes(T + 1, **REF) > cap.value
    c = synth.decode_case(seed=53, B=T, zero_frac=0.9, routing="zipf", device=cuda)
    lay = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"]) + hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
    tiles = hp.build_tiles(c["sel"], c["E"], hp.GEMM_TT)
    y_ref = _existing(c, lay, tiles)
    y = _noalloc(c, lay, tiles)
    torch.cuda.synchronize()
    assert rel_err(f32_np(y), f32_np(y_ref)) < TOL
    assert hsd_b200.device_status() == 0
    c2 = synth.decode_case(seed=54, B=T + 1, zero_frac=0.9, routing="zipf", device=cuda)
    tiles2 = hp.build_tiles(c2["sel"], c2["E"], hp.GEMM_TT)
    y2 = torch.empty((T + 1, c2["D"]), dtype=torch.float32, device=cuda)
    rc = L.lib().hsd_sparse_down_prefill_noalloc(*_args(c2, lay, tiles2, y2), L.stream_of(c2["h"]))
    assert rc == L.HSD_ERR_SHAPE


def test_noalloc_refuses_a_chunk_that_does_not_fit():
    """512 tokens at the reference shapes need far more than the fixed scratch: the call is
    refused before any device work, with the bytes it needs in the message."""
    cap = ctypes.c_size_t(0)
    L.call("hsd_prefill_noalloc_max_bytes", ctypes.byref(cap))
    assert cap.value == 64 << 20
    T, D, F, FS, topk, E = 512, 2688, 1856, 3712, 6, 128
    nr, ns = hp.num_tiles(T, topk, E, hp.GEMM_TT)
    p = ctypes.c_void_p(256)
    rc = L.lib().hsd_sparse_down_prefill_noalloc(p, L.HSD_BF16, p, p, p, nr + ns, p, p, p, L.HSD_BF16, p, p, p, None,
                                                 p, L.HSD_F32, T, D, F, FS, topk, E, None)
    assert rc == L.HSD_ERR_SHAPE
    msg = L.lib().hsd_last_error_string().decode()
    assert "scratch" in msg and str(64 << 20) in msg
    assert np.isfinite(cap.value)
