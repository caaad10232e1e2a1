"""The CPU oracle against the reference's known-answer tests and the golden fixtures,
and its restatements against each other (no GPU)."""
import os

import numpy as np
import pytest
import torch

from conftest import (GOLDEN, REF_HASHED_SHAPES, reference_down_case, reference_tile_cases, reference_words,
                      rel_err, sha256_np)
from oracle import cport
from oracle import decode as od
from oracle import layout as ol
from oracle.quant import bf16_bits_to_f32, dequantize, dequantize_neuron_major


def slow_reference_transpose(w):
    """The reference test's slow numpy method (tests/test_layout_decode.py:38-52 of the
    reference), restated: unpack every word to 8 nibbles column by column, move them,
    pack them again."""
    lead = w.shape[:-2]
    R, CW = w.shape[-2], w.shape[-1]
    C = CW * 8
    nib = np.zeros((*lead, R, C), dtype=np.uint32)
    for k in range(8):
        nib[..., k::8] = (w >> np.uint32(4 * k)) & np.uint32(0xF)
    t = np.swapaxes(nib, -1, -2)
    out = np.zeros((*lead, C, R // 8), dtype=np.uint32)
    for k in range(8):
        out |= t[..., k::8] << np.uint32(4 * k)
    return out


# the reference test's shapes (tests/test_layout_decode.py:59)
REF_SHAPES = ((5, 24, 9), (2688, 232), (1856, 336), (3712, 336), (3, 2688, 232))


@pytest.mark.parametrize("shape", REF_SHAPES)
def test_nibble_transpose_exact_and_self_inverse(shape):
    rng = np.random.default_rng(0)
    w = rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32)
    t = ol.nibble_transpose(w)
    assert t.shape == (*shape[:-2], shape[-1] * 8, shape[-2] // 8)
    assert np.array_equal(t, slow_reference_transpose(w))
    assert np.array_equal(ol.nibble_transpose(t), w)


@pytest.mark.parametrize("name", ["nibble_transpose_5x24x9.npz", "nibble_transpose_2x16x4.npz"])
def test_nibble_transpose_golden(name):
    g = np.load(os.path.join(GOLDEN, name))
    assert np.array_equal(ol.nibble_transpose(g["w"]), g["t"])
    assert np.array_equal(cport.nibble_transpose(g["w"]), g["t"])


def test_layout_matches_reference_code():
    """nibble_transpose / to_neuron_major against outputs of the reference's own
    hsd/layout.py:34-74 (run through a numpy stand-in of mlx.core): two small shapes in full,
    a 20-expert stack (the chunked branch) and a 2-D shared expert with their scale bits."""
    g = np.load(os.path.join(GOLDEN, "reference_layout.npz"))
    for key in ("5x24x9", "2x16x4"):
        assert np.array_equal(ol.nibble_transpose(g["nt_w_" + key]), g["nt_t_" + key])
        assert np.array_equal(cport.nibble_transpose(g["nt_w_" + key]), g["nt_t_" + key])
    for pre in ("ntm_", "ntm_s"):                    # keys ntm_{w,s,b,pw,ps,pb}, ntm_s{...}
        out = ol.to_neuron_major(g[pre + "w"], g[pre + "s"], g[pre + "b"])
        for got, name in zip(out, ("pw", "ps", "pb")):
            assert np.array_equal(got, g[pre + name]), (pre, name)


@pytest.mark.parametrize("shape", REF_HASHED_SHAPES)
def test_nibble_transpose_reference_hash(shape):
    """The reference test's larger shapes: the oracle's transpose of the seeded words hashes to
    the sha256 of the reference code's own transpose of the same words."""
    g = np.load(os.path.join(GOLDEN, "reference_layout.npz"))
    t = ol.nibble_transpose(reference_words(shape))
    assert sha256_np(t) == str(g["nt_sha_" + "x".join(map(str, shape))])


@pytest.mark.parametrize("case", reference_tile_cases(), ids=lambda c: c[0])
def test_build_tiles_matches_reference_code(case):
    """build_tiles against the reference's own hsd/prefill.py:247-278 on seeded routings:
    uniform, Zipf-skewed, every slot on one expert, one token, E < tt and E >= tt."""
    from oracle import prefill as op
    name, sel, E, tt, te_ref, ts_ref = case
    te, ts = op.build_tiles(sel, E, tt)
    assert np.array_equal(te, te_ref) and np.array_equal(ts, ts_ref)
    T, K = sel.shape
    assert sum(op.num_tiles(T, K, E, tt)) == te_ref.shape[0]


def test_down_projection_matches_reference_code():
    """The oracle against y of the reference test's own fp32 reference (tests/test_layout_decode.py
    :128-142 of the reference, run unmodified on a numpy stand-in of mlx.core): within the
    reference test's bound 2e-3 of max|ref| with the unrounded weights s*q + b (what the
    kernels use), and within 1e-5 once the dequantised weights are rounded to bf16 the way
    the stand-in's mx.dequantize returns them -- so the two differ by that rounding alone."""
    dims, g = reference_down_case()
    F, FS, topk = dims["F"], dims["FS"], dims["topk"]
    f = bf16_bits_to_f32
    hf = f(g["h"])
    y = od.reference_dense(hf, g["sel"], g["gains"], g["w"], f(g["s"]), f(g["b"]), g["sw"], f(g["ss"]),
                           f(g["sb"]), F=F, FS=FS, topk=topk)
    assert rel_err(y, g["y"]) < 2e-3

    def bf16(x):
        u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)

    Wd = bf16(dequantize(g["w"], f(g["s"]), f(g["b"])))           # [E, D, F]
    Ws = bf16(dequantize(g["sw"], f(g["ss"]), f(g["sb"])))          # [D, FS]
    yr = np.zeros_like(y, dtype=np.float64)
    for t in range(dims["B"]):
        for k in range(topk):
            yr[t] += g["gains"][t, k] * (Wd[g["sel"][t, k]].astype(np.float64) @ hf[t, k * F:(k + 1) * F])
        yr[t] += Ws.astype(np.float64) @ hf[t, topk * F:]
    assert rel_err(yr, g["y"]) < 1e-5


def test_c_transpose_matches_numpy():
    rng = np.random.default_rng(1)
    w = rng.integers(0, 2**32, size=(3, 64, 12), dtype=np.uint64).astype(np.uint32)
    assert np.array_equal(cport.nibble_transpose(w), ol.nibble_transpose(w))


def test_to_neuron_major_is_the_same_bytes():
    """Dequantising the neuron-major layout gives exactly the checkpoint layout's weights
    (the reference's tests/test_layout_decode.py:70-83, on synthetic weights)."""
    from hsd_b200 import synth
    gen = torch.Generator().manual_seed(3)
    w, s, b = synth.quantized_weights((4, 128, 192), gen, "cpu")
    w = w.numpy().view(np.uint32)
    s = bf16_bits_to_f32(s.view(torch.int16).numpy().view(np.uint16))
    b = bf16_bits_to_f32(b.view(torch.int16).numpy().view(np.uint16))
    pw, ps, pb = ol.to_neuron_major(w, s, b)
    ref = dequantize(w, s, b)                               # [E, D, F]
    out = dequantize_neuron_major(pw, ps, pb)               # [E, F, D]
    assert np.array_equal(np.swapaxes(out, -1, -2), ref)


def _golden_decode():
    g = np.load(os.path.join(GOLDEN, "decode_small.npz"))
    D, F, FS, E, topk, B = (int(x) for x in g["dims"])
    return g, D, F, FS, topk


def test_decode_golden_both_restatements():
    g, D, F, FS, topk = _golden_decode()
    f = bf16_bits_to_f32
    h = f(g["h"])
    y1 = od.reference_dense(h, g["sel"], g["gains"], g["w"], f(g["s"]), f(g["b"]), g["sw"], f(g["ss"]),
                            f(g["sb"]), F=F, FS=FS, topk=topk)
    assert rel_err(y1, g["y"]) < 1e-6
    y2 = od.sparse_live(h, g["sel"], g["gains"], g["pw"], f(g["ps"]), f(g["pb"]), g["spw"], f(g["sps"]),
                        f(g["spb"]), F=F, FS=FS, topk=topk)
    assert rel_err(y2, g["y"]) < 1e-5
    y3 = cport.sparse_down(h, g["sel"], g["gains"], g["pw"], g["ps"], g["pb"], g["spw"], g["sps"], g["spb"],
                           F=F, FS=FS, D=D, topk=topk)
    assert rel_err(y3, g["y"]) < 1e-5
    y4 = cport.dense_down(h, g["sel"], g["gains"], g["w"], g["s"], g["b"], g["sw"], g["ss"], g["sb"],
                          F=F, FS=FS, D=D, topk=topk)
    assert rel_err(y4, g["y"]) < 1e-5


def test_decode_restatements_agree_reference_shapes():
    """At the reference shapes (one token, 90 % zeros) the dense fp32 dequantised path and
    the live-row algebra agree to fp32 summation order."""
    from hsd_b200 import synth
    c = synth.decode_case(seed=11, B=1, E=16, zero_frac=0.9)
    f = bf16_bits_to_f32
    w = c["w"].numpy().view(np.uint32)
    s, b = (x.view(torch.int16).numpy().view(np.uint16) for x in (c["s"], c["b"]))
    sw = c["sw"].numpy().view(np.uint32)
    ss, sb = (x.view(torch.int16).numpy().view(np.uint16) for x in (c["ss"], c["sb"]))
    h = c["h"].float().numpy()
    sel, gains = c["sel"].numpy(), c["gains"].numpy()
    kw = dict(F=c["F"], FS=c["FS"], topk=c["topk"])
    y_ref = od.reference_dense(h, sel, gains, w, f(s), f(b), sw, f(ss), f(sb), **kw)
    pw, ps, pb = ol.to_neuron_major(w, s, b)
    spw, sps, spb = ol.to_neuron_major(sw, ss, sb)
    y_c = cport.sparse_down(h, sel, gains, pw, ps, pb, spw, sps, spb, D=c["D"], **kw)
    assert rel_err(y_c, y_ref) < 1e-4


def test_live_rows_and_byte_model():
    h = np.zeros((2, 3 * 64 + 128), np.float32)
    h[0, [1, 5, 64]] = 1.0
    h[1, [1, 200, 300]] = 2.0
    sel = np.array([[0, 1], [0, 2]], np.int32)
    lr = od.live_rows(h, F=96, FS=128, topk=2)
    assert list(lr[0][0]) == [1, 5, 64] and list(lr[0][1]) == [] and list(lr[1][2]) == [8, 108]
    nb = od.needed_bytes(h, sel, F=96, FS=128, D=64, topk=2)
    # rows: (0,1),(0,5),(0,64) for token 0 slot 0; (0,1) again for token 1 -> union 3; shared 2
    assert nb["rows"] == 3 + 2
    assert nb["groups"] == 2 + 2   # (0,0),(0,1) routed; (-1,0),(-1,1) shared


def test_prefill_tiles_oracle_properties():
    """The tile order restatement: every routed slot appears exactly once, in a tile of its
    expert, ascending inside the expert; shared tiles hold every token once."""
    from oracle import prefill as op
    rng = np.random.default_rng(2)
    T, K, E, tt = 100, 6, 16, 32
    sel = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    te, ts = op.build_tiles(sel, E, tt)
    nr, ns = op.num_tiles(T, K, E, tt)
    assert te.shape == (nr + ns,) and ts.shape == ((nr + ns) * tt,)
    routed = ts[:nr * tt]
    seen = routed[routed >= 0]
    assert sorted(seen.tolist()) == list(range(T * K))
    for t in range(nr):
        sl = ts[t * tt:(t + 1) * tt]
        sl = sl[sl >= 0]
        if te[t] < 0:
            assert sl.size == 0
        else:
            assert np.all(sel.reshape(-1)[sl] == te[t]) and np.all(np.diff(sl) > 0)
    assert np.all(te[nr:] == E)
    sh = ts[nr * tt:]
    assert sorted(sh[sh >= 0].tolist()) == list(range(T))


@pytest.mark.parametrize("T,topk,E,tt", [(300, 2, 8, 128), (37, 3, 8, 4), (1, 6, 128, 128), (100, 6, 16, 32),
                                           (129, 1, 2, 128), (4096, 6, 128, 128), (1000, 6, 100, 128)])
def test_routed_tile_bound_is_tight_and_holds(T, topk, E, tt):
    """The reference's fixed routed tile count T*topk//tt + E (hsd/prefill.py:266) is an upper
    bound for every routing: with T*topk = q*tt + r, the tiles needed are at most
    q + E + (r - E)/tt < q + E + 1. Checked on the routing that needs the most tiles -- one
    slot on each of E - 1 experts and the rest on one (tight when r >= E) -- and on a
    uniform one: every slot is placed."""
    from oracle import prefill as op
    N = T * topk
    flat = np.full(N, E - 1, np.int32)
    flat[:min(E - 1, N)] = np.arange(min(E - 1, N))
    rng = np.random.default_rng(T + E)
    for sel in (flat.reshape(T, topk), rng.integers(0, E, size=(T, topk)).astype(np.int32)):
        counts = np.bincount(sel.reshape(-1), minlength=E)
        need = int(((counts + tt - 1) // tt).sum())
        nr, ns = op.num_tiles(T, topk, E, tt)
        assert need <= nr == N // tt + E
        te, ts = op.build_tiles(sel, E, tt)
        routed = ts[:nr * tt]
        assert sorted(routed[routed >= 0].tolist()) == list(range(N))
    r = N % tt
    if r >= E:
        assert int(((np.bincount(flat, minlength=E) + tt - 1) // tt).sum()) == nr


def test_prefill_union_oracle_small():
    from oracle import prefill as op
    h = np.zeros((2, 2 * 64 + 64), np.float32)
    h[0, 3] = 1; h[1, 64 + 7] = 1; h[1, 128 + 5] = 1
    sel = np.array([[0, 1], [1, 0]], np.int32)
    te, ts = op.build_tiles(sel, 2, 4)
    ul, uc = op.build_union(h, te, ts, F=64, FS=64, topk=2, E=2, tt=4, umax=64)
    # expert 0: slots 0 (t0,k0: col 3) and 3 (t1,k1: col 7) -> [3, 7]; expert 1: slots 1, 2 -> []
    assert list(ul[0, :uc[0]]) == [3, 7] and uc[1] == 0 and np.all(ul[1] == -1)
    assert list(ul[te.tolist().index(2), :1]) == [5]


def _mamba_golden():
    g = np.load(os.path.join(GOLDEN, "mamba_mixer.npz"))
    H, P, G, N = (int(v) for v in g["dims"])
    p = dict(H=H, P=P, G=G, N=N, eps=float(g["eps"][0]), in_proj=g["in_proj"], conv_w=g["conv_w"],
             conv_b=g["conv_b"], A_log=g["A_log"], D=g["D"], dt_bias=g["dt_bias"], norm_w=g["norm_w"],
             out_proj=g["out_proj"])
    return g, p


def test_mamba_oracle_matches_transformers_mixer():
    """The row-by-row recurrence from a zero state equals transformers' chunked SSD path."""
    from oracle import mamba as om
    g, p = _mamba_golden()
    out, _, _ = om.mixer_rows(p, g["x"], None, None)
    assert rel_err(out, g["out"]) < 1e-4


def test_mamba_oracle_verify_then_rollback_equals_single_steps():
    """verify(L rows) then rollback(n) == n single steps (hsd/mamba.py:19-56), on the oracle."""
    from oracle import mamba as om
    g, p = _mamba_golden()
    x = g["x"]
    _, padded, states = om.mixer_rows(p, x[:5], None, None)
    conv_n, state_n = om.rollback(padded, states, 3)
    conv, st = None, None
    for t in range(3):
        _, pad1, s1 = om.mixer_rows(p, x[t:t + 1], conv, st)
        conv, st = pad1[1:], s1[0]
    # (the conv inputs come from a 5-row vs 1-row in_proj matmul: equal up to summation order)
    assert np.allclose(conv_n, conv, rtol=1e-5, atol=1e-6)
    assert np.allclose(state_n, st, rtol=1e-5, atol=1e-6)
    # and continuing after the rollback reproduces the longer run
    out_a, _, _ = om.mixer_rows(p, x[3:5], conv_n, state_n)
    out_b, _, _ = om.mixer_rows(p, x[:5], None, None)
    assert rel_err(out_a, out_b[3:5]) < 1e-5
