"""Generates the committed golden fixtures of tests/golden/ (run from the repo root:
python tests/golden/make_golden.py). Deterministic: fixed seeds.

nibble_transpose_*.npz
    Seeded uint32 words of the reference test's smallest shape (5, 24, 9) and a second
    small shape, and their transpose computed by a one-nibble-at-a-time Python loop that
    restates the reference's known-answer method (tests/test_layout_decode.py:38-52 of the
    reference: unpack each word to 8 nibbles, move them, pack them again). The loop is
    independent of the vectorised oracle it pins.
decode_small.npz
    A small MoE down-projection case (checkpoint layout and neuron-major layout, h with
    ~90 % zeros, routing, gains) and its fp32 dequantised output y, computed by the oracle's
    reference_dense (the reference test's fp32 reference, tests/test_layout_decode.py
    :128-142) after checking it agrees with the independent sparse_live restatement.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "mlx-heimr-sparse-down_b200"))


def slow_transpose(w):
    lead = w.shape[:-2]
    R, CW = w.shape[-2:]
    out = np.zeros((*lead, CW * 8, R // 8), np.uint32)
    for idx in np.ndindex(*lead) if lead else [()]:
        for r in range(R):
            for c in range(CW * 8):
                q = (int(w[idx + (r, c // 8)]) >> (4 * (c % 8))) & 0xF
                out[idx + (c, r // 8)] |= np.uint32(q << (4 * (r % 8)))
    return out


def make_layout():
    rng = np.random.default_rng(20260101)
    for shape in ((5, 24, 9), (2, 16, 4)):
        w = rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32)
        t = slow_transpose(w)
        name = "nibble_transpose_" + "x".join(map(str, shape)) + ".npz"
        np.savez_compressed(os.path.join(HERE, name), w=w, t=t)
        print("wrote", name)


def make_decode():
    import torch
    from hsd_b200 import synth
    from oracle import decode as od
    from oracle import layout as ol
    from oracle.quant import bf16_bits_to_f32

    D, F, FS, E, topk, B = 256, 128, 256, 8, 2, 3
    c = synth.decode_case(seed=7, B=B, D=D, F=F, FS=FS, E=E, topk=topk, zero_frac=0.9)
    w = c["w"].view(torch.int32).numpy().view(np.uint32)
    s = c["s"].view(torch.int16).numpy().view(np.uint16)
    b = c["b"].view(torch.int16).numpy().view(np.uint16)
    sw = c["sw"].view(torch.int32).numpy().view(np.uint32)
    ss = c["ss"].view(torch.int16).numpy().view(np.uint16)
    sb = c["sb"].view(torch.int16).numpy().view(np.uint16)
    h = c["h"].view(torch.int16).numpy().view(np.uint16)          # bf16 bits
    sel = c["sel"].numpy()
    gains = c["gains"].numpy()
    hf = bf16_bits_to_f32(h)
    y = od.reference_dense(hf, sel, gains, w, bf16_bits_to_f32(s), bf16_bits_to_f32(b), sw,
                           bf16_bits_to_f32(ss), bf16_bits_to_f32(sb), F=F, FS=FS, topk=topk)
    pw, ps, pb = ol.to_neuron_major(w, s, b)
    spw, sps, spb = ol.to_neuron_major(sw, ss, sb)
    y2 = od.sparse_live(hf, sel, gains, pw, bf16_bits_to_f32(ps), bf16_bits_to_f32(pb), spw,
                        bf16_bits_to_f32(sps), bf16_bits_to_f32(spb), F=F, FS=FS, topk=topk)
    err = np.abs(y - y2).max() / np.abs(y).max()
    assert err < 1e-5, err
    np.savez_compressed(os.path.join(HERE, "decode_small.npz"), w=w, s=s, b=b, sw=sw, ss=ss, sb=sb,
                        h=h, sel=sel, gains=gains, pw=pw, ps=ps, pb=pb, spw=spw, sps=sps, spb=spb, y=y,
                        dims=np.array([D, F, FS, E, topk, B]))
    print("wrote decode_small.npz, live fraction", float((hf != 0).mean()))


if __name__ == "__main__":
    make_layout()
    make_decode()
