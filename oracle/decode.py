"""Sparse MoE down projection for decode, numpy (test infrastructure only; see
oracle/__init__.py).

Two independent restatements that must agree:
  reference_dense   the reference test's fp32 dequantised reference
                    (tests/test_layout_decode.py:128-142): dequantise the checkpoint
                    layout, y[b] = sum_k score[b,k] * Wd[sel[b,k]] @ h[b,k] + Wsd @ hs[b]
  sparse_live       the Metal kernel's algebra on the neuron-major layout
                    (hsd/decode.py:105-144): per 64-group over the live rows only,
                    out += s * sum(h q) + b * sum(h), times the slot's gain, summed over slots
plus the active-index sets (hsd/decode.py:86-101) and the byte model of the benchmark
(bench/common.py:78-83).
"""
import numpy as np

from .quant import GS, dequantize, unpack_nibbles


def reference_dense(h, sel, gains, w, s, b, sw, ss, sb, *, F, FS, topk):
    """Checkpoint layout (w [E, D, F/8], s / b [E, D, F/64] f32; sw [D, FS/8], ss / sb
    [D, FS/64]); h [B, topk*F+FS] f32, sel [B, topk], gains [B, topk+1] -> y [B, D] f32."""
    h = np.asarray(h, np.float32)
    B = h.shape[0]
    Ws = dequantize(sw, ss, sb)                                      # [D, FS]
    D = Ws.shape[0]
    y = np.zeros((B, D), np.float32)
    cache = {}
    for bi in range(B):
        for k in range(topk):
            e = int(sel[bi, k])
            if e not in cache:
                cache[e] = dequantize(w[e], s[e], b[e])              # [D, F]
            y[bi] += np.float32(gains[bi, k]) * (cache[e] @ h[bi, k * F:(k + 1) * F])
        y[bi] += np.float32(gains[bi, topk]) * (Ws @ h[bi, topk * F:])
    return y


def _slot_live(hv, pw_rows, ps_e, pb_e):
    """One (token, slot): hv [W] f32 h of the slot, pw_rows [W, D/8] u32, ps_e / pb_e
    [W/64, D] f32 -> the slot's output [D] (per-group affine over the live rows)."""
    D = ps_e.shape[1]
    out = np.zeros(D, np.float32)
    for g in range(hv.shape[0] // GS):
        hg = hv[g * GS:(g + 1) * GS]
        live = np.flatnonzero(hg != 0)
        if live.size == 0:
            continue                                   # whole group dead: no scales, no biases
        q = unpack_nibbles(pw_rows[g * GS + live]).astype(np.float32)   # [n_live, D]
        acc = hg[live] @ q
        hsum = np.float32(hg[live].sum(dtype=np.float32))
        out += ps_e[g] * acc + pb_e[g] * hsum
    return out


def sparse_live(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS, topk):
    """Neuron-major layout (pw [E, F, D/8], ps / pb [E, F/64, D] f32; spw [FS, D/8],
    sps / spb [FS/64, D]) -> y [B, D] f32, reading live rows only."""
    h = np.asarray(h, np.float32)
    B = h.shape[0]
    D = ps.shape[-1]
    y = np.zeros((B, D), np.float32)
    for bi in range(B):
        for k in range(topk):
            e = int(sel[bi, k])
            y[bi] += np.float32(gains[bi, k]) * _slot_live(h[bi, k * F:(k + 1) * F], pw[e], ps[e], pb[e])
        y[bi] += np.float32(gains[bi, topk]) * _slot_live(h[bi, topk * F:], spw, sps, spb)
    return y


def live_rows(h, *, F, FS, topk):
    """The active-index sets: [[ascending nonzero indices of h[b, slot]] per slot] per b."""
    h = np.asarray(h)
    out = []
    for bi in range(h.shape[0]):
        row = [np.flatnonzero(h[bi, k * F:(k + 1) * F] != 0).astype(np.int32) for k in range(topk)]
        row.append(np.flatnonzero(h[bi, topk * F:] != 0).astype(np.int32))
        out.append(row)
    return out


def needed_bytes(h, sel, *, F, FS, D, topk, h_bytes=2, y_bytes=2, s_bytes=2):
    """Bytes one launch must move: the union over the batch of live (expert, neuron) rows
    x D/2, live (expert, 64-group) pairs x 2*D*s_bytes, plus h in and y out.
    -> dict(rows, groups, row_bytes, meta_bytes, io_bytes, total)."""
    h = np.asarray(h)
    sel = np.asarray(sel)
    B = h.shape[0]
    rows, groups = set(), set()
    for bi in range(B):
        for k in range(topk + 1):
            e = int(sel[bi, k]) if k < topk else -1
            hv = h[bi, k * F:(k + 1) * F] if k < topk else h[bi, topk * F:]
            nz = np.flatnonzero(hv != 0)
            rows.update((e, int(i)) for i in nz)
            groups.update((e, int(i) // GS) for i in nz)
    row_b = len(rows) * (D // 2)
    meta_b = len(groups) * 2 * D * s_bytes
    io_b = h.size * h_bytes + B * D * y_bytes
    return dict(rows=len(rows), groups=len(groups), row_bytes=row_b, meta_bytes=meta_b,
                io_bytes=io_b, total=row_b + meta_b + io_b)
