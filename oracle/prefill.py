"""Prefill path, numpy (test infrastructure only; see oracle/__init__.py).

build_tiles   restates hsd/prefill.py:247-278: slots t*topk + k sorted by expert (stable:
              ascending slot inside an expert), tiles of tt slots of one expert at
              tile_base[e] = sum of earlier experts' ceil(count / tt), a fixed routed tile
              count T*topk//tt + E, -1 for empty tiles and padding, then the
              shared expert's ceil(T/tt) tiles of tokens (expert id E).
build_union   restates hsd/prefill.py:48-93,281-291: per tile the ascending columns nonzero
              in any slot, -1 padded to umax.
prefill_y     the dequantised fp32 reference of the whole chunk: per token
              sum_k gain * Wd[sel] @ h_k + gain_s * Wsd @ h_s (hsd/prefill.py:11-16,211-221,320).
"""
import numpy as np

from .decode import reference_dense


def num_tiles(T, topk, E, tt):
    return T * topk // tt + E, (T + tt - 1) // tt


def build_tiles(sel, E, tt):
    sel = np.asarray(sel)
    T, K = sel.shape
    nr, ns = num_tiles(T, K, E, tt)
    flat = sel.reshape(-1)
    counts = np.bincount(flat, minlength=E)[:E]
    ntile = (counts + tt - 1) // tt
    tile_base = np.cumsum(ntile) - ntile
    tile_e = np.full(nr + ns, -1, np.int32)
    tile_slot = np.full((nr + ns) * tt, -1, np.int32)
    for e in range(E):
        tile_e[tile_base[e]:tile_base[e] + ntile[e]] = e
        slots = np.flatnonzero(flat == e)                 # ascending = stable
        for r, j in enumerate(slots):
            tile_slot[(tile_base[e] + r // tt) * tt + r % tt] = j
    tile_e[nr:] = E
    tile_slot[nr * tt:nr * tt + T] = np.arange(T)
    return tile_e, tile_slot


def build_union(h, tile_e, tile_slot, *, F, FS, topk, E, tt, umax):
    h = np.asarray(h)
    NT = tile_e.shape[0]
    ulist = np.full((NT, umax), -1, np.int32)
    ucount = np.zeros(NT, np.int32)
    for t in range(NT):
        e = int(tile_e[t])
        if e < 0:
            continue
        rows = []
        for m in range(tt):
            s = int(tile_slot[t * tt + m])
            if s < 0:
                continue
            if e >= E:
                rows.append(h[s, topk * F:topk * F + FS])
            else:
                rows.append(h[s // topk, (s % topk) * F:(s % topk + 1) * F])
        live = np.flatnonzero(np.any(np.stack(rows) != 0, axis=0)) if rows else np.zeros(0, np.int64)
        ulist[t, :live.size] = live
        ucount[t] = live.size
    return ulist, ucount


def prefill_y(h, sel, gains, w, s, b, sw, ss, sb, *, F, FS, topk):
    """Dense fp32 dequantised reference for a whole chunk (checkpoint layout, f32 s / b)."""
    return reference_dense(h, sel, gains, w, s, b, sw, ss, sb, F=F, FS=FS, topk=topk)
