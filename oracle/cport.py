"""numpy front end of the C oracle (test infrastructure only; see oracle/__init__.py)."""
import ctypes

import numpy as np

from .build import load


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def nibble_transpose(w):
    w = np.ascontiguousarray(w, dtype=np.uint32)
    *lead, R, CW = w.shape
    n = int(np.prod(lead)) if lead else 1
    out = np.empty((*lead, CW * 8, R // 8), np.uint32)
    load().oracle_nibble_transpose(_p(w), _p(out), n, R, CW)
    return out


def sparse_down(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS, D, topk, sl=None, nthreads=0):
    """The reference kernel's algorithm on the CPU. h f32 [B, topk*F+FS]; pw / spw uint32;
    ps / pb / sps / spb bf16 bit patterns (uint16) -> y [B, D] f32."""
    h = np.ascontiguousarray(h, np.float32)
    B = h.shape[0]
    if sl is None:
        sl = 928 if (F % 928 == 0 and FS % 928 == 0) else 64
    y = np.empty((B, D), np.float32)
    arrs = [h, np.ascontiguousarray(sel, np.int32), np.ascontiguousarray(gains, np.float32),
            np.ascontiguousarray(pw, np.uint32), np.ascontiguousarray(ps, np.uint16),
            np.ascontiguousarray(pb, np.uint16), np.ascontiguousarray(spw, np.uint32),
            np.ascontiguousarray(sps, np.uint16), np.ascontiguousarray(spb, np.uint16)]
    load().oracle_sparse_down(*[_p(a) for a in arrs], _p(y), B, D, F, FS, topk, sl, nthreads)
    return y


def dense_down(h, sel, gains, w, s, b, sw, ss, sb, *, F, FS, D, topk, nthreads=0):
    """The dequantised dense path on the checkpoint layout (bf16 bit patterns for s / b)."""
    h = np.ascontiguousarray(h, np.float32)
    B = h.shape[0]
    y = np.empty((B, D), np.float32)
    arrs = [h, np.ascontiguousarray(sel, np.int32), np.ascontiguousarray(gains, np.float32),
            np.ascontiguousarray(w, np.uint32), np.ascontiguousarray(s, np.uint16),
            np.ascontiguousarray(b, np.uint16), np.ascontiguousarray(sw, np.uint32),
            np.ascontiguousarray(ss, np.uint16), np.ascontiguousarray(sb, np.uint16)]
    load().oracle_dense_down(*[_p(a) for a in arrs], _p(y), B, D, F, FS, topk, nthreads)
    return y
