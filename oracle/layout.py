"""Neuron-major permutation, numpy (test infrastructure only; see oracle/__init__.py).

Restates hsd/layout.py:34-50 (nibble_transpose) and :53-74 (to_neuron_major) of the
reference: unpack every nibble, swap the last two axes, pack again.
"""
import numpy as np

from .quant import pack_nibbles, unpack_nibbles


def nibble_transpose(w):
    """[.., R, C/8] u32 -> [.., C, R/8] u32, out[.., c, wo] packs W[8*wo + n, c]."""
    nib = unpack_nibbles(w)                   # [.., R, C]
    nibT = np.swapaxes(nib, -1, -2)           # [.., C, R]
    return pack_nibbles(np.ascontiguousarray(nibT))


def to_neuron_major(w, s, b):
    """(w [.., D, F/8], s / b [.., D, F/64]) -> (pw [.., F, D/8], ps / pb [.., F/64, D])."""
    return (nibble_transpose(w), np.ascontiguousarray(np.swapaxes(s, -1, -2)),
            np.ascontiguousarray(np.swapaxes(b, -1, -2)))
