"""The neuron-major permutation of a quantised down projection (hsd/layout.py).

mlx-lm stores a quantised down projection as W[out=D, in=F]:

    words   [.., D, F/8]  u32   8 nibbles of one output row per word, low nibble first
    scales  [.., D, F/64]       groups along the reduction axis
    biases  [.., D, F/64]

Neuron-major (what the sparse kernels read):

    pw [.., F, D/8] u32   row i = neuron i, word w packs W[8w .. 8w+7, i]
    ps [.., F/64, D]
    pb [.., F/64, D]

so a dead neuron's weights are one contiguous D/2-byte row that is never read. The
permutation moves bytes only (no value is re-quantised) and its nibble part is
self-inverse. Packed words are carried in int32 or uint32 tensors (the same bits).
"""
import torch

from . import _lib

_WORD_DTYPES = (torch.int32, torch.uint32)


def _check_words(w, what):
    if w.dtype not in _WORD_DTYPES:
        raise TypeError(f"{what}: packed words must be int32 or uint32 (got {w.dtype})")
    _lib.require_cuda(w, what=what)


def nibble_transpose(w):
    """hsd/layout.py:34 -- [.., R, C/8] packed words -> [.., C, R/8], out[.., c, wo] packing
    W[8*wo + n, c] for n = 0..7, low nibble first. Exact and self-inverse (R % 8 == 0)."""
    _check_words(w, "nibble_transpose")
    if w.dim() < 2:
        raise ValueError("nibble_transpose: need at least 2 dims")
    *lead, R, CW = w.shape
    if R % 8:
        raise ValueError(f"nibble_transpose: rows ({R}) must be a multiple of 8")
    n_lead = 1
    for d in lead:
        n_lead *= d
    out = torch.empty((*lead, CW * 8, R // 8), dtype=w.dtype, device=w.device)
    if out.numel() == 0:
        return out
    # the kernel's grid takes up to 65535 leading blocks: split longer leading extents
    step = 65535
    wf = w.reshape(n_lead, R, CW)
    of = out.view(n_lead, CW * 8, R // 8)
    for i in range(0, n_lead, step):
        j = min(n_lead, i + step)
        _lib.call("hsd_nibble_transpose", _lib.ptr(wf[i:j]), _lib.ptr(of[i:j]), j - i, R, CW,
                  _lib.stream_of(w))
    return out


def swap_last2(x):
    """[.., R, C] 16-bit -> contiguous [.., C, R] (the scales / biases half of the layout)."""
    if x.element_size() != 2:
        raise TypeError(f"swap_last2: 16-bit tensors only (got {x.dtype})")
    _lib.require_cuda(x, what="swap_last2")
    *lead, R, C = x.shape
    n_lead = 1
    for d in lead:
        n_lead *= d
    out = torch.empty((*lead, C, R), dtype=x.dtype, device=x.device)
    if out.numel() == 0:
        return out
    step = 65535
    xf = x.reshape(n_lead, R, C)
    of = out.view(n_lead, C, R)
    for i in range(0, n_lead, step):
        j = min(n_lead, i + step)
        _lib.call("hsd_swap_last2_u16", _lib.ptr(xf[i:j]), _lib.ptr(of[i:j]), j - i, R, C,
                  _lib.stream_of(x))
    return out


def to_neuron_major(w, s, b, chunk=16):
    """hsd/layout.py:53 -- (w [.., D, F/8], s / b [.., D, F/64]) as mlx-lm stores a down
    projection -> (pw [.., F, D/8], ps [.., F/64, D], pb [.., F/64, D]).

    `chunk` is accepted for signature parity; the kernel transposes in place of MLX's
    nibble expansion, so no transient beyond the output is ever allocated."""
    del chunk
    return nibble_transpose(w), swap_last2(s), swap_last2(b)
