"""Affine 4-bit group-64 format, numpy (test infrastructure only; see oracle/__init__.py).

Format (hsd/layout.py:3-7 and hsd/decode.py:13-15,128 of the reference): uint32 words,
8 nibbles per word, low nibble first, groups of 64 along the reduction axis,
W = s * q + b with bf16 (or f16) s and b.
"""
import numpy as np

GS = 64


def bf16_bits_to_f32(u16):
    """bf16 bit patterns (uint16) -> float32, exact."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def unpack_nibbles(w):
    """[.., CW] uint32 -> [.., 8*CW] uint8, element 8j + n = nibble n of word j."""
    w = np.asarray(w, dtype=np.uint32)
    shifts = (4 * np.arange(8, dtype=np.uint32))
    nib = (w[..., None] >> shifts) & np.uint32(0xF)
    return nib.reshape(*w.shape[:-1], w.shape[-1] * 8).astype(np.uint8)


def pack_nibbles(q):
    """[.., C] values 0..15 -> [.., C/8] uint32 (inverse of unpack_nibbles)."""
    q = np.asarray(q, dtype=np.uint32)
    *lead, C = q.shape
    q = q.reshape(*lead, C // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.uint32))
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def dequantize(w, s, b, gs=GS):
    """Checkpoint layout: w [.., R, C/8] u32, s / b [.., R, C/gs] f32 -> W [.., R, C] f32."""
    q = unpack_nibbles(w).astype(np.float32)
    *lead, R, C = q.shape
    q = q.reshape(*lead, R, C // gs, gs)
    W = np.asarray(s, np.float32)[..., None] * q + np.asarray(b, np.float32)[..., None]
    return W.reshape(*lead, R, C)


def dequantize_neuron_major(pw, ps, pb, gs=GS):
    """Neuron-major layout: pw [.., F, D/8], ps / pb [.., F/gs, D] f32 -> W^T [.., F, D] f32."""
    q = unpack_nibbles(pw).astype(np.float32)                     # [.., F, D]
    s = np.repeat(np.asarray(ps, np.float32), gs, axis=-2)       # [.., F, D]
    b = np.repeat(np.asarray(pb, np.float32), gs, axis=-2)
    return s * q + b
