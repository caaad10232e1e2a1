"""The MoE front end's up projections, numpy (test infrastructure only; see
oracle/__init__.py).

hsd/model.py:110-121 of the reference: the routed up projection is mlx's gather_qmm of the
normalised token against fc1 of each selected expert (affine 4-bit g64 along the hidden
axis, checkpoint layout [E, F, D/8]), the shared expert's up_proj is a quantised linear of
the same format, and both go through relu2 = square(relu(u)). The down kernel's input is
then hcat = [h of slot 0 .. topk-1 | hs] (hsd/model.py:123-130).
"""
import numpy as np

from .quant import dequantize


def moe_up(x, sel, uw, us, ub, suw, sus, sub, *, topk):
    """x [B, D] f32, sel [B, topk]; uw [E, F, D/8] u32, us / ub [E, F, D/64] f32; suw
    [FS, D/8], sus / sub [FS, D/64] (or None) -> hcat [B, topk*F + FS] f32 after relu2."""
    x = np.asarray(x, np.float32)
    B = x.shape[0]
    parts = []
    cache = {}
    for bi in range(B):
        row = []
        for k in range(topk):
            e = int(sel[bi, k])
            if e not in cache:
                cache[e] = dequantize(uw[e], us[e], ub[e])            # [F, D]
            row.append(cache[e] @ x[bi])
        if suw is not None:
            if "shared" not in cache:
                cache["shared"] = dequantize(suw, sus, sub)           # [FS, D]
            row.append(cache["shared"] @ x[bi])
        parts.append(np.concatenate(row) if row else np.zeros(0, np.float32))
    u = np.stack(parts).astype(np.float32)
    return np.square(np.maximum(u, 0.0))
