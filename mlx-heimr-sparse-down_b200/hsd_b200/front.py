"""The MoE front end's up projections with relu2 (hsd/model.py:110-121 front), fused.

One launch of `moe_up_kernel` (csrc/hsd_up.cu) replaces the reference's gather_qmm of fc1
over the selected experts, the shared expert's quantised up_proj and the two relu2 calls,
and writes the down kernel's input hcat = [h of slots 0..topk-1 | hs] directly
(hsd/model.py:123-130 pack). The selected experts are read on the device, so the call
never synchronises with the host and can be captured in a CUDA graph.
"""
import torch

from . import _lib


def moe_up(x, sel, uw, us, ub, suw, sus, sub, *, F, FS, D, topk, out_dtype=torch.bfloat16, out=None):
    """x [B, D] (rows may be strided), sel [B, topk] int32 -> hcat [B, topk*F + FS].

    uw [E, F, D/8] u32, us / ub [E, F, D/64]: the routed experts' fc1 (checkpoint layout,
    4-bit g64 along D); suw [FS, D/8], sus / sub [FS, D/64]: the shared expert's up_proj.
    hcat[b, k*F + f] = relu(x[b] . Wu[sel[b, k], f])^2 and hcat[b, topk*F + f] =
    relu(x[b] . Wsu[f])^2, fp32 accumulation and one rounding to out_dtype."""
    what = "moe_up"
    _lib.require_cuda(sel, uw, us, ub, suw, sus, sub, out, what=what)
    if not x.is_cuda or x.dim() != 2 or x.stride(1) != 1 or x.shape[1] != D:
        raise ValueError(f"{what}: x must be a CUDA [B, {D}] tensor with contiguous rows")
    B = x.shape[0]
    E = uw.shape[0] if topk > 0 else 0
    if topk > 0:
        if sel is None or tuple(sel.shape) != (B, topk) or sel.dtype != torch.int32:
            raise ValueError(f"{what}: sel must be int32 [{B}, {topk}]")
        if tuple(uw.shape) != (E, F, D // 8) or tuple(us.shape) != (E, F, D // 64) or us.shape != ub.shape:
            raise ValueError(f"{what}: routed up weights {tuple(uw.shape)} {tuple(us.shape)} do not match F={F} D={D}")
    if FS > 0 and (tuple(suw.shape) != (FS, D // 8) or tuple(sus.shape) != (FS, D // 64) or sus.shape != sub.shape):
        raise ValueError(f"{what}: shared up weights do not match FS={FS} D={D}")
    sref = us if topk > 0 else sus
    if out is None:
        out = torch.empty((B, topk * F + FS), dtype=out_dtype, device=x.device)
    elif tuple(out.shape) != (B, topk * F + FS):
        raise ValueError(f"{what}: out must be [{B}, {topk * F + FS}]")
    if B == 0 or topk * F + FS == 0:
        return out
    _lib.call("hsd_moe_up_decode", _lib.ptr(x), _lib.dtype_code(x, what), x.stride(0), _lib.ptr(sel),
              _lib.ptr(uw), _lib.ptr(us), _lib.ptr(ub), _lib.dtype_code(sref, what), _lib.ptr(suw), _lib.ptr(sus),
              _lib.ptr(sub), _lib.ptr(out), _lib.dtype_code(out, what), B, D, F, FS, topk, E, _lib.stream_of(x))
    return out


def qlinear(x, w, s, b, *, resid=None, out_dtype=None, out=None):
    """A 4-bit g64 linear for decode rows: x [B, in_f] (rows may be strided), w [out_f, in_f/8],
    s / b [out_f, in_f/64] -> y [B, out_f] = x W^T (+ resid), fp32 accumulation, one rounding."""
    what = "qlinear"
    _lib.require_cuda(w, s, b, resid, out, what=what)
    if not x.is_cuda or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError(f"{what}: x must be a 2-D CUDA tensor with contiguous rows")
    B, in_f = x.shape
    out_f = w.shape[0]
    if tuple(w.shape) != (out_f, in_f // 8) or tuple(s.shape) != (out_f, in_f // 64) or s.shape != b.shape:
        raise ValueError(f"{what}: weights {tuple(w.shape)} {tuple(s.shape)} do not match in_f={in_f}")
    od = out_dtype or x.dtype
    if out is None:
        out = torch.empty((B, out_f), dtype=od, device=x.device)
    if resid is not None and (resid.dtype != out.dtype or tuple(resid.shape) != (B, out_f)):
        raise ValueError(f"{what}: resid must be {out.dtype} [{B}, {out_f}]")
    if B == 0:
        return out
    _lib.call("hsd_qlinear_decode", _lib.ptr(x), _lib.dtype_code(x, what), x.stride(0), _lib.ptr(w), _lib.ptr(s),
              _lib.ptr(b), _lib.dtype_code(s, what), _lib.ptr(resid), _lib.ptr(out), _lib.dtype_code(out, what),
              B, in_f, out_f, _lib.stream_of(x))
    return out
