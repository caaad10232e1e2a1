"""The MoE front end's up projections with relu2 (hsd/model.py:110-121 front), fused.

One launch of `moe_up_kernel` (csrc/hsd_up.cu) replaces the reference's gather_qmm of fc1
over the selected experts, the shared expert's quantised up_proj and the two relu2 calls,
and writes the down kernel's input hcat = [h of slots 0..topk-1 | hs] directly
(hsd/model.py:123-130 pack). The selected experts are read on the device, so the call
never synchronises with the host and can be captured in a CUDA graph.
"""
import torch

from . import _lib
from . import synth

QGEMV_ROWS = 8          # rows up to which a 4-bit linear runs the matrix-vector kernel


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


def dequant_affine4(w, s, b, dtype=torch.bfloat16):
    """Packed [.., R, C/8] words + [.., R, C/64] scales / biases -> [.., R, C] (fp32 s*q + b)."""
    shifts = 4 * torch.arange(8, device=w.device, dtype=torch.int32)
    q = (w.unsqueeze(-1) >> shifts) & 15
    q = q.reshape(*w.shape[:-1], w.shape[-1] * 8).float()
    R, C = q.shape[-2], q.shape[-1]
    qg = q.view(*q.shape[:-1], C // 64, 64)
    W = qg * s.float().unsqueeze(-1) + b.float().unsqueeze(-1)
    return W.view(*q.shape[:-2], R, C).to(dtype)


class QLinear:
    """A 4-bit g64 linear (mlx QuantizedLinear): w [out, in/8], s / b [out, in/64]. Decode rows
    (<= QGEMV_ROWS) use hsd_qlinear_decode on the packed weights; longer prompt chunks use a
    dequantised bf16 copy with cuBLAS (kept when bf16_copy)."""

    def __init__(self, out_f, in_f, gen, device, std, bf16_copy=True):
        """Seeded random weights N(0, std), quantised."""
        w, s, b = synth.quantized_weights((out_f, in_f), gen, device, std=std)
        self._set(w, s, b, bf16_copy)

    @classmethod
    def from_packed(cls, w, s, b, bf16_copy=True):
        """Existing packed weights w [out, in/8] u32, s / b [out, in/64]."""
        q = cls.__new__(cls)
        q._set(w, s, b, bf16_copy)
        return q

    def _set(self, w, s, b, bf16_copy):
        self.w, self.s, self.b = w, s, b
        self.out_f, self.in_f = w.shape[0], w.shape[1] * 8
        self.dq = dequant_affine4(w, s, b) if bf16_copy else None

    def dequant_f32(self):
        """The dequantised weights in fp32 (s*q + b), [out, in]."""
        return dequant_affine4(self.w, self.s, self.b, torch.float32)

    def __call__(self, x, resid=None, out_dtype=None):
        if x.shape[0] <= QGEMV_ROWS or self.dq is None:
            return qlinear(x, self.w, self.s, self.b, resid=resid, out_dtype=out_dtype)
        y = x @ self.dq.t()
        if resid is not None:
            y = (resid.float() + y.float()).to(resid.dtype)
        return y if out_dtype is None else y.to(out_dtype)
