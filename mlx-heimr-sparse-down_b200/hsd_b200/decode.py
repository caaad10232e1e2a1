"""Sparse MoE down projection for decode (hsd/decode.py), on the neuron-major layout.

One launch of the sm_100a kernel `sparse_down_decode_kernel` (csrc/hsd_decode.cu): it
compacts the nonzero h entries of every (token, expert) with warp ballots, stages only the
live rows' weight chunks and the live 64-groups' scale / bias chunks with 16-byte
asynchronous copies, accumulates in fp32 and sums the per-expert partials through
distributed shared memory of an 8-CTA cluster in a fixed order (deterministic, no scratch).
"""
import torch

from . import _lib


def sparse_down(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS, D, topk,
                sl=928, unr=2, nds=3, out_dtype=None, loadsc=1, resid=None, out=None, all_rows=False):
    """hsd/decode.py:164 -- the down projection over the live rows only.

    h [B, topk*F + FS] (bf16 / f16 / f32), sel [B, topk] int32 (the routed experts),
    gains [B, topk+1] f32 (routing scores, then the shared expert's gain, 1) -> y [B, D].
    pw [E, F, D/8] / ps, pb [E, F/64, D]: the routed experts, neuron-major;
    spw [FS, D/8] / sps, spb [FS/64, D]: the shared expert.

    sl / unr / nds are the Metal kernel's tuning knobs; they are accepted for signature
    parity and have no effect here. loadsc=0 skips the scale / bias loads (benchmark-only,
    as in the reference). resid [B, D] (out dtype), when given, is added in the kernel
    (y = resid + down(h)); out, when given, receives y. all_rows=True is the dense form
    (hsd_dense_down_decode_nm): every row read, the same reduction order, so the sparse form
    reproduces it bit for bit.
    """
    del sl, unr, nds
    what = "sparse_down"
    _lib.require_cuda(h, sel, gains, pw, ps, pb, spw, sps, spb, resid, out, what=what)
    if h.dim() != 2 or gains.dim() != 2:
        raise ValueError(f"{what}: h and gains must be 2-D")
    B = h.shape[0]
    E = pw.shape[0] if pw is not None else 0
    if h.shape[1] != topk * F + FS:
        raise ValueError(f"{what}: h has {h.shape[1]} columns, expected topk*F+FS = {topk * F + FS}")
    if tuple(gains.shape) != (B, topk + 1) or gains.dtype != torch.float32:
        raise ValueError(f"{what}: gains must be float32 [{B}, {topk + 1}]")
    if topk > 0:
        if sel is None or tuple(sel.shape) != (B, topk) or sel.dtype != torch.int32:
            raise ValueError(f"{what}: sel must be int32 [{B}, {topk}]")
        if tuple(pw.shape) != (E, F, D // 8) or tuple(ps.shape) != (E, F // 64, D) or ps.shape != pb.shape:
            raise ValueError(f"{what}: routed layout shapes {tuple(pw.shape)} {tuple(ps.shape)} {tuple(pb.shape)}"
                             f" do not match E={E} F={F} D={D}")
    if FS > 0:
        if tuple(spw.shape) != (FS, D // 8) or tuple(sps.shape) != (FS // 64, D) or sps.shape != spb.shape:
            raise ValueError(f"{what}: shared layout shapes do not match FS={FS} D={D}")
    sref = ps if topk > 0 else sps
    for t in (pb, sps, spb):
        if t is not None and t.dtype != sref.dtype:
            raise TypeError(f"{what}: scales and biases must share one 16-bit dtype")
    od = out_dtype or h.dtype
    if out is None:
        out = torch.empty((B, D), dtype=od, device=h.device)
    elif out.dtype != od or tuple(out.shape) != (B, D):
        raise ValueError(f"{what}: out must be {od} [{B}, {D}]")
    if resid is not None and (resid.dtype != od or tuple(resid.shape) != (B, D)):
        raise ValueError(f"{what}: resid must be {od} [{B}, {D}]")
    if B == 0:
        return out
    if all_rows:
        _lib.call("hsd_dense_down_decode_nm", _lib.ptr(h), _lib.dtype_code(h, what), _lib.ptr(sel),
                  _lib.ptr(gains), _lib.ptr(pw), _lib.ptr(ps), _lib.ptr(pb), _lib.dtype_code(sref, what),
                  _lib.ptr(spw), _lib.ptr(sps), _lib.ptr(spb), _lib.ptr(resid), _lib.ptr(out),
                  _lib.dtype_code(out, what), B, D, F, FS, topk, E, _lib.stream_of(h))
        return out
    _lib.call("hsd_sparse_down_decode", _lib.ptr(h), _lib.dtype_code(h, what), _lib.ptr(sel),
              _lib.ptr(gains), _lib.ptr(pw), _lib.ptr(ps), _lib.ptr(pb), _lib.dtype_code(sref, what),
              _lib.ptr(spw), _lib.ptr(sps), _lib.ptr(spb), _lib.ptr(resid), _lib.ptr(out),
              _lib.dtype_code(out, what), B, D, F, FS, topk, E, 1 if loadsc else 0, _lib.stream_of(h))
    return out


def live_rows(h, *, F, FS, topk):
    """The active-index sets: per (token, slot) the ascending indices of nonzero h entries,
    from the decode kernel's own ballot compaction.
    -> (live [B, topk+1, max(F, FS)] int32, valid up to count; count [B, topk+1] int32)."""
    _lib.require_cuda(h, what="live_rows")
    B = h.shape[0]
    live = torch.full((B, topk + 1, max(F, FS)), -1, dtype=torch.int32, device=h.device)
    count = torch.zeros((B, topk + 1), dtype=torch.int32, device=h.device)
    if B:
        _lib.call("hsd_decode_live_rows", _lib.ptr(h), _lib.dtype_code(h, "live_rows"), _lib.ptr(live),
                  _lib.ptr(count), B, F, FS, topk, _lib.stream_of(h))
    return live, count


def dense_down(h, sel, gains, w, s, b, sw, ss, sb, *, F, FS, D, topk, out_dtype=None, resid=None, out=None,
               workspace=None):
    """The stock dense down projection (hsd/model.py:132-133 decode_dense) on the checkpoint
    layout: every weight of the selected experts, fp32 accumulation, the slot partials summed
    in slot order. w [E, D, F/8] / s, b [E, D, F/64]; sw [D, FS/8] / ss, sb [D, FS/64]; the
    other arguments as sparse_down. workspace: fp32 [B, topk+1, D] (allocated when None)."""
    what = "dense_down"
    _lib.require_cuda(h, sel, gains, w, s, b, sw, ss, sb, resid, out, workspace, what=what)
    B = h.shape[0]
    E = w.shape[0] if topk > 0 else 0
    if h.shape[1] != topk * F + FS or tuple(gains.shape) != (B, topk + 1) or gains.dtype != torch.float32:
        raise ValueError(f"{what}: h must be [B, topk*F+FS] and gains float32 [B, topk+1]")
    if topk > 0 and (tuple(w.shape) != (E, D, F // 8) or tuple(s.shape) != (E, D, F // 64)):
        raise ValueError(f"{what}: routed weights {tuple(w.shape)} do not match the checkpoint layout [E, D, F/8]")
    if FS > 0 and (tuple(sw.shape) != (D, FS // 8) or tuple(ss.shape) != (D, FS // 64)):
        raise ValueError(f"{what}: shared weights do not match [D, FS/8]")
    sref = s if topk > 0 else ss
    od = out_dtype or h.dtype
    if out is None:
        out = torch.empty((B, D), dtype=od, device=h.device)
    if workspace is None:
        workspace = torch.empty((B, topk + 1, D), dtype=torch.float32, device=h.device)
    elif workspace.numel() < B * (topk + 1) * D or workspace.dtype != torch.float32:
        raise ValueError(f"{what}: workspace must hold {B * (topk + 1) * D} fp32")
    if B == 0:
        return out
    _lib.call("hsd_dense_down_decode", _lib.ptr(h), _lib.dtype_code(h, what), _lib.ptr(sel), _lib.ptr(gains),
              _lib.ptr(w), _lib.ptr(s), _lib.ptr(b), _lib.dtype_code(sref, what), _lib.ptr(sw), _lib.ptr(ss),
              _lib.ptr(sb), _lib.ptr(resid), _lib.ptr(out), _lib.dtype_code(out, what), _lib.ptr(workspace),
              B, D, F, FS, topk, E, _lib.stream_of(h))
    return out
