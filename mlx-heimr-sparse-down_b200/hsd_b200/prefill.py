"""Sparse MoE down projection for prefill (hsd/prefill.py), on the neuron-major layout.

The (token, expert-slot) pairs of a chunk are sorted by expert into tiles of slots with a
FIXED tile count (no host readback), each tile's h rows are gathered as fp16, and a
tcgen05 grouped GEMM (csrc/hsd_prefill_gemm.cu) multiplies them with the expert's weights,
dequantised to fp16 in shared memory per 64-neuron group and accumulated in fp32 in TMEM;
the routing gain is applied in the epilogue and each token's topk+1 partial rows are summed
in a fixed order. The GEMM's tile is 128 slots.
"""
import ctypes

import torch

from . import _lib

GEMM_TT = 128      # slots per tile of the tensor-core GEMM (its M)


def num_tiles(T, topk, E, tt):
    """(nt_routed, nt_shared) of the fixed tile order."""
    a, b = ctypes.c_int(0), ctypes.c_int(0)
    _lib.call("hsd_prefill_num_tiles", T, topk, E, tt, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def build_tiles(sel, E, tt):
    """hsd/prefill.py:247 -- sel [T, topk] int32 -> (tile_e [NT] int32, tile_slot [NT*tt] int32).

    Routed tiles hold slots t*topk + k of one expert in ascending order, then the shared
    expert's tiles (expert id E) hold tokens t; empty tiles carry -1, padding slots -1."""
    _lib.require_cuda(sel, what="build_tiles")
    if sel.dim() != 2 or sel.dtype != torch.int32:
        raise ValueError("build_tiles: sel must be int32 [T, topk]")
    T, topk = sel.shape
    nr, ns = num_tiles(T, topk, E, tt)
    tile_e = torch.empty(nr + ns, dtype=torch.int32, device=sel.device)
    tile_slot = torch.empty((nr + ns) * tt, dtype=torch.int32, device=sel.device)
    _lib.call("hsd_prefill_build_tiles", _lib.ptr(sel), T, topk, E, tt, _lib.ptr(tile_e), _lib.ptr(tile_slot),
              _lib.stream_of(sel))
    return tile_e, tile_slot


def build_union(h, tile_e, tile_slot, *, F, FS, topk, E, tt, kc=32, nth=256):
    """hsd/prefill.py:281 -- per tile the ascending union of the columns nonzero in any of its
    slots -> (ulist [NT, UMAX] int32, -1 padded; ucount [NT] int32), UMAX = max(F, FS)
    rounded up to kc. nth is the Metal kernel's thread count (no effect here)."""
    del nth
    _lib.require_cuda(h, tile_e, tile_slot, what="build_union")
    NT = tile_e.shape[0]
    umax = (max(F, FS) + kc - 1) // kc * kc
    ulist = torch.empty((NT, umax), dtype=torch.int32, device=h.device)
    ucount = torch.empty(NT, dtype=torch.int32, device=h.device)
    _lib.call("hsd_prefill_build_union", _lib.ptr(h), _lib.dtype_code(h, "build_union"), _lib.ptr(tile_e),
              _lib.ptr(tile_slot), NT, tt, F, FS, topk, E, umax, _lib.ptr(ulist), _lib.ptr(ucount),
              _lib.stream_of(h))
    return ulist, ucount


def workspace_bytes(T, D, F, FS, topk, E):
    n = ctypes.c_size_t(0)
    _lib.call("hsd_prefill_workspace_bytes", T, D, F, FS, topk, E, ctypes.byref(n))
    return n.value


def sparse_down_prefill(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS, D, topk, E,
                        tt=32, nb=64, kc=32, nsg=4, tiles=None, union=None, out_dtype=None,
                        resid=None, out=None, workspace=None):
    """hsd/prefill.py:294 -- the MoE down projection over a prompt chunk.

    h [T, topk*F + FS], sel [T, topk] int32, gains [T, topk+1] f32 -> y [T, D] (out_dtype or
    h's dtype). tt / nb / kc / nsg are the Metal kernel's tuning knobs and have no effect:
    the GEMM tiles 128 slots x 192 outputs x 64 neurons. `tiles` is used when it was built
    with tt = 128, otherwise the tile order is rebuilt on the device; `union` is accepted for
    signature parity (the GEMM reads every 64-group). resid [T, D] is added in the reduce;
    `workspace` (uint8, >= workspace_bytes()) avoids an allocation per call."""
    del tt, nb, kc, nsg, union
    what = "sparse_down_prefill"
    _lib.require_cuda(h, sel, gains, pw, ps, pb, spw, sps, spb, resid, out, what=what)
    T = h.shape[0]
    if h.shape[1] != topk * F + FS or tuple(sel.shape) != (T, topk) or tuple(gains.shape) != (T, topk + 1):
        raise ValueError(f"{what}: h / sel / gains shapes do not match T={T} topk={topk} F={F} FS={FS}")
    if sel.dtype != torch.int32 or gains.dtype != torch.float32:
        raise ValueError(f"{what}: sel must be int32 and gains float32")
    od = out_dtype or h.dtype
    if out is None:
        out = torch.empty((T, D), dtype=od, device=h.device)
    if T == 0:
        return out
    nr, ns = num_tiles(T, topk, E, GEMM_TT)
    if tiles is None or tiles[0].shape[0] != nr + ns or tiles[1].shape[0] != (nr + ns) * GEMM_TT:
        tiles = build_tiles(sel, E, GEMM_TT)
    tile_e, tile_slot = tiles
    need = workspace_bytes(T, D, F, FS, topk, E)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=h.device)
    _lib.call("hsd_sparse_down_prefill", _lib.ptr(h), _lib.dtype_code(h, what), _lib.ptr(gains), _lib.ptr(tile_e),
              _lib.ptr(tile_slot), tile_e.shape[0], _lib.ptr(pw), _lib.ptr(ps), _lib.ptr(pb), _lib.dtype_code(ps, what),
              _lib.ptr(spw), _lib.ptr(sps), _lib.ptr(spb), _lib.ptr(resid), _lib.ptr(out), _lib.dtype_code(out, what),
              T, D, F, FS, topk, E, _lib.ptr(workspace), workspace.numel(), _lib.stream_of(h))
    return out
