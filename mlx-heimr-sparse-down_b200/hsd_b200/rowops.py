"""Per-row operators of the decode step around the hot path (csrc/hsd_norm.cu): RMSNorm,
the Mamba-2 gated norm and the MoE router, each one launch, no host reads (capturable)."""
import torch

from . import _lib


def rms_norm(x, w, eps, out=None):
    """NemotronH RMSNorm: w * cast(x * rsqrt(mean(x^2) + eps)); x [B, D] (rows may be strided)."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("rms_norm: x must be 2-D with contiguous rows")
    B, D = x.shape
    if out is None:
        out = torch.empty((B, D), dtype=x.dtype, device=x.device)
    _lib.call("hsd_rms_norm", _lib.ptr(x), _lib.dtype_code(x, "rms_norm"), x.stride(0), _lib.ptr(w),
              _lib.dtype_code(w, "rms_norm"), _lib.ptr(out), _lib.dtype_code(out, "rms_norm"), B, D, float(eps),
              _lib.stream_of(x))
    return out


def gated_rms_norm(y, gate, w, group, eps, out_dtype):
    """The Mamba-2 gated norm: w * cast(g * rsqrt(mean_group(g^2) + eps)), g = y * silu(gate)."""
    if y.dim() != 2 or y.stride(1) != 1 or gate.stride(1) != 1 or gate.shape != y.shape:
        raise ValueError("gated_rms_norm: y and gate must be 2-D [B, I] with contiguous rows")
    B, I = y.shape
    out = torch.empty((B, I), dtype=out_dtype, device=y.device)
    _lib.call("hsd_gated_rms_norm", _lib.ptr(y), _lib.dtype_code(y, "y"), y.stride(0), _lib.ptr(gate),
              _lib.dtype_code(gate, "gate"), gate.stride(0), _lib.ptr(w), _lib.dtype_code(w, "w"), _lib.ptr(out),
              _lib.dtype_code(out, "out"), B, I, group, float(eps), _lib.stream_of(y))
    return out


class Router:
    """The MoE router with its scratch (scores, ticket) kept across calls."""

    def __init__(self, R, topk):
        if R.dtype != torch.float32 or R.dim() != 2 or not R.is_contiguous():
            raise ValueError("Router: R must be a contiguous fp32 [E, D] tensor")
        self.R, self.topk = R, topk
        self.E, self.D = R.shape
        self.ticket = torch.zeros(1, dtype=torch.int32, device=R.device)
        self._scores = {}

    def __call__(self, x):
        """x [B, D] -> (sel [B, topk] int32, gains [B, topk+1] f32)."""
        B = x.shape[0]
        sc = self._scores.get(B)
        if sc is None:
            sc = self._scores[B] = torch.empty((B, self.E), dtype=torch.float32, device=x.device)
        sel = torch.empty((B, self.topk), dtype=torch.int32, device=x.device)
        gains = torch.empty((B, self.topk + 1), dtype=torch.float32, device=x.device)
        _lib.call("hsd_router_topk", _lib.ptr(x), _lib.dtype_code(x, "router"), x.stride(0), _lib.ptr(self.R), B,
                  self.D, self.E, self.topk, _lib.ptr(sc), _lib.ptr(self.ticket), _lib.ptr(sel), _lib.ptr(gains),
                  _lib.stream_of(x))
        return sel, gains


class DecodeAttention:
    """GQA attention of decode rows over a fixed-size cache with a device-side position
    (hsd_attn_decode): q [L, QH*HD] (rows may be strided), k / v caches [KVH, max_len, HD]
    bf16, pos int64 [1] on the device -> out [L, QH*HD] bf16. Keeps its fp32 workspace."""

    def __init__(self, q_heads, kv_heads, head_dim, max_len, rows, device):
        import ctypes
        self.QH, self.KVH, self.HD, self.max_len, self.rows = q_heads, kv_heads, head_dim, max_len, rows
        nb = ctypes.c_size_t(0)
        _lib.call("hsd_attn_decode_workspace_bytes", rows, q_heads, max_len, ctypes.byref(nb))
        self.ws = torch.empty(nb.value // 4, dtype=torch.float32, device=device)
        self.scale = head_dim ** -0.5

    def __call__(self, q, kc, vc, pos):
        L = q.shape[0]
        if L > self.rows or q.dtype != torch.bfloat16 or q.stride(1) != 1:
            raise ValueError(f"DecodeAttention: at most {self.rows} bf16 rows with contiguous columns")
        out = torch.empty((L, self.QH * self.HD), dtype=torch.bfloat16, device=q.device)
        _lib.call("hsd_attn_decode", _lib.ptr(q), q.stride(0), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(pos),
                  _lib.ptr(out), _lib.ptr(self.ws), L, self.QH, self.KVH, self.HD, self.max_len, float(self.scale),
                  _lib.stream_of(q))
        return out
