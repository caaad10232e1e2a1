"""Multi-row Mamba-2 steps with rollback, for speculative decoding (hsd/mamba.py).

A Mamba-2 layer's recurrent state (conv window, SSM state) advances by every row a verify
step processes. The reference records the verify's inputs and, on rollback, re-runs
mlx-lm's ssm_update over the kept rows. Here the verify kernel (csrc/hsd_mamba.cu) writes
the state after EVERY row while it runs (the per-row checkpoints, [L, H, P, N] fp32) and
the conv kernel keeps the padded window, so a rollback selects a checkpoint on the device
-- no recomputation and no host round trip. Rows run exactly as single steps would, so the
state after row n of a verify equals n single steps bit for bit.

The cache is a two-entry list like mlx-lm's ArraysCache: cache[0] the conv window
[K-1, conv_dim] (bf16, None at the start), cache[1] the SSM state [H, P, N] (fp32, None
at the start). Every piece of the block runs this library's kernels: in_proj / out_proj are
4-bit g64 linears like the reference checkpoint's QuantizedLinear (hsd_qlinear_decode for
verify and decode rows, the residual added inside out_proj's kernel; prompt chunks longer
than 8 rows use the linear's dequantised bf16 copy), the pre-norm and the gated norm are
hsd_rms_norm / hsd_gated_rms_norm, and the causal conv, the selective scan and the rollback
are csrc/hsd_mamba.cu.
"""
from dataclasses import dataclass

import torch

from . import _lib
from .front import QLinear
from .rowops import gated_rms_norm, rms_norm


@dataclass
class Mamba2Block:
    """One Mamba-2 block (pre-norm + mixer) of the Nemotron-H layer stack.

    norm_w [D]; in_proj a 4-bit linear [I + conv_dim + H, D] (gate | conv input | dt); conv_w
    [conv_dim, K] f32, conv_b [conv_dim] f32; A_log, D, dt_bias [H] f32; gate_norm_w [I];
    out_proj a 4-bit linear [D, I]."""
    norm_w: torch.Tensor
    in_proj: QLinear
    conv_w: torch.Tensor
    conv_b: torch.Tensor
    A_log: torch.Tensor
    D: torch.Tensor
    dt_bias: torch.Tensor
    gate_norm_w: torch.Tensor
    out_proj: QLinear
    H: int
    P: int
    G: int
    N: int
    K: int = 4
    eps: float = 1e-5
    time_step_limit: tuple = (0.0, float("inf"))

    @property
    def I(self):  # noqa: E743 -- the reference's intermediate_size
        return self.H * self.P

    @property
    def conv_dim(self):
        return self.H * self.P + 2 * self.G * self.N


def random_mamba2(seed, hidden=2688, H=64, P=64, G=8, N=128, K=4, device="cuda", dtype=torch.bfloat16,
                  std=0.02):
    """A seeded random-init block with the reference model's Mamba-2 shapes; the linears'
    weights N(0, std) quantised to 4-bit g64."""
    gen = torch.Generator(device=device).manual_seed(seed)
    I = H * P
    conv_dim = I + 2 * G * N

    return Mamba2Block(
        norm_w=(1.0 + 0.1 * torch.randn(hidden, generator=gen, device=device)).to(dtype),
        in_proj=QLinear(I + conv_dim + H, hidden, gen, device, std),
        conv_w=torch.randn((conv_dim, K), generator=gen, device=device) * 0.3,
        conv_b=torch.randn(conv_dim, generator=gen, device=device) * 0.1,
        A_log=torch.log(torch.linspace(1.0, 16.0, H, device=device)),
        D=torch.ones(H, device=device),
        dt_bias=torch.linspace(-4.0, -1.0, H, device=device),
        gate_norm_w=(1.0 + 0.1 * torch.randn(I, generator=gen, device=device)).to(dtype),
        out_proj=QLinear(hidden, I, gen, device, std),
        H=H, P=P, G=G, N=N, K=K)


def conv_verify(conv_in, conv_state, conv_w, conv_b, out_dtype=torch.bfloat16):
    """conv_in [L, C] (rows may be strided) -> (silu(conv) [L, C], padded [K-1+L, C])."""
    L, C = conv_in.shape
    K = conv_w.shape[1]
    _lib.require_cuda(conv_w, conv_b, what="conv_verify")
    if conv_in.stride(1) != 1:
        raise ValueError("conv_verify: conv_in rows must be contiguous")
    out = torch.empty((L, C), dtype=out_dtype, device=conv_in.device)
    padded = torch.empty((K - 1 + L, C), dtype=conv_in.dtype, device=conv_in.device)
    if conv_state is not None and (conv_state.dtype != conv_in.dtype or not conv_state.is_contiguous()):
        conv_state = conv_state.to(conv_in.dtype).contiguous()
    _lib.call("hsd_mamba_conv_verify", _lib.ptr(conv_in), _lib.dtype_code(conv_in, "conv_in"), conv_in.stride(0),
              _lib.ptr(conv_state), _lib.ptr(conv_w), _lib.dtype_code(conv_w, "conv_w"), _lib.ptr(conv_b),
              _lib.ptr(out), _lib.dtype_code(out, "out"), _lib.ptr(padded), L, C, K, _lib.stream_of(conv_in))
    return out, padded


def ssm_verify(xbc, dt, A_log, D, dt_bias, state0, *, H, P, G, N, time_step_limit=(0.0, float("inf")),
               y_dtype=torch.float32, checkpoints=True):
    """xbc [L, >= H*P + 2GN] (x | B | C), dt [L, >= H] -> (y [L, H*P], states [L, H, P, N] fp32:
    the state after every row; with checkpoints=False only the final one, [1, H, P, N])."""
    L = xbc.shape[0]
    if xbc.stride(1) != 1 or dt.stride(1) != 1:
        raise ValueError("ssm_verify: rows must be contiguous")
    if state0 is not None and (state0.dtype != torch.float32 or not state0.is_contiguous()):
        state0 = state0.float().contiguous()
    y = torch.empty((L, H * P), dtype=y_dtype, device=xbc.device)
    states = torch.empty((L if checkpoints else 1, H, P, N), dtype=torch.float32, device=xbc.device)
    lo, hi = time_step_limit
    _lib.call("hsd_mamba_ssm_verify", _lib.ptr(xbc), _lib.dtype_code(xbc, "xbc"), xbc.stride(0), _lib.ptr(dt),
              _lib.dtype_code(dt, "dt"), dt.stride(0), _lib.ptr(A_log), _lib.ptr(D), _lib.ptr(dt_bias), float(lo),
              float(hi), _lib.ptr(state0), _lib.ptr(states), _lib.ptr(y), _lib.dtype_code(y, "y"), L, H, P, G, N,
              0 if checkpoints else 1, _lib.stream_of(xbc))
    return y, states


def mamba_verify(block, x3, cache, records, checkpoints=True):
    """hsd/mamba.py:19 -- one Mamba-2 block on x3 [1, L, D] with the cache advanced by L rows;
    `records` gets what a later rollback needs (the padded conv window and the per-row states).
    checkpoints=False (a prompt chunk, never rolled back) keeps the final state only and records
    nothing. Returns x3 + mixer(norm(x3))."""
    b = block
    x = x3[0]
    L = x.shape[0]
    I, Cd = b.I, b.conv_dim
    h = rms_norm(x, b.norm_w, b.eps)
    proj = b.in_proj(h)                                           # [L, I + conv_dim + H]
    co, padded = conv_verify(proj[:, I:I + Cd], cache[0], b.conv_w, b.conv_b)
    y, states = ssm_verify(co, proj[:, I + Cd:], b.A_log, b.D, b.dt_bias, cache[1], H=b.H, P=b.P, G=b.G, N=b.N,
                           time_step_limit=b.time_step_limit, checkpoints=checkpoints)
    cache[0] = padded[L:]                                         # the last K-1 rows of the window
    cache[1] = states[-1]
    if checkpoints:
        records.append((cache, padded, states, b.K))
    yn = gated_rms_norm(y, proj[:, :I], b.gate_norm_w, I // b.G, b.eps, x.dtype)
    return b.out_proj(yn, resid=x)[None]                          # x3 + out_proj(yn), one rounding


def mamba_rollback(records, n_keep):
    """hsd/mamba.py:47 -- put every cache in `records` back at the state after the first
    n_keep rows: the conv window is padded[n_keep : n_keep+K-1] and the SSM state the
    verify's checkpoint of row n_keep-1. Views on the device; nothing is recomputed."""
    for cache, padded, states, K in records:
        if not 1 <= n_keep <= states.shape[0]:
            raise ValueError(f"mamba_rollback: n_keep {n_keep} outside 1..{states.shape[0]}")
        cache[0] = padded[n_keep:n_keep + K - 1]
        cache[1] = states[n_keep - 1]


def conv_step(conv_in, padded, n_keep, conv_w, conv_b, out_dtype=torch.bfloat16):
    """Resident-buffer conv: the window is padded[n_keep .. n_keep+K-2] (n_keep a device int32
    tensor holding the previous call's kept row count); padded [rows + K-1, C] receives the
    window and the L new rows in place. -> silu(conv) [L, C]."""
    L, C = conv_in.shape
    K = conv_w.shape[1]
    rows = padded.shape[0] - (K - 1)
    if conv_in.stride(1) != 1 or not padded.is_contiguous() or padded.dtype != conv_in.dtype:
        raise ValueError("conv_step: conv_in rows and padded must be contiguous, padded in conv_in's dtype")
    out = torch.empty((L, C), dtype=out_dtype, device=conv_in.device)
    _lib.call("hsd_mamba_conv_step", _lib.ptr(conv_in), _lib.dtype_code(conv_in, "conv_in"), conv_in.stride(0),
              _lib.ptr(padded), _lib.ptr(n_keep), rows, _lib.ptr(conv_w), _lib.dtype_code(conv_w, "conv_w"),
              _lib.ptr(conv_b), _lib.ptr(out), _lib.dtype_code(out, "out"), L, C, K, _lib.stream_of(conv_in))
    return out


def ssm_step(xbc, dt, A_log, D, dt_bias, states, n_keep, *, H, P, G, N, time_step_limit=(0.0, float("inf")),
             y_dtype=torch.float32):
    """Resident-buffer selective scan: the state is states[n_keep-1] (n_keep a device int32
    tensor), and the state after each of the L rows is written to states[0 .. L-1] in place
    (states [rows, H, P, N] fp32). -> y [L, H*P]."""
    L = xbc.shape[0]
    if xbc.stride(1) != 1 or dt.stride(1) != 1 or not states.is_contiguous() or states.dtype != torch.float32:
        raise ValueError("ssm_step: rows must be contiguous and states fp32 contiguous")
    y = torch.empty((L, H * P), dtype=y_dtype, device=xbc.device)
    lo, hi = time_step_limit
    _lib.call("hsd_mamba_ssm_step", _lib.ptr(xbc), _lib.dtype_code(xbc, "xbc"), xbc.stride(0), _lib.ptr(dt),
              _lib.dtype_code(dt, "dt"), dt.stride(0), _lib.ptr(A_log), _lib.ptr(D), _lib.ptr(dt_bias), float(lo),
              float(hi), _lib.ptr(states), _lib.ptr(n_keep), states.shape[0], _lib.ptr(y), _lib.dtype_code(y, "y"),
              L, H, P, G, N, _lib.stream_of(xbc))
    return y


class ResidentMambaCache:
    """A Mamba-2 layer's decode state in fixed buffers, for graph-replayed decode loops:
    padded [rows + K-1, conv_dim] (the conv window and the last call's rows) and states
    [rows, H, P, N] (the state after each row of the last call). The kept row count lives in
    one device int32 shared by all layers of a model (`n_keep`), so a rollback after a verify
    is a single device write."""

    def __init__(self, block, rows, device, dtype=torch.bfloat16):
        self.rows = rows
        self.padded = torch.zeros((rows + block.K - 1, block.conv_dim), dtype=dtype, device=device)
        self.states = torch.zeros((rows, block.H, block.P, block.N), dtype=torch.float32, device=device)

    def load(self, cache, n_keep_host=1):
        """Seed from an ArraysCache-style [conv window [K-1, C], state [H, P, N]] (prefill's
        result): window to padded[n_keep .. n_keep+K-2], state to states[n_keep-1]."""
        conv, st = cache
        k = n_keep_host
        self.padded.zero_()
        self.states.zero_()
        if conv is not None:
            self.padded[k:k + conv.shape[0]].copy_(conv)
        if st is not None:
            self.states[k - 1].copy_(st)


def mamba_step_resident(block, x, rc, n_keep):
    """One Mamba-2 block on x [L, D] (L <= rc.rows) over a ResidentMambaCache: the conv window
    and state come from the previous call's rows selected by n_keep, and every row's state is
    kept for a later rollback. Graph-capturable (no host reads, fixed buffers).
    Returns x + mixer(norm(x))."""
    b = block
    I, Cd = b.I, b.conv_dim
    h = rms_norm(x, b.norm_w, b.eps)
    proj = b.in_proj(h)
    co = conv_step(proj[:, I:I + Cd], rc.padded, n_keep, b.conv_w, b.conv_b)
    y = ssm_step(co, proj[:, I + Cd:], b.A_log, b.D, b.dt_bias, rc.states, n_keep, H=b.H, P=b.P, G=b.G, N=b.N,
                 time_step_limit=b.time_step_limit)
    yn = gated_rms_norm(y, proj[:, :I], b.gate_norm_w, I // b.G, b.eps, x.dtype)
    return b.out_proj(yn, resid=x)


def rollback_into(padded, states, n_keep, conv_out, state_out):
    """The rollback as copies into fixed buffers (for callers whose cache tensors must keep
    their addresses, e.g. a captured CUDA graph): conv_out [K-1, C] <- padded[n_keep:],
    state_out [H, P, N] <- states[n_keep-1]."""
    L, H, P, N = states.shape
    C = padded.shape[1]
    K = padded.shape[0] - L + 1
    _lib.call("hsd_mamba_rollback", _lib.ptr(states), _lib.ptr(padded), padded.element_size(), n_keep, L, H, P, N,
              C, K, _lib.ptr(state_out), _lib.ptr(conv_out), _lib.stream_of(states))
