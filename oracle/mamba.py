"""Mamba-2 layer for multi-row verify and rollback, numpy float32 (test infrastructure only;
see oracle/__init__.py).

Restates hsd/mamba.py:19-56 of the reference with mlx-lm's ssm_update (mlx-lm 0.31.3, not
vendored; its published Mamba-2 selective state update):

    dt_t   = clip(softplus(dt[t] + dt_bias), *time_step_limit)       per head
    dA     = exp(dt_t * A),  A = -exp(A_log)
    state  = state * dA + (dt_t * x[t]) outer B[t, group(h)]          [H, P, N]
    y[t]   = state . C[t, group(h)] + D * x[t]

rows processed one after another from state0, the conv window crossing the verify boundary
(padded = [conv_state; conv_in], out = silu(depthwise conv, kernel 4, + bias)), the gated
group RMSNorm (y * silu(gate), RMS per group, times the weight) and the block around it
(x + out_proj(norm(...(in_proj(rms_norm(x)))))). Rollback to n_keep rows keeps
padded[n_keep : n_keep + 3] and the state after row n_keep - 1.
Pinned against transformers' NemotronHMamba2Mixer (tests/golden/make_mamba_golden.py).
"""
import numpy as np


def softplus(x):
    x = np.asarray(x, np.float32)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def silu(x):
    x = np.asarray(x, np.float32)
    return (x / (1.0 + np.exp(-x))).astype(np.float32)


def rms_norm(x, w, eps):
    x = np.asarray(x, np.float32)
    var = (x * x).mean(-1, keepdims=True)
    return (x / np.sqrt(var + eps) * np.asarray(w, np.float32)).astype(np.float32)


def gated_rms_norm(y, gate, w, group_size, eps):
    y = np.asarray(y, np.float32) * silu(gate)
    *lead, last = y.shape
    g = y.reshape(*lead, last // group_size, group_size)
    g = g / np.sqrt((g * g).mean(-1, keepdims=True) + eps)
    return (g.reshape(*lead, last) * np.asarray(w, np.float32)).astype(np.float32)


def conv_rows(conv_in, conv_state, w, bias):
    """conv_in [L, C], conv_state [K-1, C] (None: zeros), w [C, K], bias [C] or None ->
    (silu(conv) [L, C], padded [K-1+L, C])."""
    conv_in = np.asarray(conv_in, np.float32)
    L, C = conv_in.shape
    K = w.shape[1]
    st = np.zeros((K - 1, C), np.float32) if conv_state is None else np.asarray(conv_state, np.float32)
    padded = np.concatenate([st, conv_in], 0)
    out = np.zeros((L, C), np.float32)
    for j in range(K):
        out += padded[j:j + L] * np.asarray(w, np.float32)[:, j]
    if bias is not None:
        out += np.asarray(bias, np.float32)
    return silu(out), padded


def ssm_rows(x, B, C, dt, A_log, D, dt_bias, state0, time_step_limit=(0.0, np.inf)):
    """x [L, H, P], B / C [L, G, N], dt [L, H]; A_log, D, dt_bias [H]; state0 [H, P, N] (None:
    zeros) -> (y [L, H, P], states [L, H, P, N]: the state after each row)."""
    x = np.asarray(x, np.float32)
    L, H, P = x.shape
    G, N = B.shape[1], B.shape[2]
    rep = H // G
    A = -np.exp(np.asarray(A_log, np.float32))
    state = np.zeros((H, P, N), np.float32) if state0 is None else np.array(state0, np.float32)
    ys = np.zeros((L, H, P), np.float32)
    states = np.zeros((L, H, P, N), np.float32)
    lo, hi = time_step_limit
    for t in range(L):
        dtt = np.clip(softplus(np.asarray(dt[t], np.float32) + np.asarray(dt_bias, np.float32)), lo, hi)
        dA = np.exp(dtt * A).astype(np.float32)                               # [H]
        Bh = np.repeat(np.asarray(B[t], np.float32), rep, axis=0)             # [H, N]
        Ch = np.repeat(np.asarray(C[t], np.float32), rep, axis=0)
        state = state * dA[:, None, None] + (dtt[:, None] * x[t])[:, :, None] * Bh[:, None, :]
        ys[t] = (state * Ch[:, None, :]).sum(-1) + np.asarray(D, np.float32)[:, None] * x[t]
        states[t] = state
    return ys, states


def mixer_rows(p, h, conv_state, state0, time_step_limit=(0.0, np.inf)):
    """The Mamba-2 mixer on h [L, hidden] (already normed): in_proj -> (gate, conv_in, dt) ->
    conv + silu -> (x, B, C) -> ssm -> gated norm -> out_proj. p: dict with in_proj [proj, hidden],
    conv_w [C, K], conv_b [C], A_log, D, dt_bias [H], norm_w [I], out_proj [hidden, I], and the
    sizes H, P, G, N, eps. -> (out [L, hidden], padded, states)."""
    H, P, G, N = p["H"], p["P"], p["G"], p["N"]
    I = H * P
    conv_dim = I + 2 * G * N
    proj = np.asarray(h, np.float32) @ np.asarray(p["in_proj"], np.float32).T
    gate, conv_in, dt = proj[:, :I], proj[:, I:I + conv_dim], proj[:, I + conv_dim:]
    co, padded = conv_rows(conv_in, conv_state, p["conv_w"], p.get("conv_b"))
    L = h.shape[0]
    x = co[:, :I].reshape(L, H, P)
    Bm = co[:, I:I + G * N].reshape(L, G, N)
    Cm = co[:, I + G * N:].reshape(L, G, N)
    y, states = ssm_rows(x, Bm, Cm, dt, p["A_log"], p["D"], p["dt_bias"], state0, time_step_limit)
    yn = gated_rms_norm(y.reshape(L, I), gate, p["norm_w"], I // G, p["eps"])
    return yn @ np.asarray(p["out_proj"], np.float32).T, padded, states


def rollback(padded, states, n_keep, kernel=4):
    """The reference's rollback (hsd/mamba.py:47-56) on recorded quantities: the conv window
    after n_keep rows and the state after row n_keep - 1."""
    return padded[n_keep:n_keep + kernel - 1], states[n_keep - 1]
