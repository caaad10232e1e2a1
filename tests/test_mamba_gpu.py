"""Mamba-2 verify / rollback on the GPU (hsd/mamba.py:19-56; the reference's
tests/test_verify_rollback.py structure): the conv and scan kernels against the oracle, a
verify of L rows then a rollback to n equal to n single steps (bit for bit: the same
kernel runs the same row sequence), and the whole block against the oracle's mixer."""
import numpy as np
import pytest
import torch

from conftest import f32_np, rel_err
from oracle import mamba as om

from hsd_b200 import mamba as hm

# config 3: 64 heads x 64, state 128, 8 groups, conv 4 -> I 4096, conv_dim 6144
H, P, G, N, K = 64, 64, 8, 128, 4


def _inputs(L, seed, device, dtype=torch.bfloat16):
    gen = torch.Generator(device=device).manual_seed(seed)
    I, Cd = H * P, H * P + 2 * G * N
    xbc = torch.randn((L, Cd), generator=gen, device=device).to(dtype)
    dt = (torch.randn((L, H), generator=gen, device=device) * 0.5).to(dtype)
    A_log = torch.log(torch.linspace(1.0, 16.0, H, device=device))
    D = torch.rand(H, generator=gen, device=device) + 0.5
    dt_bias = torch.linspace(-4.0, -1.0, H, device=device)
    state0 = torch.randn((H, P, N), generator=gen, device=device) * 0.1
    return xbc, dt, A_log, D, dt_bias, state0


@pytest.mark.gpu
@pytest.mark.parametrize("L", [1, 3, 4])
def test_ssm_kernel_vs_oracle(cuda, L):
    xbc, dt, A_log, D, dt_bias, state0 = _inputs(L, 10 + L, cuda)
    y, states = hm.ssm_verify(xbc, dt, A_log, D, dt_bias, state0, H=H, P=P, G=G, N=N)
    I = H * P
    xb = f32_np(xbc)
    oy, ost = om.ssm_rows(xb[:, :I].reshape(L, H, P), xb[:, I:I + G * N].reshape(L, G, N),
                          xb[:, I + G * N:].reshape(L, G, N), f32_np(dt), f32_np(A_log), f32_np(D), f32_np(dt_bias),
                          f32_np(state0))
    assert rel_err(f32_np(states), ost) < 1e-5
    assert rel_err(f32_np(y).reshape(L, H, P), oy) < 1e-5


@pytest.mark.gpu
def test_conv_kernel_vs_oracle(cuda):
    L, Cd = 3, H * P + 2 * G * N
    gen = torch.Generator(device=cuda).manual_seed(3)
    proj = torch.randn((L, Cd + 100), generator=gen, device=cuda).to(torch.bfloat16)
    conv_in = proj[:, 50:50 + Cd]                                  # strided rows, as from in_proj
    state = torch.randn((K - 1, Cd), generator=gen, device=cuda).to(torch.bfloat16)
    w = torch.randn((Cd, K), generator=gen, device=cuda) * 0.3
    b = torch.randn(Cd, generator=gen, device=cuda) * 0.1
    out, padded = hm.conv_verify(conv_in, state, w, b, out_dtype=torch.float32)
    oout, opad = om.conv_rows(f32_np(conv_in), f32_np(state), f32_np(w), f32_np(b))
    assert np.array_equal(f32_np(padded), opad)
    assert rel_err(f32_np(out), oout) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("L,n_keep", [(3, 1), (3, 2), (3, 3), (4, 2)])
def test_verify_then_rollback_equals_single_steps(cuda, L, n_keep):
    """The reference's test_rollback_equals_n_single_steps (tests/test_verify_rollback.py:153-161)
    at the block level: verify(L) -> rollback(n) leaves the caches where n single steps do."""
    blk = hm.random_mamba2(5, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(6)
    x = torch.randn((1, L, 2688), generator=gen, device=cuda).to(torch.bfloat16)
    warm = torch.randn((1, 5, 2688), generator=gen, device=cuda).to(torch.bfloat16)
    c0 = [None, None]
    hm.mamba_verify(blk, warm, c0, [])                              # some history first
    cv = list(c0)
    rec = []
    out_v = hm.mamba_verify(blk, x, cv, rec)
    hm.mamba_rollback(rec, n_keep)
    cs = list(c0)
    outs = []
    for t in range(n_keep):
        outs.append(hm.mamba_verify(blk, x[:, t:t + 1], cs, []))
    # every piece computes a row independently of the call's other rows (the 4-bit linears, the
    # norms, the conv and the scan), so the rolled-back window and state are the single-step
    # ones bit for bit, and so are the outputs of the kept rows
    assert torch.equal(cv[0], cs[0])
    assert torch.equal(cv[1], cs[1])
    for t in range(n_keep):
        assert torch.equal(out_v[0, t], outs[t][0, 0])


@pytest.mark.gpu
def test_rollback_is_exact_on_identical_rows(cuda):
    """With the row inputs fixed (the scan kernel alone), the rolled-back state is the
    single-step state bit for bit."""
    L = 4
    xbc, dt, A_log, D, dt_bias, state0 = _inputs(L, 21, cuda)
    _, states = hm.ssm_verify(xbc, dt, A_log, D, dt_bias, state0, H=H, P=P, G=G, N=N)
    st = state0
    for t in range(3):
        _, s1 = hm.ssm_verify(xbc[t:t + 1], dt[t:t + 1], A_log, D, dt_bias, st, H=H, P=P, G=G, N=N)
        st = s1[0]
    assert torch.equal(states[2], st)
    # the copying rollback gives the same bits
    padded = torch.randn((K - 1 + L, 100), device=cuda).to(torch.bfloat16)
    conv_out = torch.empty((K - 1, 100), dtype=torch.bfloat16, device=cuda)
    state_out = torch.empty((H, P, N), device=cuda)
    hm.rollback_into(padded, states, 3, conv_out, state_out)
    assert torch.equal(state_out, st) and torch.equal(conv_out, padded[3:3 + K - 1])


@pytest.mark.gpu
def test_block_vs_oracle_mixer(cuda):
    blk = hm.random_mamba2(7, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(8)
    x = torch.randn((1, 3, 2688), generator=gen, device=cuda).to(torch.bfloat16)
    out = hm.mamba_verify(blk, x, [None, None], [])
    p = dict(H=H, P=P, G=G, N=N, eps=blk.eps, in_proj=f32_np(blk.in_proj.dequant_f32()),
             conv_w=f32_np(blk.conv_w), conv_b=f32_np(blk.conv_b), A_log=f32_np(blk.A_log), D=f32_np(blk.D),
             dt_bias=f32_np(blk.dt_bias), norm_w=f32_np(blk.gate_norm_w),
             out_proj=f32_np(blk.out_proj.dequant_f32()))
    hn = om.rms_norm(f32_np(x[0]), f32_np(blk.norm_w), blk.eps)
    ref, _, _ = om.mixer_rows(p, hn, None, None)
    assert rel_err(f32_np(out[0] - x[0]), ref) < 3e-2              # bf16 matmuls and activations


@pytest.mark.gpu
def test_long_chunk_final_state_only(cuda):
    """A prompt chunk of 300 rows (no rollback): the final state alone equals the last
    checkpoint of the full run, and the conv window is the chunk's last rows."""
    L = 300
    xbc, dt, A_log, D, dt_bias, state0 = _inputs(L, 31, cuda)
    y1, s_all = hm.ssm_verify(xbc, dt, A_log, D, dt_bias, state0, H=H, P=P, G=G, N=N)
    y2, s_last = hm.ssm_verify(xbc, dt, A_log, D, dt_bias, state0, H=H, P=P, G=G, N=N, checkpoints=False)
    assert s_last.shape[0] == 1 and torch.equal(s_last[0], s_all[-1]) and torch.equal(y1, y2)
    conv_in = torch.randn((L, 512), device=cuda).to(torch.bfloat16)
    w = torch.randn((512, K), device=cuda)
    out, padded = hm.conv_verify(conv_in, None, w, None, out_dtype=torch.float32)
    oout, opad = om.conv_rows(f32_np(conv_in), None, f32_np(w), None)
    assert np.array_equal(f32_np(padded), opad) and rel_err(f32_np(out), oout) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("accepts", [[0, 2, 1, 2], [2, 2, 0, 0]])
def test_resident_buffers_match_the_verify_rollback_path(cuda, accepts):
    """The graph-friendly form (conv / scan in place over fixed buffers, the rollback one
    device integer) against mamba_verify + mamba_rollback: a prefill, then verifies of 3 rows
    each followed by a rollback to the accepted prefix -- every output and the final state
    bit-identical."""
    blk = hm.random_mamba2(seed=4, hidden=512, H=16, P=32, G=4, N=64, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(9)
    x0 = torch.randn((1, 7, 512), generator=gen, device=cuda).to(torch.bfloat16)
    cache = [None, None]
    hm.mamba_verify(blk, x0, cache, [], checkpoints=False)
    rc = hm.ResidentMambaCache(blk, rows=3, device=cuda)
    rc.load(cache)
    n_keep = torch.ones(1, dtype=torch.int32, device=cuda)
    for step, a in enumerate(accepts):
        x = torch.randn((1, 3, 512), generator=gen, device=cuda).to(torch.bfloat16)
        rec = []
        ref = hm.mamba_verify(blk, x, cache, rec)[0]
        out = hm.mamba_step_resident(blk, x[0], rc, n_keep)
        assert torch.equal(out, ref), f"verify {step}: outputs differ"
        hm.mamba_rollback(rec, a + 1)
        n_keep.fill_(a + 1)
    assert torch.equal(rc.states[n_keep.item() - 1], cache[1])
    k = n_keep.item()
    assert torch.equal(rc.padded[k:k + blk.K - 1], cache[0])
    assert hm._lib.lib() is not None


@pytest.mark.gpu
def test_resident_single_steps_match_plain_steps(cuda):
    """A plain decode step is the resident form with L = 1 and n_keep = 1."""
    blk = hm.random_mamba2(seed=5, hidden=512, H=16, P=32, G=4, N=64, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(11)
    cache = [None, None]
    rc = hm.ResidentMambaCache(blk, rows=3, device=cuda)
    n_keep = torch.ones(1, dtype=torch.int32, device=cuda)
    for _ in range(5):
        x = torch.randn((1, 1, 512), generator=gen, device=cuda).to(torch.bfloat16)
        ref = hm.mamba_verify(blk, x, cache, [])[0]
        out = hm.mamba_step_resident(blk, x[0], rc, n_keep)
        assert torch.equal(out, ref)
    assert torch.equal(rc.states[0], cache[1])


@pytest.mark.gpu
def test_resident_bad_keep_is_flagged(cuda):
    import hsd_b200
    blk = hm.random_mamba2(seed=6, hidden=512, H=16, P=32, G=4, N=64, device=cuda)
    rc = hm.ResidentMambaCache(blk, rows=3, device=cuda)
    hsd_b200.device_status()
    n_keep = torch.full((1,), 9, dtype=torch.int32, device=cuda)
    x = torch.randn((1, 512), device=cuda).to(torch.bfloat16)
    hm.mamba_step_resident(blk, x, rc, n_keep)
    torch.cuda.synchronize()
    assert hsd_b200.device_status() == hsd_b200._lib.HSD_ERR_INDEX
