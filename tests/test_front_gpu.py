"""The fused 4-bit matrix-vector kernels of the decode step on the GPU against the oracle:

  moe_up      the MoE front end's up projections + relu2 (hsd/model.py:110-121) vs
              oracle/front.py (fp32 dequantised weights, numpy matmul)
  dense_down  the stock dense down projection (hsd/model.py:132-133) vs the C oracle's fp32
              dequantised reference (the same one the sparse kernel is checked against)

Bars: 1e-3 of max|ref| for fp32 outputs (fp32 accumulation both sides, different order),
1e-2 for bf16 outputs (one bf16 rounding); an expert id outside [0, E) gives zeros for its
slot and HSD_ERR_INDEX in the device status word."""
import numpy as np
import pytest
import torch

from conftest import bits16_np, f32_np, rel_err, words_np
from oracle import cport
from oracle import front as ofront
from oracle.quant import bf16_bits_to_f32

import hsd_b200
from hsd_b200 import synth
from hsd_b200.decode import dense_down
from hsd_b200.front import moe_up

TOL32 = 1e-3
TOL16 = 1e-2


def up_case(seed, B, D, F, FS, E, topk, device):
    gen = torch.Generator(device=device).manual_seed(seed)
    uw, us, ub = synth.quantized_weights((E, F, D), gen, device)
    suw, sus, sub = synth.quantized_weights((FS, D), gen, device) if FS else (None, None, None)
    x = torch.randn((B, D), generator=gen, device=device).to(torch.bfloat16)
    logits = torch.randn((B, E), generator=gen, device=device)
    sel, _ = synth.route_topk(logits, topk) if topk else (torch.zeros((B, 0), dtype=torch.int32, device=device), None)
    return x, sel.to(torch.int32).contiguous(), (uw, us, ub), (suw, sus, sub)


def oracle_up(x, sel, up, sup, topk):
    uw, us, ub = up
    suw, sus, sub = sup
    f = lambda t: bf16_bits_to_f32(bits16_np(t)) if t is not None else None  # noqa: E731
    return ofront.moe_up(f32_np(x), sel.cpu().numpy(), words_np(uw) if uw is not None else None, f(us), f(ub),
                         words_np(suw) if suw is not None else None, f(sus), f(sub), topk=topk)


@pytest.mark.gpu
@pytest.mark.parametrize("B,D,F,FS,E,topk", [(1, 2688, 1856, 3712, 128, 6), (3, 2688, 1856, 3712, 128, 6),
                                              (5, 384, 256, 512, 16, 4), (2, 4096, 128, 64, 4, 2)])
def test_moe_up_vs_oracle(cuda, B, D, F, FS, E, topk):
    x, sel, up, sup = up_case(7 + B, B, D, F, FS, E, topk, cuda)
    ref = oracle_up(x, sel, up, sup, topk)
    h32 = moe_up(x, sel, *up, *sup, F=F, FS=FS, D=D, topk=topk, out_dtype=torch.float32)
    h16 = moe_up(x, sel, *up, *sup, F=F, FS=FS, D=D, topk=topk)
    assert rel_err(f32_np(h32), ref) < TOL32
    assert rel_err(f32_np(h16), ref) < TOL16
    assert float(h32.min()) >= 0.0
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
def test_moe_up_strided_rows_and_forms(cuda):
    """x rows with a stride (a view into a wider buffer), the shared-only (topk = 0) and the
    routed-only (FS = 0) forms."""
    B, D, F, FS, E, topk = 3, 384, 256, 512, 8, 3
    x, sel, up, sup = up_case(21, B, D, F, FS, E, topk, cuda)
    wide = torch.zeros((B, D + 64), dtype=x.dtype, device=cuda)
    wide[:, 32:32 + D] = x
    xv = wide[:, 32:32 + D]
    ref = oracle_up(x, sel, up, sup, topk)
    h = moe_up(xv, sel, *up, *sup, F=F, FS=FS, D=D, topk=topk, out_dtype=torch.float32)
    assert rel_err(f32_np(h), ref) < TOL32
    hs = moe_up(x, None, None, None, None, *sup, F=F, FS=FS, D=D, topk=0, out_dtype=torch.float32)
    assert rel_err(f32_np(hs), ref[:, topk * F:]) < TOL32
    hr = moe_up(x, sel, *up, None, None, None, F=F, FS=0, D=D, topk=topk, out_dtype=torch.float32)
    assert rel_err(f32_np(hr), ref[:, :topk * F]) < TOL32


@pytest.mark.gpu
def test_moe_up_bad_expert_id_is_zero_and_flagged(cuda):
    B, D, F, FS, E, topk = 2, 384, 256, 512, 8, 2
    x, sel, up, sup = up_case(5, B, D, F, FS, E, topk, cuda)
    hsd_b200.device_status()
    sel[1, 0] = E + 3
    h = moe_up(x, sel, *up, *sup, F=F, FS=FS, D=D, topk=topk, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float(h[1, :F].abs().max()) == 0.0
    assert hsd_b200.device_status() == hsd_b200._lib.HSD_ERR_INDEX
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("B,z", [(1, 0.9), (3, 0.8), (8, 0.97)])
def test_dense_down_vs_oracle(cuda, B, z):
    c = synth.decode_case(seed=300 + B, B=B, zero_frac=z, device=cuda)
    ref = cport.dense_down(f32_np(c["h"]), c["sel"].cpu().numpy(), c["gains"].cpu().numpy(), words_np(c["w"]),
                           bits16_np(c["s"]), bits16_np(c["b"]), words_np(c["sw"]), bits16_np(c["ss"]),
                           bits16_np(c["sb"]), F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"])
    y = dense_down(c["h"], c["sel"], c["gains"], c["w"], c["s"], c["b"], c["sw"], c["ss"], c["sb"], F=c["F"],
                   FS=c["FS"], D=c["D"], topk=c["topk"], out_dtype=torch.float32)
    assert rel_err(f32_np(y), ref) < TOL32
    # with the residual, rounded once to bf16
    resid = torch.randn((B, c["D"]), device=cuda).to(torch.bfloat16)
    yr = dense_down(c["h"], c["sel"], c["gains"], c["w"], c["s"], c["b"], c["sw"], c["ss"], c["sb"], F=c["F"],
                    FS=c["FS"], D=c["D"], topk=c["topk"], resid=resid)
    assert rel_err(f32_np(yr), f32_np(resid) + ref) < TOL16
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
def test_dense_and_sparse_down_agree(cuda):
    """The two down projections on the same inputs (checkpoint vs neuron-major layout): fp32
    accumulation in different orders, so they agree to fp32 rounding, not bit for bit."""
    c = synth.decode_case(seed=311, B=3, zero_frac=0.9, device=cuda)
    pw, ps, pb = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"])
    spw, sps, spb = hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
    ys = hsd_b200.sparse_down(c["h"], c["sel"], c["gains"], pw, ps, pb, spw, sps, spb, F=c["F"], FS=c["FS"],
                              D=c["D"], topk=c["topk"], out_dtype=torch.float32)
    yd = dense_down(c["h"], c["sel"], c["gains"], c["w"], c["s"], c["b"], c["sw"], c["ss"], c["sb"], F=c["F"],
                    FS=c["FS"], D=c["D"], topk=c["topk"], out_dtype=torch.float32)
    assert rel_err(f32_np(ys), f32_np(yd)) < 1e-5
    assert np.isfinite(f32_np(yd)).all()


@pytest.mark.gpu
@pytest.mark.parametrize("B,in_f,out_f", [(1, 2688, 10304), (3, 4096, 2688), (2, 5376, 2688), (4, 8192, 96),
                                          (1, 64, 40)])
def test_qlinear_vs_oracle(cuda, B, in_f, out_f):
    from oracle.quant import dequantize
    from hsd_b200.front import qlinear
    gen = torch.Generator(device=cuda).manual_seed(in_f + out_f + B)
    w, s, b = synth.quantized_weights((out_f, in_f), gen, cuda)
    x = torch.randn((B, in_f), generator=gen, device=cuda).to(torch.bfloat16)
    Wf = dequantize(words_np(w), bf16_bits_to_f32(bits16_np(s)), bf16_bits_to_f32(bits16_np(b)))
    ref = f32_np(x) @ Wf.T
    y32 = qlinear(x, w, s, b, out_dtype=torch.float32)
    assert rel_err(f32_np(y32), ref) < TOL32
    resid = torch.randn((B, out_f), generator=gen, device=cuda).to(torch.bfloat16)
    y16 = qlinear(x, w, s, b, resid=resid)
    assert rel_err(f32_np(y16), f32_np(resid) + ref) < TOL16


def torch_rms_norm(x, w, eps):
    """fp32 torch reference of NemotronH's RMSNorm: w * cast(x * rsqrt(mean(x^2) + eps))."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def torch_gated_rms_norm(y, gate, w, group_size, eps, out_dtype):
    """fp32 torch reference of the Mamba-2 gated norm: y * silu(gate), RMS-normalised per group."""
    yf = y.float() * torch.nn.functional.silu(gate.float())
    *lead, last = yf.shape
    g = yf.view(*lead, last // group_size, group_size)
    g = g * torch.rsqrt(g.square().mean(-1, keepdim=True) + eps)
    return w * g.view(*lead, last).to(out_dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("B,D", [(1, 2688), (3, 2688), (5, 384)])
def test_rms_norm_vs_torch(cuda, B, D):
    from hsd_b200.rowops import rms_norm
    gen = torch.Generator(device=cuda).manual_seed(B * D)
    x = (torch.randn((B, D + 16), generator=gen, device=cuda) * 3).to(torch.bfloat16)[:, 8:8 + D]
    w = (1 + 0.1 * torch.randn(D, generator=gen, device=cuda)).to(torch.bfloat16)
    ref = torch_rms_norm(x, w, 1e-5)
    y = rms_norm(x, w, 1e-5)
    assert rel_err(f32_np(y), f32_np(ref)) < TOL16


@pytest.mark.gpu
def test_gated_rms_norm_vs_torch(cuda):
    from hsd_b200.rowops import gated_rms_norm
    gen = torch.Generator(device=cuda).manual_seed(3)
    B, I, G = 3, 4096, 8
    y = torch.randn((B, I), generator=gen, device=cuda)
    proj = torch.randn((B, I + 100), generator=gen, device=cuda).to(torch.bfloat16)
    gate = proj[:, :I]
    w = (1 + 0.1 * torch.randn(I, generator=gen, device=cuda)).to(torch.bfloat16)
    ref = torch_gated_rms_norm(y, gate, w, I // G, 1e-5, torch.bfloat16)
    out = gated_rms_norm(y, gate, w, I // G, 1e-5, torch.bfloat16)
    assert rel_err(f32_np(out), f32_np(ref)) < TOL16


@pytest.mark.gpu
@pytest.mark.parametrize("B,E,topk", [(1, 128, 6), (3, 128, 6), (4, 16, 4), (2, 256, 8), (1, 1000, 6)])
def test_router_vs_torch(cuda, B, E, topk):
    from hsd_b200.rowops import Router
    gen = torch.Generator(device=cuda).manual_seed(E + B)
    D = 2688
    R = torch.randn((E, D), generator=gen, device=cuda) * 0.02
    x = torch.randn((B, D), generator=gen, device=cuda).to(torch.bfloat16)
    router = Router(R, topk)
    for _ in range(2):                                   # the ticket resets between calls
        sel, gains = router(x)
        sc = torch.sigmoid(x.float() @ R.t())
        top, ref_sel = torch.topk(sc, topk, dim=-1)
        assert torch.equal(torch.sort(sel.long(), -1).values, torch.sort(ref_sel, -1).values)
        ref_g = top / top.sum(-1, keepdim=True)
        order = torch.argsort(sel.long(), -1)
        ref_order = torch.argsort(ref_sel, -1)
        assert torch.allclose(gains[:, :topk].gather(1, order), ref_g.gather(1, ref_order), rtol=1e-5, atol=1e-6)
        assert torch.all(gains[:, topk] == 1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("L,pos,HD,QH,KVH", [(1, 0, 128, 32, 2), (3, 200, 128, 32, 2), (4, 1000, 64, 4, 2),
                                             (1, 4095, 128, 32, 2), (2, 63, 128, 16, 1)])
def test_decode_attention_vs_fp32_softmax(cuda, L, pos, HD, QH, KVH):
    """hsd_attn_decode against an fp32 softmax(q K^T / sqrt(HD)) V over each row's keys, and
    a row's result equals the same row computed alone (bit for bit)."""
    from hsd_b200.rowops import DecodeAttention
    max_len = 4096
    gen = torch.Generator(device=cuda).manual_seed(L + pos + HD)
    kc = torch.randn((KVH, max_len, HD), generator=gen, device=cuda).to(torch.bfloat16)
    vc = torch.randn((KVH, max_len, HD), generator=gen, device=cuda).to(torch.bfloat16)
    wide = torch.randn((L, QH * HD + 3 * 8 * HD), generator=gen, device=cuda).to(torch.bfloat16)
    q = wide[:, :QH * HD]                                    # strided rows, as the qkv slice
    p = torch.tensor([pos], dtype=torch.int64, device=cuda)
    att = DecodeAttention(QH, KVH, HD, max_len, 8, cuda)
    out = att(q, kc, vc, p)
    g = QH // KVH
    for l in range(L):
        n = pos + l + 1
        qf = q[l].float().view(QH, HD)
        kf = kc[:, :n].float().repeat_interleave(g, 0)       # [QH, n, HD]
        vf = vc[:, :n].float().repeat_interleave(g, 0)
        w = torch.softmax(torch.einsum("hd,hnd->hn", qf, kf) / HD ** 0.5, -1)
        ref = torch.einsum("hn,hnd->hd", w, vf).reshape(-1)
        assert rel_err(f32_np(out[l]), f32_np(ref)) < TOL16
        alone = att(q[l:l + 1], kc, vc, p + l)
        assert torch.equal(alone[0], out[l])
    assert hsd_b200.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("B", [2, 3, 5, 8])
def test_qlinear_rows_equal_single_rows(cuda, B):
    """A multi-row call reads the weights once for all rows, and each row's output equals the
    same row computed alone, bit for bit (the verify-row property)."""
    from hsd_b200.front import qlinear
    gen = torch.Generator(device=cuda).manual_seed(40 + B)
    w, s, b = synth.quantized_weights((2688, 4096), gen, cuda)
    x = torch.randn((B, 4096), generator=gen, device=cuda).to(torch.bfloat16)
    resid = torch.randn((B, 2688), generator=gen, device=cuda).to(torch.bfloat16)
    yb = qlinear(x, w, s, b, resid=resid)
    for r in range(B):
        y1 = qlinear(x[r:r + 1], w, s, b, resid=resid[r:r + 1])
        assert torch.equal(y1[0], yb[r])


_FORMS_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from hsd_b200 import synth
from hsd_b200.front import moe_up, qlinear
dev = torch.device("cuda", 0)
out = {}
for B in (1, 3, 8):
    gen = torch.Generator(device=dev).manual_seed(300 + B)
    uw, us, ub = synth.quantized_weights((16, 256, 2688), gen, dev)
    suw, sus, sub = synth.quantized_weights((512, 2688), gen, dev)
    x = torch.randn((B, 2688), generator=gen, device=dev).to(torch.bfloat16)
    sel, _ = synth.route_topk(torch.randn((B, 16), generator=gen, device=dev), 6)
    out[f"up{B}"] = moe_up(x, sel.to(torch.int32).contiguous(), uw, us, ub, suw, sus, sub, F=256, FS=512, D=2688,
                           topk=6, out_dtype=torch.float32).cpu()
    w, s, b = synth.quantized_weights((1040, 2688), gen, dev)
    resid = torch.randn((B, 1040), generator=gen, device=dev).to(torch.bfloat16)
    out[f"lin{B}"] = qlinear(x, w, s, b, resid=resid).cpu()
torch.save(out, sys.argv[2])
"""


@pytest.mark.gpu
def test_streaming_form_agrees_with_block_form(cuda, tmp_path):
    """The streaming form of the 4-bit tensor-core products (persistent blocks fed by bulk
    copies, used for up to 8 rows) and the one-tile-per-block form (HSD_QMMA_STREAM=0, read
    once per process) compute the same exact per-group MMA sums and differ only in how the
    fp32 group terms are split over warps: they agree to fp32 rounding, for the MoE up
    projections and a plain linear, at 1, 3 and 8 rows."""
    import os
    import subprocess
    import sys
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mlx-heimr-sparse-down_b200")
    outs = []
    for stream in ("1", "0"):
        f = tmp_path / f"forms_{stream}.pt"
        env = dict(os.environ, HSD_QMMA_STREAM=stream)
        subprocess.run([sys.executable, "-c", _FORMS_SCRIPT, pkg, str(f)], env=env, check=True, timeout=300)
        outs.append(torch.load(f))
    for k in outs[0]:
        a, b = outs[0][k].float(), outs[1][k].float()
        tol = 1e-5 if k.startswith("up") else 1e-2     # the linear's output is bf16 (one rounding)
        assert float((a - b).abs().max()) <= tol * float(b.abs().max()), k
