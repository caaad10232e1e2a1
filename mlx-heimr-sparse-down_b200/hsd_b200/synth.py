"""Seeded synthetic inputs with the reference model's shapes and value distributions.

There is no checkpoint here, so weights are drawn N(0, 0.02), quantised to the affine
4-bit group-64 format in the checkpoint layout (w [.., D, F/8] packed words, s / b
[.., D, F/64] bf16), and activations are relu(x)^2 with x ~ N(mu, 1), mu = -Phi^-1(z),
which makes a fraction z of them exactly zero. Everything is torch and runs on the
tensor's device (the GPU for full-size benchmarks, the CPU for small test cases).

The quantiser is this package's own: per 64-group, bias = min and scale = (max - min) / 15,
both rounded to bf16, q = round((W - bias) / scale) clamped to 0..15. Both the kernels and
the oracle consume the same packed bytes, so the quantiser's rounding choices do not
enter any parity comparison.
"""
import math

import torch

GS = 64

# reference shapes (Nemotron 3.5 Lightning 30B-A3B MoE layer)
D_REF, F_REF, FS_REF, E_REF, TOPK_REF = 2688, 1856, 3712, 128, 6


def _phi_inv(p):
    """Inverse standard normal CDF (Acklam's rational approximation, |error| < 1.2e-9)."""
    a = [-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
         1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00]
    b = [-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
         6.680131188771972e+01, -1.328068155288572e+01]
    c = [-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
         -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00]
    d = [7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00, 3.754408661907416e+00]
    if p < 0.02425:
        q = math.sqrt(-2 * math.log(p))
        return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) / \
               ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1)
    if p > 1 - 0.02425:
        return -_phi_inv(1 - p)
    q = p - 0.5
    r = q * q
    return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q / \
           (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1)


def zero_mean(z):
    """The Gaussian mean that makes relu(x)^2 exactly zero with probability z."""
    return -_phi_inv(z)


def pack_nibbles(q):
    """q [.., C] integers 0..15 -> [.., C/8] int32 words, nibble n of word j = q[8j + n]."""
    *lead, C = q.shape
    q = q.reshape(*lead, C // 8, 8).to(torch.int64)
    shifts = (4 * torch.arange(8, device=q.device, dtype=torch.int64))
    words = (q << shifts).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def quantize_affine4(W, gs=GS):
    """W [.., R, C] float -> (w [.., R, C/8] int32, s [.., R, C/gs] bf16, b [.., R, C/gs] bf16)."""
    *lead, R, C = W.shape
    Wg = W.float().reshape(*lead, R, C // gs, gs)
    lo = Wg.amin(-1)
    hi = Wg.amax(-1)
    s = ((hi - lo) / 15.0).to(torch.bfloat16)
    b = lo.to(torch.bfloat16)
    sf = s.float().unsqueeze(-1)
    bf = b.float().unsqueeze(-1)
    q = torch.where(sf > 0, torch.round((Wg - bf) / torch.where(sf > 0, sf, torch.ones_like(sf))),
                    torch.zeros_like(Wg)).clamp_(0, 15)
    w = pack_nibbles(q.reshape(*lead, R, C).to(torch.uint8))
    return w, s, b


def quantized_weights(shape, gen, device, std=0.02, chunk=16):
    """Checkpoint-layout 4-bit weights of `shape` [.., R, C] drawn N(0, std), generated
    `chunk` leading slices at a time to bound the fp32 transient."""
    *lead, R, C = shape
    if not lead:
        W = torch.randn((R, C), generator=gen, device=device, dtype=torch.float32) * std
        return quantize_affine4(W.to(torch.bfloat16))
    n = lead[0]
    ws, ss, bs = [], [], []
    for i in range(0, n, chunk):
        m = min(chunk, n - i)
        W = torch.randn((m, *lead[1:], R, C), generator=gen, device=device, dtype=torch.float32) * std
        w, s, b = quantize_affine4(W.to(torch.bfloat16))
        ws.append(w)
        ss.append(s)
        bs.append(b)
        del W
    return torch.cat(ws), torch.cat(ss), torch.cat(bs)


def relu2_activations(shape, zero_frac, gen, device, dtype=torch.bfloat16):
    """relu(x)^2, x ~ N(-Phi^-1(zero_frac), 1), in `dtype` (a fraction zero_frac exactly zero)."""
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) + zero_mean(zero_frac)
    return torch.relu(x).square().to(dtype)


def route_topk(logits, topk):
    """softmax -> top-k -> renormalise (the config's router) -> (sel int32, scores f32)."""
    p = torch.softmax(logits.float(), dim=-1)
    sc, sel = torch.topk(p, topk, dim=-1)
    sc = sc / sc.sum(-1, keepdim=True)
    return sel.to(torch.int32), sc.float()


def route_zipf(T, E, topk, gen, device, alpha=1.1):
    """Top-k without replacement under a Zipf(alpha) expert popularity (Gumbel-top-k on
    log p_e); gains = softmax over the selected perturbed logits."""
    e = torch.arange(1, E + 1, device=device, dtype=torch.float32)
    logp = -alpha * torch.log(e)
    logp = logp - torch.logsumexp(logp, 0)
    u = torch.rand((T, E), generator=gen, device=device, dtype=torch.float32).clamp_(1e-12, 1 - 1e-7)
    g = logp[None, :] - torch.log(-torch.log(u))
    top, sel = torch.topk(g, topk, dim=-1)
    sc = torch.softmax(top, dim=-1)
    return sel.to(torch.int32), sc.float()


def decode_case(seed=0, B=1, D=D_REF, F=F_REF, FS=FS_REF, E=E_REF, topk=TOPK_REF,
                zero_frac=0.90, device="cpu", h_dtype=torch.bfloat16, routing="softmax"):
    """One MoE layer's down projection inputs in the checkpoint layout.

    -> dict(w, s, b: routed [E, D, F/8] / [E, D, F/64]; sw, ss, sb: shared [D, FS/8] /
    [D, FS/64]; h [B, topk*F+FS]; sel [B, topk] int32; gains [B, topk+1] f32 (last = 1))."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w, s, b = quantized_weights((E, D, F), gen, device)
    sw, ss, sb = quantized_weights((D, FS), gen, device)
    if routing == "zipf":
        sel, sc = route_zipf(B, E, topk, gen, device)
    else:
        logits = torch.randn((B, E), generator=gen, device=device, dtype=torch.float32)
        sel, sc = route_topk(logits, topk)
    gains = torch.cat([sc, torch.ones((B, 1), device=device, dtype=torch.float32)], dim=1).contiguous()
    h = relu2_activations((B, topk * F + FS), zero_frac, gen, device, h_dtype)
    return dict(w=w, s=s, b=b, sw=sw, ss=ss, sb=sb, h=h, sel=sel.contiguous(), gains=gains,
                D=D, F=F, FS=FS, E=E, topk=topk)
