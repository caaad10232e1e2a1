"""A random-init Nemotron-H-style hybrid model around the hot path (hsd/model.py, hsd/mtp.py).

This is the caller of the operators, for the end-to-end configs: 52 layers (23 Mamba-2, 23 MoE,
6 GQA attention), hidden 2688, vocab 131072, every linear weight affine 4-bit g64 from
N(0, 0.02). There is no checkpoint here, so the weights are seeded random and the layer
pattern is a fixed one with the reference's counts and its named MoE layer indices
(hsd/model.py:46, tests/test_layout_decode.py:21, bench/decode_layers.py:24).

  dense   the MoE down projection dequantised in fp32 over every weight of the selected
          experts (the arithmetic mlx-lm's gather_qmm performs on the checkpoint layout, with
          fp32 accumulation as the sparse path has)
  sparse  the down projection on the neuron-major layout through this library's sparse
          decode kernel (hsd_sparse_down_decode) and, for prompt chunks, its tcgen05 prefill
          GEMM (hsd_sparse_down_prefill)
  mtp     greedy speculative decoding with a random-init MTP head (hsd/mtp.py): k drafts,
          one (k+1)-row verify step, attention KV trim and the Mamba-2 checkpoint rollback
          (hsd_mamba_*), in the reference's loop (hsd/model.py:366-443)

The up projections, router, attention, norms and Mamba in/out projections are dense torch
ops on dequantised bf16 copies of the 4-bit weights (outside the hot path). Batch-1
generation reads one token back per step, as the reference's loop does (`y.item()`).
"""
import time
from dataclasses import dataclass, field

import torch

from . import mamba as hm
from . import synth
from .decode import sparse_down
from .layout import to_neuron_major
from .prefill import sparse_down_prefill

MODES = ("dense", "sparse")


def layer_pattern(n_layers=52, n_moe=23, n_attn=6):
    """A fixed hybrid pattern: MoE at the reference's named indices (1, 10, 17, 20, 22, 24, 27,
    29, 31, 51) plus others, attention at 6 spread positions, Mamba-2 elsewhere."""
    named = [1, 10, 17, 20, 22, 24, 27, 29, 31, 51]
    attn = [5, 14, 25, 34, 42, 47] if n_layers == 52 else list(range(2, n_layers, max(2, n_layers // max(1, n_attn))))[:n_attn]
    types = ["M"] * n_layers
    for i in attn:
        types[i] = "*"
    moe = [i for i in named if i < n_layers]
    for i in range(1, n_layers, 2):
        if len(moe) >= n_moe:
            break
        if i not in moe and types[i] == "M":
            moe.append(i)
    for i in range(n_layers):
        if len(moe) >= n_moe:
            break
        if i not in moe and types[i] == "M":
            moe.append(i)
    for i in moe:
        types[i] = "E"
    return "".join(types)


@dataclass
class ModelArgs:
    hidden: int = 2688
    vocab: int = 131072
    n_layers: int = 52
    n_moe: int = 23
    n_attn: int = 6
    E: int = 128
    topk: int = 6
    F: int = 1856
    FS: int = 3712
    mamba_heads: int = 64
    mamba_head_dim: int = 64
    mamba_groups: int = 8
    mamba_state: int = 128
    conv_kernel: int = 4
    q_heads: int = 32
    kv_heads: int = 2
    head_dim: int = 128
    eps: float = 1e-5
    std: float = 0.02
    max_len: int = 4096
    pattern: str = field(default="")

    def __post_init__(self):
        if not self.pattern:
            self.pattern = layer_pattern(self.n_layers, self.n_moe, self.n_attn)

    @classmethod
    def tiny(cls):
        """A reduced model for tests: the same structure at small sizes."""
        return cls(hidden=384, vocab=2048, n_layers=8, n_moe=3, n_attn=2, E=16, topk=4, F=256, FS=512,
                   mamba_heads=8, mamba_head_dim=32, mamba_groups=2, mamba_state=64, q_heads=4, kv_heads=2,
                   head_dim=64, max_len=1024, pattern="ME*MEM*E")


def dequant_affine4(w, s, b, dtype=torch.bfloat16):
    """Packed [.., R, C/8] words + [.., R, C/64] scales / biases -> [.., R, C] (fp32 s*q + b)."""
    shifts = 4 * torch.arange(8, device=w.device, dtype=torch.int32)
    q = (w.unsqueeze(-1) >> shifts) & 15
    q = q.reshape(*w.shape[:-1], w.shape[-1] * 8).float()
    R, C = q.shape[-2], q.shape[-1]
    qg = q.view(*q.shape[:-1], C // 64, 64)
    W = qg * s.float().unsqueeze(-1) + b.float().unsqueeze(-1)
    return W.view(*q.shape[:-2], R, C).to(dtype)


def quantized_linear(out_f, in_f, gen, device, std):
    """A 4-bit g64 weight [out_f, in_f], returned as its dequantised bf16 copy."""
    w, s, b = synth.quantized_weights((out_f, in_f), gen, device, std=std)
    return dequant_affine4(w, s, b)


def rms_norm(x, w, eps):
    return hm.rms_norm(x, w, eps)


def _expert_groups(flat):
    """(expert, slot indices) for every expert present in flat [n] (one host read)."""
    order = torch.argsort(flat, stable=True)
    uniq, counts = torch.unique_consecutive(flat[order], return_counts=True)
    out, i = [], 0
    for e, c in zip(uniq.tolist(), counts.tolist()):
        out.append((e, order[i:i + c]))
        i += c
    return out


class MoEBlock:
    """One MoE block: router (sigmoid scores, normalised top-k, as Nemotron-H routes), 4-bit
    routed and shared up projections with ReLU^2, and the down projection in either mode."""

    def __init__(self, a, gen, device):
        self.a = a
        D, E, F, FS = a.hidden, a.E, a.F, a.FS
        self.norm_w = (1.0 + 0.1 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
        self.router = torch.randn((E, D), generator=gen, device=device) * a.std
        self.up = quantized_linear(E * F, D, gen, device, a.std).view(E, F, D)
        self.shared_up = quantized_linear(FS, D, gen, device, a.std)
        # the down projections in the checkpoint layout, then the neuron-major one
        self.w, self.s, self.b = synth.quantized_weights((E, D, F), gen, device, std=a.std)
        self.sw, self.ss, self.sb = synth.quantized_weights((D, FS), gen, device, std=a.std)
        self.pw, self.ps, self.pb = to_neuron_major(self.w, self.s, self.b)
        self.spw, self.sps, self.spb = to_neuron_major(self.sw, self.ss, self.sb)

    def front(self, x):
        """x [B, D] -> (sel [B, topk] int32, gains [B, topk+1] f32, hcat [B, topk*F + FS] bf16)."""
        a = self.a
        xn = rms_norm(x, self.norm_w, a.eps)
        scores = torch.sigmoid(xn.float() @ self.router.t())
        top, sel = torch.topk(scores, a.topk, dim=-1)
        gains = torch.cat([top / (top.sum(-1, keepdim=True) + 1e-20), torch.ones_like(top[:, :1])], 1)
        # routed up projections, grouped by expert: one GEMM per selected expert on a view of
        # its weight (the expert ids come back to the host once per layer)
        B = x.shape[0]
        h = torch.empty((B * a.topk, a.F), dtype=torch.float32, device=x.device)
        flat = sel.reshape(-1)
        for e, rows in _expert_groups(flat):
            h[rows] = (xn[rows // a.topk] @ self.up[e].t()).float()
        h = torch.relu(h).square().view(B, a.topk, a.F)
        hs = torch.relu(xn @ self.shared_up.t()).square()
        hcat = torch.cat([h.reshape(x.shape[0], -1), hs], 1).to(torch.bfloat16).contiguous()
        return sel.to(torch.int32).contiguous(), gains.float().contiguous(), hcat

    def down_dense(self, hcat, sel, gains):
        """The dequantised fp32 down projection over every weight of the selected experts
        (each expert's weights dequantised once per call, every neuron multiplied)."""
        a = self.a
        B = hcat.shape[0]
        hf = hcat.float()
        hr = hf[:, :a.topk * a.F].reshape(B * a.topk, a.F)
        g = gains[:, :a.topk].reshape(-1)
        y = torch.zeros((B, a.hidden), dtype=torch.float32, device=hcat.device)
        for e, rows in _expert_groups(sel.reshape(-1)):
            We = dequant_affine4(self.w[e], self.s[e], self.b[e], torch.float32)          # [D, F]
            y.index_add_(0, rows // a.topk, (hr[rows] @ We.t()) * g[rows, None])
        Ws = dequant_affine4(self.sw, self.ss, self.sb, torch.float32)
        return y + gains[:, a.topk:] * (hf[:, a.topk * a.F:] @ Ws.t())

    def decode(self, x, mode):
        sel, gains, hcat = self.front(x)
        a = self.a
        if mode == "dense":
            # the residual added in fp32 and rounded once, as the kernels do
            return (x.float() + self.down_dense(hcat, sel, gains)).to(x.dtype)
        return sparse_down(hcat, sel, gains, self.pw, self.ps, self.pb, self.spw, self.sps, self.spb, F=a.F,
                           FS=a.FS, D=a.hidden, topk=a.topk, resid=x)

    def prefill(self, x, mode):
        if mode == "dense" or self.a.hidden % 192 != 0:
            return self.decode(x, mode)
        sel, gains, hcat = self.front(x)
        a = self.a
        return sparse_down_prefill(hcat, sel, gains, self.pw, self.ps, self.pb, self.spw, self.sps, self.spb, F=a.F,
                                   FS=a.FS, D=a.hidden, topk=a.topk, E=a.E, resid=x)


class KVCache:
    """Preallocated keys / values [max_len, kv_heads, head_dim] with a host-side offset."""

    def __init__(self, a, device):
        self.k = torch.empty((a.max_len, a.kv_heads, a.head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.empty_like(self.k)
        self.offset = 0

    def trim(self, n):
        self.offset -= n

    def clone(self):
        c = KVCache.__new__(KVCache)
        c.k, c.v, c.offset = self.k.clone(), self.v.clone(), self.offset
        return c


class AttnBlock:
    """Pre-norm GQA self-attention without positional encoding (Nemotron-H's attention)."""

    def __init__(self, a, gen, device):
        self.a = a
        D = a.hidden
        self.norm_w = (1.0 + 0.1 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
        self.wq = quantized_linear(a.q_heads * a.head_dim, D, gen, device, a.std)
        self.wk = quantized_linear(a.kv_heads * a.head_dim, D, gen, device, a.std)
        self.wv = quantized_linear(a.kv_heads * a.head_dim, D, gen, device, a.std)
        self.wo = quantized_linear(D, a.q_heads * a.head_dim, gen, device, a.std)

    def __call__(self, x, cache):
        """x [L, D]: L new positions after cache.offset; the cache is advanced by L."""
        a = self.a
        L = x.shape[0]
        xn = rms_norm(x, self.norm_w, a.eps)
        q = (xn @ self.wq.t()).view(L, a.q_heads, a.head_dim)
        o0 = cache.offset
        cache.k[o0:o0 + L] = (xn @ self.wk.t()).view(L, a.kv_heads, a.head_dim)
        cache.v[o0:o0 + L] = (xn @ self.wv.t()).view(L, a.kv_heads, a.head_dim)
        cache.offset = o0 + L
        k = cache.k[:o0 + L].repeat_interleave(a.q_heads // a.kv_heads, dim=1)
        v = cache.v[:o0 + L].repeat_interleave(a.q_heads // a.kv_heads, dim=1)
        mask = None
        if L > 1:
            pos = torch.arange(o0 + L, device=x.device)
            mask = pos[None, :] <= (o0 + torch.arange(L, device=x.device))[:, None]
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                                             attn_mask=mask)
        return x + o.transpose(0, 1).reshape(L, -1) @ self.wo.t()


class MambaLayer:
    """A Mamba-2 block whose in / out projections are 4-bit weights (dequantised bf16 copies)."""

    def __init__(self, a, gen, device):
        H, P, G, N, K = a.mamba_heads, a.mamba_head_dim, a.mamba_groups, a.mamba_state, a.conv_kernel
        I = H * P
        conv_dim = I + 2 * G * N
        self.blk = hm.Mamba2Block(
            norm_w=(1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=device)).to(torch.bfloat16),
            in_proj=quantized_linear(I + conv_dim + H, a.hidden, gen, device, a.std),
            conv_w=torch.randn((conv_dim, K), generator=gen, device=device) * 0.3,
            conv_b=torch.randn(conv_dim, generator=gen, device=device) * 0.1,
            A_log=torch.log(torch.linspace(1.0, 16.0, H, device=device)),
            D=torch.ones(H, device=device),
            dt_bias=torch.linspace(-4.0, -1.0, H, device=device),
            gate_norm_w=(1.0 + 0.1 * torch.randn(I, generator=gen, device=device)).to(torch.bfloat16),
            out_proj=quantized_linear(a.hidden, I, gen, device, a.std),
            H=H, P=P, G=G, N=N, K=K, eps=a.eps)


class NemotronModel:
    """The random-init hybrid model with the reference's generation loops (hsd/model.py:178-443)."""

    def __init__(self, args=None, seed=0, device="cuda", mode="sparse"):
        self.args = a = args or ModelArgs()
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        self.types = [{"M": "mamba", "*": "attention", "E": "moe"}[c] for c in a.pattern]
        self.embeddings = (torch.randn((a.vocab, a.hidden), generator=gen, device=self.device) * 1.0).to(torch.bfloat16)
        self.blocks = []
        for t in self.types:
            if t == "moe":
                self.blocks.append(MoEBlock(a, gen, self.device))
            elif t == "attention":
                self.blocks.append(AttnBlock(a, gen, self.device))
            else:
                self.blocks.append(MambaLayer(a, gen, self.device))
        self.norm_f = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=self.device)).to(torch.bfloat16)
        self.lm_head = quantized_linear(a.vocab, a.hidden, gen, self.device, a.std)
        self.mode = mode
        self._records = []

    def set_mode(self, mode):
        assert mode in MODES, mode
        self.mode = mode

    # ---- pieces shared with the MTP head
    def embed(self, ids):
        return self.embeddings[ids]

    def head_fn(self, h):
        """Logits in fp32 (bf16 operands, fp32 output): bf16 logits near 4 are 1/32 apart, which
        turns many greedy choices into exact ties."""
        if h.is_cuda:
            return torch.mm(h.reshape(-1, h.shape[-1]), self.lm_head.t(), out_dtype=torch.float32).view(
                *h.shape[:-1], -1)
        return h.float() @ self.lm_head.float().t()

    def logits(self, x):
        return self.head_fn(rms_norm(x, self.norm_f, self.args.eps))

    def make_cache(self):
        return [[None, None] if t == "mamba" else KVCache(self.args, self.device) if t == "attention" else None
                for t in self.types]

    # ---- forward
    def _layers(self, x, cache, records, multi):
        for l, t in enumerate(self.types):
            blk = self.blocks[l]
            if t == "moe":
                x = blk.prefill(x, self.mode) if multi == "prefill" else blk.decode(x, self.mode)
            elif t == "attention":
                x = blk(x, cache[l])
            else:
                x = hm.mamba_verify(blk.blk, x[None], cache[l], records, checkpoints=multi != "prefill")[0]
        return x

    def prefill(self, tokens, cache, chunk=512, on_hidden=None):
        """tokens [T] -> the residual stream of the last position [1, D] (hsd/model.py:259)."""
        last = None
        for i in range(0, tokens.shape[0], chunk):
            x = self.embed(tokens[i:i + chunk])
            x = self._layers(x, cache, [], "prefill")
            if on_hidden is not None:
                on_hidden(i, x)
            last = x[-1:]
        return last

    def step(self, x, cache):
        """One decode step on x [1, D] (hsd/model.py:281)."""
        return self._layers(x, cache, [], "decode")

    def verify_step(self, x, cache):
        """x [B, D]: B consecutive positions in ONE step, every cache advanced by B rows; the
        Mamba layers keep their per-row checkpoints for rollback() (hsd/model.py:333)."""
        self._records = []
        return self._layers(x, cache, self._records, "decode")

    def rollback(self, cache, n_keep, B):
        """Undo a verify_step of B rows beyond its first n_keep (hsd/model.py:348): attention
        caches trimmed, Mamba states set to the checkpoints of row n_keep-1."""
        if n_keep == B:
            return
        for l, t in enumerate(self.types):
            if t == "attention":
                cache[l].trim(B - n_keep)
        hm.mamba_rollback(self._records, n_keep)

    # ---- generation (greedy)
    def _pick(self, x):
        """Greedy choice for the last row of x: (token, top-1 minus top-2 logit), one host read."""
        top = torch.topk(self.logits(x[-1:]), 2, dim=-1)
        v, i = top.values[0], top.indices[0]
        tok, margin = torch.stack([i[0].float(), v[0] - v[1]]).tolist()
        return int(tok), margin

    def generate(self, prompt, max_tokens=128, chunk=512, forced=None):
        """Greedy decoding (hsd/model.py:291) -> (tokens, stats). stats["margins"] holds the
        top-1 minus top-2 logit of every choice. With `forced` (a token list) the loop feeds
        forced[i] instead of its own choice (teacher forcing) and still returns its choices."""
        prompt = torch.as_tensor(prompt, dtype=torch.long, device=self.device)
        cache = self.make_cache()
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        h = self.prefill(prompt, cache, chunk)
        tok, mg = self._pick(h)
        t1 = time.perf_counter()
        out, margins = [tok], [mg]
        while len(out) < max_tokens:
            feed = forced[len(out) - 1] if forced is not None else tok
            x = self.step(self.embed(torch.tensor([feed], device=self.device)), cache)
            tok, mg = self._pick(x)
            out.append(tok)
            margins.append(mg)
        t2 = time.perf_counter()
        return out, dict(mode=self.mode, prompt_tokens=int(prompt.shape[0]), prompt_s=t1 - t0, gen_tokens=len(out),
                         decode_s=t2 - t1, decode_tps=(len(out) - 1) / max(t2 - t1, 1e-9), margins=margins)

    def generate_mtp(self, prompt, mtp, n_draft=2, max_tokens=128, chunk=512, replay=None):
        """Greedy speculative decoding with the MTP head (hsd/model.py:366-443) -> (tokens, stats).

        replay (a token list, e.g. an earlier greedy run's output) replaces the head's drafts
        with the tokens that follow in that list -- forced acceptance, which times the verify
        and rollback at acceptances a = 0..k that a random-init head never reaches. The accept
        rule is unchanged, so the output is still this model's own greedy sequence."""
        prompt = torch.as_tensor(prompt, dtype=torch.long, device=self.device)
        cache = self.make_cache()
        mtp.reset()
        last_h = []

        def on_hidden(i, x):                       # the head's prefill: rows (h_p, tok_{p+1})
            nxt = prompt[i + 1:i + 1 + x.shape[0]]
            if nxt.shape[0] > 0 and replay is None:
                mtp(x[:nxt.shape[0]], nxt)
            last_h.append(x[-1:])

        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        x_last = self.prefill(prompt, cache, chunk, on_hidden=on_hidden)
        tok = int(torch.argmax(self.logits(x_last), -1).item())
        t1 = time.perf_counter()
        out = [tok]
        pend_h, pend_t = [last_h[-1]], [tok]
        steps, acc = 0, []
        bs = n_draft + 1
        while len(out) < max_tokens:
            if replay is None:
                d, hd = mtp(torch.cat(pend_h, 0), torch.tensor(pend_t, device=self.device))
                drafts = [d[-1:]]
                hd = hd[-1:]
                for _ in range(1, n_draft):        # chain the head on its own hidden output
                    d, hd = mtp(hd, drafts[-1])
                    drafts.append(d)
                draft = torch.cat(drafts)
            else:
                nxt = replay[len(out):len(out) + n_draft]
                draft = torch.tensor(nxt + [0] * (n_draft - len(nxt)), device=self.device)
            ids = torch.cat([torch.tensor([tok], device=self.device), draft])
            x = self.verify_step(self.embed(ids), cache)
            tgt = torch.argmax(self.logits(x), -1)
            dl, tl = draft.tolist(), tgt.tolist()
            a = next((i for i in range(bs - 1) if dl[i] != tl[i]), bs - 1)
            new = (dl[:a] + [tl[a]])[:max_tokens - len(out)]
            self.rollback(cache, a + 1, bs)
            if n_draft > 1 and replay is None:
                mtp.trim(n_draft - 1)              # drop the chained speculative rows
            pend_h = [x[i:i + 1] for i in range(len(new))]
            pend_t = list(new)
            steps += 1
            acc.append(a)
            out.extend(new)
            tok = new[-1]
        t2 = time.perf_counter()
        return out, dict(mode=self.mode, n_draft=n_draft, steps=steps, accepted_mean=sum(acc) / max(1, len(acc)),
                         accepted_hist=[acc.count(k) for k in range(n_draft + 1)], gen_tokens=len(out),
                         prompt_s=t1 - t0, decode_s=t2 - t1, decode_tps=(len(out) - 1) / max(t2 - t1, 1e-9),
                         replay=replay is not None)


def identical_prefix(a, b):
    """Length of the common prefix of two token lists."""
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


class MTPHead:
    """The MTP drafter (hsd/mtp.py:41-88): x = eh_proj([rms(embed(tok)), rms(h)]) -> attention
    block (own KV cache) -> MoE block (dense down, as the reference's head runs) -> final norm
    -> the target's lm_head argmax. Random init here."""

    def __init__(self, target, seed=1):
        a = target.args
        self.target, self.eps = target, a.eps
        gen = torch.Generator(device=target.device).manual_seed(seed)
        dev = target.device
        self.enorm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.hnorm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.eh_proj = quantized_linear(a.hidden, 2 * a.hidden, gen, dev, a.std)
        self.attn = AttnBlock(a, gen, dev)
        self.moe = MoEBlock(a, gen, dev)
        self.final_norm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.reset()

    def reset(self):
        self.kv = KVCache(self.target.args, self.target.device)

    def trim(self, n):
        self.kv.trim(n)

    def __call__(self, h, toks):
        """h [R, D] (the target's pre-norm hidden state), toks [R] -> (pred [R], hn [R, D])."""
        e = rms_norm(self.target.embed(toks), self.enorm, self.eps)
        hh = rms_norm(h, self.hnorm, self.eps)
        x = torch.cat([e, hh], -1) @ self.eh_proj.t()
        x = self.attn(x, self.kv)
        x = self.moe.decode(x, "dense")
        hn = rms_norm(x, self.final_norm, self.eps)
        return torch.argmax(self.target.head_fn(hn), -1), hn
