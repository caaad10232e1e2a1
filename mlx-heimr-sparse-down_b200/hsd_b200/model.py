"""A random-init Nemotron-H-style hybrid model around the hot path (hsd/model.py, hsd/mtp.py).

This is the caller of the operators, for the end-to-end configs: 52 layers (23 Mamba-2, 23 MoE,
6 GQA attention), hidden 2688, vocab 131072, every linear weight affine 4-bit g64 from
N(0, 0.02). There is no checkpoint here, so the weights are seeded random and the layer
pattern is a fixed one with the reference's counts and its named MoE layer indices
(hsd/model.py:46, tests/test_layout_decode.py:21, bench/decode_layers.py:24).

  dense   the MoE down projection over every weight of the selected experts, on the
          neuron-major layout in the sparse kernel's own reduction order
          (hsd_dense_down_decode_nm): the reference for greedy-token identity, which the
          sparse path reproduces bit for bit (a zero h adds an exact zero where sparse skips)
  stock   the same dense work on the checkpoint layout (hsd_dense_down_decode, what mlx-lm's
          gather_qmm computes without the layout change): the speed comparison
  sparse  the down projection on the neuron-major layout through this library's sparse
          decode kernel (hsd_sparse_down_decode) and, for prompt chunks, its tcgen05 prefill
          GEMM (hsd_sparse_down_prefill; prefill_gemm=False keeps prompt chunks on the decode
          kernel, so a whole generation is bit-identical to dense mode)
  mtp     greedy speculative decoding with a random-init MTP head (hsd/mtp.py): k drafts,
          one (k+1)-row verify step, attention KV positions and the Mamba-2 checkpoint
          selection rolled back on the device, in the reference's loop (hsd/model.py:366-443)

Decode rows (at most QGEMV_ROWS) run only this library's kernels and fixed-shape torch ops on
state kept in fixed device buffers (DecodeState: the attention caches with a device-side
position, the Mamba-2 windows / per-row states with a device-side kept-row count), so a
whole decode step -- or a whole MTP iteration: drafts, verify, accept rule, rollback -- is
captured once as a CUDA graph and replayed; the host reads back one small tensor per step,
as the reference's loop reads `y.item()`. Prompt chunks run eagerly: the linears on
dequantised bf16 copies with cuBLAS, the MoE down projection on the prefill GEMM.
"""
import time
from dataclasses import dataclass, field

import torch

from . import mamba as hm
from . import synth
from .decode import dense_down, sparse_down
from .front import QGEMV_ROWS, QLinear, moe_up
from .layout import to_neuron_major
from .prefill import sparse_down_prefill
from .rowops import DecodeAttention, Router, gated_rms_norm, rms_norm

MODES = ("dense", "sparse", "stock")


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


class MoEBlock:
    """One MoE block (NemotronH "E": norm, router, routed + shared experts, residual): the
    router (sigmoid scores, normalised top-k), the fused 4-bit up projections with relu2
    (hsd_moe_up_decode, the reference's front, hsd/model.py:110-121) and the down projection
    in either mode. Up weights in the checkpoint layout [E, F, D/8]; the down weights in the
    checkpoint layout (dense mode) and, permuted once at load, the neuron-major one (sparse)."""

    def __init__(self, a, gen, device):
        self.a = a
        D, E, F, FS = a.hidden, a.E, a.F, a.FS
        self.norm_w = (1.0 + 0.1 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
        self.router = Router((torch.randn((E, D), generator=gen, device=device) * a.std).contiguous(), a.topk)
        self.uw, self.us, self.ub = synth.quantized_weights((E, F, D), gen, device, std=a.std)
        self.suw, self.sus, self.sub = synth.quantized_weights((FS, D), gen, device, std=a.std)
        self.w, self.s, self.b = synth.quantized_weights((E, D, F), gen, device, std=a.std)
        self.sw, self.ss, self.sb = synth.quantized_weights((D, FS), gen, device, std=a.std)
        self.pw, self.ps, self.pb = to_neuron_major(self.w, self.s, self.b)
        self.spw, self.sps, self.spb = to_neuron_major(self.sw, self.ss, self.sb)

    def front(self, x):
        """x [T, D] -> (sel [T, topk] int32, gains [T, topk+1] f32, hcat [T, topk*F + FS] bf16)."""
        a = self.a
        xn = rms_norm(x, self.norm_w, a.eps)
        sel, gains = self.router(xn)
        hcat = moe_up(xn, sel, self.uw, self.us, self.ub, self.suw, self.sus, self.sub, F=a.F, FS=a.FS, D=a.hidden,
                      topk=a.topk)
        return sel, gains, hcat

    def down(self, hcat, sel, gains, x, mode, prefill_gemm=True):
        a = self.a
        if mode == "stock":
            return dense_down(hcat, sel, gains, self.w, self.s, self.b, self.sw, self.ss, self.sb, F=a.F, FS=a.FS,
                              D=a.hidden, topk=a.topk, resid=x)
        if mode == "dense":
            return sparse_down(hcat, sel, gains, self.pw, self.ps, self.pb, self.spw, self.sps, self.spb, F=a.F,
                               FS=a.FS, D=a.hidden, topk=a.topk, resid=x, all_rows=True)
        if prefill_gemm and x.shape[0] > QGEMV_ROWS and a.hidden % 192 == 0:
            return sparse_down_prefill(hcat, sel, gains, self.pw, self.ps, self.pb, self.spw, self.sps, self.spb,
                                       F=a.F, FS=a.FS, D=a.hidden, topk=a.topk, E=a.E, resid=x)
        return sparse_down(hcat, sel, gains, self.pw, self.ps, self.pb, self.spw, self.sps, self.spb, F=a.F,
                           FS=a.FS, D=a.hidden, topk=a.topk, resid=x)

    def __call__(self, x, mode, prefill_gemm=True):
        """x [T, D] -> x + moe(norm(x)), the residual added in fp32 inside the down kernel."""
        sel, gains, hcat = self.front(x)
        return self.down(hcat, sel, gains, x, mode, prefill_gemm)


class KVCache:
    """Keys / values [kv_heads, max_len, head_dim] (zeros) of one attention layer. The
    position is not stored here: every layer of a model is at the same one, a device tensor
    of the DecodeState."""

    def __init__(self, a, device):
        self.k = torch.zeros((a.kv_heads, a.max_len, a.head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)

    def reset(self):
        self.k.zero_()
        self.v.zero_()

    def clone(self):
        c = KVCache.__new__(KVCache)
        c.k, c.v = self.k.clone(), self.v.clone()
        return c


class AttnBlock:
    """Pre-norm GQA self-attention without positional encoding (Nemotron-H's attention). The
    L new rows are written at positions pos .. pos+L-1 (pos a device int64 [1]) and attend
    to every position up to their own, over the fixed-size cache with a mask, so the shapes
    never depend on the position (capturable)."""

    def __init__(self, a, gen, device):
        self.a = a
        D = a.hidden
        self.norm_w = (1.0 + 0.1 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
        self.wqkv = QLinear((a.q_heads + 2 * a.kv_heads) * a.head_dim, D, gen, device, a.std)
        self.wo = QLinear(D, a.q_heads * a.head_dim, gen, device, a.std)
        self.keys = torch.arange(a.max_len, device=device)
        self.attn = DecodeAttention(a.q_heads, a.kv_heads, a.head_dim, a.max_len, QGEMV_ROWS, device)

    def rows(self, x, kv, pos):
        a = self.a
        L = x.shape[0]
        qh, kvh, hd = a.q_heads, a.kv_heads, a.head_dim
        g = qh // kvh
        xn = rms_norm(x, self.norm_w, a.eps)
        qkv = self.wqkv(xn)
        q = qkv[:, :qh * hd].reshape(L, kvh, g, hd)
        k = qkv[:, qh * hd:(qh + kvh) * hd].reshape(L, kvh, hd)
        v = qkv[:, (qh + kvh) * hd:].reshape(L, kvh, hd)
        rows = torch.arange(L, device=x.device)
        kv.k.index_copy_(1, pos + rows, k.transpose(0, 1))
        kv.v.index_copy_(1, pos + rows, v.transpose(0, 1))
        sdpa = torch.nn.functional.scaled_dot_product_attention
        if L <= QGEMV_ROWS:
            # decode rows: hsd_attn_decode over the keys up to each row's position, a row's
            # result independent of the launch's other rows (a verify row equals the token
            # decoded alone bit for bit)
            o = self.attn(qkv[:, :qh * hd], kv.k, kv.v, pos)
        else:
            # the g query heads of a KV head as g*L rows (row r = head j*L + l), one mask row each
            qg = q.permute(1, 2, 0, 3).reshape(1, kvh, g * L, hd)
            lim = pos + rows.repeat(g)
            mask = self.keys[None, :] <= lim[:, None]
            o = sdpa(qg, kv.k[None], kv.v[None], attn_mask=mask[None, None])
            o = o.reshape(kvh, g, L, hd).permute(2, 0, 1, 3).reshape(L, qh * hd)
        return self.wo(o, resid=x)


class MambaLayer:
    """A Mamba-2 block whose in / out projections are 4-bit linears; the causal conv, the
    selective scan and the rollback are this library's kernels (hsd_b200.mamba)."""

    def __init__(self, a, gen, device):
        H, P, G, N, K = a.mamba_heads, a.mamba_head_dim, a.mamba_groups, a.mamba_state, a.conv_kernel
        I = H * P
        conv_dim = I + 2 * G * N
        self.in_proj = QLinear(I + conv_dim + H, a.hidden, gen, device, a.std)
        self.out_proj = QLinear(a.hidden, I, gen, device, a.std)
        self.blk = hm.Mamba2Block(
            norm_w=(1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=device)).to(torch.bfloat16),
            in_proj=self.in_proj,
            conv_w=torch.randn((conv_dim, K), generator=gen, device=device) * 0.3,
            conv_b=torch.randn(conv_dim, generator=gen, device=device) * 0.1,
            A_log=torch.log(torch.linspace(1.0, 16.0, H, device=device)),
            D=torch.ones(H, device=device),
            dt_bias=torch.linspace(-4.0, -1.0, H, device=device),
            gate_norm_w=(1.0 + 0.1 * torch.randn(I, generator=gen, device=device)).to(torch.bfloat16),
            out_proj=self.out_proj,
            H=H, P=P, G=G, N=N, K=K, eps=a.eps)

    def _mix(self, x, conv_scan):
        b = self.blk
        I, Cd = b.I, b.conv_dim
        h = rms_norm(x, b.norm_w, b.eps)
        proj = self.in_proj(h)                                     # [L, I + conv_dim + H]
        y = conv_scan(proj[:, I:I + Cd], proj[:, I + Cd:])
        yn = gated_rms_norm(y, proj[:, :I], b.gate_norm_w, I // b.G, b.eps, x.dtype)
        return self.out_proj(yn, resid=x)

    def rows(self, x, rc, n_keep):
        """Decode rows over the resident buffers (window / state of the previous call's kept
        rows, every row's state kept for a rollback)."""
        b = self.blk

        def conv_scan(conv_in, dt):
            co = hm.conv_step(conv_in, rc.padded, n_keep, b.conv_w, b.conv_b)
            return hm.ssm_step(co, dt, b.A_log, b.D, b.dt_bias, rc.states, n_keep, H=b.H, P=b.P, G=b.G, N=b.N,
                               time_step_limit=b.time_step_limit)

        return self._mix(x, conv_scan)

    def prefill(self, x, rc):
        """A prompt chunk of any length: the final window / state only, stored where a kept
        row count of 1 points (padded[1 .. K-1], states[0])."""
        b = self.blk
        L = x.shape[0]

        def conv_scan(conv_in, dt):
            co, padded = hm.conv_verify(conv_in, rc.padded[1:b.K], b.conv_w, b.conv_b)
            y, states = hm.ssm_verify(co, dt, b.A_log, b.D, b.dt_bias, rc.states[0], H=b.H, P=b.P, G=b.G, N=b.N,
                                      time_step_limit=b.time_step_limit, checkpoints=False)
            rc.padded[1:b.K].copy_(padded[L:])
            rc.states[0].copy_(states[0])
            return y

        return self._mix(x, conv_scan)


class DecodeState:
    """Everything a decode loop changes, in fixed device buffers: the attention caches and
    the position pos (tokens already in them, int64 [1]), every Mamba-2 layer's resident
    window / per-row states, and the kept-row count n_keep (int32 [1]) that selects the
    window and state the next call starts from. rows = the longest verify step."""

    def __init__(self, model, rows):
        self.rows = rows
        dev = model.device
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.n_keep = torch.ones(1, dtype=torch.int32, device=dev)
        self.kv = [KVCache(model.args, dev) if t == "attention" else None for t in model.types]
        self.mamba = [hm.ResidentMambaCache(b.blk, rows, dev) if t == "mamba" else None
                      for t, b in zip(model.types, model.blocks)]

    def reset(self):
        self.pos.zero_()
        self.n_keep.fill_(1)
        for c in self.kv:
            if c is not None:
                c.reset()
        for m in self.mamba:
            if m is not None:
                m.padded.zero_()
                m.states.zero_()

    def clone(self):
        c = DecodeState.__new__(DecodeState)
        c.rows, c.pos, c.n_keep = self.rows, self.pos.clone(), self.n_keep.clone()
        c.kv = [None if k is None else k.clone() for k in self.kv]
        c.mamba = []
        for m in self.mamba:
            if m is None:
                c.mamba.append(None)
            else:
                r = hm.ResidentMambaCache.__new__(hm.ResidentMambaCache)
                r.rows, r.padded, r.states = m.rows, m.padded.clone(), m.states.clone()
                c.mamba.append(r)
        return c

    def mamba_now(self, l):
        """(conv window [K-1, C], SSM state [H, P, N]) of Mamba layer l at the current kept row."""
        k = int(self.n_keep.item())
        m = self.mamba[l]
        K = m.padded.shape[0] - m.rows + 1
        return m.padded[k:k + K - 1], m.states[k - 1]


class _Graph:
    def __init__(self, graph, out):
        self.graph, self.out = graph, out


class NemotronModel:
    """The random-init hybrid model with the reference's generation loops (hsd/model.py:178-443)."""

    def __init__(self, args=None, seed=0, device="cuda", mode="sparse", verify_rows=4):
        self.args = a = args or ModelArgs()
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        self.types = [{"M": "mamba", "*": "attention", "E": "moe"}[c] for c in a.pattern]
        self.embeddings = torch.randn((a.vocab, a.hidden), generator=gen, device=self.device).to(torch.bfloat16)
        self.blocks = []
        for t in self.types:
            if t == "moe":
                self.blocks.append(MoEBlock(a, gen, self.device))
            elif t == "attention":
                self.blocks.append(AttnBlock(a, gen, self.device))
            else:
                self.blocks.append(MambaLayer(a, gen, self.device))
        self.norm_f = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=self.device)).to(torch.bfloat16)
        self.lm_head = QLinear(a.vocab, a.hidden, gen, self.device, a.std, bf16_copy=False)
        self.mode = mode
        self.prefill_gemm = True                          # prompt chunks of sparse mode on the GEMM
        self.state = DecodeState(self, verify_rows)      # the state the captured graphs run on
        self._graphs = {}
        self._io = None

    def set_mode(self, mode):
        assert mode in MODES, mode
        self.mode = mode

    def make_state(self, rows=None):
        return DecodeState(self, rows or self.state.rows)

    # ---- pieces shared with the MTP head
    def embed(self, ids):
        return self.embeddings[ids]

    def head_fn(self, hn):
        """lm_head on normed rows -> fp32 logits (hsd/model.py:226)."""
        return self.lm_head(hn, out_dtype=torch.float32)

    def logits(self, x):
        return self.head_fn(rms_norm(x, self.norm_f, self.args.eps))

    # ---- forward
    def forward_rows(self, x, st):
        """Decode rows x [L, D] (L <= st.rows) at position st.pos from the kept row st.n_keep;
        every cache gets the L rows, the position is not advanced (step / rollback do that)."""
        for l, t in enumerate(self.types):
            blk = self.blocks[l]
            if t == "moe":
                x = blk(x, self.mode)
            elif t == "attention":
                x = blk.rows(x, st.kv[l], st.pos)
            else:
                x = blk.rows(x, st.mamba[l], st.n_keep)
        return x

    def prefill(self, tokens, st, chunk=512, on_hidden=None):
        """tokens [T] -> the residual stream of the last position [1, D] (hsd/model.py:259).
        st must be fresh (reset) or at a kept row count of 1."""
        last = None
        for i in range(0, tokens.shape[0], chunk):
            x = self.embed(tokens[i:i + chunk])
            for l, t in enumerate(self.types):
                blk = self.blocks[l]
                if t == "moe":
                    x = blk(x, self.mode, self.prefill_gemm)
                elif t == "attention":
                    x = blk.rows(x, st.kv[l], st.pos)
                else:
                    x = blk.prefill(x, st.mamba[l])
            st.pos.add_(x.shape[0])
            if on_hidden is not None:
                on_hidden(i, x)
            last = x[-1:]
        st.n_keep.fill_(1)
        return last

    def step(self, x, st):
        """One decode step on x [1, D] (hsd/model.py:281)."""
        y = self.forward_rows(x, st)
        st.pos.add_(1)
        st.n_keep.fill_(1)
        return y

    def verify_step(self, x, st):
        """x [B, D]: B consecutive positions in ONE step (hsd/model.py:333); every Mamba layer
        keeps the state after each row. rollback() must follow."""
        return self.forward_rows(x, st)

    def rollback(self, st, n_keep, B):
        """Keep the first n_keep rows of the last verify_step of B rows (hsd/model.py:348): the
        attention position advances by n_keep (the rows past it are overwritten by the next
        step) and the Mamba layers continue from their row n_keep-1 checkpoint."""
        if not 1 <= n_keep <= B:
            raise ValueError(f"rollback: n_keep {n_keep} outside 1..{B}")
        st.pos.add_(n_keep)
        st.n_keep.fill_(n_keep)

    # ---- captured decode steps
    def _capture(self, key, body):
        g = self._graphs.get(key)
        if g is not None:
            return g
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):                    # warm-up: library state, cuBLAS handles
                body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = body()
        torch.cuda.synchronize(self.device)
        g = self._graphs[key] = _Graph(graph, out)
        return g

    def _io_buffers(self):
        if self._io is None:
            a, dev, R = self.args, self.device, self.state.rows
            self._io = dict(tok=torch.zeros(1, dtype=torch.int64, device=dev),
                            pend_h=torch.zeros((R, a.hidden), dtype=torch.bfloat16, device=dev),
                            pend_t=torch.zeros(R, dtype=torch.int64, device=dev),
                            cnt=torch.ones(1, dtype=torch.int64, device=dev),
                            replay=torch.zeros(R, dtype=torch.int64, device=dev),
                            ar=torch.arange(R, device=dev))
        return self._io

    def _step_body(self):
        """One greedy step from io.tok: -> [token, top-1 minus top-2 logit] (fp32; ids < 2^24)."""
        st, io = self.state, self._io_buffers()
        x = self.step(self.embed(io["tok"]), st)
        top = torch.topk(self.logits(x), 2, dim=-1)
        io["tok"].copy_(top.indices[0, :1])
        return torch.stack([top.indices[0, 0].float(), top.values[0, 0] - top.values[0, 1]])

    def _mtp_body(self, mtp, n_draft, replay):
        """One speculative iteration (hsd/model.py:397-437) on the device: the head drafts
        n_draft tokens from the pending rows (or the replay buffer holds them), one verify
        step of n_draft+1 rows, the greedy accept rule, the rollback (position += a+1, the
        Mamba layers keep row a) and the next pending rows. -> [tokens (n_draft+1), a]: the
        first a+1 tokens are the new ones."""
        st, io = self.state, self._io_buffers()
        bs = n_draft + 1
        if replay:
            drafts = io["replay"][:n_draft]
        else:
            pred, hn = mtp.rows(io["pend_h"][:bs], io["pend_t"][:bs], mtp.pos)
            i = io["cnt"] - 1
            d, hd = pred.index_select(0, i), hn.index_select(0, i)
            mtp.pos.add_(io["cnt"])
            ds = [d]
            for j in range(1, n_draft):           # chained rows: past the head's position, dropped
                d, hd = mtp.rows(hd, d, mtp.pos + (j - 1))
                ds.append(d)
            drafts = torch.cat(ds)
        ids = torch.cat([io["tok"], drafts])
        x = self.forward_rows(self.embed(ids), st)
        tgt = torch.argmax(self.logits(x), dim=-1)
        acc = torch.cumprod((drafts == tgt[:n_draft]).long(), 0).sum().view(1)
        st.pos.add_(acc + 1)
        st.n_keep.copy_(acc + 1)
        io["tok"].copy_(tgt.index_select(0, acc))
        io["pend_h"][:bs].copy_(x)
        io["pend_t"][:bs].copy_(tgt)
        io["cnt"].copy_(acc + 1)
        return torch.cat([tgt, acc])

    # ---- generation (greedy)
    def _first(self, h):
        top = torch.topk(self.logits(h), 2, dim=-1)
        tok, margin = torch.stack([top.indices[0, 0].float(), top.values[0, 0] - top.values[0, 1]]).tolist()
        return int(tok), margin

    def generate(self, prompt, max_tokens=128, chunk=512, forced=None, graphs=True):
        """Greedy decoding (hsd/model.py:291) -> (tokens, stats). stats["margins"] holds the
        top-1 minus top-2 logit of every choice. With `forced` (a token list) the loop feeds
        forced[i] instead of its own choice (teacher forcing) and still returns its choices.
        graphs=True replays one captured step per token; False runs the same ops eagerly."""
        prompt = torch.as_tensor(prompt, dtype=torch.long, device=self.device)
        io = self._io_buffers()
        g = self._capture(("step", self.mode), self._step_body) if graphs else None
        st = self.state
        st.reset()
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        h = self.prefill(prompt, st, chunk)
        tok, mg = self._first(h)
        t1 = time.perf_counter()
        out, margins = [tok], [mg]
        io["tok"].fill_(tok)
        while len(out) < max_tokens:
            if forced is not None:
                io["tok"].fill_(forced[len(out) - 1])
            if g is not None:
                g.graph.replay()
                r = g.out.tolist()
            else:
                r = self._step_body().tolist()
            out.append(int(r[0]))
            margins.append(r[1])
        t2 = time.perf_counter()
        return out, dict(mode=self.mode, prompt_tokens=int(prompt.shape[0]), prompt_s=t1 - t0, gen_tokens=len(out),
                         decode_s=t2 - t1, decode_tps=(len(out) - 1) / max(t2 - t1, 1e-9), margins=margins,
                         graphs=graphs)

    def generate_mtp(self, prompt, mtp, n_draft=2, max_tokens=128, chunk=512, replay=None, graphs=True):
        """Greedy speculative decoding with the MTP head (hsd/model.py:366-443) -> (tokens, stats).

        replay (a token list, e.g. an earlier greedy run's output) replaces the head's drafts
        with the tokens that follow in that list -- forced acceptance, which times the verify
        and rollback at acceptances a = 0..k that a random-init head never reaches. The accept
        rule is unchanged, so the output is still this model's own greedy sequence."""
        if n_draft + 1 > self.state.rows:
            raise ValueError(f"generate_mtp: n_draft {n_draft} needs verify_rows >= {n_draft + 1}")
        prompt = torch.as_tensor(prompt, dtype=torch.long, device=self.device)
        io = self._io_buffers()
        body = lambda: self._mtp_body(mtp, n_draft, replay is not None)  # noqa: E731
        g = self._capture(("mtp", self.mode, n_draft, replay is not None, id(mtp)), body) if graphs else None
        st = self.state
        st.reset()
        mtp.reset()
        last_h = []

        def on_hidden(i, x):                       # the head's prefill: rows (h_p, tok_{p+1})
            nxt = prompt[i + 1:i + 1 + x.shape[0]]
            if nxt.shape[0] > 0 and replay is None:
                mtp.rows(x[:nxt.shape[0]], nxt, mtp.pos)
                mtp.pos.add_(nxt.shape[0])
            last_h.append(x[-1:])

        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        x_last = self.prefill(prompt, st, chunk, on_hidden=on_hidden)
        tok, _ = self._first(x_last)
        t1 = time.perf_counter()
        out = [tok]
        io["tok"].fill_(tok)
        io["pend_h"][:1].copy_(last_h[-1])
        io["pend_t"][:1].fill_(tok)
        io["cnt"].fill_(1)
        steps, acc = 0, []
        while len(out) < max_tokens:
            if replay is not None:
                nxt = replay[len(out):len(out) + n_draft]
                nxt = nxt + [0] * (n_draft - len(nxt))
                io["replay"][:n_draft].copy_(torch.tensor(nxt, dtype=torch.int64))
            if g is not None:
                g.graph.replay()
                r = g.out.tolist()
            else:
                r = body().tolist()
            a = int(r[-1])
            new = [int(t) for t in r[:a + 1]][:max_tokens - len(out)]
            steps += 1
            acc.append(a)
            out.extend(new)
        t2 = time.perf_counter()
        return out, dict(mode=self.mode, n_draft=n_draft, steps=steps, accepted_mean=sum(acc) / max(1, len(acc)),
                         accepted_hist=[acc.count(k) for k in range(n_draft + 1)], gen_tokens=len(out),
                         prompt_s=t1 - t0, decode_s=t2 - t1, decode_tps=(len(out) - 1) / max(t2 - t1, 1e-9),
                         replay=replay is not None, graphs=graphs)


class MTPHead:
    """The MTP drafter (hsd/mtp.py:41-88): x = eh_proj([rms(embed(tok)), rms(h)]) -> attention
    block (own KV cache and position) -> MoE block -> final norm -> the target's lm_head
    argmax. Random init here. The head's MoE runs `mode` (the reference's head is a stock
    mlx block, i.e. the dense down projection)."""

    def __init__(self, target, seed=1, mode="dense"):
        a = target.args
        self.target, self.eps, self.mode = target, a.eps, mode
        gen = torch.Generator(device=target.device).manual_seed(seed)
        dev = target.device
        self.enorm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.hnorm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.eh_proj = QLinear(a.hidden, 2 * a.hidden, gen, dev, a.std)
        self.attn = AttnBlock(a, gen, dev)
        self.moe = MoEBlock(a, gen, dev)
        self.final_norm = (1.0 + 0.1 * torch.randn(a.hidden, generator=gen, device=dev)).to(torch.bfloat16)
        self.kv = KVCache(a, dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)

    def reset(self):
        self.kv.reset()
        self.pos.zero_()

    def rows(self, h, toks, pos):
        """h [R, D] (the target's pre-norm hidden state), toks [R] (the token after each row's
        position), pos the head cache position of row 0 -> (pred [R] int64, hn [R, D]). The
        head's cache gets the R rows; the position is advanced by the caller."""
        e = rms_norm(self.target.embed(toks), self.enorm, self.eps)
        hh = rms_norm(h, self.hnorm, self.eps)
        x = self.eh_proj(torch.cat([e, hh], -1))
        x = self.attn.rows(x, self.kv, pos)
        x = self.moe(x, self.mode, self.target.prefill_gemm)
        hn = rms_norm(x, self.final_norm, self.eps)
        return torch.argmax(self.target.head_fn(hn), -1), hn


def identical_prefix(a, b):
    """Length of the common prefix of two token lists."""
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n
