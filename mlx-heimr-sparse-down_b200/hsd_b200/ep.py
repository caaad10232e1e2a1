"""Expert-parallel MoE down projection over the GPUs of one box (a multi-GPU form of
hsd/decode.py's sparse_down and hsd/prefill.py's sparse_down_prefill; the reference itself
runs on one Apple GPU).

Placement: routed expert e lives on rank e % G (local index e // G), round robin, so that the
popular low-numbered experts of a skewed router spread over every rank (under the Zipf(1.1)
routing of the benchmark the busiest rank gets ~1.7x the mean slot count, against ~4.9x for
contiguous blocks of E/G experts at G = 8). The shared expert is replicated. Tokens stay on
their home rank.

ExpertParallelDown (the product) runs one call as three library calls on the caller's stream,
exchanging through peer memory: every rank's inbox (PeerInboxes) is mapped into every other
rank's process and written with plain stores over NVLink, ordered by release / acquire flags
(include/hsd.h, hsd_ep_*):

  dispatch  each (token, slot)'s h row, local expert id and gain go straight into its owner's
            inbox (the counts travel the same way first, so nothing is read back to the host)
  expert    the owner runs the tcgen05 grouped GEMM over the rows it received; the epilogue
            stores each fp32 partial row, times its gain, into its home rank's inbox
  combine   the home rank sums each token's topk partials in slot order plus its shared-expert
            row (the owner's GEMM launch also runs the shared expert's tiles of the rank's own
            tokens, so one persistent grid covers both)

The partials stay fp32: six bf16-rounded partials per token would cost ~2^-9 relative each,
most of the parity budget. With one GPU the same path runs with the rank's own inbox.

ExpertParallelDownCollective is the same computation with torch.distributed all_to_all
exchanges (NCCL on GPUs, gloo on CPU): the baseline the bench measures beside the product, and
the form the CPU tests drive with the oracle's arithmetic in place of the kernels.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib as L
from .decode import sparse_down
from .prefill import sparse_down_prefill

GEMM_MIN_SLOTS = 64         # owners with at least this many slots use the tensor-core GEMM
GEMM_MIN_ROWS = 32          # the shared expert of at least this many tokens uses the GEMM (measured crossover ~28)


def owned_experts(E, rank, world):
    """The global ids of the routed experts rank `rank` holds (round robin: e % world == rank),
    in local-index order."""
    return list(range(rank, E, world))


def expert_placement(E, world, replicated=()):
    """Where every routed expert lives. Expert e belongs to rank e % world (round robin) unless it
    is in `replicated`, a list of hot experts held by EVERY rank: a slot routed to one of those is
    computed on its own home rank and never crosses NVLink (under the benchmark's Zipf(1.1)
    routing, replicating the 8 most used experts cuts the busiest rank's slots from 1.70x to
    1.09x the mean at 8 GPUs, for 8 more expert stacks per rank). Rank r's local experts are its
    owned ones in ascending id, then the replicated ones in the given order.
    -> (local: per rank the global ids in local-id order, emap: per rank a list of E ints,
    owner << 16 | local id at the owner, replicated experts mapped to the rank itself)."""
    rep = list(dict.fromkeys(int(e) for e in replicated))
    if any(not 0 <= e < E for e in rep):
        raise ValueError(f"expert_placement: replicated ids must be in [0, {E})")
    repset = set(rep)
    owned = [[e for e in range(E) if e % world == r and e not in repset] for r in range(world)]
    where = {e: (r, i) for r in range(world) for i, e in enumerate(owned[r])}
    local = [owned[r] + rep for r in range(world)]
    emap = []
    for r in range(world):
        m = []
        for e in range(E):
            if e in repset:
                m.append((r << 16) | (len(owned[r]) + rep.index(e)))
            else:
                o, i = where[e]
                m.append((o << 16) | i)
        emap.append(m)
    return local, emap


def hottest_experts(sel, E, n, group=None):
    """The n experts with the most slots in `sel` (summed over the ranks of `group` when a process
    group is up): a one-time calibration for `replicated`."""
    cnt = torch.bincount(sel.reshape(-1).long(), minlength=E).to(torch.float64)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(cnt, group=group)
    return [int(e) for e in torch.argsort(cnt, descending=True, stable=True)[:n].tolist()]


def shard_experts(pw, ps, pb, rank, world, replicated=()):
    """This rank's stack of a full neuron-major expert stack ([E, ...] each), in local-id order
    (expert_placement), contiguous."""
    ids = expert_placement(pw.shape[0], world, replicated)[0][rank]
    idx = torch.tensor(ids, dtype=torch.long, device=pw.device)
    return tuple(t.index_select(0, idx).contiguous() for t in (pw, ps, pb))


def _kernel_local_down(pw, ps, pb, F, D, E_local):
    """Routed-only down projection of received slots with this library's kernels: the tcgen05
    prefill GEMM from GEMM_MIN_SLOTS slots (its cost follows the number of non-empty expert
    tiles), the decode kernel's per-slot form below (each slot costs a whole launch row of
    clusters for one expert's groups: measured ~4.5 us per slot at 192 slots)."""

    def run(h, local_ids, gains):
        R = h.shape[0]
        g2 = torch.stack([gains, torch.zeros_like(gains)], 1).contiguous()
        sel = local_ids.view(R, 1).to(torch.int32).contiguous()
        if R >= GEMM_MIN_SLOTS and D % 192 == 0:
            return sparse_down_prefill(h, sel, g2, pw, ps, pb, None, None, None, F=F, FS=0, D=D, topk=1,
                                       E=E_local, out_dtype=torch.float32)
        return sparse_down(h, sel, g2, pw, ps, pb, None, None, None, F=F, FS=0, D=D, topk=1,
                           out_dtype=torch.float32)

    return run


def _kernel_shared_down(spw, sps, spb, FS, D):
    """The shared expert of the home rank's tokens: the decode kernel's shared-only form, or for
    many tokens the prefill GEMM with the shared expert as the single routed expert."""
    one = None if spw is None else (spw.view(1, *spw.shape), sps.view(1, *sps.shape), spb.view(1, *spb.shape))

    def run(hs, gain):
        B = hs.shape[0]
        if B >= GEMM_MIN_ROWS and D % 192 == 0:
            sel = torch.zeros((B, 1), dtype=torch.int32, device=hs.device)
            g2 = torch.cat([gain.reshape(B, 1), torch.zeros_like(gain.reshape(B, 1))], 1).contiguous()
            return sparse_down_prefill(hs, sel, g2, *one, None, None, None, F=FS, FS=0, D=D, topk=1, E=1,
                                       out_dtype=torch.float32)
        return sparse_down(hs, None, gain.contiguous(), None, None, None, spw, sps, spb, F=64, FS=FS, D=D, topk=0,
                           out_dtype=torch.float32)

    return run


class ExpertParallelDownCollective:
    """The MoE down projection with routed experts sharded round robin over `group`, exchanged
    with torch.distributed all_to_all (the baseline of ExpertParallelDown).

    pw / ps / pb: this rank's experts (owned_experts order) [E/G, F, D/8] / [E/G, F/64, D]
    (neuron-major; shard_experts slices a full stack); spw / sps / spb: the shared expert
    (replicated). local_down / shared_down replace the kernels (the CPU tests pass the
    oracle's arithmetic; the product passes nothing). Without an initialised process group
    the object runs alone (world size 1). timing=True records CUDA events around the phases
    of every call; phase_ms() reads the last call's."""

    def __init__(self, E, F, FS, D, topk, pw=None, ps=None, pb=None, spw=None, sps=None, spb=None, group=None,
                 local_down=None, shared_down=None, timing=False):
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        if E % self.world:
            raise ValueError(f"ExpertParallelDown: E={E} is not divisible by {self.world} ranks")
        self.E, self.F, self.FS, self.D, self.topk = E, F, FS, D, topk
        self.E_local = E // self.world
        self.local_down = local_down or _kernel_local_down(pw, ps, pb, F, D, self.E_local)
        self.shared_down = shared_down or _kernel_shared_down(spw, sps, spb, FS, D)
        self.timing = timing
        self._events = None

    def owner(self, e):
        return e % self.world

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _mark(self, i):
        if self._events is not None:
            self._events[i].record()

    def phase_ms(self):
        """The last timed call's device time per phase (ms): dispatch (counts + packed rows),
        compute (the owner's kernels), combine (partials back, slot sums, shared expert)."""
        if self._events is None:
            return None
        self._events[-1].synchronize()
        e = self._events
        return {"dispatch": e[0].elapsed_time(e[1]), "compute": e[1].elapsed_time(e[2]),
                "combine": e[2].elapsed_time(e[3]), "total": e[0].elapsed_time(e[3])}

    def __call__(self, hcat, sel, gains):
        """hcat [B, topk*F + FS], sel [B, topk] int32 (global ids), gains [B, topk+1] f32 ->
        y [B, D] f32 for this rank's B tokens (B may be 0; every rank must call)."""
        B, K, F, D = hcat.shape[0], self.topk, self.F, self.D
        dev = hcat.device
        if self.timing and dev.type == "cuda":
            self._events = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        self._mark(0)
        flat = sel.reshape(-1).long()                                   # slot j = b*K + k
        dest = flat % self.world
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        if self.world == 1:
            recv_counts = send_counts
        else:
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        # one packed byte row per slot: h (2F bytes) | local expert id (int32) | gain (f32),
        # queued before the host read so that the read waits on work already launched
        rb = 2 * F + 8
        packed = torch.empty((B * K, rb), dtype=torch.uint8, device=dev)
        packed[:, :2 * F] = hcat[:, :K * F].reshape(B * K, F)[order].contiguous().view(torch.uint8)
        packed[:, 2 * F:2 * F + 4] = (flat // self.world)[order].to(torch.int32).view(-1, 1).view(torch.uint8)
        packed[:, 2 * F + 4:] = gains[:, :K].reshape(-1)[order].contiguous().view(-1, 1).view(torch.uint8)
        sc, rc = send_counts.tolist(), recv_counts.tolist()             # the one host read
        R = sum(rc)
        recv = torch.empty((R, rb), dtype=torch.uint8, device=dev)
        self._a2a(recv.view(-1), packed.view(-1), [c * rb for c in rc], [c * rb for c in sc])
        self._mark(1)
        if R > 0:
            h_recv = recv[:, :2 * F].contiguous().view(hcat.dtype)
            ids_recv = recv[:, 2 * F:2 * F + 4].contiguous().view(torch.int32).view(-1)
            g_recv = recv[:, 2 * F + 4:].contiguous().view(torch.float32).view(-1)
            y_recv = self.local_down(h_recv, ids_recv, g_recv)
        else:
            y_recv = torch.empty((0, D), dtype=torch.float32, device=dev)
        self._mark(2)
        y_back = torch.empty((B * K, D), dtype=torch.float32, device=dev)
        self._a2a(y_back, y_recv.contiguous(), sc, rc)
        y_slots = torch.empty_like(y_back)
        y_slots[order] = y_back                                         # back to slot order j
        y = y_slots.view(B, K, D).sum(1) if K > 0 else torch.zeros((B, D), dtype=torch.float32, device=dev)
        if self.FS > 0 and B > 0:
            y = y + self.shared_down(hcat[:, K * F:].contiguous(), gains[:, K:])
        self._mark(3)
        return y


class PeerInboxes:
    """One rank's expert-parallel buffers: its inbox (hsd_ep_alloc memory that every other rank
    maps and writes) and its private workspace, with the inboxes of all ranks as this process
    addresses them stored in the workspace. Construction is collective over `group` (an
    all_gather of the 64-byte IPC handles and of the configuration, which must agree). One
    PeerInboxes serves every call and every layer of the rank. close() is collective too: it
    synchronises the device, waits for every rank, unmaps the peers' inboxes and frees this
    rank's; without it the memory stays until the process exits."""

    def __init__(self, world, rank, max_tokens, topk, F, FS, D, E, device, group=None, n_local=0):
        self.world, self.rank, self.max_tokens = world, rank, max_tokens
        self.topk, self.F, self.FS, self.D, self.E = topk, F, FS, D, E
        self.n_local = n_local if n_local > 0 else E // world
        self.device = torch.device(device)
        self.group = group
        ib, wb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        L.call("hsd_ep_buffer_bytes", world, max_tokens, topk, F, FS, D, E, self.n_local, ctypes.byref(ib),
               ctypes.byref(wb))
        self.inbox_bytes, self.workspace_bytes = ib.value, wb.value
        with torch.cuda.device(self.device):
            p = ctypes.c_void_p(0)
            L.call("hsd_ep_alloc", ib.value, ctypes.byref(p))
            self.inbox = p.value
            self.workspace = torch.empty(wb.value, dtype=torch.uint8, device=self.device)
            self._opened = []
            addrs = [0] * world
            addrs[rank] = self.inbox
            if world > 1:
                handle = (ctypes.c_ubyte * 64)()
                L.call("hsd_ep_ipc_handle", ctypes.c_void_p(self.inbox), ctypes.cast(handle, ctypes.c_void_p))
                mine = (bytes(handle), (world, max_tokens, topk, F, FS, D, E))
                everyone = [None] * world
                dist.all_gather_object(everyone, mine, group=group)
                for r, (h, cfg) in enumerate(everyone):
                    if cfg != mine[1]:
                        raise ValueError(f"PeerInboxes: rank {r} has configuration {cfg}, this rank {mine[1]}")
                    if r == rank:
                        continue
                    q = ctypes.c_void_p(0)
                    L.call("hsd_ep_ipc_open", ctypes.cast((ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.c_void_p),
                           ctypes.byref(q))
                    self._opened.append(q.value)
                    addrs[r] = q.value
            table = (ctypes.c_uint64 * world)(*addrs)
            L.call("hsd_ep_set_peers", L.ptr(self.workspace), ctypes.cast(table, ctypes.c_void_p), world,
                   L.stream_of(self.workspace))

    def close(self):
        if self.inbox is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for q in self._opened:
            L.call("hsd_ep_ipc_close", ctypes.c_void_p(q))
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)            # nobody maps this inbox any more
        L.call("hsd_ep_free", ctypes.c_void_p(self.inbox))
        self.inbox = None


class ExpertParallelDown:
    """The MoE down projection with routed experts sharded round robin over `group`, exchanged
    through peer memory with this library's kernels (no host synchronisation per call: a call
    can be captured in a CUDA graph).

    pw / ps / pb: this rank's experts (owned_experts order) [E/G, F, D/8] / [E/G, F/64, D]
    (neuron-major; shard_experts slices a full stack); spw / sps / spb: the shared expert
    (replicated). replicated: hot expert ids every rank holds (expert_placement; pw / ps / pb then
    hold this rank's owned experts followed by those, as shard_experts(..., replicated) gives).
    max_tokens bounds B per call (it sizes the inbox); inboxes: a PeerInboxes to share between
    layers with the same placement (else one is made, collectively). Without an initialised process group
    the object runs alone (world size 1) on its own inbox. timing=True records CUDA events
    around the phases of every call; phase_ms() reads the last call's. Every rank must make
    the same calls in the same order (B may differ, and may be 0)."""

    def __init__(self, E, F, FS, D, topk, pw, ps, pb, spw=None, sps=None, spb=None, group=None, max_tokens=512,
                 inboxes=None, timeout_s=10.0, timing=False, replicated=()):
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        if E % self.world:
            raise ValueError(f"ExpertParallelDown: E={E} is not divisible by {self.world} ranks")
        self.E, self.F, self.FS, self.D, self.topk = E, F, FS, D, topk
        local, emap = expert_placement(E, self.world, replicated)
        self.local_ids = local[self.rank]
        self.E_local = len(self.local_ids)
        L.require_cuda(pw, ps, pb, spw, sps, spb, what="ExpertParallelDown")
        if pw.shape[0] != self.E_local:
            raise ValueError(f"ExpertParallelDown: {pw.shape[0]} local experts given, {self.E_local} expected")
        self.emap = (torch.tensor(emap[self.rank], dtype=torch.int32, device=pw.device) if len(replicated) else None)
        self.pw, self.ps, self.pb = pw, ps, pb
        self.s_code = L.dtype_code(ps, "ExpertParallelDown scales")
        self.max_tokens = max_tokens
        self.inboxes = inboxes or PeerInboxes(self.world, self.rank, max_tokens, topk, F, FS, D, E, pw.device, group,
                                              n_local=self.E_local)
        ib = self.inboxes
        if (ib.world, ib.rank, ib.max_tokens, ib.topk, ib.F, ib.FS, ib.D, ib.E, ib.n_local) != (
                self.world, self.rank, max_tokens, topk, F, FS, D, E, self.E_local):
            raise ValueError("ExpertParallelDown: the inboxes were made for another configuration")
        if FS > 0 and (spw is None or sps is None or spb is None):
            raise ValueError("ExpertParallelDown: FS > 0 needs the shared expert's spw, sps, spb")
        self.spw, self.sps, self.spb = spw, sps, spb
        self.timeout_s = float(timeout_s)
        self.timing = timing
        self._events = None

    def owner(self, e):
        return e % self.world

    def _mark(self, i):
        if self._events is not None:
            self._events[i].record()

    def phase_ms(self):
        """The last timed call's device time per phase (ms) on this rank: dispatch (routing and
        the rows out), expert (waiting for the rows in, the one GEMM over the received rows and
        this rank's shared expert, the partial rows out), combine (waiting for the partials in
        and the sums)."""
        if self._events is None:
            return None
        self._events[-1].synchronize()
        e = self._events
        return {"dispatch": e[0].elapsed_time(e[1]), "expert": e[1].elapsed_time(e[2]),
                "combine": e[2].elapsed_time(e[3]), "total": e[0].elapsed_time(e[3])}

    def __call__(self, hcat, sel, gains):
        """hcat [B, topk*F + FS] bf16 / f16, sel [B, topk] int32 (global ids), gains [B, topk+1]
        f32 -> y [B, D] f32 for this rank's B tokens (B may be 0; every rank must call)."""
        B, K, F, D = hcat.shape[0], self.topk, self.F, self.D
        what = "ExpertParallelDown"
        L.require_cuda(hcat, sel, gains, what=what)
        if B > self.max_tokens:
            raise ValueError(f"{what}: {B} tokens, more than max_tokens={self.max_tokens}")
        if tuple(hcat.shape) != (B, K * F + self.FS) or tuple(sel.shape) != (B, K) or tuple(gains.shape) != (B, K + 1):
            raise ValueError(f"{what}: shapes hcat {tuple(hcat.shape)}, sel {tuple(sel.shape)}, gains "
                             f"{tuple(gains.shape)} do not match topk={K}, F={F}, FS={self.FS}")
        if sel.dtype != torch.int32 or gains.dtype != torch.float32:
            raise TypeError(f"{what}: sel must be int32 and gains float32")
        h_code = L.dtype_code(hcat, what)
        if h_code == L.HSD_F32:
            raise TypeError(f"{what}: hcat must be bf16 or f16")
        dev = hcat.device
        st = L.stream_of(hcat)
        ib = self.inboxes
        ws = L.ptr(ib.workspace)
        if self.timing:
            self._events = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        hp = L.ptr(hcat) if B else None
        self._mark(0)
        L.call("hsd_ep_dispatch", ws, self.rank, self.world, self.max_tokens, hp, h_code, L.ptr(sel) if B else None,
               L.ptr(gains) if B else None, B, K, F, self.FS, D, self.E, L.ptr(self.emap), self.timeout_s, st)
        self._mark(1)
        L.call("hsd_ep_expert", ws, ctypes.c_void_p(ib.inbox), self.rank, self.world, self.max_tokens, hp, h_code, B,
               L.ptr(self.pw), L.ptr(self.ps), L.ptr(self.pb), L.ptr(self.spw), L.ptr(self.sps), L.ptr(self.spb),
               self.s_code, K, F, self.FS, D, self.E, self.E_local, self.timeout_s, st)
        self._mark(2)
        y = torch.empty((B, D), dtype=torch.float32, device=dev)
        L.call("hsd_ep_combine", ws, self.rank, self.world, self.max_tokens, L.ptr(y) if B else None, B, K, F, self.FS,
               D, self.E, self.timeout_s, st)
        self._mark(3)
        return y
