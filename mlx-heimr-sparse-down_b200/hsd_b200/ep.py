"""Expert-parallel MoE down projection over the GPUs of one box (a multi-GPU form of
hsd/decode.py's sparse_down and hsd/prefill.py's sparse_down_prefill; the reference itself
runs on one Apple GPU).

Placement: routed expert e lives on rank e % G (local index e // G), round robin, so that the
popular low-numbered experts of a skewed router spread over every rank (under the Zipf(1.1)
routing of the benchmark the busiest rank gets ~1.7x the mean slot count, against ~4.9x for
contiguous blocks of E/G experts at G = 8). The shared expert is replicated. Tokens stay on
their home rank. One MoE down projection is:

  dispatch  every (token, slot) goes to its expert's owner as one packed byte row -- its h
            row (F values), its expert id local to the owner and its routing gain -- in ONE
            all_to_all_single over NCCL, after an all_to_all of the per-rank slot counts
  compute   the owner runs this library's kernels on the slots it received, one slot per row
            (the tcgen05 prefill GEMM, or the decode kernel's routed-only form for a handful of
            slots), the gain applied in the kernel, fp32 out
  combine   the fp32 partial rows go back with a second all_to_all_single; the home rank sums
            each token's topk partials in slot order and adds its own shared-expert part (the
            decode kernel's shared-only form, or the GEMM with the shared expert as the one
            routed expert for many tokens). The partials stay fp32: six bf16-rounded
            partials per token would cost ~2^-9 relative each, most of the parity budget.

The only host synchronisation is the read of the received slot counts (all_to_all_single
takes its split sizes on the host). Batch-1 latency stays on one GPU (no exchange); this path
is for batch decode and prefill chunks. With no process group (a single GPU) the exchanges
are local copies, so the same code path gives the one-GPU baseline.
"""
import torch
import torch.distributed as dist

from .decode import sparse_down
from .prefill import sparse_down_prefill

GEMM_MIN_SLOTS = 64         # owners with at least this many slots use the tensor-core GEMM
GEMM_MIN_ROWS = 256         # the shared expert of at least this many tokens uses the GEMM


def owned_experts(E, rank, world):
    """The global ids of the routed experts rank `rank` holds (round robin: e % world == rank),
    in local-index order."""
    return list(range(rank, E, world))


def shard_experts(pw, ps, pb, rank, world):
    """This rank's slice of a full neuron-major expert stack ([E, ...] each), contiguous."""
    return tuple(t[rank::world].contiguous() for t in (pw, ps, pb))


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


class ExpertParallelDown:
    """The MoE down projection with routed experts sharded round robin over `group`.

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
