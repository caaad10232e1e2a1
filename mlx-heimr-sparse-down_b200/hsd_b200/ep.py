"""Expert-parallel MoE down projection over the GPUs of one box (a multi-GPU form of
hsd/decode.py's sparse_down and hsd/prefill.py's sparse_down_prefill; the reference itself
runs on one Apple GPU).

Placement: routed expert e lives on rank e // (E / G) (E / G contiguous experts per GPU); the
shared expert is replicated. Tokens stay on their home rank. One MoE down projection is:

  dispatch  every (token, slot) goes to its expert's owner: its h row (F values), its expert
            id local to the owner and its routing gain, with all_to_all_single over NCCL
            (counts first, then the payloads in expert-owner order)
  compute   the owner runs this library's kernels on the slots it received, one slot per row
            (the decode kernel's routed-only form for few slots, the tcgen05 prefill GEMM for
            many), the gain applied in the kernel, fp32 out
  combine   the fp32 partial rows go back with all_to_all_single; the home rank sums each
            token's topk partials in slot order and adds its own shared-expert part (the
            decode kernel's shared-only form) -- a fixed order, so the result does not
            depend on the number of GPUs beyond fp32 rounding of the same terms

The only host synchronisation is the read of the per-rank slot counts. Batch-1 latency stays
on one GPU (no exchange); this path is for batch decode and prefill chunks.
"""
import torch
import torch.distributed as dist

from .decode import sparse_down
from .prefill import sparse_down_prefill

PREFILL_MIN_SLOTS = 256     # owners with at least this many slots use the tensor-core GEMM


def _kernel_local_down(pw, ps, pb, F, D, E_local):
    """Routed-only down projection of received slots with this library's kernels."""

    def run(h, local_ids, gains):
        R = h.shape[0]
        g2 = torch.stack([gains, torch.zeros_like(gains)], 1).contiguous()
        sel = local_ids.view(R, 1).to(torch.int32).contiguous()
        if R >= PREFILL_MIN_SLOTS and D % 192 == 0:
            return sparse_down_prefill(h, sel, g2, pw, ps, pb, None, None, None, F=F, FS=0, D=D, topk=1,
                                       E=E_local, out_dtype=torch.float32)
        return sparse_down(h, sel, g2, pw, ps, pb, None, None, None, F=F, FS=0, D=D, topk=1,
                           out_dtype=torch.float32)

    return run


def _kernel_shared_down(spw, sps, spb, FS, D):
    def run(hs, gain):
        return sparse_down(hs, None, gain.contiguous(), None, None, None, spw, sps, spb, F=64, FS=FS, D=D, topk=0,
                           out_dtype=torch.float32)

    return run


class ExpertParallelDown:
    """The MoE down projection with routed experts sharded over `group`.

    pw / ps / pb: this rank's experts [E/G, F, D/8] / [E/G, F/64, D] (neuron-major);
    spw / sps / spb: the shared expert (replicated). local_down / shared_down replace the
    kernels (the CPU tests pass the oracle's arithmetic; the product passes nothing)."""

    def __init__(self, E, F, FS, D, topk, pw=None, ps=None, pb=None, spw=None, sps=None, spb=None, group=None,
                 local_down=None, shared_down=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.world:
            raise ValueError(f"ExpertParallelDown: E={E} is not divisible by {self.world} ranks")
        self.E, self.F, self.FS, self.D, self.topk = E, F, FS, D, topk
        self.E_local = E // self.world
        self.local_down = local_down or _kernel_local_down(pw, ps, pb, F, D, self.E_local)
        self.shared_down = shared_down or _kernel_shared_down(spw, sps, spb, FS, D)

    def owner(self, e):
        return e // self.E_local

    def __call__(self, hcat, sel, gains):
        """hcat [B, topk*F + FS], sel [B, topk] int32 (global ids), gains [B, topk+1] f32 ->
        y [B, D] f32 for this rank's B tokens (B may be 0; every rank must call)."""
        B, K, F, D = hcat.shape[0], self.topk, self.F, self.D
        dev = hcat.device
        flat = sel.reshape(-1).long()                                   # slot j = b*K + k
        dest = flat // self.E_local
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()             # the one host read
        R = sum(rc)
        h_slots = hcat[:, :K * F].reshape(B * K, F)[order].contiguous()
        local_ids = (flat - dest * self.E_local)[order].contiguous()     # the owner's expert index
        g_slots = gains[:, :K].reshape(-1)[order].contiguous()
        h_recv = torch.empty((R, F), dtype=hcat.dtype, device=dev)
        ids_recv = torch.empty(R, dtype=torch.int64, device=dev)
        g_recv = torch.empty(R, dtype=torch.float32, device=dev)
        dist.all_to_all_single(h_recv, h_slots, rc, sc, group=self.group)
        dist.all_to_all_single(ids_recv, local_ids, rc, sc, group=self.group)
        dist.all_to_all_single(g_recv, g_slots, rc, sc, group=self.group)
        y_recv = self.local_down(h_recv, ids_recv, g_recv) if R > 0 else \
            torch.empty((0, D), dtype=torch.float32, device=dev)
        y_back = torch.empty((B * K, D), dtype=torch.float32, device=dev)
        dist.all_to_all_single(y_back, y_recv.contiguous(), sc, rc, group=self.group)
        y_slots = torch.empty_like(y_back)
        y_slots[order] = y_back                                         # back to slot order j
        y = y_slots.view(B, K, D).sum(1) if K > 0 else torch.zeros((B, D), dtype=torch.float32, device=dev)
        if self.FS > 0 and B > 0:
            y = y + self.shared_down(hcat[:, K * F:].contiguous(), gains[:, K:])
        return y
