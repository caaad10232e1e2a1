"""Expert-parallel dispatch / combine on CPU ranks (gloo, world size 2): the exchange logic of
hsd_b200.ep's collective form (round-robin expert placement, one packed dispatch exchange) with
the oracle's arithmetic standing in for the kernels, against the single-process oracle; and the
placement helpers the peer-memory form shares with it. No GPU (the peer-memory exchange runs in
CUDA kernels: tests/test_ep_gpu.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

D, F, FS, E, TOPK = 128, 128, 128, 8, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case():
    from hsd_b200 import synth
    return synth.decode_case(seed=3, B=12, D=D, F=F, FS=FS, E=E, topk=TOPK, zero_frac=0.7)


def _worker(rank, world, port, tokens_per_rank, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for pth in (os.path.join(os.path.dirname(here), "mlx-heimr-sparse-down_b200"), os.path.dirname(here), here):
        sys.path.insert(0, pth)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import decode as od
        from oracle import layout as ol
        from oracle.quant import bf16_bits_to_f32, dequantize_neuron_major
        from hsd_b200.ep import ExpertParallelDownCollective
        c = _case()
        u16 = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        w = c["w"].numpy().view(np.uint32)
        pw, ps, pb = ol.to_neuron_major(w, u16(c["s"]), u16(c["b"]))
        Wt = dequantize_neuron_major(pw, bf16_bits_to_f32(ps), bf16_bits_to_f32(pb))       # [E, F, D]
        spw, sps, spb = ol.to_neuron_major(c["sw"].numpy().view(np.uint32), u16(c["ss"]), u16(c["sb"]))
        Wst = dequantize_neuron_major(spw, bf16_bits_to_f32(sps), bf16_bits_to_f32(spb))   # [FS, D]
        def local_down(h, ids, g):          # the owner's arithmetic, oracle-side (fp32)
            hf = h.float().numpy()               # local expert i of this rank is global i * world + rank
            y = np.stack([g[r].item() * (hf[r] @ Wt[int(ids[r]) * world + rank]) for r in range(h.shape[0])])
            return torch.from_numpy(y.astype(np.float32))

        def shared_down(hs, g):
            return torch.from_numpy((hs.float().numpy() @ Wst).astype(np.float32)) * g

        ep = ExpertParallelDownCollective(E, F, FS, D, TOPK, group=None, local_down=local_down, shared_down=shared_down)
        lo = sum(tokens_per_rank[:rank])
        hi = lo + tokens_per_rank[rank]
        y = ep(c["h"][lo:hi].contiguous(), c["sel"][lo:hi].contiguous(), c["gains"][lo:hi].contiguous())
        f = bf16_bits_to_f32
        ref = od.reference_dense(c["h"].float().numpy()[lo:hi], c["sel"].numpy()[lo:hi], c["gains"].numpy()[lo:hi],
                                 w, f(u16(c["s"])), f(u16(c["b"])), c["sw"].numpy().view(np.uint32), f(u16(c["ss"])),
                                 f(u16(c["sb"])), F=F, FS=FS, topk=TOPK)
        err = float(np.abs(y.numpy() - ref).max() / max(np.abs(ref).max(), 1e-30)) if hi > lo else 0.0
        q.put((rank, err, tuple(y.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens_per_rank", [(7, 5), (12, 0)])
def test_ep_dispatch_combine_gloo(tokens_per_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, tokens_per_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, shape in res:
        assert shape == (tokens_per_rank[rank], D)
        assert err < 1e-5, (rank, err)


def test_owned_experts_round_robin():
    from hsd_b200.ep import owned_experts, shard_experts
    assert owned_experts(8, 1, 4) == [1, 5]
    assert sorted(sum((owned_experts(128, r, 8) for r in range(8)), [])) == list(range(128))
    w = torch.arange(8 * 3).view(8, 3)
    a, _, _ = shard_experts(w, w, w, 2, 4)
    assert torch.equal(a, w[[2, 6]])


def test_round_robin_balances_zipf_routing():
    """Under the benchmark's Zipf(1.1) routing the busiest rank's slot count stays within 2x the
    mean with round-robin placement (contiguous blocks of E/G experts: ~4.9x at G = 8)."""
    from hsd_b200 import synth
    gen = torch.Generator().manual_seed(5)
    sel, _ = synth.route_zipf(4096, 128, 6, gen, "cpu")
    for G in (2, 4, 8):
        rr = torch.bincount(sel.reshape(-1).long() % G, minlength=G).float()
        blk = torch.bincount(sel.reshape(-1).long() // (128 // G), minlength=G).float()
        assert rr.max() / rr.mean() < 2.0, (G, rr)
        assert blk.max() / blk.mean() > rr.max() / rr.mean()


def test_placement_table_with_replicated_experts():
    """expert_placement: every rank's local stack is its owned experts (e % G == rank, not
    replicated) then the replicated ones; the table sends a replicated expert's slots to the
    rank itself and every other expert to its owner, at the owner's local index."""
    from hsd_b200.ep import expert_placement, shard_experts
    E, G, hot = 16, 4, [0, 3, 9]
    local, emap = expert_placement(E, G, hot)
    for r in range(G):
        assert local[r][-len(hot):] == hot
        assert all(e % G == r and e not in hot for e in local[r][:-len(hot)])
        for e in range(E):
            owner, lid = emap[r][e] >> 16, emap[r][e] & 0xFFFF
            if e in hot:
                assert owner == r
            else:
                assert owner == e % G
            assert local[owner][lid] == e
    owned = sorted(e for r in range(G) for e in local[r][:-len(hot)])
    assert owned == sorted(set(range(E)) - set(hot))
    # no replication: the round-robin placement (owner e % G, local index e // G)
    local0, emap0 = expert_placement(E, G)
    assert all(emap0[r][e] == ((e % G) << 16 | e // G) for r in range(G) for e in range(E))
    w = torch.arange(E * 2).view(E, 2)
    a, _, _ = shard_experts(w, w, w, 1, G, replicated=hot)
    assert torch.equal(a, w[local[1]])


def test_replicating_hot_experts_balances_zipf_routing():
    """With the 8 most used experts on every rank (their slots computed at home) the busiest
    rank's slots come within 1.2x of the mean at 8 ranks under the Zipf(1.1) routing."""
    from hsd_b200 import synth
    from hsd_b200.ep import expert_placement
    G, E = 8, 128
    load = torch.zeros(G)
    sels = []
    for r in range(G):
        gen = torch.Generator().manual_seed(100 + r)
        sels.append(synth.route_zipf(512, E, 6, gen, "cpu")[0])
    cnt = torch.bincount(torch.cat(sels).reshape(-1).long(), minlength=E)
    hot = torch.argsort(cnt, descending=True)[:8].tolist()
    _, emap = expert_placement(E, G, hot)
    for r in range(G):
        owners = torch.tensor([emap[r][e] >> 16 for e in sels[r].reshape(-1).tolist()])
        load += torch.bincount(owners, minlength=G).float()
    assert load.max() / load.mean() < 1.2, load
