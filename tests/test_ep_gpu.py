"""Expert-parallel down projection on GPUs: the peer-memory form (ExpertParallelDown: the
hsd_ep_* kernels, inboxes mapped over CUDA IPC) and the collective baseline
(ExpertParallelDownCollective, NCCL all_to_all) give the same outputs as the single-GPU
operators on the same tokens, for batch decode rows and a prefill chunk, at world size 2 (needs
2 GPUs) and at world size 1 (any GPU). A call of the peer-memory form reads nothing back to the
host: it is captured in a CUDA graph and replayed. A bounded device-side wait that runs out
(a flag no rank sets) returns HSD_ERR_TIMEOUT through the status word, with the context intact."""
import ctypes
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import rel_err

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _single(hsd_b200, c, lo, hi, pw, ps, pb, spw, sps, spb):
    args = (c["h"][lo:hi].contiguous(), c["sel"][lo:hi].contiguous(), c["gains"][lo:hi].contiguous(),
            pw, ps, pb, spw, sps, spb)
    return hsd_b200.sparse_down(*args, F=c["F"], FS=c["FS"], D=c["D"], topk=c["topk"], out_dtype=torch.float32)


def _worker(rank, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for pth in (os.path.join(os.path.dirname(here), "mlx-heimr-sparse-down_b200"), os.path.dirname(here), here):
        sys.path.insert(0, pth)
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import hsd_b200
        from hsd_b200 import synth
        from hsd_b200.ep import ExpertParallelDown, ExpertParallelDownCollective, shard_experts
        out = []
        inboxes = rep_inboxes = None
        for T in (8, 512):                  # batch decode rows, a prefill chunk, per rank
            c = synth.decode_case(seed=5, B=T * WORLD, zero_frac=0.9, device=dev, routing="zipf")
            pw, ps, pb = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"])
            spw, sps, spb = hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
            mine = shard_experts(pw, ps, pb, rank, WORLD)
            lo, hi = rank * T, (rank + 1) * T
            # rank 1 brings one token fewer: B may differ between ranks
            hi -= rank
            x = (c["h"][lo:hi].contiguous(), c["sel"][lo:hi].contiguous(), c["gains"][lo:hi].contiguous())
            ref = _single(hsd_b200, c, lo, hi, pw, ps, pb, spw, sps, spb)
            p2p = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], *mine, spw, sps, spb, max_tokens=512,
                                     inboxes=inboxes)
            inboxes = p2p.inboxes                # one inbox set for both shapes (and every layer)
            ys = [p2p(*x) for _ in range(3)]     # three calls: epochs advance, buffers reused
            coll = ExpertParallelDownCollective(c["E"], c["F"], c["FS"], c["D"], c["topk"], *mine, spw, sps, spb)
            yc = coll(*x)
            # hot experts on every rank: their slots stay home (placement table in the dispatch)
            hot = [0, 1, 2, 5]
            rep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"],
                                     *shard_experts(pw, ps, pb, rank, WORLD, replicated=hot), spw, sps, spb,
                                     max_tokens=512, replicated=hot, inboxes=rep_inboxes)
            rep_inboxes = rep.inboxes
            yr = rep(*x)
            torch.cuda.synchronize()
            r = ref.cpu().numpy()
            out.append((T, [rel_err(y.cpu().numpy(), r) for y in ys] + [rel_err(yr.cpu().numpy(), r)],
                        rel_err(yc.cpu().numpy(), r), all(torch.equal(ys[0], y) for y in ys),
                        hsd_b200.device_status()))
        inboxes.close()
        rep_inboxes.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_two_gpus_matches_single_gpu(cuda):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs on one machine")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, out in res:
        for T, errs, err_coll, same, status in out:
            assert status == 0, (rank, T, status)
            assert max(errs) < 5e-3, (rank, T, errs)   # GEMM form: fp16 operands, fp32 accumulation
            assert err_coll < 5e-3, (rank, T, err_coll)
            assert same, (rank, T)                       # repeated calls give the same bits


def _case(cuda, T, seed=6):
    import hsd_b200
    from hsd_b200 import synth
    c = synth.decode_case(seed=seed, B=T, zero_frac=0.9, device=cuda, routing="zipf")
    pw, ps, pb = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"])
    spw, sps, spb = hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
    return c, (pw, ps, pb, spw, sps, spb)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [8, 512])
def test_ep_one_gpu_path_matches_operator(cuda, T):
    """Both forms at world size 1 (no process group: the rank's own inbox, every expert local)
    equal the single-GPU operator on the same tokens."""
    import hsd_b200
    from hsd_b200.ep import ExpertParallelDown, ExpertParallelDownCollective
    c, wts = _case(cuda, T)
    ref = _single(hsd_b200, c, 0, T, *wts).cpu().numpy()
    ep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], *wts, max_tokens=512, timing=True)
    y = ep(c["h"], c["sel"], c["gains"])
    ph = ep.phase_ms()
    coll = ExpertParallelDownCollective(c["E"], c["F"], c["FS"], c["D"], c["topk"], *wts, timing=True)
    yc = coll(c["h"], c["sel"], c["gains"])
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) < 5e-3
    assert rel_err(yc.cpu().numpy(), ref) < 5e-3
    assert ph["total"] > 0 and set(ph) == {"dispatch", "expert", "combine", "total"}
    assert set(coll.phase_ms()) == {"dispatch", "compute", "combine", "total"}
    assert hsd_b200.device_status() == 0
    ep.inboxes.close()


@pytest.mark.gpu
def test_ep_placement_table_with_replicated_experts(cuda):
    """A placement with replicated experts at world size 1: the local stack is the owned experts
    then the replicated ones (a permutation of all 128), reached through the dispatch's table;
    the output is the single-GPU operator's."""
    import hsd_b200
    from hsd_b200.ep import ExpertParallelDown, hottest_experts, shard_experts
    T = 256
    c, wts = _case(cuda, T, seed=11)
    hot = hottest_experts(c["sel"], c["E"], 8)
    assert hot[0] == 0                        # Zipf routing: expert 0 is the most used
    ref = _single(hsd_b200, c, 0, T, *wts).cpu().numpy()
    ep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], *shard_experts(*wts[:3], 0, 1, replicated=hot),
                            *wts[3:], max_tokens=T, replicated=hot)
    y = ep(c["h"], c["sel"], c["gains"])
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) < 5e-3
    assert hsd_b200.device_status() == 0
    ep.inboxes.close()


@pytest.mark.gpu
def test_ep_call_replays_from_a_cuda_graph(cuda):
    """The peer-memory call reads nothing back to the host, so it captures: replays of the graph
    (each a new epoch of the flags) reproduce the eager call's bits on new inputs copied in."""
    import hsd_b200
    from hsd_b200.ep import ExpertParallelDown
    T = 64
    c, wts = _case(cuda, T, seed=8)
    c2, _ = _case(cuda, T, seed=9)          # other tokens, same weights (seed of the weights differs: unused)
    ep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], *wts, max_tokens=T)
    h, sel, g = c["h"].clone(), c["sel"].clone(), c["gains"].clone()
    ep(h, sel, g)                            # warm-up outside the capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            y_g = ep(h, sel, g)
    torch.cuda.current_stream().wait_stream(s)
    for src in (c, c2, c):
        h.copy_(src["h"])
        sel.copy_(src["sel"])
        g.copy_(src["gains"])
        graph.replay()
        torch.cuda.synchronize()
        y_e = ep(src["h"], src["sel"], src["gains"])
        torch.cuda.synchronize()
        assert torch.equal(y_g, y_e)
    assert hsd_b200.device_status() == 0
    del graph
    ep.inboxes.close()


@pytest.mark.gpu
def test_ep_wait_for_a_missing_rank_times_out_with_status(cuda):
    """A world of 2 whose second rank never runs: both inbox entries name this process's own
    inbox, so every count row, row and arrival lands here -- but the count flag of rank 1 is
    never set, and the dispatch's wait for it runs out (0.2 s). The call returns, the status
    word says HSD_ERR_TIMEOUT, and the context stays usable."""
    import hsd_b200
    import hsd_b200._lib as L
    c, wts = _case(cuda, 8, seed=7)
    E, F, FS, D, K = c["E"], c["F"], c["FS"], c["D"], c["topk"]
    assert hsd_b200.device_status() == 0
    ib, wb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    L.call("hsd_ep_buffer_bytes", 2, 8, K, F, FS, D, E, 0, ctypes.byref(ib), ctypes.byref(wb))
    p = ctypes.c_void_p(0)
    L.call("hsd_ep_alloc", ib.value, ctypes.byref(p))
    try:
        ws = torch.empty(wb.value, dtype=torch.uint8, device=cuda)
        table = (ctypes.c_uint64 * 2)(p.value, p.value)
        st = L.stream_of(ws)
        L.call("hsd_ep_set_peers", L.ptr(ws), ctypes.cast(table, ctypes.c_void_p), 2, st)
        pw, ps, pb = (t[0::2].contiguous() for t in wts[:3])
        spw, sps, spb = wts[3:]
        y = torch.empty((8, D), dtype=torch.float32, device=cuda)
        L.call("hsd_ep_dispatch", L.ptr(ws), 0, 2, 8, L.ptr(c["h"]), L.HSD_BF16, L.ptr(c["sel"]), L.ptr(c["gains"]),
               8, K, F, FS, D, E, None, 0.2, st)
        L.call("hsd_ep_expert", L.ptr(ws), p, 0, 2, 8, L.ptr(c["h"]), L.HSD_BF16, 8, L.ptr(pw), L.ptr(ps), L.ptr(pb),
               L.ptr(spw), L.ptr(sps), L.ptr(spb), L.HSD_BF16, K, F, FS, D, E, 0, 0.2, st)
        L.call("hsd_ep_combine", L.ptr(ws), 0, 2, 8, L.ptr(y), 8, K, F, FS, D, E, 0.2, st)
        torch.cuda.synchronize()
        assert hsd_b200.device_status() == L.HSD_ERR_TIMEOUT
        assert hsd_b200.device_status() == 0                    # read and cleared
        torch.ones(4, device=cuda).sum().item()                 # the context still works
    finally:
        torch.cuda.synchronize()
        L.call("hsd_ep_free", p)
