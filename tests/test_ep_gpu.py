"""Expert-parallel down projection over 2 GPUs (NCCL): the same outputs as the single-GPU
kernels on the same tokens, for batch decode (few slots per owner: the decode kernel) and a
prefill chunk (many slots per owner: the tcgen05 GEMM). Needs 2 GPUs."""
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


def _worker(rank, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for pth in (os.path.join(os.path.dirname(here), "mlx-heimr-sparse-down_b200"), os.path.dirname(here), here):
        sys.path.insert(0, pth)
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import hsd_b200
        from hsd_b200 import synth
        from hsd_b200.ep import ExpertParallelDown, shard_experts
        out = []
        for T in (8, 512):                  # batch decode rows, a prefill chunk, per rank
            c = synth.decode_case(seed=5, B=T * WORLD, zero_frac=0.9, device=dev, routing="zipf")
            pw, ps, pb = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"])
            spw, sps, spb = hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
            ep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], *shard_experts(pw, ps, pb, rank, WORLD),
                                    spw, sps, spb)
            lo, hi = rank * T, (rank + 1) * T
            y = ep(c["h"][lo:hi].contiguous(), c["sel"][lo:hi].contiguous(), c["gains"][lo:hi].contiguous())
            ref = hsd_b200.sparse_down(c["h"][lo:hi].contiguous(), c["sel"][lo:hi].contiguous(),
                                       c["gains"][lo:hi].contiguous(), pw, ps, pb, spw, sps, spb, F=c["F"],
                                       FS=c["FS"], D=c["D"], topk=c["topk"], out_dtype=torch.float32)
            torch.cuda.synchronize()
            out.append((T, rel_err(y.cpu().numpy(), ref.cpu().numpy())))
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
        for T, err in out:
            assert err < 5e-3, (rank, T, err)      # decode-kernel form exact to fp32 order; GEMM form fp16 operands


@pytest.mark.gpu
@pytest.mark.parametrize("T", [8, 512])
def test_ep_one_gpu_path_matches_operator(cuda, T):
    """The expert-parallel code path at world size 1 (no process group: the exchanges are local
    copies, every expert local) equals the single-GPU operator on the same tokens: the packing,
    the slot order, the per-slot kernels and the combine, on the hardware of a 1-GPU box."""
    import hsd_b200
    from hsd_b200 import synth
    from hsd_b200.ep import ExpertParallelDown
    c = synth.decode_case(seed=6, B=T, zero_frac=0.9, device=cuda, routing="zipf")
    pw, ps, pb = hsd_b200.to_neuron_major(c["w"], c["s"], c["b"])
    spw, sps, spb = hsd_b200.to_neuron_major(c["sw"], c["ss"], c["sb"])
    ep = ExpertParallelDown(c["E"], c["F"], c["FS"], c["D"], c["topk"], pw, ps, pb, spw, sps, spb, timing=True)
    y = ep(c["h"], c["sel"], c["gains"])
    ref = hsd_b200.sparse_down(c["h"], c["sel"], c["gains"], pw, ps, pb, spw, sps, spb, F=c["F"], FS=c["FS"],
                               D=c["D"], topk=c["topk"], out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < 5e-3
    ph = ep.phase_ms()
    assert ph["total"] > 0 and set(ph) == {"dispatch", "compute", "combine", "total"}
