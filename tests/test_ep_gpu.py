"""Expert parallelism on GPUs: one GPU (local all-to-all) and, with 2+ GPUs, NCCL ranks."""

import os
import socket

import pytest
import torch

from oracle import ffn as off

pytestmark = pytest.mark.gpu

H, I, E, K, T = 1024, 512, 16, 4, 8


def _inputs(rank: int):
    g = torch.Generator().manual_seed(321)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    gt = torch.Generator().manual_seed(2000 + rank)
    x = torch.randn(T, H, generator=gt).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=gt)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, K, generator=gt)
    w = (w / w.sum(-1, keepdim=True)).float()
    return w1, w2, x, ids, w


def _run_rank(rank: int, world: int, dev: int):
    """Expert-parallel layer on this rank; returns (gpu out, oracle out) on the CPU."""
    import tideway_b200 as tw
    from tideway_b200.ep import ExpertParallelMoE

    w1, w2, x, ids, w = _inputs(rank)
    Eg = E // world
    lo, hi = rank * Eg, (rank + 1) * Eg
    cache = tw.OffloadMoeCache(num_layers=1, num_experts=Eg, cache_size=Eg, device=f"cuda:{dev}")
    cache.set_bank_sources({"gate_up": [w1[lo:hi].contiguous().pin_memory()],
                            "down": [w2[lo:hi].contiguous().pin_memory()]})
    ep = ExpertParallelMoE(E, K, H, I, T, device=f"cuda:{dev}")
    out = torch.empty(T, H, dtype=torch.bfloat16, device=f"cuda:{dev}")
    for _ in range(2):  # the second call runs with every local expert already resident
        ep.forward(x.cuda(dev), w.cuda(dev), ids.cuda(dev), 0, cache, out)
    torch.cuda.synchronize(dev)
    return out.cpu(), off.moe_decode(x, w1, w2, w, ids)


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


def test_expert_parallel_one_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    out, ref = _run_rank(0, 1, 0)
    assert _rel(out, ref) <= 2e-2


def _worker(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        out, ref = _run_rank(rank, world, rank)
        q.put((rank, _rel(out, ref)))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) <= 2e-2, errs
