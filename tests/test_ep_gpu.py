"""Expert parallelism on GPUs: one GPU and, with 2+ GPUs, one process per GPU.

Both transports -- NVLink peer stores from our own kernels ("p2p") and NCCL all-to-alls
("nccl") -- against the oracle (the single-process expert FFN over all experts) and against
each other bit for bit, with the p2p combine also forming the next residual RMSNorm
(bit-identical to the all-to-all combine followed by tw_rmsnorm).  Failures of the
multi-process case are host-side only: every wait in the exchange kernels is bounded.
"""

import datetime
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
    resid = torch.randn(T, H, generator=gt).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(H, generator=gt)).to(torch.bfloat16)
    return w1, w2, x, ids, w, resid, norm_w


def _run_rank(rank: int, world: int, dev: int) -> dict:
    """Both transports on this rank; returns the errors and bit-equalities to report."""
    import tideway_b200 as tw
    from tideway_b200 import ops
    from tideway_b200.ep import ExpertParallelMoE

    w1, w2, x, ids, w, resid, norm_w = _inputs(rank)
    d = f"cuda:{dev}"
    Eg = E // world
    lo, hi = rank * Eg, (rank + 1) * Eg
    outs = {}
    for transport in ("nccl", "p2p"):
        cache = tw.OffloadMoeCache(num_layers=1, num_experts=Eg, cache_size=Eg, device=d)
        cache.set_bank_sources({"gate_up": [w1[lo:hi].contiguous().pin_memory()],
                                "down": [w2[lo:hi].contiguous().pin_memory()]})
        ep = ExpertParallelMoE(E, K, H, I, T, device=d, transport=transport)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=d)
        for _ in range(3):  # later calls run with every local expert resident; flags step on
            ep.forward(x.to(d), w.to(d), ids.to(d), 0, cache, out)
        torch.cuda.synchronize(dev)
        outs[transport] = out.cpu()
        if transport == "p2p":
            r_out = resid.to(d).clone()
            h = torch.empty(T, H, dtype=torch.bfloat16, device=d)
            ep.forward(x.to(d), w.to(d), ids.to(d), 0, cache, None, residual=r_out,
                       residual_out=r_out, norm_w=norm_w.to(d), eps=1e-6, h_out=h)
            want_h = ops.rmsnorm(outs["nccl"].to(d), norm_w.to(d), 1e-6,
                                 residual=resid.to(d), residual_out=(want_r := torch.empty_like(h)))
            torch.cuda.synchronize(dev)
            outs["norm_equal"] = torch.equal(h, want_h) and torch.equal(r_out, want_r)
            outs["error_word"] = ep.error()
            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            ep.close()
    ref = off.moe_decode(x, w1, w2, w, ids)
    rel = lambda a: float((a.float() - ref.float()).abs().max() / ref.float().abs().max())
    return {"nccl": rel(outs["nccl"]), "p2p": rel(outs["p2p"]),
            "same": torch.equal(outs["nccl"], outs["p2p"]), "norm_equal": outs["norm_equal"],
            "error_word": outs["error_word"]}


def _check(r: dict) -> None:
    assert r["nccl"] <= 2e-2 and r["p2p"] <= 2e-2, r
    assert r["same"] and r["norm_equal"] and r["error_word"] == 0, r


def test_expert_parallel_one_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _check(_run_rank(0, 1, 0))


def _worker(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        q.put((rank, _run_rank(rank, world, rank)))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus():
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
    for _ in range(2):
        _check(q.get(timeout=5)[1])
