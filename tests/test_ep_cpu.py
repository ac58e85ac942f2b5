"""Expert-parallel dataflow on two and four CPU ranks (gloo) against the single-process expert
FFN."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep as oep
from oracle import ffn as off

H, I, E, K, T = 256, 128, 8, 2, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(rank: int):
    g = torch.Generator().manual_seed(123)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    gt = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=gt).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=gt)[:K] for _ in range(T)]).to(torch.int32)
    ids[1, 1] = -1  # a padded route
    w = torch.rand(T, K, generator=gt)
    w = (w / w.sum(-1, keepdim=True)).float()
    return w1, w2, x, ids, w


def _rank(rank: int, world: int, port: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w1, w2, x, ids, w = _inputs(rank)
        Eg = E // world
        out = oep.expert_parallel_decode(
            x, w, ids, w1[rank * Eg:(rank + 1) * Eg], w2[rank * Eg:(rank + 1) * Eg], rank, world,
            lambda o, i: dist.all_to_all_single(o, i))
        ref = off.moe_decode(x, w1, w2, w, ids)
        err = float((out.float() - ref.float()).abs().max() / ref.float().abs().max())
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_cpu_ranks_match_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=5) for _ in range(world))
    # partial sums are rounded to bf16 per GPU before the cross-GPU sum
    assert max(errs.values()) <= 2e-2, errs


def test_expert_parallel_single_rank_is_exact():
    w1, w2, x, ids, w = _inputs(0)
    out = oep.expert_parallel_decode(x, w, ids, w1, w2, 0, 1, lambda o, i: o.copy_(i))
    assert torch.equal(out, off.moe_decode(x, w1, w2, w, ids))
