"""Expert-parallel dispatch/combine restatement (CPU, test infrastructure only).

The reference has no multi-GPU MoE path (src/tideway/offload/paged_decode_graph.py:62-63);
this restates the expert-parallel dataflow the build defines, so that it can be checked on
CPU ranks (gloo) against the single-process expert FFN: experts [d*Eg, (d+1)*Eg) live on
rank d; each rank sends, per destination and token, the token's row and the routes the
destination owns; the owner computes one partial sum per received row (routes in k order);
the source adds the partials in rank order.
"""

from __future__ import annotations

import torch

from . import ffn as off


def expert_parallel_decode(x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                           w1_local: torch.Tensor, w2_local: torch.Tensor, rank: int,
                           world: int, all_to_all) -> torch.Tensor:
    """``all_to_all(out, inp)`` exchanges equal dim-0 chunks (rank d's chunk goes to rank d)."""
    T, H = x.shape
    K = topk_ids.shape[1]
    Eg = w1_local.shape[0]
    ids = topk_ids.to(torch.int64)
    send_x = torch.zeros(world, T, H, dtype=torch.bfloat16)
    send_ids = torch.full((world, T, K), -1, dtype=torch.int64)
    send_w = torch.zeros(world, T, K)
    for d in range(world):
        mine = (ids >= 0) & (ids // Eg == d)
        send_ids[d] = torch.where(mine, ids % Eg, torch.full_like(ids, -1))
        send_w[d] = topk_w
        send_x[d] = x
    recv_x, recv_ids, recv_w = (torch.empty_like(send_x), torch.empty_like(send_ids),
                                torch.empty_like(send_w))
    all_to_all(recv_x, send_x)
    all_to_all(recv_ids, send_ids)
    all_to_all(recv_w, send_w)
    part = off.moe_decode(recv_x.view(world * T, H), w1_local, w2_local,
                          recv_w.view(world * T, K), recv_ids.view(world * T, K).to(torch.int32))
    back = torch.empty(world, T, H, dtype=torch.bfloat16)
    all_to_all(back, part.view(world, T, H))
    return back.float().sum(dim=0).to(torch.bfloat16)
