"""Router top-k restatements (CPU, test infrastructure only).

Each function cites the reference routine whose arithmetic it restates.
"""

from __future__ import annotations

import numpy as np
import torch


def _stable_topk_desc(values: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k along the last dim, descending, ties broken toward the lower index."""
    order = torch.sort(values, dim=-1, descending=True, stable=True).indices[..., :k]
    return torch.gather(values, -1, order), order


def softmax_topk(
    logits: torch.Tensor,
    topk: int,
    renormalize: bool,
    num_token_non_padded: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax router: fp32 softmax over all experts, top-k, optional renormalisation.

    Restates ``_torch_fused_topk`` (backends/freetoken_tideway/freetoken/moe/fused.py:16-35),
    the path ``fused_topk`` takes when ``triton_kernels`` is absent (fused.py:51-63).
    Ties are broken toward the lower expert id.  Rows at or past
    ``num_token_non_padded`` get id -1 (fused.py:32-34).
    """
    probs = torch.softmax(logits.float(), dim=-1)
    w, ids = _stable_topk_desc(probs, topk)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    ids = ids.to(torch.int32)
    if num_token_non_padded is not None:
        ids[num_token_non_padded:, :] = -1
    return w.contiguous(), ids.contiguous()


def gemma_topk(
    logits: torch.Tensor, per_expert_scale: torch.Tensor, topk: int
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gemma routing: top-k logits (ties -> lower id), softmax over those k, x scale[id].

    Restates ``_routing_with_copy`` (src/tideway/gemma_route_copy_kernel.py:28-70): the
    packed-key sort orders by logit descending and then by id ascending (:47-54); the
    softmax runs over the selected logits only (:58-62); each weight is multiplied by
    ``per_expert_scale[id]`` (:63-66); the ids are written twice (:69-70).
    """
    lf = logits.float()
    top, ids = _stable_topk_desc(lf, topk)
    m = top.max(dim=-1, keepdim=True).values
    e = torch.exp(top - m)
    d = e.sum(dim=-1, keepdim=True)
    w = e / torch.where(d > 0, d, torch.ones_like(d))
    w = w * per_expert_scale.float()[ids]
    ids = ids.to(torch.int32)
    return w.contiguous(), ids.contiguous(), ids.clone()


def sigmoid_group_topk(
    logits: torch.Tensor,
    topk: int,
    n_group: int,
    topk_group: int,
    routed_scaling_factor: float,
    renormalize: bool = True,
    bias: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """DeepSeek-style sigmoid scoring with group-limited top-k (parity unpinned).

    The reference consumes this gate's output (src/tideway/offload/ffn_front_graph.py:24-30,
    contract at :331-336) but its code lives in the absent FreeToken model.  This restates
    the published DeepSeek-V3 routing: s = sigmoid(logit); choice = s + bias; a group's
    score is the sum of its two best choice scores; keep the ``topk_group`` best groups;
    pick the ``topk`` best experts of the kept groups; weight = s (without bias),
    renormalised over the k picks, times ``routed_scaling_factor``.  Ties go to the lower
    index at every selection.
    """
    T, E = logits.shape
    s = torch.sigmoid(logits.float())
    choice = s if bias is None else s + bias.float()
    g = choice.view(T, n_group, E // n_group)
    top2 = _stable_topk_desc(g, 2)[0].sum(dim=-1)
    _, gidx = _stable_topk_desc(top2, topk_group)
    gmask = torch.zeros(T, n_group, dtype=torch.bool)
    gmask.scatter_(1, gidx, True)
    emask = gmask.unsqueeze(-1).expand(T, n_group, E // n_group).reshape(T, E)
    masked = torch.where(emask, choice, torch.full_like(choice, float("-inf")))
    _, ids = _stable_topk_desc(masked, topk)
    w = torch.gather(s, 1, ids)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    w = w * routed_scaling_factor
    return w.contiguous(), ids.to(torch.int32).contiguous()


def topk_margin(logits: torch.Tensor, topk: int) -> np.ndarray:
    """Per-token gap between the k-th and (k+1)-th largest logit (near-tie diagnostics)."""
    v = torch.sort(logits.float(), dim=-1, descending=True).values
    return (v[:, topk - 1] - v[:, topk]).numpy()
