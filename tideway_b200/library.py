"""The hot-path entry points as ``torch.library`` custom ops (namespace ``tideway_b200``).

``torch.ops.tideway_b200.<name>`` runs the same CUDA kernels as ``tideway_b200.ops``; each
op declares its schema (which arguments it mutates) and a fake implementation giving its
output shapes, so the ops can sit inside ``torch.compile`` graphs (fullgraph, no graph
breaks) and be traced by ``torch.export``.  Functional ops allocate their outputs; the slot
table updates mutate the table tensors and rewrite the routed ids in place, as the
reference's ``ensure_experts`` does (backends/.../moe/offload_cache.py:851-864).

This module registers the ops when imported (``import tideway_b200`` does so).
"""

from typing import Optional

import torch

from . import ops

_NS = "tideway_b200"


def _op(name: str, mutates_args=()):
    return torch.library.custom_op(f"{_NS}::{name}", mutates_args=mutates_args,
                                   device_types="cuda")


# ---------------------------------------------------------------- routing

@_op("fused_topk")
def fused_topk(gating_output: torch.Tensor, topk: int,
               renormalize: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax router (``fused_topk``, backends/.../moe/fused.py:38-85)."""
    logits = gating_output if gating_output.dtype in (torch.float32, torch.bfloat16) \
        else gating_output.float()
    return ops.softmax_topk(logits.contiguous(), topk, renormalize)


@fused_topk.register_fake
def _(gating_output, topk, renormalize):
    T = gating_output.shape[0]
    return (gating_output.new_empty(T, topk, dtype=torch.float32),
            gating_output.new_empty(T, topk, dtype=torch.int32))


@_op("gemma_topk")
def gemma_topk(logits: torch.Tensor, per_expert_scale: torch.Tensor,
               topk: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gemma routing (src/tideway/gemma_route_copy_kernel.py:28-102): weights, ids, ids."""
    return ops.gemma_topk(logits.contiguous(), per_expert_scale, topk)


@gemma_topk.register_fake
def _(logits, per_expert_scale, topk):
    T = logits.shape[0]
    return (logits.new_empty(T, topk, dtype=torch.float32),
            logits.new_empty(T, topk, dtype=torch.int32),
            logits.new_empty(T, topk, dtype=torch.int32))


@_op("sigmoid_group_topk")
def sigmoid_group_topk(logits: torch.Tensor, topk: int, n_group: int, topk_group: int,
                       routed_scaling_factor: float, renormalize: bool,
                       bias: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor]:
    """DeepSeek-style sigmoid scoring with group-limited top-k."""
    return ops.sigmoid_group_topk(logits.contiguous(), topk, n_group, topk_group,
                                  routed_scaling_factor, renormalize, bias=bias)


@sigmoid_group_topk.register_fake
def _(logits, topk, n_group, topk_group, routed_scaling_factor, renormalize, bias):
    T = logits.shape[0]
    return (logits.new_empty(T, topk, dtype=torch.float32),
            logits.new_empty(T, topk, dtype=torch.int32))


@_op("router_logits")
def router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """fp32 logits [T, E] = x . w^T (bf16 inputs)."""
    return ops.router_logits(x, w)


@router_logits.register_fake
def _(x, w):
    return x.new_empty(x.shape[0], w.shape[0], dtype=torch.float32)


# ---------------------------------------------------------------- norms and merges

@_op("rmsnorm")
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, weight_bias: float) -> torch.Tensor:
    return ops.rmsnorm(x.contiguous(), w, eps, weight_bias)


@rmsnorm.register_fake
def _(x, w, eps, weight_bias):
    return torch.empty_like(x)


@_op("router_norm_pair")
def router_norm_pair(x: torch.Tensor, ones: torch.Tensor, routed_weight: torch.Tensor,
                     scale: torch.Tensor, eps: float,
                     root: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(router input, routed input) from one RMSNorm reduction
    (src/tideway/cute_router_norm_pair.py:252-312)."""
    return ops.router_norm_pair(x.contiguous(), ones, routed_weight, scale, eps, root)


@router_norm_pair.register_fake
def _(x, ones, routed_weight, scale, eps, root):
    return torch.empty_like(x), torch.empty_like(x)


@_op("router_norm_triple")
def router_norm_triple(x: torch.Tensor, ones: torch.Tensor, routed_weight: torch.Tensor,
                       scale: torch.Tensor, shared_weight: torch.Tensor, eps: float,
                       root: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The router pair plus the shared expert's pre-norm, from one reduction."""
    return ops.router_norm_triple(x.contiguous(), ones, routed_weight, scale, shared_weight,
                                  eps, root)


@router_norm_triple.register_fake
def _(x, ones, routed_weight, scale, shared_weight, eps, root):
    return torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)


@_op("dual_norm_merge")
def dual_norm_merge(a: torch.Tensor, b: torch.Tensor, x: torch.Tensor, w1: torch.Tensor,
                    w2: torch.Tensor, w3: torch.Tensor, eps1: float, eps2: float, eps3: float,
                    scalar: float) -> torch.Tensor:
    """bf16(bf16(x + N3(bf16(N1(a) + N2(b)))) * scalar) (src/tideway/overlap_shared_expert.py)."""
    return ops.dual_norm_merge(a, b, x, w1, w2, w3, eps1, eps2, eps3, scalar)


@dual_norm_merge.register_fake
def _(a, b, x, w1, w2, w3, eps1, eps2, eps3, scalar):
    return torch.empty_like(x)


@_op("add_shared")
def add_shared(routed: torch.Tensor, shared: torch.Tensor) -> torch.Tensor:
    return ops.add_shared(routed, shared)


@add_shared.register_fake
def _(routed, shared):
    return torch.empty_like(routed)


# ---------------------------------------------------------------- slot table

@_op("lru_ensure", mutates_args=("ids", "slot_for_id", "id_of_slot", "usage", "step",
                                 "evict_slots", "src_indices", "num_indices"))
def lru_ensure(ids: torch.Tensor, slot_for_id: torch.Tensor, id_of_slot: torch.Tensor,
               usage: torch.Tensor, step: torch.Tensor, num_experts: int, layer_id: int,
               evict_slots: torch.Tensor, src_indices: torch.Tensor,
               num_indices: torch.Tensor) -> None:
    """``ensure_experts``: rewrite ``ids`` into slot ids in place and stage the misses."""
    ops.lru_ensure(ids, slot_for_id, id_of_slot, usage, step, num_experts, layer_id,
                   evict_slots, src_indices, num_indices)


@lru_ensure.register_fake
def _(ids, slot_for_id, id_of_slot, usage, step, num_experts, layer_id, evict_slots,
      src_indices, num_indices):
    return None


@_op("hybrid_ensure", mutates_args=("ids", "slot_for_id", "id_of_slot", "usage", "step",
                                    "active_mask", "evict_slots", "src_indices",
                                    "num_indices", "num_missing_full", "recency"))
def hybrid_ensure(ids: torch.Tensor, slot_for_id: torch.Tensor, id_of_slot: torch.Tensor,
                  usage: torch.Tensor, step: torch.Tensor, num_experts: int, layer_id: int,
                  active_mask: torch.Tensor, evict_slots: torch.Tensor,
                  src_indices: torch.Tensor, num_indices: torch.Tensor,
                  num_missing_full: torch.Tensor, recency: Optional[torch.Tensor],
                  max_fetch: int, fetch_frac_q16: int) -> None:
    """``ensure_experts_hybrid``: capped-fetch LRU (misses beyond the cap become -1)."""
    ops.hybrid_ensure(ids, slot_for_id, id_of_slot, usage, step, num_experts, layer_id,
                      active_mask, evict_slots, src_indices, num_indices, num_missing_full,
                      recency, max_fetch, fetch_frac_q16)


@hybrid_ensure.register_fake
def _(ids, slot_for_id, id_of_slot, usage, step, num_experts, layer_id, active_mask,
      evict_slots, src_indices, num_indices, num_missing_full, recency, max_fetch,
      fetch_frac_q16):
    return None


@_op("materialize_layer", mutates_args=("slot_for_id", "id_of_slot", "usage", "step",
                                        "evict_slots", "src_indices", "num_indices"))
def materialize_layer(slot_for_id: torch.Tensor, id_of_slot: torch.Tensor, usage: torch.Tensor,
                      step: torch.Tensor, num_experts: int, layer_id: int,
                      evict_slots: torch.Tensor, src_indices: torch.Tensor,
                      num_indices: torch.Tensor) -> None:
    """Make every expert of one layer resident (``materialize_layer``)."""
    ops.materialize_layer(slot_for_id, id_of_slot, usage, step, num_experts, layer_id,
                          evict_slots, src_indices, num_indices)


@materialize_layer.register_fake
def _(slot_for_id, id_of_slot, usage, step, num_experts, layer_id, evict_slots, src_indices,
      num_indices):
    return None


@_op("reset_slots", mutates_args=("slot_for_id", "id_of_slot", "usage", "step",
                                  "num_indices"))
def reset_slots(slot_for_id: torch.Tensor, id_of_slot: torch.Tensor, usage: torch.Tensor,
                step: torch.Tensor, num_indices: torch.Tensor) -> None:
    """Empty the slot table (``reset``)."""
    ops.reset_slots(slot_for_id, id_of_slot, usage, step, num_indices)


@reset_slots.register_fake
def _(slot_for_id, id_of_slot, usage, step, num_indices):
    return None


# ---------------------------------------------------------------- expert FFN

@_op("moe_ffn_bf16")
def moe_ffn_bf16(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                 topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """Slot-indirect SwiGLU expert FFN + combine over BF16 banks
    (``fused_experts_decode_impl``, backends/.../moe/fused.py:367-450)."""
    return ops.moe_ffn_bf16(x, w1, w2, topk_weights, topk_ids)


@moe_ffn_bf16.register_fake
def _(x, w1, w2, topk_weights, topk_ids):
    return torch.empty_like(x)


@_op("moe_ffn_bf16_residual_norm")
def moe_ffn_bf16_residual_norm(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                               topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                               residual: torch.Tensor, norm_w: torch.Tensor,
                               eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """The FFN with its combine fused into the next residual RMSNorm:
    (residual_out = bf16(y + residual), h = rmsnorm(residual_out))."""
    residual_out, h = torch.empty_like(residual), torch.empty_like(residual)
    ops.moe_ffn_bf16_residual_norm(x, w1, w2, topk_weights, topk_ids, residual, residual_out,
                                   norm_w, eps, h)
    return residual_out, h


@moe_ffn_bf16_residual_norm.register_fake
def _(x, w1, w2, topk_weights, topk_ids, residual, norm_w, eps):
    return torch.empty_like(residual), torch.empty_like(residual)


@_op("moe_ffn_bf16_dual_merge")
def moe_ffn_bf16_dual_merge(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                            topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                            shared: torch.Tensor, residual: torch.Tensor, w1n: torch.Tensor,
                            w2n: torch.Tensor, w3n: torch.Tensor, eps1: float, eps2: float,
                            eps3: float, scalar: float) -> torch.Tensor:
    """The FFN with its combine fused into the Gemma shared/routed dual-norm merge."""
    return ops.moe_ffn_bf16_dual_merge(x, w1, w2, topk_weights, topk_ids, shared, residual,
                                       w1n, w2n, w3n, eps1, eps2, eps3, scalar)


@moe_ffn_bf16_dual_merge.register_fake
def _(x, w1, w2, topk_weights, topk_ids, shared, residual, w1n, w2n, w3n, eps1, eps2, eps3,
      scalar):
    return torch.empty_like(residual)


@_op("moe_ffn_nvfp4")
def moe_ffn_nvfp4(x: torch.Tensor, w1_packed: torch.Tensor, w1_scale: torch.Tensor,
                  w1_global: torch.Tensor, w2_packed: torch.Tensor, w2_scale: torch.Tensor,
                  w2_global: torch.Tensor, topk_weights: torch.Tensor,
                  topk_ids: torch.Tensor) -> torch.Tensor:
    """The same FFN over NVFP4 banks (e2m1 codes, e4m3 scales per 16, fp32 row scale)."""
    return ops.moe_ffn_nvfp4(x, (w1_packed, w1_scale, w1_global),
                             (w2_packed, w2_scale, w2_global), topk_weights, topk_ids)


@moe_ffn_nvfp4.register_fake
def _(x, w1_packed, w1_scale, w1_global, w2_packed, w2_scale, w2_global, topk_weights,
      topk_ids):
    return torch.empty_like(x)


@_op("ffn_dense_bf16")
def ffn_dense_bf16(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """Dense SwiGLU FFN of one expert over every row (the shared expert)."""
    return ops.ffn_dense_bf16(x, w1, w2)


@ffn_dense_bf16.register_fake
def _(x, w1, w2):
    return torch.empty_like(x)


@_op("moe_align_block_size")
def moe_align_block_size(topk_ids: torch.Tensor, block_size: int,
                         num_experts: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(sorted_ids, expert_ids, num_tokens_post_padded) (backends/.../moe/fused.py:88-158)."""
    return ops.moe_align_block_size(topk_ids, block_size, num_experts)


@moe_align_block_size.register_fake
def _(topk_ids, block_size, num_experts):
    numel = topk_ids.numel()
    if numel < num_experts + 1:
        padded = numel * block_size
    else:
        padded = numel + (num_experts + 1) * (block_size - 1)
    padded = max(padded, 1)
    return (topk_ids.new_empty(padded, dtype=torch.int32),
            topk_ids.new_empty(-(-padded // block_size), dtype=torch.int32),
            topk_ids.new_empty(1, dtype=torch.int32))


@_op("nvfp4_dequantize")
def nvfp4_dequantize(packed: torch.Tensor, scale: torch.Tensor,
                     global_: torch.Tensor) -> torch.Tensor:
    return ops.nvfp4_dequantize(packed, scale, global_)


@nvfp4_dequantize.register_fake
def _(packed, scale, global_):
    return packed.new_empty(*packed.shape[:-1], 2 * packed.shape[-1], dtype=torch.float32)


OPS = ("fused_topk", "gemma_topk", "sigmoid_group_topk", "router_logits", "rmsnorm",
       "router_norm_pair", "router_norm_triple", "dual_norm_merge", "add_shared", "lru_ensure",
       "hybrid_ensure", "materialize_layer", "reset_slots", "moe_ffn_bf16",
       "moe_ffn_bf16_residual_norm", "moe_ffn_bf16_dual_merge", "moe_ffn_nvfp4",
       "ffn_dense_bf16", "moe_align_block_size", "nvfp4_dequantize")
