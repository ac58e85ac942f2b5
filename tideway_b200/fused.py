"""Drop-in replacements for the reference's fused-MoE entry points.

Same names, argument meaning, asserts and return contracts as
backends/freetoken_tideway/freetoken/moe/fused.py; the arithmetic runs in the
tideway_b200 CUDA library (sm_100a).  There is no CPU path.
"""

from __future__ import annotations

import torch

from . import ops

# The routes one FFN launch handles (the library's per-launch limit); larger prefill
# chunks are processed in slices of whole tokens.
_MAX_ROUTES = 65535


def fused_topk(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int,
               renormalize: bool, num_token_non_padded: torch.Tensor | None = None):
    """Softmax router: (topk_weights fp32 [T, K], topk_ids int32 [T, K]).

    Mirrors fused_topk / _torch_fused_topk (fused.py:16-85): fp32 softmax over all
    experts, top-k, optional renormalisation, rows >= num_token_non_padded get id -1.
    Exactly tied probabilities are ordered by ascending expert id.
    """
    assert hidden_states.shape[0] == gating_output.shape[0], "Number of tokens mismatch"
    logits = gating_output
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.float()
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return ops.softmax_topk(logits, topk, renormalize, num_token_non_padded)


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int):
    """(sorted_token_ids, expert_ids, num_tokens_post_padded); see fused.py:88-158."""
    return ops.moe_align_block_size(topk_ids, block_size, num_experts)


def _check(hidden_states, w1, w2, topk_weights, topk_ids, activation):
    assert hidden_states.shape[1] == w1.shape[2], "Hidden size mismatch"
    assert w1.shape[0] == w2.shape[0], "Expert cache size mismatch"
    assert w1.shape[1] == 2 * w2.shape[2], "Intermediate size mismatch"
    assert w2.shape[1] == hidden_states.shape[1], "Output hidden size mismatch"
    assert topk_weights.shape == topk_ids.shape, "topk shape mismatch"
    assert hidden_states.is_contiguous(), "Hidden_states must be contiguous"
    assert w1.is_contiguous(), "Expert weights1 must be contiguous"
    assert w2.is_contiguous(), "Expert weights2 must be contiguous"
    assert topk_weights.is_contiguous(), "topk_weights must be contiguous"
    assert topk_ids.is_contiguous(), "topk_ids must be contiguous"
    assert hidden_states.dtype == torch.bfloat16, "the B200 path computes bf16 activations"
    assert w1.dtype == hidden_states.dtype and w2.dtype == hidden_states.dtype
    assert topk_weights.dtype == torch.float32
    assert topk_ids.dtype == torch.int32
    if activation not in ops.ACTIVATIONS:
        raise ValueError(f"Unsupported activation: {activation}")


def _ffn_sliced(x, w1, w2, topk_weights, topk_ids, out, activation="silu", w_in=False):
    T, K = topk_ids.shape
    step = max(1, _MAX_ROUTES // K)
    for t0 in range(0, T, step):
        t1 = min(T, t0 + step)
        ops.moe_ffn_bf16(x[t0:t1], w1, w2, topk_weights[t0:t1], topk_ids[t0:t1],
                         out=out[t0:t1], activation=activation, weight_on_input=w_in)
    return out


def fused_experts_decode_impl(hidden_states, w1, w2, topk_weights, topk_ids,
                              activation: str = "silu",
                              apply_router_weight_on_input: bool = False) -> torch.Tensor:
    """Decode expert FFN over a slot bank; allocates its output (fused.py:367-450).

    ``topk_ids`` index the bank's first dimension (slot ids).  The router weight is
    applied on the down projection, or with ``apply_router_weight_on_input`` on the up
    projection (before its bf16 rounding) and not on the down projection.
    """
    _check(hidden_states, w1, w2, topk_weights, topk_ids, activation)
    out = torch.empty_like(hidden_states)
    return _ffn_sliced(hidden_states, w1, w2, topk_weights, topk_ids, out, activation,
                       apply_router_weight_on_input)


def fused_experts_impl(hidden_states, w1, w2, topk_weights, topk_ids, activation: str = "silu",
                       apply_router_weight_on_input: bool = False) -> torch.Tensor:
    """Prefill expert FFN; returns ``hidden_states`` overwritten with the routed output
    (fused.py:261-364).  Read the input before the call if it is still needed."""
    _check(hidden_states, w1, w2, topk_weights, topk_ids, activation)
    T, K = topk_ids.shape
    w_in = apply_router_weight_on_input
    if T * K <= _MAX_ROUTES:
        return ops.moe_ffn_bf16(hidden_states, w1, w2, topk_weights, topk_ids, out=hidden_states,
                                activation=activation, weight_on_input=w_in)
    # slices read the input before their outputs land, so stage the input once
    x = hidden_states.clone()
    return _ffn_sliced(x, w1, w2, topk_weights, topk_ids, hidden_states, activation, w_in)


class FusedMoe:
    """Backend object with the reference's ``forward`` signature (fused.py:453-479)."""

    def forward(self, hidden_states, w1, w2, gating_output, topk: int, renormalize: bool,
                activation: str = "silu", apply_router_weight_on_input: bool = False):
        topk_weights, topk_ids = fused_topk(hidden_states, gating_output, topk, renormalize)
        return fused_experts_impl(hidden_states, w1, w2, topk_weights, topk_ids, activation,
                                  apply_router_weight_on_input)
