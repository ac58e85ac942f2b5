"""Expert FFN, combine, RMSNorm and token-permutation restatements (CPU, test only).

Floating-point restatements use torch on the CPU in fp32 with the bf16 rounding points of
the reference orchestration; integer restatements use numpy.
"""

from __future__ import annotations

import numpy as np
import torch

bf16 = torch.bfloat16


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, weight_bias: float = 0.0) -> torch.Tensor:
    """bf16(x * rsqrt(mean(x^2) + eps) * (w + weight_bias)) with an fp32 reduction.

    Restates the RMSNorm arithmetic the reference's CuTe kernel keeps from FlashInfer
    (src/tideway/cute_router_norm_pair.py:252-260, routed output at :300-306).
    """
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * rstd * (w.float() + weight_bias)).to(bf16)


def router_norm_pair(x, ones, routed_weight, scale, eps: float, root: float):
    """Two RMSNorm outputs sharing one reduction, with the router's bf16 cast chain.

    Restates ``RouterNormPairKernel`` (src/tideway/cute_router_norm_pair.py:252-312):
    router = bf16(bf16(bf16(x*rstd*ones) * scale) * root); routed = bf16(x*rstd*w).
    """
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    h0 = (xf * rstd * ones.float()).to(bf16).float()
    h1 = (h0 * scale.float()).to(bf16).float()
    router = (h1 * root).to(bf16)
    routed = (xf * rstd * routed_weight.float()).to(bf16)
    return router, routed


def dual_norm_merge(a, b, x, w1, w2, w3, eps1, eps2, eps3, scalar):
    """Shared/routed post-FFN merge (the reference calls FreeToken's
    gemma_dual_rmsnorm_residual_scalar, src/tideway/overlap_shared_expert.py:265-276, which is
    absent, with the layer's residual and ``layer_scalar``): bf16(bf16(x + N3(bf16(N1(a) +
    N2(b)))) * scalar) -- the Gemma 4 decoder layer's order (transformers 5.5
    Gemma4TextDecoderLayer.forward: post-FFN norms of the dense and expert branches, their
    sum, the post-feedforward norm, the residual add, then ``*= layer_scalar``)."""
    m = (rmsnorm(a, w1, eps1).float() + rmsnorm(b, w2, eps2).float()).to(bf16)
    h = (x.float() + rmsnorm(m, w3, eps3).float()).to(bf16)
    return (h.float() * scalar).to(bf16)


def gate_activation(g: torch.Tensor, activation: str) -> torch.Tensor:
    """The gate half's activation in fp32, by the names ``fused_experts_impl`` accepts
    (backends/.../moe/fused.py:343, :393-394, :428: silu, gelu, gelu_tanh).  The
    activation kernels themselves live in the absent FreeToken; these are the published
    forms: silu(g) = g / (1 + e^-g); gelu(g) = g/2 (1 + erf(g / sqrt 2)); gelu_tanh(g) =
    g/2 (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))) (Hendrycks and Gimpel, 2016)."""
    if activation == "silu":
        return g / (1.0 + torch.exp(-g))
    if activation == "gelu":
        return torch.nn.functional.gelu(g)
    if activation == "gelu_tanh":
        return torch.nn.functional.gelu(g, approximate="tanh")
    raise ValueError(f"Unsupported activation: {activation}")


def silu_mul(c1: torch.Tensor, activation: str = "silu") -> torch.Tensor:
    """bf16(act(gate) * up) with gate = first half (src/tideway/offload/geometry.py:197-203)."""
    I = c1.shape[-1] // 2
    g = c1[..., :I].float()
    u = c1[..., I:].float()
    return (gate_activation(g, activation) * u).to(bf16)


def expert_ffn_routes(x_rows: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                      route_w: torch.Tensor, activation: str = "silu",
                      weight_on_input: bool = False) -> torch.Tensor:
    """c3 for a batch of routes that share one expert: [n, H] -> [n, H] bf16.

    c1 = bf16(x . w1^T); c2 = bf16(act(c1_gate) * c1_up); c3 = bf16((c2 . w2^T) * w).
    Rounding points of ``fused_experts_decode_impl`` (backends/.../moe/fused.py:406-446):
    cache1/cache2/cache3 are bf16 tensors, the router weight is applied on the second GEMM
    (``not apply_router_weight_on_input``, :442) -- or, with ``weight_on_input``, on the
    first GEMM's fp32 accumulator before its bf16 rounding (the first kernel's
    ``apply_router_weight_on_input`` flag, :410-420), and not on the second.
    """
    wcol = route_w.float().unsqueeze(-1)
    acc1 = x_rows.float() @ w1.float().t()
    c1 = (acc1 * wcol if weight_on_input else acc1).to(bf16)
    c2 = silu_mul(c1, activation)
    acc2 = c2.float() @ w2.float().t()
    return (acc2 if weight_on_input else acc2 * wcol).to(bf16)


def moe_decode(x: torch.Tensor, w1_bank: torch.Tensor, w2_bank: torch.Tensor,
               topk_w: torch.Tensor, topk_ids: torch.Tensor, activation: str = "silu",
               weight_on_input: bool = False) -> torch.Tensor:
    """Slot-indirect decode FFN plus combine: out[t] = bf16(sum_k c3[t, k]).

    Restates ``fused_experts_decode_impl`` (backends/.../moe/fused.py:367-450) with
    ``moe_sum_reduce`` (:448-449) as an fp32 sum over k in index order.  ``topk_ids``
    index the bank's first dimension (slot ids in decode, expert ids in prefill).
    Routes with a negative id contribute nothing.
    """
    T, K = topk_ids.shape
    H = x.shape[1]
    c3 = torch.zeros(T, K, H, dtype=bf16)
    ids = topk_ids.to(torch.int64)
    for s in torch.unique(ids[ids >= 0]).tolist():
        t_idx, k_idx = torch.nonzero(ids == s, as_tuple=True)
        c3[t_idx, k_idx] = expert_ffn_routes(x[t_idx], w1_bank[s], w2_bank[s],
                                             topk_w[t_idx, k_idx], activation, weight_on_input)
    return c3.float().sum(dim=1).to(bf16)


def moe_prefill(x: torch.Tensor, w1_bank: torch.Tensor, w2_bank: torch.Tensor,
                topk_w: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """Prefill grouped FFN; same arithmetic as decode (backends/.../moe/fused.py:261-364).

    The reference writes the result into ``hidden_states`` (fused.py:270-273, :312); the
    product path keeps that contract, the oracle returns a fresh tensor.
    """
    return moe_decode(x, w1_bank, w2_bank, topk_w, topk_ids)


def shared_expert(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """Always-active dense SwiGLU expert, same rounding points as a routed one with w = 1."""
    return expert_ffn_routes(x, w1, w2, torch.ones(x.shape[0]))


def moe_align_block_size(topk_ids: np.ndarray, block_size: int, num_experts: int
                         ) -> tuple[np.ndarray, np.ndarray, int]:
    """Stable by-expert permutation of the flattened routes, each expert padded to a block.

    Restates ``moe_align_block_size`` (backends/.../moe/fused.py:88-158, worked example at
    :113-126): routes are flattened in (token, k) order, grouped by expert id ascending
    keeping their flat order, each group padded to a multiple of ``block_size`` with the
    sentinel ``numel``; experts with no route get no block.  Returns
    (sorted_ids, expert_of_block, num_tokens_post_padded).
    """
    flat = np.asarray(topk_ids, np.int64).reshape(-1)
    numel = flat.size
    sorted_ids: list[int] = []
    block_expert: list[int] = []
    for e in range(num_experts):
        rows = np.flatnonzero(flat == e).tolist()
        if not rows:
            continue
        pad = (-len(rows)) % block_size
        rows += [numel] * pad
        sorted_ids += rows
        block_expert += [e] * (len(rows) // block_size)
    return (np.asarray(sorted_ids, np.int32), np.asarray(block_expert, np.int32),
            len(sorted_ids))
