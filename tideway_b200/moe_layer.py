"""Offloaded MoE layer with the reference's operator signatures.

Mirrors ``OffloadMoELayer`` (backends/freetoken_tideway/freetoken/layers/moe.py:204-649):
``forward(hidden, router_logits)`` splits on the batch phase, ``routed_forward`` takes a
precomputed routing, decode rewrites ids into slot ids in place through the cache, and
``_expert_gemm`` dispatches on ``cache.quant_format`` (``bf16``, ``nvfp4``, and ``ds_fp4``
experts held as NVFP4 slot banks).  The phase comes from
``batch_context()`` (the reference reads ``get_global_ctx().batch.is_prefill``).
"""

from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass

import torch

from . import ops
from .fused import fused_experts_decode_impl, fused_experts_impl, fused_topk
from .offload_cache import OffloadMoeCache


@dataclass
class _Batch:
    is_prefill: bool = False


_ctx = threading.local()


def current_batch() -> _Batch:
    b = getattr(_ctx, "batch", None)
    if b is None:
        b = _ctx.batch = _Batch()
    return b


@contextlib.contextmanager
def batch_context(is_prefill: bool):
    prev = current_batch().is_prefill
    current_batch().is_prefill = is_prefill
    try:
        yield
    finally:
        current_batch().is_prefill = prev


class OffloadMoELayer:
    def __init__(self, layer_id: int, num_experts: int, top_k: int, hidden_size: int,
                 intermediate_size: int, renormalize: bool = True, activation: str = "silu",
                 apply_router_weight_on_input: bool = False, tp_group=None):
        if activation not in ops.ACTIVATIONS:
            raise ValueError(f"Unsupported activation: {activation}")
        self.layer_id = layer_id
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.activation = activation
        self.apply_router_weight_on_input = apply_router_weight_on_input
        # tensor parallelism: every rank of tp_group holds its slice of each expert's
        # intermediate dimension (its banks are [S, 2I/tp, H] and [S, H, I/tp]), and the
        # partial outputs are summed across the group
        self.tp_group = tp_group
        self.offload_cache: OffloadMoeCache | None = None

    @property
    def tp_size(self) -> int:
        if self.tp_group is None:
            return 1
        import torch.distributed as dist

        return dist.get_world_size(self.tp_group)

    def _maybe_all_reduce(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """Sum the partial outputs of a tensor-parallel group in place (NCCL on the GPUs),
        as the reference's layer does for tp_size > 1 (layers/moe.py:91-94)."""
        if self.tp_size > 1:
            import torch.distributed as dist

            dist.all_reduce(hidden_states, group=self.tp_group)
        return hidden_states

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor | None = None):
        if current_batch().is_prefill:
            out = self.prefill_forward(hidden_states, router_logits)
        else:
            out = self.decode_forward(hidden_states, router_logits)
        return self._maybe_all_reduce(out)

    __call__ = forward

    def routed_forward(self, hidden_states, topk_weights, topk_ids):
        """Expert compute for an external routing; ``topk_ids`` is rewritten in place."""
        if current_batch().is_prefill:
            out = self._prefill_routed(hidden_states, topk_weights, topk_ids)
        else:
            out = self._decode_routed(hidden_states, topk_weights, topk_ids)
        return self._maybe_all_reduce(out)

    def decode_forward(self, hidden_states, router_logits=None):
        w, ids = fused_topk(hidden_states, router_logits, self.top_k, self.renormalize)
        return self._decode_routed(hidden_states, w, ids)

    def prefill_forward(self, hidden_states, router_logits=None):
        w, ids = fused_topk(hidden_states, router_logits, self.top_k, self.renormalize)
        return self._prefill_routed(hidden_states, w, ids)

    def _decode_routed(self, hidden_states, topk_weights, topk_ids):
        cache = self.offload_cache
        assert cache is not None
        if cache.is_cpu_layer(self.layer_id):
            # the reference hands such layers to its host executor (layers/moe.py:313-316)
            raise NotImplementedError(f"layer {self.layer_id} is marked for whole-layer host "
                                      "decode (cpu_layer_ids), which is not on the B200 path")
        if cache.decode_target == "hybrid":
            return self._decode_hybrid(cache, hidden_states, topk_weights, topk_ids)
        cache.ensure_experts(self.layer_id, topk_ids)
        cache.copy_missing()
        return self._expert_gemm(cache, hidden_states, topk_weights, topk_ids,
                                 views=cache.bank_views(), n=None,
                                 alphas=cache.alphas_for_slots(self.layer_id), is_prefill=False)

    def _decode_hybrid(self, cache, hidden_states, topk_weights, topk_ids):
        """Hybrid decode (backends/.../layers/moe.py:331-378): the capped-fetch ensure gives
        each route its slot (hit or fetched) or -1; the caller's executor is handed the -1
        routes (raw ids, -1 elsewhere) before the fetch and the GPU FFN start, so both run
        at once; the GPU FFN skips the -1 routes itself (no clamped slot, no zeroed
        weight); the two partials add in the hidden dtype."""
        executor = cache.cpu_executor
        if executor is None:
            raise RuntimeError("decode_target='hybrid' needs cache.set_cpu_executor(...)")
        raw = topk_ids.clone()
        cache.ensure_experts_hybrid(self.layer_id, topk_ids)
        if cache.collect_stats:
            cache.record_decode_stats_hybrid(self.layer_id)
        cpu_ids = torch.where(topk_ids >= 0, torch.full_like(raw, -1), raw)
        pending = executor.decode_submit(self.layer_id, hidden_states, topk_weights, cpu_ids)
        cache.copy_missing()
        gpu_out = self._expert_gemm(cache, hidden_states, topk_weights, topk_ids,
                                    views=cache.bank_views(), n=None,
                                    alphas=cache.alphas_for_slots(self.layer_id),
                                    is_prefill=False)
        return gpu_out + executor.decode_sync(pending)

    def _prefill_routed(self, hidden_states, topk_weights, topk_ids):
        cache = self.offload_cache
        assert cache is not None
        if cache.prefill_overlap:
            if self.layer_id == 0:
                cache.begin_prefill()
            cache.prefetch_prefill_layer(self.layer_id)
            cache.prefetch_prefill_layer(self.layer_id + 1)
            views = cache.wait_prefill_layer(self.layer_id)
            out = self._expert_gemm(cache, hidden_states, topk_weights, topk_ids, views=views,
                                    n=self.num_experts,
                                    alphas=cache.alphas_for_layer(self.layer_id), is_prefill=True)
            cache.release_prefill_layer(self.layer_id)
            return out
        cache.materialize_layer(self.layer_id)
        cache.copy_missing()
        return self._expert_gemm(cache, hidden_states, topk_weights, topk_ids,
                                 views=cache.bank_views(self.num_experts), n=self.num_experts,
                                 alphas=cache.alphas_for_layer(self.layer_id), is_prefill=True)

    def _expert_gemm(self, cache, hidden_states, topk_weights, topk_ids, *, views, n, alphas,
                     is_prefill: bool):
        fmt = cache.quant_format
        if fmt == "ds_fp4":
            # re-encoded as NVFP4 slot banks; the clamped SwiGLU of the reference's DS-FP4
            # kernels (moe.py:606-637) is not computed here
            limit = getattr(self, "swiglu_limit", None)
            if limit is not None and limit != float("inf"):
                raise NotImplementedError("ds_fp4 experts with a finite swiglu_limit")
            fmt = "nvfp4"
        if fmt == "nvfp4":
            gp, gs, gg, dp, ds, dg = views
            out = hidden_states if is_prefill else None
            if is_prefill:
                hidden_states = hidden_states.clone()
            return ops.moe_ffn_nvfp4(hidden_states, (gp, gs, gg), (dp, ds, dg), topk_weights,
                                     topk_ids, out=out, activation=self.activation,
                                     weight_on_input=self.apply_router_weight_on_input)
        assert fmt == "bf16", f"unknown quant_format {fmt!r}"
        gate_up, down = views
        impl = fused_experts_impl if is_prefill else fused_experts_decode_impl
        return impl(hidden_states, gate_up, down, topk_weights, topk_ids, self.activation,
                    self.apply_router_weight_on_input)


def iter_offload_moe_layers(model):
    """The offloaded MoE layers of a model, in attribute order (the reference's walk,
    backends/.../moe/offload_cache.py:1057-1079): a model that names its layers through an
    ``_iter_offload_moe_layers()`` hook is taken at its word; otherwise an OffloadMoELayer is
    yielded and every object reachable through attributes, lists, tuples and dicts (a torch
    module's submodules included) is searched, each once.  Tensors and caches are not
    searched."""
    seen: set[int] = set()

    def walk(obj):
        if id(obj) in seen or isinstance(obj, (torch.Tensor, OffloadMoeCache, str, bytes)):
            return
        seen.add(id(obj))
        if isinstance(obj, OffloadMoELayer):
            yield obj
            return
        hook = getattr(type(obj), "_iter_offload_moe_layers", None)
        if hook is not None:
            yield from obj._iter_offload_moe_layers()
            return
        if isinstance(obj, (list, tuple)):
            items = obj
        elif isinstance(obj, dict):
            items = obj.values()
        elif hasattr(obj, "__dict__") and not isinstance(obj, type):
            items = vars(obj).values()
        else:
            return
        for item in items:
            yield from walk(item)

    yield from walk(model)


def attach_offload_moe_cache(model, cache: OffloadMoeCache) -> list:
    """Point every offloaded MoE layer of ``model`` (a model object, or a list of layers)
    at ``cache`` and return them (offload_cache.py:1082-1086)."""
    layers = list(iter_offload_moe_layers(model))
    for layer in layers:
        layer.offload_cache = cache
    return layers
