"""OffloadMoELayer's host-side dispatch (decode_target="hybrid", activation arguments) against
recording stand-ins for the slot cache, the executor and the expert GEMM; no GPU needed."""

from __future__ import annotations

import pytest
import torch

from tideway_b200.moe_layer import OffloadMoELayer, batch_context


class FakeHybridCache:
    """ensure_experts_hybrid keeps even expert ids (as their own slots) and leaves odd ids to
    the executor (-1), the way the capped fetch leaves misses past its cap."""

    decode_target = "hybrid"
    quant_format = "bf16"
    collect_stats = False

    def __init__(self, executor):
        self.cpu_executor = executor
        self.log = []

    def is_cpu_layer(self, layer):
        return False

    def ensure_experts_hybrid(self, layer, ids):
        self.log.append(("ensure", layer))
        ids.copy_(torch.where(ids % 2 == 0, ids, torch.full_like(ids, -1)))

    def copy_missing(self):
        self.log.append(("copy",))

    def bank_views(self, n=None):
        return ("gate_up", "down")

    def alphas_for_slots(self, layer):
        return None


class FakeExecutor:
    def __init__(self, log):
        self.log = log
        self.submitted = None

    def decode_submit(self, layer, hidden, weights, ids):
        self.log.append(("submit", layer))
        self.submitted = ids.clone()
        return "handle"

    def decode_sync(self, handle):
        assert handle == "handle"
        self.log.append(("sync",))
        return torch.full((2, 4), 0.25, dtype=torch.bfloat16)


def test_hybrid_decode_splits_routes_and_adds_the_partials():
    log = []
    ex = FakeExecutor(log)
    cache = FakeHybridCache(ex)
    cache.log = log
    layer = OffloadMoELayer(3, 8, 2, 4, 4)
    layer.offload_cache = cache
    seen = {}

    def fake_gemm(c, hidden, weights, ids, *, views, n, alphas, is_prefill):
        log.append(("gemm",))
        seen["ids"] = ids.clone()
        assert views == ("gate_up", "down") and n is None and not is_prefill
        return torch.full((2, 4), 0.5, dtype=torch.bfloat16)

    layer._expert_gemm = fake_gemm
    ids = torch.tensor([[0, 3], [5, 6]], dtype=torch.int32)
    w = torch.tensor([[0.6, 0.4], [0.3, 0.7]])
    with batch_context(is_prefill=False):
        out = layer.routed_forward(torch.zeros(2, 4, dtype=torch.bfloat16), w, ids)
    # the executor gets the raw ids of the routes left at -1, before the copy and the GEMM
    assert torch.equal(ex.submitted, torch.tensor([[-1, 3], [5, -1]], dtype=torch.int32))
    assert torch.equal(seen["ids"], torch.tensor([[0, -1], [-1, 6]], dtype=torch.int32))
    assert [e[0] for e in log] == ["ensure", "submit", "copy", "gemm", "sync"]
    assert torch.equal(out, torch.full((2, 4), 0.75, dtype=torch.bfloat16))


def test_hybrid_decode_needs_an_executor():
    cache = FakeHybridCache(None)
    layer = OffloadMoELayer(0, 8, 2, 4, 4)
    layer.offload_cache = cache
    with batch_context(is_prefill=False), pytest.raises(RuntimeError):
        layer.routed_forward(torch.zeros(1, 4, dtype=torch.bfloat16), torch.ones(1, 2),
                             torch.zeros(1, 2, dtype=torch.int32))


def test_layer_passes_activation_and_weight_placement():
    """The layer hands its activation and apply_router_weight_on_input to the expert FFN."""
    import tideway_b200.moe_layer as ml

    calls = {}

    def fake_decode(hidden, w1, w2, weights, ids, activation, w_in):
        calls.update(activation=activation, w_in=w_in)
        return hidden

    layer = OffloadMoELayer(0, 8, 2, 4, 4, activation="gelu_tanh",
                            apply_router_weight_on_input=True)

    class Cache:
        quant_format = "bf16"

    orig = ml.fused_experts_decode_impl
    ml.fused_experts_decode_impl = fake_decode
    try:
        layer._expert_gemm(Cache(), torch.zeros(1, 4), torch.ones(1, 2),
                           torch.zeros(1, 2, dtype=torch.int32), views=("a", "b"), n=None,
                           alphas=None, is_prefill=False)
    finally:
        ml.fused_experts_decode_impl = orig
    assert calls == {"activation": "gelu_tanh", "w_in": True}


def test_cache_takes_the_engines_alpha_call():
    """An engine hands every cache its format's folded alphas (the reference's engine calls
    set_alphas unconditionally): (None, None) is accepted, real alphas are refused, and the
    cache exposes no alphas."""
    from tideway_b200.offload_cache import OffloadMoeCache

    cache = object.__new__(OffloadMoeCache)  # the table tensors need a GPU; this does not
    cache.gate_up_alpha = cache.down_alpha = None
    cache.set_alphas(None, None)
    with pytest.raises(NotImplementedError):
        cache.set_alphas(torch.ones(4), torch.ones(4))
    assert cache.alphas_for_slots(0) is None and cache.alphas_for_layer(0) is None
    assert cache.gate_up_alpha is None and cache.down_alpha is None


def test_layer_refuses_layers_marked_for_host_decode():
    """An engine that marks a layer for whole-layer host decode (cpu_layer_ids, the
    reference's decode_target 'cpu') gets an error instead of a silent GPU decode."""
    cache = FakeHybridCache(FakeExecutor([]))
    cache.decode_target = "gpu"
    cache.is_cpu_layer = lambda layer: layer == 2
    layer = OffloadMoELayer(2, 8, 2, 4, 4)
    layer.offload_cache = cache
    with batch_context(is_prefill=False), pytest.raises(NotImplementedError):
        layer.routed_forward(torch.zeros(1, 4, dtype=torch.bfloat16), torch.ones(1, 2),
                             torch.zeros(1, 2, dtype=torch.int32))
