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


def _cpu_cache(L=2, E=4, S=6, hybrid=False):
    """An OffloadMoeCache's state on CPU tensors, for the host-side methods (the real
    constructor insists on a CUDA device)."""
    from tideway_b200 import ops
    from tideway_b200.offload_cache import OffloadMoeCache

    c = object.__new__(OffloadMoeCache)
    c.num_layers, c.num_experts, c.cache_size = L, E, S
    c.device, c.decode_target, c.prefill_overlap = torch.device("cpu"), \
        "hybrid" if hybrid else "gpu", False
    c.slot_for_id = torch.full((L, E), -1, dtype=torch.int32)
    c.id_of_slot = torch.arange(S, dtype=torch.int32)
    c.usage = torch.arange(S, dtype=torch.int64)
    c.step = torch.tensor(9)
    for name in ("num_indices", "num_missing_full"):
        setattr(c, name, torch.ones(1, dtype=torch.int64))
    c.active_mask = torch.ones(E, dtype=torch.int32)
    c.expert_recency = torch.ones(L, E, dtype=torch.int64)
    c.decode_freq = torch.zeros(L, E, dtype=torch.int64)
    c.lru_stats = torch.zeros(L, 4, dtype=torch.int64)
    c.hybrid_stats = torch.zeros(4, dtype=torch.int64) if hybrid else None
    c.hybrid_stats_layer = torch.zeros(L, 4, dtype=torch.int64) if hybrid else None
    c.pinned_slots = torch.zeros(S, dtype=torch.int32)
    c._pending_src_layer = 1
    c.bank_schema = ("gate_up", "down")
    c.bank_sources = {"gate_up": [torch.randn(E, 8, 4) for _ in range(L)],
                      "down": [torch.randn(E, 4, 4) for _ in range(L)]}
    c.bank_caches = {"gate_up": torch.zeros(S, 8, 4), "down": torch.zeros(S, 4, 4)}
    c.banks = [(c.bank_sources[n], c.bank_caches[n]) for n in c.bank_schema]
    c._copy_plans = [ops.CopyPlan([b for _, b in c.banks], [p[l] for p, _ in c.banks])
                     for l in range(L)]
    c.prefill_bank_buffers, c.prefill_copy_stream = [], None
    c.prefill_ready_events, c.prefill_release_events = [], []
    c._prefill_buffer_layer = [None, None]
    c._prefill_buffer_released = [True, True]
    c._prefill_has_release = [False, False]
    return c


def test_rebuild_resizes_the_slot_cache_cold():
    """rebuild() (the reference's in-place resize) keeps the host sources, reallocates the
    slot banks and slot-sized tables at the new size, empties every slot and clears the
    statistics; validate_rebuild refuses sizes below one slot per expert or above what one
    ensure launch ranks."""
    c = _cpu_cache()
    src = c.bank_sources
    c.lru_stats += 3
    c.decode_freq += 2
    c.rebuild(10)
    assert c.cache_size == 10 and c.bank_sources is src
    assert [tuple(b.shape) for _, b in c.banks] == [(10, 8, 4), (10, 4, 4)]
    assert c.id_of_slot.shape == (10,) and bool((c.id_of_slot == -1).all())
    assert bool((c.slot_for_id == -1).all()) and int(c.usage.sum()) == 0 and int(c.step) == 0
    assert c.pinned_slots is None and c._pending_src_layer is None
    assert int(c.lru_stats.sum()) == 0 and int(c.decode_freq.sum()) == 0
    assert len(c._copy_plans) == 2 and c._copy_plans[1].dst[0] == c.banks[0][1].data_ptr()
    for bad in (3, 16385):
        with pytest.raises(ValueError):
            c.validate_rebuild(bad)


def test_per_layer_and_routing_statistics():
    """decode_miss_stats_per_layer and decode_routing_stats report with the reference's keys:
    per layer steps, active / missing / fetched per step and the miss rate; over the
    histogram the working set, the experts covering 90% of the routes, the normalised
    entropy and the best hit rate of a layer keeping its most-routed experts."""
    import math

    c = _cpu_cache(L=2, E=4, S=4)
    c.lru_stats[0, :3] = torch.tensor([12, 3, 4])  # active, missing, calls
    rep = c.decode_miss_stats_per_layer()["per_layer"]
    assert rep[0] == {"layer": 0, "steps": 4, "active_per_step": 3.0, "missing_per_step": 0.75,
                      "miss_rate": 0.25, "fetched_per_step": 0.75}
    assert rep[1]["steps"] == 0 and rep[1]["miss_rate"] == 0.0
    h = _cpu_cache(L=2, E=4, S=4, hybrid=True)
    h.hybrid_stats_layer[1] = torch.tensor([6, 2, 10, 5])  # missing, fetched, active, calls
    r1 = h.decode_miss_stats_per_layer()["per_layer"][1]
    assert (r1["missing_per_step"], r1["fetched_per_step"], r1["miss_rate"]) == (1.2, 0.4, 0.6)
    assert c.decode_routing_stats() == {}
    c.decode_freq[0] = torch.tensor([6, 2, 2, 0])  # layer 1 routed nothing
    s = c.decode_routing_stats()
    p = [0.6, 0.2, 0.2]
    assert s["slots_per_layer"] == 2.0 and s["working_set_max"] == 3
    assert s["working_set_mean"] == 3.0 and s["experts_for_90pct"] == 3.0
    assert abs(s["oracle_hit_at_slots"] - 0.8) < 1e-12
    assert abs(s["norm_entropy"] + sum(q * math.log(q) for q in p) / math.log(4)) < 1e-12
    c.record_decode_stats(0)  # the ensure launch counts by itself


def _tp_rank(rank: int, world: int, port: int, q) -> None:
    import os

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = OffloadMoELayer(0, 8, 2, 4, 4, tp_group=dist.group.WORLD)
        # each rank's partial output: its slice of the intermediate dimension
        layer._decode_routed = lambda h, w, ids: h * (rank + 1)
        with batch_context(is_prefill=False):
            out = layer.routed_forward(torch.ones(2, 4), torch.ones(2, 2),
                                       torch.zeros(2, 2, dtype=torch.int32))
        q.put((rank, layer.tp_size, out.tolist()))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_partials_are_summed():
    """With a tensor-parallel group the layer sums the ranks' partial outputs (the
    reference's _maybe_all_reduce); without one it returns its own output untouched."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = dict((r, (n, o)) for r, n, o in (q.get(timeout=5) for _ in range(2)))
    assert all(n == 2 and o == [[3.0] * 4] * 2 for n, o in got.values())
    solo = OffloadMoELayer(0, 8, 2, 4, 4)
    assert solo.tp_size == 1
    x = torch.ones(2, 4)
    assert solo._maybe_all_reduce(x) is x


def test_attach_walks_a_model_for_its_layers():
    """attach_offload_moe_cache takes a model object as the reference's does: the layers
    found through attributes, lists and torch submodules (each once), or those a model's
    _iter_offload_moe_layers hook names; a plain list of layers still works."""
    from tideway_b200.moe_layer import attach_offload_moe_cache

    layers = [OffloadMoELayer(i, 8, 2, 4, 4) for i in range(3)]

    class Block(torch.nn.Module):
        def __init__(self, layer):
            super().__init__()
            self.norm = torch.nn.LayerNorm(4)
            self.moe = layer

    class Model:
        def __init__(self):
            self.blocks = torch.nn.ModuleList([Block(layers[0]), Block(layers[1])])
            self.extra = {"tail": layers[2], "again": layers[0]}
            self.weight = torch.zeros(3)

    cache = object()
    got = attach_offload_moe_cache(Model(), cache)
    assert got == layers and all(l.offload_cache is cache for l in layers)

    class Hooked:
        def _iter_offload_moe_layers(self):
            return iter(layers[1:])

    assert attach_offload_moe_cache(Hooked(), None) == layers[1:]
    assert attach_offload_moe_cache(layers, cache) == layers
