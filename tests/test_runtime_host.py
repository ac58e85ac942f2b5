"""The B200 offload manager's host logic (entry-point ownership, prefill sequencing,
install/uninstall) against a recording stand-in for the slot cache; no GPU needed."""

from __future__ import annotations

import pytest

from tideway_b200 import runtime
from tideway_b200.moe_layer import OffloadMoELayer


class FakeCache:
    def __init__(self, L=3, E=4, overlap=True):
        self.num_layers, self.num_experts, self.cache_size = L, E, 4 * E
        self.prefill_overlap = overlap
        self.banks = [("sources", "slots")]
        self.log = []

    def ensure_experts(self, layer, ids):
        self.log.append(("ensure", layer, ids))

    def copy_missing(self):
        self.log.append(("copy",))

    def begin_prefill(self):
        self.log.append(("begin",))

    def prefetch_prefill_layer(self, layer):
        self.log.append(("prefetch", layer))

    def wait_prefill_layer(self, layer):
        self.log.append(("wait", layer))
        return ("views", layer)

    def release_prefill_layer(self, layer):
        self.log.append(("release", layer))

    def alphas_for_layer(self, layer):
        return None


class FakeLayer:
    def __init__(self, layer_id):
        self.layer_id = layer_id
        self.calls = []

    def _expert_gemm(self, cache, hidden, weights, ids, *, views, n, alphas, is_prefill):
        self.calls.append((hidden, views, n, is_prefill))
        return ("out", self.layer_id)


def test_manager_owns_ensure_and_copy():
    c = FakeCache()
    m = runtime.TidewayOffload(c)
    assert c.ensure_experts == m.ensure
    c.ensure_experts(2, "ids")
    c.copy_missing()                         # the manager's no-op: ensure already copied
    assert c.log == [("ensure", 2, "ids"), ("copy",)]
    assert m.stats["ensure_calls"] == 1
    m.close()
    assert "ensure_experts" not in vars(c) and "copy_missing" not in vars(c)
    c.ensure_experts(1, "x")
    assert c.log[-1] == ("ensure", 1, "x")


def test_prefill_streams_layers_in_order():
    c = FakeCache(L=3)
    m = runtime.TidewayOffload(c)
    layers = [FakeLayer(i) for i in range(3)]
    outs = [m.prefill(layer, f"h{i}", "w", "ids") for i, layer in enumerate(layers)]
    assert outs == [("out", 0), ("out", 1), ("out", 2)]
    assert c.log == [("begin",), ("prefetch", 0), ("wait", 0), ("release", 0), ("prefetch", 1),
                     ("prefetch", 1), ("wait", 1), ("release", 1), ("prefetch", 2),
                     ("prefetch", 2), ("wait", 2), ("release", 2)]
    assert layers[1].calls == [("h1", ("views", 1), 4, True)]
    assert m.snapshot()["prefill_layers"] == 3 and m.snapshot()["double_buffer"] == 8


def test_manager_needs_banks_and_the_double_buffer():
    c = FakeCache()
    c.banks = []
    with pytest.raises(RuntimeError):
        runtime.TidewayOffload(c)
    with pytest.raises(ValueError):
        runtime.TidewayOffload(FakeCache(overlap=False))


def test_install_patches_prefill_and_uninstall_restores():
    class Layer(OffloadMoELayer):
        pass

    c = FakeCache(L=2)
    original = Layer._prefill_routed
    session = runtime.install(c, layer_classes=(Layer,))
    layer = Layer(0, 4, 2, 64, 32)
    layer.offload_cache = c
    fake = FakeLayer(0)
    layer._expert_gemm = fake._expert_gemm
    assert layer._prefill_routed("h", "w", "ids") == ("out", 0)
    assert ("wait", 0) in c.log and c.ensure_experts == session.manager.ensure
    session.uninstall()
    assert Layer._prefill_routed is original and "_prefill_routed" not in vars(Layer)
    assert "ensure_experts" not in vars(c)


def test_install_takes_the_reference_keywords():
    """install(cache, geo=, host_rows=, reader=, arm=, ...) as the reference's installer takes
    them: its arms, its reader/geometry check, host banks read through the reader when the
    cache has none, and a refusal of the tiers this path does not have."""
    class Geo:
        name, total_experts = "g", 8

    class Reader:
        geo = Geo()

        def __init__(self):
            self.reads = []

        def layer_banks(self, layer, pin=True):
            self.reads.append(layer)
            return {"gate_up": ("gu", layer), "down": ("dn", layer)}

    class Layer(OffloadMoELayer):
        pass

    c = FakeCache(L=2)
    with pytest.raises(ValueError):
        runtime.install(c, layer_classes=(Layer,), arm="bounded")
    other = type("Other", (), {"name": "h"})()
    with pytest.raises(ValueError):
        runtime.install(c, layer_classes=(Layer,), geo=other, reader=Reader())
    big = type("Big", (), {"name": "g", "total_experts": 100})()
    with pytest.raises(NotImplementedError):  # 1 host row + 16 slots < 100 experts: SSD tier
        runtime.install(c, layer_classes=(Layer,), geo=big, host_rows=1)
    with pytest.raises(TypeError):
        runtime.install(c, layer_classes=(Layer,), not_an_option=1)
    for name, value in (("ssd_prefetch_rows", 4), ("phase_policy", "adaptive"),
                        ("core_rows", 3), ("volatile_mirror_rows", 2), ("prior", [1])):
        with pytest.raises(NotImplementedError):
            runtime.install(c, layer_classes=(Layer,), **{name: value})
    # a cache without host banks gets them through the reader (per layer, pinned)
    c = FakeCache(L=2)
    c.banks = []
    got = {}

    def set_bank_sources(sources):
        got.update(sources)
        c.banks = [("sources", "slots")]

    c.set_bank_sources = set_bank_sources
    reader = Reader()
    session = runtime.install(c, layer_classes=(Layer,), geo=reader.geo, host_rows=8,
                              reader=reader, arm="tideway_hybrid", writeback=False,
                              dma_decode=False, phase_policy="off")
    assert reader.reads == [0, 1]
    assert got == {"gate_up": [("gu", 0), ("gu", 1)], "down": [("dn", 0), ("dn", 1)]}
    session.uninstall()


def test_manager_payload_audit_against_the_checkpoint(tmp_path):
    """verify_payload checks every host bank row against the checkpoint through the reader
    install() was given, then the slot copies through the cache's own audit, and reports with
    the reference's keys; a corrupted host byte or slot is named."""
    import torch

    from tests.golden import synthetic_checkpoints as sc
    from tideway_b200 import geometry as G

    geo = G.from_checkpoint(sc.write_fused(tmp_path, "qwen"))
    with G.CheckpointReader(geo) as reader:
        c = FakeCache(L=geo.layers, E=geo.experts)
        per_layer = [reader.layer_banks(layer) for layer in range(geo.layers)]
        c.bank_sources = {b.name: [banks[b.name] for banks in per_layer] for b in geo.banks}
        audit = {"rows": 5, "mismatches": []}
        c.verify_payload = lambda raise_on_mismatch=True: audit
        session = runtime.install(c, layer_classes=(type("L", (OffloadMoELayer,), {}),),
                                  geo=geo, reader=reader)
        try:
            rep = session.manager.verify_payload()
            assert rep["all_resident_payloads_equal"] is True
            assert rep["checked_copies"] == geo.layers * geo.experts + 5 and rep["wall_s"] >= 0
            name = geo.banks[1].name
            row = c.bank_sources[name][1][2].view(torch.uint8).view(-1)
            row[0] ^= 1
            with pytest.raises(AssertionError, match="host"):
                session.manager.verify_payload()
            row[0] ^= 1
            audit["mismatches"] = [(7, 1, 3, name)]
            with pytest.raises(AssertionError, match="GPU"):
                session.manager.verify_payload()
        finally:
            session.uninstall()
