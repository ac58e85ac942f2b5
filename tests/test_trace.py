"""Routing trace ring and histograms (CPU tensors; the same device ops run on the GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tideway_b200 import runtime
from tideway_b200.trace import RouteTrace, accumulate_histogram
from tests.test_runtime_host import FakeCache, FakeLayer


def test_ring_pads_orders_and_wraps():
    t = RouteTrace(rows=4, width=6, device="cpu")
    recs = [(l % 3, torch.arange(n, dtype=torch.int32) + 10 * l) for l, n in
            enumerate([6, 4, 6, 1, 6, 5])]
    for layer, ids in recs[:3]:
        t.record(layer, ids.view(-1, 2) if ids.numel() % 2 == 0 else ids)
    layers, ids, total = t.read()
    assert total == 3 and layers.tolist() == [0, 1, 2]
    assert ids[1].tolist() == [10, 11, 12, 13, -1, -1]
    for layer, x in recs[3:]:
        t.record(layer, x)
    layers, ids, total = t.read()
    assert total == 6 and layers.tolist() == [2, 0, 1, 2]      # the last four, oldest first
    assert ids[1].tolist() == [30, -1, -1, -1, -1, -1]
    assert ids[3].tolist() == [50, 51, 52, 53, 54, -1]
    with pytest.raises(ValueError):
        t.record(0, torch.zeros(7, dtype=torch.int32))
    t.reset()
    assert t.read()[2] == 0


def test_histogram_skips_padding():
    h = torch.zeros(2, 5, dtype=torch.int64)
    accumulate_histogram(h, 1, torch.tensor([[0, 4], [4, -1]], dtype=torch.int32))
    assert h.tolist() == [[0] * 5, [1, 0, 0, 0, 2]]


class TracingCache(FakeCache):
    def __init__(self, **kw):
        super().__init__(**kw)
        self.slot_for_id = torch.zeros(1)
        self.route_trace = None

    def enable_route_trace(self, steps, width):
        self.route_trace = RouteTrace(steps * self.num_layers, width, "cpu")
        return self.route_trace

    def ensure_experts(self, layer, ids):
        if self.route_trace is not None:
            self.route_trace.record(layer, ids)
        super().ensure_experts(layer, ids)


def test_manager_dumps_the_reference_trace_keys(tmp_path):
    c = TracingCache(L=2, E=4)
    m = runtime.TidewayOffload(c)
    m.enable_trace(steps=8, width=4)
    for step in range(3):
        for layer in range(2):
            c.ensure_experts(layer, torch.tensor([[step, layer]], dtype=torch.int32))
        m.mark_case()
    m.prefill(FakeLayer(1), "h", "w", torch.tensor([[0, 3], [3, -1]]))
    info = m.dump_trace(tmp_path / "trace.npz")
    d = np.load(tmp_path / "trace.npz")
    assert set(d.files) == {"decode_layers", "decode_ids", "case_marks", "prefill_hist",
                            "experts_per_layer", "layers_total", "gpu_slots", "host_rows"}
    assert d["decode_layers"].tolist() == [0, 1] * 3
    assert d["decode_ids"][3].tolist() == [1, 1, -1, -1]
    assert d["case_marks"].tolist() == [2, 4, 6]
    assert d["prefill_hist"].tolist() == [0, 0, 0, 0, 1, 0, 0, 2]
    assert info["decode_records"] == 6 and info["prefill_accesses"] == 3
