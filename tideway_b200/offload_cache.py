"""Fixed-address expert slot cache with device-side tables (graph-safe).

Mirrors ``OffloadMoeCache`` (backends/freetoken_tideway/freetoken/moe/offload_cache.py):
same constructor fields, bank schemas, table tensors and entry points
(``set_bank_sources``, ``bank_views``, ``ensure_experts``, ``copy_missing``,
``materialize_layer``, ``reset``, the prefill double buffer, miss statistics).  The table
updates and row copies are the tideway_b200 CUDA kernels; ``ensure_experts`` rewrites the
routed ids into slot ids in place and ``copy_missing`` moves the missing rows from the
pinned host banks, both without a host sync, so the decode step stays capturable.
"""

from __future__ import annotations

import math
import os
import warnings
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .trace import RouteTrace, accumulate_histogram

# quant_format -> bank names in registration order (offload_cache.py:32-74 for the names).
BANK_SCHEMAS: dict[str, tuple[str, ...]] = {
    "bf16": ("gate_up", "down"),
    "nvfp4": ("gate_up_packed", "gate_up_scale", "gate_up_global",
              "down_packed", "down_scale", "down_global"),
    # DeepSeek-V4 FP4 sources (e8m0 per-32 scales); registered as NVFP4 slot banks, each
    # row re-encoded exactly (tideway_b200/ds_fp4.py)
    "ds_fp4": ("gate_up_packed", "gate_up_scale", "down_packed", "down_scale"),
}

# lru_stats columns (ACTIVE unique experts, MISS, CALLS)
STAT_ACTIVE, STAT_MISS, STAT_CALLS = 0, 1, 2
N_STATS = 4
# slots one ensure launch can rank (its radix-select keys hold the slot in 14 bits)
MAX_SLOTS = 16384


@dataclass
class OffloadMoeCache:
    num_layers: int
    num_experts: int
    cache_size: int
    device: torch.device
    cache_policy: str = "lru"
    prefill_overlap: bool = False
    prefill_hit_d2d: bool = False
    quant_format: str = "bf16"
    decode_target: str = "gpu"
    hybrid_max_fetch: int = 1 << 30       # ensure_experts_hybrid: fetches per step
    hybrid_fetch_fraction: float = 0.0    # > 0: bandwidth-matched share of the misses
    hybrid_fetch_by_recency: bool = True  # fetch order: recency (else lowest id)

    def __post_init__(self) -> None:
        self.device = torch.device(self.device)
        if self.device.type != "cuda":
            raise RuntimeError("OffloadMoeCache lives on a CUDA device (no CPU path)")
        assert self.cache_policy == "lru", self.cache_policy
        if self.decode_target == "cpu":
            # whole layers decoded on the host cores (the reference's CpuMoeExecutor) are a
            # host engine, not the B200 expert path
            raise NotImplementedError("decode_target='cpu' is not on the B200 path")
        assert self.decode_target in ("gpu", "hybrid"), self.decode_target
        assert self.quant_format in BANK_SCHEMAS, f"unknown quant_format {self.quant_format!r}"
        if self.cache_size < self.num_experts:
            raise ValueError(f"cache_size {self.cache_size} < num_experts {self.num_experts}")
        assert not self.prefill_overlap or self.cache_size >= 2 * self.num_experts, (
            "prefill overlap borrows two expert-layer buffers: cache_size >= 2 * num_experts")
        if self.prefill_hit_d2d:
            # an auto-fallback option in the reference (offload_cache.py:702-724): say once
            # that the fallback, whole layers from the host banks, is what runs
            warnings.warn("prefill_hit_d2d: every prefill layer streams whole from the host "
                          "banks (the hit/miss split copy is not wired); outputs are the same",
                          stacklevel=2)
        dev = self.device
        L, E, S = self.num_layers, self.num_experts, self.cache_size
        self.slot_for_id = torch.full((L, E), -1, dtype=torch.int32, device=dev)
        self.id_of_slot = torch.full((S,), -1, dtype=torch.int32, device=dev)
        self.usage = torch.zeros((S,), dtype=torch.int64, device=dev)
        self.step = torch.zeros((), dtype=torch.int64, device=dev)
        self.evict_slots = torch.zeros((E,), dtype=torch.int32, device=dev)
        self.src_indices = torch.zeros((E,), dtype=torch.int32, device=dev)
        self.num_indices = torch.zeros((1,), dtype=torch.int64, device=dev)
        self.lru_stats = torch.zeros((L, N_STATS), dtype=torch.int64, device=dev)
        # hybrid (capped-fetch) ensure state
        self.active_mask = torch.zeros((E,), dtype=torch.int32, device=dev)
        self.num_missing_full = torch.zeros((1,), dtype=torch.int64, device=dev)
        self.expert_recency = torch.zeros((L, E), dtype=torch.int64, device=dev)
        self.collect_stats = False
        # hybrid decode: misses (before the fetch cap), fetches, active experts and calls, in
        # total and per layer, accumulated on the device by record_decode_stats_hybrid
        hybrid = self.decode_target == "hybrid"
        self.hybrid_stats = torch.zeros((4,), dtype=torch.int64, device=dev) if hybrid else None
        self.hybrid_stats_layer = (torch.zeros((L, 4), dtype=torch.int64, device=dev)
                                   if hybrid else None)
        # decode_target == "hybrid": the caller's engine for the misses the capped fetch
        # leaves out (set_cpu_executor); this package computes the GPU share only
        self.cpu_executor = None
        # the reference's Tideway-Shift phase-policy state; its callers skip it when None
        self.shift = None
        # layers an engine sends wholly to a host executor (decode_target 'cpu'): none here
        self.cpu_layer_ids: frozenset = frozenset()
        # folded per-expert alphas of the reference's pre-tiled layouts: never set here
        self.gate_up_alpha: torch.Tensor | None = None
        self.down_alpha: torch.Tensor | None = None
        # routing observability (backends/.../moe/offload_cache.py:211-240): a per-layer
        # routed-expert histogram and a device ring of each ensure's raw ids, both recorded
        # before the ids are rewritten, both device-only (kept by captured graphs)
        self.collect_decode_freq = False
        self.decode_freq = torch.zeros((L, E), dtype=torch.int64, device=dev)
        self.route_trace: RouteTrace | None = None
        steps = int(os.environ.get("TIDEWAY_SHIFT_TRACE_STEPS", "0") or 0)
        if steps > 0:
            self.enable_route_trace(steps, width=8)
        self.pinned_slots: torch.Tensor | None = None
        # slot banks in registration order; DS-FP4 experts live in NVFP4 slot banks
        self.bank_schema = BANK_SCHEMAS["nvfp4" if self.quant_format == "ds_fp4"
                                        else self.quant_format]
        self.ds_fp4_flushed_blocks = 0
        self.bank_sources: dict[str, list[torch.Tensor]] = {}
        self.bank_generation = 0  # bumped by every set_bank_sources
        self.bank_caches: dict[str, torch.Tensor] = {}
        self.banks: list[tuple[list[torch.Tensor], torch.Tensor]] = []
        self._copy_plans: list[ops.CopyPlan] = []
        self._pending_src_layer: int | None = None
        self.prefill_bank_buffers: list[torch.Tensor] = []
        self.prefill_copy_stream: torch.cuda.Stream | None = None
        self.prefill_ready_events: list[torch.cuda.Event] = []
        self.prefill_release_events: list[torch.cuda.Event] = []
        self._prefill_buffer_layer: list[int | None] = [None, None]
        self._prefill_buffer_released = [True, True]
        self._prefill_has_release = [False, False]

    # ------------------------------------------------------------ banks
    def set_bank_sources(self, sources: dict[str, list[torch.Tensor]],
                         layer_residency: list[str] | None = None) -> None:
        """Attach per-layer host banks (pinned, [E, ...] each) and allocate the slot banks.
        ``ds_fp4`` sources are re-encoded as NVFP4 host banks here (a one-time copy of the
        scales; the packed codes are kept)."""
        schema = BANK_SCHEMAS[self.quant_format]
        assert set(sources) == set(schema), (
            f"banks {sorted(sources)} do not match the {self.quant_format!r} schema {schema}")
        if self.quant_format == "ds_fp4":
            sources = self._reencode_ds_fp4(sources)
        if layer_residency is not None and any(r != "pinned" for r in layer_residency):
            raise NotImplementedError("only pinned host bank layers are served")
        for name in self.bank_schema:
            per_layer = sources[name]
            assert len(per_layer) == self.num_layers, (name, len(per_layer))
            head = per_layer[0]
            for layer_id, src in enumerate(per_layer):
                assert src.is_contiguous(), f"bank {name!r} layer {layer_id} must be contiguous"
                assert src.size(0) == self.num_experts, (name, layer_id, tuple(src.shape))
                assert src.shape == head.shape and src.dtype == head.dtype, (name, layer_id)
                if not src.is_cuda and not src.is_pinned():
                    raise ValueError(f"bank {name!r} layer {layer_id}: host banks must be pinned")
            self.bank_sources[name] = list(per_layer)
            self.bank_caches[name] = torch.empty((self.cache_size, *head.shape[1:]),
                                                 dtype=head.dtype, device=self.device)
        self.banks = [(self.bank_sources[n], self.bank_caches[n]) for n in self.bank_schema]
        self.bank_generation += 1
        self._copy_plans = [
            ops.CopyPlan([cache for _, cache in self.banks],
                         [per_layer[layer] for per_layer, _ in self.banks])
            for layer in range(self.num_layers)
        ]
        if self.prefill_overlap:
            self._init_prefill_overlap_buffers()

    def _reencode_ds_fp4(self, sources: dict) -> dict:
        from . import ds_fp4

        for name in ds_fp4.DS_FP4_BANKS:
            assert len(sources[name]) == self.num_layers, (name, len(sources[name]))
        out: dict[str, list[torch.Tensor]] = {name: [] for name in ds_fp4.NVFP4_BANKS}
        self.ds_fp4_flushed_blocks = 0
        for layer in range(self.num_layers):
            banks, flushed = ds_fp4.expert_banks(
                *(sources[name][layer] for name in ds_fp4.DS_FP4_BANKS))
            self.ds_fp4_flushed_blocks += flushed
            for name, t in banks.items():
                out[name].append(t if t.is_cuda or t.is_pinned() else t.pin_memory())
        return out

    def bank_views(self, n: int | None = None) -> tuple[torch.Tensor, ...]:
        """Per-bank slot caches in registration order: all ``[S]`` slots or the first n."""
        assert self.banks, "set_bank_sources must register the banks first"
        if n is None:
            return tuple(cache for _, cache in self.banks)
        return tuple(cache[:n] for _, cache in self.banks)

    def set_alphas(self, gate_up_alpha: torch.Tensor | None,
                   down_alpha: torch.Tensor | None) -> None:
        """The reference's hook for per-expert global scales folded out of the pre-tiled
        nvfp4_marlin / nvfp4_b12x layouts (backends/.../moe/offload_cache.py:493-509), which
        an engine calls with whatever its format carries.  ``(None, None)`` is a no-op, as
        there; this build serves no folded-alpha layout (its NVFP4 banks keep their row
        globals), so real alphas are refused."""
        if gate_up_alpha is None and down_alpha is None:
            return
        raise NotImplementedError("folded per-expert alphas belong to the nvfp4_marlin / "
                                  "nvfp4_b12x layouts, which this build does not serve")

    def alphas_for_slots(self, layer_id: int):
        """Per-slot folded alphas (offload_cache.py:527-535): none here, the NVFP4 banks
        carry their own row globals."""
        return None

    def alphas_for_layer(self, layer_id: int):
        """Per-layer folded alphas (offload_cache.py:537-545): none here."""
        return None

    # ------------------------------------------------------------ decode
    def ensure_experts(self, layer_id: int, expert_ids: torch.Tensor) -> None:
        """Make this layer's routed experts resident; rewrite ``expert_ids`` (int32, any
        shape, contiguous) to slot ids in place.  Misses are staged for copy_missing."""
        assert 0 <= layer_id < self.num_layers, layer_id
        if self.collect_decode_freq:
            accumulate_histogram(self.decode_freq, layer_id, expert_ids)
        if self.route_trace is not None and expert_ids.numel() <= self.route_trace.width:
            self.route_trace.record(layer_id, expert_ids)
        self._pending_src_layer = layer_id
        ops.lru_ensure(expert_ids, self.slot_for_id, self.id_of_slot, self.usage, self.step,
                       self.num_experts, layer_id, self.evict_slots, self.src_indices,
                       self.num_indices,
                       stats=self.lru_stats[layer_id] if self.collect_stats else None,
                       pinned=self.pinned_slots)

    def ensure_experts_grouped(self, layer_id: int, expert_ids: torch.Tensor, ws: torch.Tensor,
                               hidden: int, inter: int) -> None:
        """``ensure_experts`` on a decode batch's ids [T, K] that also groups the rewritten
        routes by slot into the expert FFN's workspace ``ws`` in the same launch; the FFN
        then runs with ``pregrouped=True`` (one launch fewer per layer)."""
        assert 0 <= layer_id < self.num_layers, layer_id
        if self.collect_decode_freq:
            accumulate_histogram(self.decode_freq, layer_id, expert_ids)
        if self.route_trace is not None and expert_ids.numel() <= self.route_trace.width:
            self.route_trace.record(layer_id, expert_ids)
        self._pending_src_layer = layer_id
        ops.lru_ensure_group(expert_ids, self.slot_for_id, self.id_of_slot, self.usage,
                             self.step, self.num_experts, layer_id, self.evict_slots,
                             self.src_indices, self.num_indices, hidden, inter, ws,
                             stats=self.lru_stats[layer_id] if self.collect_stats else None,
                             pinned=self.pinned_slots,
                             nvfp4=self.bank_schema != BANK_SCHEMAS["bf16"])

    def ensure_experts_hybrid(self, layer_id: int, expert_ids: torch.Tensor) -> None:
        """Capped-fetch LRU (the reference's hybrid backend,
        backends/.../moe/offload_cache.py:866-884): like ensure_experts, but only
        ``hybrid_max_fetch`` -- or ``~hybrid_fetch_fraction * misses`` when the fraction is
        set -- of this step's misses get a slot and a pending copy; ``expert_ids`` becomes
        the slot (hit or fetched) or -1 (a miss left to another engine).  ``num_indices`` =
        fetches (copy_missing), ``num_missing_full`` = misses.  Device-side, graph-safe."""
        assert 0 <= layer_id < self.num_layers, layer_id
        if self.collect_decode_freq:  # before the kernel rewrites the ids in place
            accumulate_histogram(self.decode_freq, layer_id, expert_ids)
        self._pending_src_layer = layer_id
        # Q16 fixed point, so that the cap is computed without floats on the device
        frac_q16 = min(1 << 16, max(0, round(self.hybrid_fetch_fraction * (1 << 16))))
        ops.hybrid_ensure(expert_ids, self.slot_for_id, self.id_of_slot, self.usage, self.step,
                          self.num_experts, layer_id, self.active_mask, self.evict_slots,
                          self.src_indices, self.num_indices, self.num_missing_full,
                          self.expert_recency if self.hybrid_fetch_by_recency else None,
                          min(self.hybrid_max_fetch, 1 << 30), frac_q16)

    def set_cpu_executor(self, executor) -> None:
        """Attach the engine that computes the routes ``ensure_experts_hybrid`` leaves at -1
        (backends/.../moe/offload_cache.py:511-521).  It needs two methods:
        ``decode_submit(layer_id, hidden, topk_weights, ids) -> handle`` (``ids`` holds raw
        expert ids for its routes and -1 elsewhere) and ``decode_sync(handle) -> Tensor``,
        the [T, H] partial output on this cache's device in the hidden dtype."""
        if self.decode_target != "hybrid":
            raise ValueError("set_cpu_executor requires decode_target='hybrid'")
        self.cpu_executor = executor

    def is_cpu_layer(self, layer_id: int) -> bool:
        """Whether ``layer_id`` is in ``cpu_layer_ids``, the layers an engine routes wholly to
        a host executor (offload_cache.py:134, :520-522).  That is decode_target 'cpu',
        which this build refuses, so the set stays empty unless an engine fills it, and the
        layer then refuses to decode it."""
        return layer_id in self.cpu_layer_ids

    def record_decode_stats_hybrid(self, layer_id: int) -> None:
        """Add this hybrid ensure's misses, fetches and active experts to the device
        counters (cf. backends/.../moe/offload_cache.py:920-938); no host sync."""
        assert 0 <= layer_id < self.num_layers, layer_id
        assert self.hybrid_stats is not None, "hybrid statistics need decode_target='hybrid'"
        v = torch.stack([self.num_missing_full[0], self.num_indices[0],
                         self.active_mask.sum().to(torch.int64),
                         torch.ones((), dtype=torch.int64, device=self.device)])
        self.hybrid_stats += v
        self.hybrid_stats_layer[layer_id] += v

    def enable_route_trace(self, steps: int, width: int) -> RouteTrace:
        """Record the raw routed ids of every ensure call (up to ``width`` ids each; larger
        calls are not recorded) in a device ring of ``steps`` x layers rows."""
        self.route_trace = RouteTrace(int(steps) * self.num_layers, width, self.device)
        return self.route_trace

    def copy_missing(self) -> None:
        """Copy the staged missing rows of every bank (count read on the device)."""
        assert self.banks, "set_bank_sources must register the banks first"
        layer_id = self._pending_src_layer
        assert layer_id is not None, "no staged misses (ensure_experts/materialize_layer first)"
        ops.copy_rows(self._copy_plans[layer_id], self.evict_slots, self.src_indices,
                      self.num_indices, self.num_experts)

    def materialize_layer(self, layer_id: int) -> None:
        self._pending_src_layer = layer_id
        ops.materialize_layer(self.slot_for_id, self.id_of_slot, self.usage, self.step,
                              self.num_experts, layer_id, self.evict_slots, self.src_indices,
                              self.num_indices)

    def reset(self) -> None:
        ops.reset_slots(self.slot_for_id, self.id_of_slot, self.usage, self.step,
                        self.num_indices)

    def seed_resident(self, layer_experts: dict[int, list[int]]) -> None:
        """Place experts into free slots (setup-time, host side) and copy their rows."""
        slots = iter(torch.nonzero(self.id_of_slot.cpu() < 0).flatten().tolist())
        sfi = self.slot_for_id.cpu()
        ios = self.id_of_slot.cpu()
        for layer, experts in layer_experts.items():
            for e in experts:
                s = next(slots)
                ios[s] = layer * self.num_experts + e
                sfi[layer, e] = s
                for (per_layer, cache) in self.banks:
                    cache[s].copy_(per_layer[layer][e], non_blocking=True)
        self.slot_for_id.copy_(sfi)
        self.id_of_slot.copy_(ios)

    def validate_rebuild(self, cache_size: int) -> None:
        """Check a slot count for rebuild() without touching the device (the reference's
        pre-teardown check, backends/.../moe/offload_cache.py:401-416): at least one slot per
        expert of a layer, and no more than one ensure launch ranks."""
        if cache_size < self.num_experts:
            raise ValueError(f"cache_size {cache_size} < num_experts {self.num_experts}")
        if cache_size > MAX_SLOTS:
            raise ValueError(f"cache_size {cache_size} > {MAX_SLOTS}, the most slots one "
                             "ensure launch ranks")

    def rebuild(self, cache_size: int) -> None:
        """Resize the slot cache to ``cache_size`` slots in place (offload_cache.py:418-486):
        the pinned host sources stay registered, the slot banks and the slot-sized tables are
        freed and allocated again, every slot starts empty, the statistics, histogram and
        pinned slots are cleared, and the prefill double buffer is set up again if it still
        fits (else turned off).  The object stays the same, so attached layers keep it; any
        captured graph now fails its address check and must be captured again."""
        assert self.banks, "set_bank_sources must register the banks first"
        self.validate_rebuild(cache_size)
        dev = self.device
        # the double buffer's views alias the old slot banks: drop them first
        self.prefill_bank_buffers = []
        self.prefill_copy_stream = None
        self.prefill_ready_events, self.prefill_release_events = [], []
        self._prefill_buffer_layer = [None, None]
        self._prefill_buffer_released = [True, True]
        self._prefill_has_release = [False, False]
        shapes = {name: (tuple(cache.shape[1:]), cache.dtype)
                  for name, cache in self.bank_caches.items()}
        self.banks, self.bank_caches, self._copy_plans = [], {}, []
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
            torch.cuda.empty_cache()
        self.cache_size = S = cache_size
        for name in self.bank_schema:
            tail, dtype = shapes[name]
            self.bank_caches[name] = torch.empty((S, *tail), dtype=dtype, device=dev)
        self.banks = [(self.bank_sources[n], self.bank_caches[n]) for n in self.bank_schema]
        self._copy_plans = [
            ops.CopyPlan([cache for _, cache in self.banks],
                         [per_layer[layer] for per_layer, _ in self.banks])
            for layer in range(self.num_layers)
        ]
        self.slot_for_id.fill_(-1)
        self.id_of_slot = torch.full((S,), -1, dtype=torch.int32, device=dev)
        self.usage = torch.zeros((S,), dtype=torch.int64, device=dev)
        self.step.zero_()
        self.pinned_slots = None  # pins named slots of the old layout
        for t in (self.num_indices, self.num_missing_full, self.active_mask,
                  self.expert_recency, self.decode_freq):
            t.zero_()
        self.reset_stats()
        self._pending_src_layer = None
        if self.prefill_overlap and S < 2 * self.num_experts:
            warnings.warn(f"prefill overlap turned off by rebuild: {S} slots < "
                          f"2 * {self.num_experts} experts")
            self.prefill_overlap = False
        if self.prefill_overlap:
            self._init_prefill_overlap_buffers()

    def record_decode_stats(self, layer_id: int) -> None:
        """Nothing to do (offload_cache.py:913-918): the ensure launch adds its unique,
        missing and call counts to ``lru_stats`` itself when ``collect_stats`` is set."""

    def reset_stats(self) -> None:
        self.lru_stats.zero_()
        if self.hybrid_stats is not None:
            self.hybrid_stats.zero_()
            self.hybrid_stats_layer.zero_()

    def decode_miss_stats_per_layer(self) -> dict:
        """Per-layer decode statistics since the last reset_stats (one device read), with
        the keys of the reference's report (offload_cache.py:962-990).  Without the hybrid
        cap every miss is fetched."""
        if self.decode_target == "hybrid":
            missing, fetched, active, steps = self.hybrid_stats_layer.cpu().numpy().T
        else:
            active, missing, steps = self.lru_stats[:, :3].cpu().numpy().T
            fetched = missing

        def per(v, d):
            return float(v) / float(d) if d else 0.0

        return {"per_layer": [
            {"layer": l, "steps": int(steps[l]),
             "active_per_step": per(active[l], steps[l]),
             "missing_per_step": per(missing[l], steps[l]),
             "miss_rate": per(missing[l], active[l]),
             "fetched_per_step": per(fetched[l], steps[l])}
            for l in range(self.num_layers)]}

    def decode_routing_stats(self) -> dict:
        """How concentrated each layer's decode routing is, from the ``collect_decode_freq``
        histogram (the reference's report, offload_cache.py:992-1022), averaged over the
        layers that routed anything: distinct experts routed, how many of the most-routed
        experts carry 90% of the routes, the entropy of the route shares over log(E), and
        the hit rate a layer holding its share of the slots (``cache_size / num_layers``)
        would get if it always kept its most-routed experts."""
        f = self.decode_freq.cpu().numpy().astype(np.float64)
        total = f.sum(axis=1)
        live = total > 0
        if not live.any():
            return {}
        f, total = f[live], total[live]
        share = f / total[:, None]
        ranked = -np.sort(-share, axis=1)
        slots_per_layer = self.cache_size / self.num_layers
        keep = max(1, int(round(slots_per_layer)))
        covered = np.cumsum(ranked, axis=1)
        entropy = -(share * np.log(np.maximum(share, 1e-12))).sum(axis=1)
        distinct = (f > 0).sum(axis=1)
        return {
            "slots_per_layer": slots_per_layer,
            "working_set_mean": float(distinct.mean()),
            "working_set_max": int(distinct.max()),
            "experts_for_90pct": float(((covered < 0.9).sum(axis=1) + 1).mean()),
            "oracle_hit_at_slots": float(ranked[:, :keep].sum(axis=1).mean()),
            "norm_entropy": float((entropy / math.log(self.num_experts)).mean()),
        }

    def decode_miss_stats(self) -> dict:
        if self.decode_target == "hybrid":
            missing, fetched, active, calls = (int(v) for v in self.hybrid_stats.tolist())
        else:
            active, missing, calls = (int(v) for v in self.lru_stats[:, :3].sum(0).tolist())
            fetched = missing
        out = {
            "layer_calls": calls,
            "active_per_layer": active / calls if calls else 0.0,
            "missing_per_layer": missing / calls if calls else 0.0,
            "miss_rate": missing / active if active else 0.0,
        }
        if self.decode_target == "hybrid":  # how the misses split between fetch and the engine
            out.update(fetched_per_layer=fetched / calls if calls else 0.0,
                       cpu_per_layer=(missing - fetched) / calls if calls else 0.0,
                       fetch_rate=fetched / missing if missing else 0.0)
        return out

    def graph_signature(self) -> tuple:
        """Everything a captured decode step bakes in from this cache: the address, shape,
        strides and dtype of every device tensor its kernels read or write (slot banks,
        tables, ensure scratch, statistics, histogram, routing-trace ring and cursor, pinned
        slots), and every host source row pointer its miss copies read.  A graph controller
        compares it before each replay (cf. the fixed-address checks of
        src/tideway/offload/paged_decode_graph.py:255-282)."""
        ts = [cache for _, cache in self.banks] + [
            self.slot_for_id, self.id_of_slot, self.usage, self.step, self.evict_slots,
            self.src_indices, self.num_indices, self.lru_stats, self.active_mask,
            self.num_missing_full, self.expert_recency, self.decode_freq]
        if self.hybrid_stats is not None:
            ts += [self.hybrid_stats, self.hybrid_stats_layer]
        if self.route_trace is not None:
            rt = self.route_trace
            ts += [rt.ids, rt.layer, rt.pos, rt._row]
        if self.pinned_slots is not None:
            ts.append(self.pinned_slots)
        sig = tuple((t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype) for t in ts)
        sources = tuple(tuple(t.data_ptr() for t in per_layer) for per_layer, _ in self.banks)
        return sig + (sources, self.bank_generation, self.route_trace is None,
                      self.pinned_slots is None)

    def verify_tables(self) -> None:
        """Host audit of the slot <-> id bijection (cf. src/tideway/offload/native_verify.py)."""
        sfi = self.slot_for_id.flatten().cpu()
        ios = self.id_of_slot.cpu()
        mapped = torch.nonzero(sfi >= 0).flatten()
        if not torch.equal(ios[sfi[mapped].long()].long(), mapped):
            raise RuntimeError("slot table corrupt: slot_for_id -> id_of_slot mismatch")
        occ = torch.nonzero(ios >= 0).flatten()
        if not torch.equal(sfi[ios[occ].long()].long(), occ):
            raise RuntimeError("slot table corrupt: id_of_slot -> slot_for_id mismatch")

    def verify_payload(self, raise_on_mismatch: bool = True) -> dict:
        """Audit every resident slot against its host source row, bank by bank (cf. the
        reference's ``verify_payload``, src/tideway/offload/runtime.py:1068-1109): the bytes
        a slot holds must equal the bytes of the expert the table says it holds.  A host
        audit: synchronises, and streams each resident row's source over the host link.
        Returns {"rows": checked slots, "mismatches": [(slot, layer, expert, bank)]}."""
        assert self.banks, "set_bank_sources must register the banks first"
        torch.cuda.synchronize(self.device)
        ios = self.id_of_slot.cpu()
        occ = torch.nonzero(ios >= 0).flatten()
        mismatches = []
        E = self.num_experts
        for layer in range(self.num_layers):
            here = occ[(ios[occ] // E) == layer]
            if here.numel() == 0:
                continue
            experts = (ios[here] % E).long()
            for name, (per_layer, cache) in zip(self.bank_schema, self.banks):
                want = per_layer[layer].index_select(0, experts.to(per_layer[layer].device))
                have = cache.index_select(0, here.to(self.device)).to(want.device)
                same = (have.reshape(len(here), -1).view(torch.uint8)
                        == want.reshape(len(here), -1).view(torch.uint8)).all(dim=1)
                for i in torch.nonzero(~same).flatten().tolist():
                    mismatches.append((int(here[i]), layer, int(experts[i]), name))
        if mismatches and raise_on_mismatch:
            raise RuntimeError(f"slot payload differs from its host source: {mismatches[:8]}")
        return {"rows": int(occ.numel()), "mismatches": mismatches}

    # ------------------------------------------------------------ prefill double buffer
    def _init_prefill_overlap_buffers(self) -> None:
        E = self.num_experts
        self.prefill_bank_buffers = [cache[:2 * E].view(2, E, *cache.shape[1:])
                                     for _, cache in self.banks]
        self.prefill_copy_stream = torch.cuda.Stream(device=self.device)
        self.prefill_ready_events = [torch.cuda.Event() for _ in range(2)]
        self.prefill_release_events = [torch.cuda.Event() for _ in range(2)]
        self._prefill_buffer_layer = [None, None]
        self._prefill_buffer_released = [True, True]
        self._prefill_has_release = [False, False]

    def _invalidate_prefill_buffer(self, buffer_id: int) -> None:
        """Unmap the experts held in buffer ``buffer_id``'s slots, without a host sync: the
        empty slots (-1) are sent to a spare trailing entry of a copy of the table."""
        E = self.num_experts
        lo, hi = buffer_id * E, (buffer_id + 1) * E
        old = self.id_of_slot[lo:hi]
        sfi = self.slot_for_id.view(-1)
        n = sfi.numel()
        table = torch.cat([sfi, sfi.new_full((1,), -1)])
        table.index_fill_(0, torch.where(old >= 0, old, n).long(), -1)
        sfi.copy_(table[:n])
        old.fill_(-1)
        self.usage[lo:hi].zero_()

    def begin_prefill(self) -> None:
        if not self.prefill_overlap:
            return
        self._prefill_buffer_layer = [None, None]
        self._prefill_buffer_released = [True, True]
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.prefill_copy_stream.wait_event(ev)

    def prefetch_prefill_layer(self, layer_id: int) -> None:
        if not self.prefill_overlap or layer_id >= self.num_layers:
            return
        if layer_id < 0:
            raise ValueError(f"Invalid prefill layer id: {layer_id}")
        b = layer_id % 2
        if self._prefill_buffer_layer[b] == layer_id:
            return
        if self._prefill_buffer_layer[b] is not None:
            assert self._prefill_buffer_released[b], "prefill buffer reused before release"
        with torch.cuda.stream(self.prefill_copy_stream):
            if self._prefill_has_release[b]:
                self.prefill_copy_stream.wait_event(self.prefill_release_events[b])
            self._invalidate_prefill_buffer(b)
            for (per_layer, _), buf in zip(self.banks, self.prefill_bank_buffers):
                buf[b].copy_(per_layer[layer_id], non_blocking=True)
            self.prefill_ready_events[b].record(self.prefill_copy_stream)
        self._prefill_buffer_layer[b] = layer_id
        self._prefill_buffer_released[b] = False

    def wait_prefill_layer(self, layer_id: int) -> tuple[torch.Tensor, ...]:
        b = layer_id % 2
        assert self._prefill_buffer_layer[b] == layer_id, "layer was not prefetched"
        torch.cuda.current_stream(self.device).wait_event(self.prefill_ready_events[b])
        return tuple(buf[b] for buf in self.prefill_bank_buffers)

    def release_prefill_layer(self, layer_id: int) -> None:
        if not self.prefill_overlap:
            return
        b = layer_id % 2
        if self._prefill_buffer_layer[b] != layer_id:
            return
        self.prefill_release_events[b].record(torch.cuda.current_stream(self.device))
        self._prefill_has_release[b] = True
        self._prefill_buffer_released[b] = True
