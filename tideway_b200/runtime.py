"""B200 counterpart of Tideway's offload manager and its installer.

Mirrors ``TidewayOffload`` (src/tideway/offload/runtime.py:291-1030) and ``install``
(src/tideway/offload/install.py:138-283) for the path this package covers: the manager
takes ownership of the cache's ``ensure_experts`` / ``copy_missing`` entry points
(runtime.py:374-380) and the layers' ``_prefill_routed`` is patched to ``manager.prefill``
(install.py:187-236), with the same signatures:

* ``ensure(layer, expert_ids)`` (runtime.py:583) -- make one layer's routed experts
  resident and rewrite ``expert_ids`` into slot ids in place;
* ``prefill(layer, hidden, weights, ids)`` (runtime.py:882) -- run one layer's routed
  experts over a prefill chunk from the layer's whole-layer buffer, streaming the next
  layer in behind it;
* ``begin_prefill()``, ``load_layer(layer)``, ``reset_stats()``, ``snapshot()``,
  ``close()``.

What differs, by design: the reference's manager keeps a bounded RAM tier over an SSD
reader and a host-side LRU, so every ensure reads the routed ids back to the host
(runtime.py:598) before it can plan its copies.  Here every expert row lives in pinned
host banks and the slot LRU runs on the device, so ``ensure`` only enqueues the table
update and the copy of the missing rows -- no host synchronisation, and a decode step built
on it is one CUDA graph.  Prefill streams whole layers into the two layer buffers at slots
[0, 2E) on a copy stream (buffer = layer % 2), ordered by events against the GEMM that
reads them.  RAM/SSD tiering, write-back and phase policies are not part of this path.
"""

from __future__ import annotations

import time

import numpy as np
import torch

_ABSENT = object()


class TidewayOffload:
    """Owns the slot cache's entry points; see the module docstring."""

    def __init__(self, cache):
        if not getattr(cache, "banks", None):
            raise RuntimeError("register the host banks first (cache.set_bank_sources)")
        if not getattr(cache, "prefill_overlap", False):
            raise ValueError("the manager streams prefill layers through the double buffer: "
                             "construct the cache with prefill_overlap=True")
        self.cache = cache
        self.E, self.L = int(cache.num_experts), int(cache.num_layers)
        self.DOUBLE = 2 * self.E
        # the cache's own implementations, called by the manager
        self._ensure = cache.ensure_experts
        self._copy_missing = cache.copy_missing
        self._restore = [(name, vars(cache).get(name, _ABSENT))
                         for name in ("ensure_experts", "copy_missing")]
        cache.ensure_experts = self.ensure
        cache.copy_missing = lambda: None   # ensure moves the rows itself
        self.closed = False
        self.trace, self.trace_marks, self.prefill_hist = None, [], None
        self.reader = None  # the checkpoint reader install() read the host banks with
        self.reset_stats()

    def reset_stats(self) -> None:
        self.stats = {"ensure_calls": 0, "prefill_layers": 0, "prefill_loads": 0}

    # ------------------------------------------------------------ decode
    def ensure(self, layer, expert_ids) -> None:
        """Rewrite ``expert_ids`` (one layer's routed expert ids, int32) into slot ids in
        place; the missing rows are copied from the host banks on the same stream."""
        self._ensure(int(layer), expert_ids)
        self._copy_missing()
        self.stats["ensure_calls"] += 1

    # ------------------------------------------------------------ prefill
    def begin_prefill(self) -> None:
        self.cache.begin_prefill()

    def load_layer(self, layer) -> None:
        """Stream layer ``layer`` (an index) into its buffer; a no-op past the last layer
        or when the buffer already holds it."""
        layer = int(layer)
        if layer < self.L:
            self.cache.prefetch_prefill_layer(layer)
            self.stats["prefill_loads"] += 1

    def prefill(self, layer, hidden, weights, ids):
        """One layer's routed experts over a prefill chunk (``ids`` are expert ids)."""
        number = int(layer.layer_id)
        if number == 0:
            self.begin_prefill()
        self.load_layer(number)
        if self.prefill_hist is not None:
            flat = ids.reshape(-1).long()
            self.prefill_hist.scatter_add_(0, flat.clamp(min=0) + number * self.E,
                                           (flat >= 0).long())
        views = self.cache.wait_prefill_layer(number)
        result = layer._expert_gemm(self.cache, hidden, weights, ids, views=views, n=self.E,
                                    alphas=self.cache.alphas_for_layer(number),
                                    is_prefill=True)
        self.cache.release_prefill_layer(number)
        self.load_layer(number + 1)   # the next layer's upload overlaps this layer's GEMM
        self.stats["prefill_layers"] += 1
        return result

    # ------------------------------------------------------------ tracing
    def enable_trace(self, steps: int = 4096, width: int = 8) -> None:
        """Record decode routes (the cache's device ring, ``steps`` decode steps of rows of
        up to ``width`` ids) and prefill expert counts (runtime.py:1037-1041)."""
        import torch

        self.trace = self.cache.enable_route_trace(steps, width)
        self.trace_marks = []
        self.prefill_hist = torch.zeros(self.L * self.E, dtype=torch.int64,
                                        device=self.cache.slot_for_id.device)

    def mark_case(self) -> None:
        """Mark a request boundary at the current trace position (synchronises)."""
        if self.trace is not None:
            self.trace_marks.append(int(self.trace.pos.item()))

    def dump_trace(self, path):
        """Write routes, request marks and prefill expert counts to an NPZ file with the
        reference's keys (runtime.py:1043-1066); decode rows are padded with -1."""
        if self.trace is None:
            return None
        layers, ids, total = self.trace.read()
        hist = self.prefill_hist.cpu().numpy()
        np.savez_compressed(
            path, decode_layers=layers.astype(np.int16), decode_ids=ids.astype(np.int16),
            case_marks=np.array(self.trace_marks, dtype=np.int64), prefill_hist=hist,
            experts_per_layer=self.E, layers_total=self.L, gpu_slots=int(self.cache.cache_size),
            host_rows=self.L * self.E)
        return dict(path=str(path), decode_records=int(len(layers)),
                    decode_records_total=total, prefill_accesses=int(hist.sum()))

    # ------------------------------------------------------------ audits
    def verify_payload(self, reader=None) -> dict:
        """Check every resident copy (the reference's audit, runtime.py:1068-1109): with a
        checkpoint reader (this call's, or the one install() read the banks with), every
        expert's host bank rows against its checkpoint bytes; then every occupied slot's
        bytes against its host rows (``cache.verify_payload``).  A mismatch raises
        AssertionError naming the tier, the expert (layer * E + e) and the bank.  Synchronises;
        reads the whole checkpoint when a reader is used."""
        start = time.monotonic()
        reader = reader if reader is not None else self.reader
        checked = 0
        if reader is not None:
            sources = self.cache.bank_sources
            for expert in range(self.L * self.E):
                layer, e = divmod(expert, self.E)
                views = reader.geo.host_views(torch.from_numpy(reader.read(expert)))
                for name, want in views.items():
                    got = sources[name][layer][e]
                    if not torch.equal(got.contiguous().view(torch.uint8).flatten(),
                                       want.contiguous().view(torch.uint8).flatten()):
                        raise AssertionError(("host", expert, name))
                checked += 1
        audit = self.cache.verify_payload(raise_on_mismatch=False)
        if audit["mismatches"]:
            slot, layer, e, name = audit["mismatches"][0]
            raise AssertionError(("GPU", layer * self.E + e, name))
        checked += audit["rows"]
        return dict(all_resident_payloads_equal=True, checked_copies=checked,
                    wall_s=time.monotonic() - start)

    # ------------------------------------------------------------ reporting / teardown
    def snapshot(self) -> dict:
        out = dict(self.stats)
        out.update(layers=self.L, experts=self.E, slots=int(self.cache.cache_size),
                   double_buffer=self.DOUBLE)
        return out

    def close(self) -> None:
        """Give the cache its own entry points back."""
        if self.closed:
            return
        for name, value in self._restore:
            if value is _ABSENT:
                vars(self.cache).pop(name, None)
            else:
                setattr(self.cache, name, value)
        self.closed = True


class Session:
    """What ``install`` changed, and how to undo it (install.py's session)."""

    def __init__(self, manager: TidewayOffload, classes: tuple, restore: list):
        self.manager, self.classes, self.restore = manager, classes, restore

    def uninstall(self) -> None:
        for klass, name, original in reversed(self.restore):
            if original is _ABSENT:
                if name in vars(klass):
                    delattr(klass, name)
            else:
                setattr(klass, name, original)
        self.restore = []
        self.manager.close()


# The reference installer's arms (src/tideway/offload/install.py:108-109): the bounded pager
# and the static GPU-core layout.  Both map to this manager: its host tier holds every expert
# row in pinned memory and its decode is device-side, as the hybrid arm's is.
ARMS = ("tideway", "tideway_hybrid")

# The reference installer's tier options (install.py:82-101) and their defaults.  Those that
# select a tier or policy this path does not have must stay at their default; the others
# tune its RAM tier's write-back and host-side guards, and have nothing to act on here.
_TIER_FEATURES = {"prior": None, "core_rows": None, "ssd_prefetch_rows": 0,
                  "volatile_mirror_rows": 0, "phase_policy": None}
_TIER_TOGGLES = {"writeback": True, "seed_tail": False, "prefill_guard": False,
                 "writeback_ahead": "auto", "dma_decode": True, "kernel_guard": True,
                 "batch_prefill": True}


def install(cache, layer_classes=None, *, geo=None, host_rows=None, reader=None,
            arm: str = "tideway", **tier_options) -> Session:
    """Build the manager over ``cache`` and route the layers' prefill through it.

    ``layer_classes`` are the MoE layer classes to patch (default: this package's
    ``OffloadMoELayer``); as in the reference, the patch is on the class, so every layer of
    those classes prefills through this manager until ``Session.uninstall()``.

    The reference's keywords are taken as it takes them (``install(cache, geo=...,
    host_rows=..., reader=..., arm=..., ...)``): ``arm`` must name one of its arms
    (``ValueError`` otherwise); ``reader`` must have been built from ``geo``
    (``ValueError``); a cache without host banks gets them read through ``reader``
    (``geometry.CheckpointReader.layer_banks``, pinned); ``host_rows`` too small for the
    experts the slot cache cannot hold would need the SSD tier, and a non-default SSD,
    mirror, prior, core-row or phase-policy option a tier this path does not have: both raise
    ``NotImplementedError``.  The write-back and guard toggles are accepted and have nothing
    to act on (no RAM tier to write back to).
    """
    from .moe_layer import OffloadMoELayer

    if arm not in ARMS:
        raise ValueError(f"unknown arm {arm!r}; the arms are {list(ARMS)}")
    unknown = set(tier_options) - set(_TIER_FEATURES) - set(_TIER_TOGGLES)
    if unknown:
        raise TypeError(f"install() got unexpected keyword arguments {sorted(unknown)}")
    for name, default in _TIER_FEATURES.items():
        value = tier_options.get(name, default)
        if value != default and not (name == "phase_policy" and value in ("off", {})):
            raise NotImplementedError(f"install({name}={value!r}): that tier is not on the "
                                      "B200 path (every expert row is in pinned host memory)")
    if reader is not None and geo is not None:
        rg = getattr(reader, "geo", None)
        if rg is not geo and getattr(rg, "name", None) != getattr(geo, "name", None):
            raise ValueError("the reader was built from another checkpoint geometry than geo")
    if host_rows is not None and geo is not None:
        if int(host_rows) + int(cache.cache_size) < int(geo.total_experts):
            raise NotImplementedError(
                f"host_rows={host_rows} + cache_size={cache.cache_size} < "
                f"{geo.total_experts} experts: the rest would live on the SSD tier, which is "
                "not on the B200 path")
    if not getattr(cache, "banks", None) and reader is not None:
        layers = range(cache.num_layers)
        per_layer = [reader.layer_banks(layer, pin=True) for layer in layers]
        cache.set_bank_sources({name: [banks[name] for banks in per_layer]
                                for name in per_layer[0]})

    classes = tuple(layer_classes or (OffloadMoELayer,))
    manager = TidewayOffload(cache)
    manager.reader = reader
    restore = []
    try:
        for klass in classes:
            restore.append((klass, "_prefill_routed", vars(klass).get("_prefill_routed",
                                                                       _ABSENT)))

            def replacement(layer, hidden, weights, ids, *, _manager=manager):
                return _manager.prefill(layer, hidden, weights, ids)

            klass._prefill_routed = replacement
        if getattr(cache.ensure_experts, "__self__", None) is not manager:
            raise RuntimeError("cache.ensure_experts is not bound to the installed manager")
    except BaseException:
        Session(manager, classes, restore).uninstall()
        raise
    return Session(manager, classes, restore)
