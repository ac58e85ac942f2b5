"""Expert-slot table restatements (numpy, test infrastructure only).

The slot table is the reference's ``OffloadMoeCache`` device state
(backends/freetoken_tideway/freetoken/moe/offload_cache.py:143-173):

* ``slot_for_id``  int32 [L*E]  flat id (layer*E + expert) -> slot, -1 if absent
* ``id_of_slot``   int32 [S]    slot -> flat id, -1 if empty
* ``usage``        int64 [S]    last step that touched the slot
* ``step``         int64 scalar step counter
* ``evict_slots`` / ``src_indices`` int32 [E], ``num_indices`` int64 [1] -- pending copies
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

USAGE_MAX = np.iinfo(np.int64).max


@dataclass
class SlotTable:
    num_layers: int
    num_experts: int
    num_slots: int
    slot_for_id: np.ndarray = field(init=False)
    id_of_slot: np.ndarray = field(init=False)
    usage: np.ndarray = field(init=False)
    step: int = field(init=False, default=0)
    evict_slots: np.ndarray = field(init=False)
    src_indices: np.ndarray = field(init=False)
    num_indices: int = field(init=False, default=0)
    stats: np.ndarray = field(init=False)

    def __post_init__(self) -> None:
        self.slot_for_id = np.full(self.num_layers * self.num_experts, -1, np.int32)
        self.id_of_slot = np.full(self.num_slots, -1, np.int32)
        self.usage = np.zeros(self.num_slots, np.int64)
        self.evict_slots = np.zeros(self.num_experts, np.int32)
        self.src_indices = np.zeros(self.num_experts, np.int32)
        self.stats = np.zeros(4, np.int64)

    def copy(self) -> "SlotTable":
        t = SlotTable(self.num_layers, self.num_experts, self.num_slots)
        for k in ("slot_for_id", "id_of_slot", "usage", "evict_slots", "src_indices", "stats"):
            setattr(t, k, getattr(self, k).copy())
        t.step, t.num_indices = self.step, self.num_indices
        return t

    def seed(self, layer_experts: dict[int, list[int]], slots: list[int] | None = None) -> None:
        """Place experts in slots (untimed initial residency); usage stays 0."""
        it = iter(slots if slots is not None else range(self.num_slots))
        for layer, experts in layer_experts.items():
            for e in experts:
                s = next(it)
                fid = layer * self.num_experts + e
                self.id_of_slot[s] = fid
                self.slot_for_id[fid] = s


def lru_ensure(table: SlotTable, ids: np.ndarray, layer_id: int,
               pinned: np.ndarray | None = None) -> np.ndarray:
    """Make one layer's routed experts resident and return the ids rewritten to slots.

    Restates the sequential-argmin LRU of the reference's vendored ``lru_ensure``
    (backends/freetoken_tideway/freetoken/moe/shift.py:698-777, pinned mask all zero by
    default), which ``ensure_experts`` calls with ``id_base = layer * E``
    (backends/.../moe/offload_kernels.py:19-51):

    1. ``step += 1``; hits set ``usage[slot] = step``.
    2. First-occurrence misses are ranked by ascending flat id (shift.py:708-713).
    3. For miss rank i: the victim is argmin ``usage`` over slots not touched this step
       (and not pinned), the first index winning ties; its old id is unmapped, the new id
       mapped, ``evict_slots[i] = victim``, ``src_indices[i] = expert`` (layer-local).
    4. ``num_indices = #misses``; stats += (#unique, #misses, 1).

    Negative ids (padding rows) are passed through as -1 and take no part (the reference
    would index ``slot_for_id[id_base - 1]`` for them; this build defines them as inert).
    """
    E = table.num_experts
    base = layer_id * E
    flat = np.asarray(ids, np.int64).reshape(-1)
    valid = flat >= 0
    q = np.where(valid, flat + base, -1)
    table.step += 1
    step = table.step
    s = np.where(valid, table.slot_for_id[np.where(valid, q, 0)], -1).astype(np.int64)
    hit = valid & (s >= 0)
    miss = valid & (s < 0)
    table.usage[s[hit]] = step
    uniq = np.unique(q[valid])
    missing = np.unique(q[miss])  # ascending flat ids == the reference's miss rank
    M = len(missing)
    table.num_indices = M
    out = np.where(hit, s, -1)
    if M:
        u = table.usage.copy()
        u[u == step] = USAGE_MAX
        if pinned is not None:
            u[np.asarray(pinned) != 0] = USAGE_MAX
        for i, e in enumerate(missing):
            victim = int(np.argmin(u))  # first index among equal minima
            old = int(table.id_of_slot[victim])
            if old >= 0:
                table.slot_for_id[old] = -1
            table.id_of_slot[victim] = e
            table.slot_for_id[e] = victim
            table.usage[victim] = step
            table.evict_slots[i] = victim
            table.src_indices[i] = e - base
            out[miss & (q == e)] = victim
            u[victim] = USAGE_MAX
    table.stats[:3] += (len(uniq), M, 1)
    return out.astype(np.int32).reshape(np.shape(ids))


def hybrid_fetch_cap(num_missing: int, max_fetch: int, frac_q16: int) -> int:
    """Fetches allowed this step: ``max_fetch``, or with ``frac_q16`` > 0 the integer F near
    ``frac * M`` minimising max(F * (1 - frac), (M - F) * frac) in Q16 fixed point (the
    reference computes this in-kernel, backends/.../moe/offload_kernels.py:350-360, and in
    its CPU mirror, :165-169)."""
    if frac_q16 > 0:
        m, q = num_missing, 1 << 16
        lo = (m * frac_q16) >> 16
        cost = lambda f: max(f * (q - frac_q16), (m - f) * frac_q16)  # noqa: E731
        max_fetch = lo if cost(lo) <= cost(lo + 1) else lo + 1
    return min(num_missing, max_fetch)


def hybrid_ensure(table: SlotTable, recency: np.ndarray, ids: np.ndarray, layer_id: int,
                  max_fetch: int, frac_q16: int, by_recency: bool = True
                  ) -> tuple[np.ndarray, np.ndarray, int]:
    """Capped-fetch LRU of the hybrid backend; returns (ids rewritten, active mask [E],
    pre-cap miss count).  ``recency`` is the [L, E] int64 per-expert recency table.

    Restates ``_ensure_experts_hybrid_cpu`` (backends/.../moe/offload_kernels.py:135-195,
    the reference's CPU mirror of its kernel at :295-415):

    1. ``step += 1``; the active set is this step's distinct experts; hits set
       ``usage[slot] = step``.
    2. The misses are ordered by (recency descending, id ascending) -- or by id when not
       ``by_recency`` -- and only the first ``hybrid_fetch_cap`` of them are fetched.
    3. Fetch i takes the victim argmin (usage, slot) over the slots not touched this step,
       as ``lru_ensure`` does; ``num_indices`` = fetches, ``num_missing_full`` = misses.
    4. ``by_recency``: every active expert's recency becomes ``step``.
    5. ids are rewritten to slots; misses left unfetched become -1 (computed elsewhere).
    """
    E = table.num_experts
    base = layer_id * E
    flat = np.asarray(ids, np.int64).reshape(-1)
    active = np.zeros(E, np.int32)
    active[np.unique(flat[(flat >= 0) & (flat < E)])] = 1
    table.step += 1
    step = table.step
    experts = np.flatnonzero(active)
    slots = table.slot_for_id[base + experts]
    table.usage[slots[slots >= 0]] = step
    missing = experts[slots < 0]
    if by_recency:
        rec = recency[layer_id]
        missing = np.array(sorted(missing.tolist(), key=lambda e: (-int(rec[e]), e)), np.int64)
    num_fetch = hybrid_fetch_cap(len(missing), max_fetch, frac_q16)
    table.num_indices = num_fetch
    if num_fetch:
        u = table.usage.copy()
        u[u == step] = USAGE_MAX
        for i in range(num_fetch):
            e = int(missing[i])
            victim = int(np.argmin(u))  # first index among equal minima
            old = int(table.id_of_slot[victim])
            if old >= 0:
                table.slot_for_id[old] = -1
            table.id_of_slot[victim] = base + e
            table.slot_for_id[base + e] = victim
            table.usage[victim] = step
            table.evict_slots[i] = victim
            table.src_indices[i] = e
            u[victim] = USAGE_MAX
    if by_recency:
        recency[layer_id, experts] = step
    valid = (flat >= 0) & (flat < E)
    out = np.where(valid, table.slot_for_id[base + np.where(valid, flat, 0)], -1)
    return out.astype(np.int32).reshape(np.shape(ids)), active, len(missing)


def materialize_layer(table: SlotTable, layer_id: int) -> None:
    """Map layer ``layer_id``'s experts onto slots [0, E) for a whole-layer copy.

    Restates ``_materialize_layer_kernel`` (backends/.../moe/offload_kernels.py:256-292).
    """
    E = table.num_experts
    base = layer_id * E
    old = table.id_of_slot.copy()
    same = (old >= base) & (old < base + E)
    table.id_of_slot[same] = -1
    table.usage[same] = 0
    low = np.arange(table.num_slots) < E
    clear = low & (old >= 0) & ~same
    table.slot_for_id[old[clear]] = -1
    table.step += 1
    off = np.arange(E)
    table.id_of_slot[off] = base + off
    table.slot_for_id[base + off] = off
    table.usage[off] = table.step
    table.evict_slots[:E] = off
    table.src_indices[:E] = off
    table.num_indices = E


def reset(table: SlotTable) -> None:
    """Restates ``_reset_cache_kernel`` (backends/.../moe/offload_kernels.py:233-253)."""
    table.slot_for_id[:] = -1
    table.id_of_slot[:] = -1
    table.usage[:] = 0
    table.step = 0
    table.num_indices = 0


def prefill_hit_compact(table: SlotTable, layer_id: int, buffer_id: int
                        ) -> tuple[np.ndarray, np.ndarray, int]:
    """Compact a layer's resident experts outside the double buffer into gather lists.

    Restates ``_prefill_hit_compact_kernel`` (backends/.../moe/offload_kernels.py:418-436):
    hit = slot >= 2E; dst = buffer_id*E + expert, src = slot, in expert order.
    """
    E = table.num_experts
    row = table.slot_for_id[layer_id * E:(layer_id + 1) * E]
    hits = np.flatnonzero(row >= 2 * E)
    return (buffer_id * E + hits).astype(np.int32), row[hits].astype(np.int32), len(hits)


def copy_rows(dst_bank: np.ndarray, src_bank: np.ndarray, evict_slots: np.ndarray,
              src_indices: np.ndarray, num: int) -> None:
    """``bank[evict_slots[i]] = host_layer[src_indices[i]]`` for i < num.

    Restates what ``copy_missing`` asks of ``fast_index_copy_multi_jit``
    (backends/.../moe/offload_cache.py:1024-1054).
    """
    for i in range(num):
        dst_bank[evict_slots[i]] = src_bank[src_indices[i]]
