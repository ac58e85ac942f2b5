"""Pin the CPU oracle against the golden vectors produced by the reference's own code."""

import numpy as np
import torch

from oracle import ffn, routing, slot_cache
from tests.conftest import load_golden


def canonical_topk(w: np.ndarray, ids: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Order each row by (weight descending, id ascending).

    ``torch.topk`` on the CPU leaves equal values in an implementation-defined order
    (measured: about half of tied pairs come out higher-id first), so the reference
    router's order among exactly tied probabilities is not part of its contract.  This
    build breaks ties toward the lower id; comparisons canonicalise both sides.
    """
    order = np.lexsort((ids, -w), axis=-1)
    return np.take_along_axis(w, order, -1), np.take_along_axis(ids, order, -1)


def test_softmax_topk_matches_reference_fused_topk():
    for name, c in load_golden("fused_topk").items():
        logits = torch.from_numpy(c["logits"])
        if bool(c["is_bf16"]):
            logits = logits.to(torch.bfloat16)
        ntp = int(c["ntp"])
        w, ids = routing.softmax_topk(logits, int(c["K"]), bool(c["renorm"]),
                                      None if ntp < 0 else ntp)
        if name != "bf16_logits":  # fp32 logits: no exact ties, exact order
            assert np.array_equal(ids.numpy(), c["ids"]), name
        w_o, ids_o = canonical_topk(w.numpy(), ids.numpy())
        w_r, ids_r = canonical_topk(c["w"], c["ids"])
        assert np.array_equal(ids_o, ids_r), name
        np.testing.assert_allclose(w_o, w_r, rtol=1e-6, atol=1e-7, err_msg=name)


def test_gemma_topk_matches_reference_kernel():
    for name, c in load_golden("gemma_routing").items():
        w, ids, priv = routing.gemma_topk(torch.from_numpy(c["logits"]),
                                          torch.from_numpy(c["scale"]), int(c["K"]))
        assert np.array_equal(ids.numpy(), c["ids"]), name
        assert np.array_equal(priv.numpy(), c["private"]), name
        np.testing.assert_allclose(w.numpy(), c["w"], rtol=2e-6, atol=1e-7, err_msg=name)


def _replay_lru(c):
    L, E, S = int(c["L"]), int(c["E"]), int(c["S"])
    t = slot_cache.SlotTable(L, E, S)
    t.slot_for_id[:] = c["init_slot_of_id"]
    t.id_of_slot[:] = c["init_id_of_slot"]
    return t


def test_lru_ensure_matches_reference_kernel():
    for name, c in load_golden("lru_ensure").items():
        t = _replay_lru(c)
        for i in range(int(c["steps"])):
            out = slot_cache.lru_ensure(t, c[f"s{i}_ids"], int(c[f"s{i}_layer"]))
            n = int(c[f"s{i}_num"])
            assert np.array_equal(out, c[f"s{i}_out"]), (name, i)
            assert t.num_indices == n, (name, i)
            assert np.array_equal(t.evict_slots[:n], c[f"s{i}_dst"]), (name, i)
            assert np.array_equal(t.src_indices[:n], c[f"s{i}_src"]), (name, i)
            assert np.array_equal(t.slot_for_id, c[f"s{i}_slot_of_id"]), (name, i)
            assert np.array_equal(t.id_of_slot, c[f"s{i}_id_of_slot"]), (name, i)
            assert np.array_equal(t.usage, c[f"s{i}_usage"]), (name, i)
            assert t.step == int(c[f"s{i}_step"]), (name, i)
        assert np.array_equal(t.stats[:3], c["stats"][:3]), name


def test_hybrid_ensure_matches_reference_mirror():
    """The capped-fetch LRU restatement equals the reference's own CPU mirror
    (offload_kernels.py:135-195) step for step: rewritten ids, fetch lists, caps, recency,
    active mask and every table tensor."""
    for name, c in load_golden("hybrid_ensure").items():
        t = _replay_lru(c)
        rec = np.zeros((int(c["L"]), int(c["E"])), np.int64)
        for i in range(int(c["steps"])):
            out, active, full = slot_cache.hybrid_ensure(
                t, rec, c[f"s{i}_ids"], int(c[f"s{i}_layer"]), int(c["max_fetch"]),
                int(c["frac_q16"]), bool(c["by_recency"]))
            n = int(c[f"s{i}_num"])
            assert np.array_equal(out, c[f"s{i}_out"]), (name, i)
            assert t.num_indices == n and full == int(c[f"s{i}_num_full"]), (name, i)
            assert np.array_equal(t.evict_slots[:n], c[f"s{i}_dst"]), (name, i)
            assert np.array_equal(t.src_indices[:n], c[f"s{i}_src"]), (name, i)
            assert np.array_equal(t.slot_for_id, c[f"s{i}_slot_of_id"]), (name, i)
            assert np.array_equal(t.id_of_slot, c[f"s{i}_id_of_slot"]), (name, i)
            assert np.array_equal(t.usage, c[f"s{i}_usage"]), (name, i)
            assert np.array_equal(rec, c[f"s{i}_recency"]), (name, i)
            assert np.array_equal(active, c[f"s{i}_active"]), (name, i)
            assert t.step == int(c[f"s{i}_step"]), (name, i)


def test_moe_align_docstring_example():
    c = load_golden("moe_align")["docstring"]
    sorted_ids, blocks, npad = ffn.moe_align_block_size(c["topk_ids"], int(c["block_size"]),
                                                        int(c["num_experts"]))
    assert np.array_equal(sorted_ids, c["sorted_ids"])
    assert npad == 16
    assert blocks.tolist() == [1, 2, 3, 4]


def test_slot_table_bijection_after_random_traffic():
    """Host-side invariant the reference audits (src/tideway/offload/native_verify.py:13-41)."""
    rng = np.random.default_rng(7)
    t = slot_cache.SlotTable(6, 32, 64)
    for it in range(200):
        layer = it % 6
        slot_cache.lru_ensure(t, rng.integers(0, 32, size=(4, 4)), layer)
        mapped = np.flatnonzero(t.slot_for_id >= 0)
        assert np.array_equal(t.id_of_slot[t.slot_for_id[mapped]], mapped)
        occ = np.flatnonzero(t.id_of_slot >= 0)
        assert np.array_equal(t.slot_for_id[t.id_of_slot[occ]], occ)
