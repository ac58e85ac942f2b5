"""Pin the CPU oracle against the golden vectors produced by the reference's own code."""

import numpy as np
import pytest
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


@pytest.mark.parametrize("stem", ["lru_ensure", "lru_ensure_pinned"])
def test_lru_ensure_matches_reference_kernel(stem):
    """Replays of the reference's lru_ensure (shift.py:698-777); the second fixture sets the
    pinned flag on some resident slots, which are then never chosen as victims."""
    for name, c in load_golden(stem).items():
        t = _replay_lru(c)
        pinned = c.get("pinned")
        for i in range(int(c["steps"])):
            out = slot_cache.lru_ensure(t, c[f"s{i}_ids"], int(c[f"s{i}_layer"]), pinned)
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


def test_hybrid_fetch_cap_edges():
    """The cap arithmetic at its ends: a fixed cap clamps to the misses, a zero cap fetches
    nothing, fraction 1.0 fetches every miss, and the bandwidth-matched split picks the
    integer neighbour of frac * M that balances the two sides."""
    assert slot_cache.hybrid_fetch_cap(5, 3, 0) == 3
    assert slot_cache.hybrid_fetch_cap(2, 3, 0) == 2
    assert slot_cache.hybrid_fetch_cap(7, 0, 0) == 0
    assert slot_cache.hybrid_fetch_cap(9, 0, 1 << 16) == 9
    assert slot_cache.hybrid_fetch_cap(0, 4, 30000) == 0
    # frac = 0.4, M = 10: F = 4 gives max(4 * 0.6, 6 * 0.4) = 2.4 vs F = 5: max(3.0, 2.0)
    assert slot_cache.hybrid_fetch_cap(10, 1 << 30, round(0.4 * (1 << 16))) == 4
    # frac = 0.45, M = 10: F = 4 -> max(2.2, 2.7) = 2.7, F = 5 -> max(2.75, 2.25) = 2.75
    assert slot_cache.hybrid_fetch_cap(10, 1 << 30, round(0.45 * (1 << 16))) == 4


def test_hybrid_ensure_all_hits_and_zero_cap():
    """Every routed expert resident: nothing fetched, usage bumped, recency set.  With a
    zero cap every miss comes back as -1 and the table keeps its mapping."""
    t = slot_cache.SlotTable(1, 8, 8)
    t.seed({0: list(range(8))})
    rec = np.zeros((1, 8), np.int64)
    ids = np.array([[0, 3], [5, 3]], np.int32)
    out, active, full = slot_cache.hybrid_ensure(t, rec, ids, 0, 4, 0, True)
    assert np.array_equal(out, t.slot_for_id[ids]) and full == 0 and t.num_indices == 0
    assert active.tolist() == [1, 0, 0, 1, 0, 1, 0, 0] and rec[0, 3] == t.step == 1
    t2 = slot_cache.SlotTable(1, 8, 4)
    before = t2.slot_for_id.copy()
    out2, _, full2 = slot_cache.hybrid_ensure(t2, np.zeros((1, 8), np.int64),
                                              np.array([[1, 2]], np.int32), 0, 0, 0, False)
    assert (out2 == -1).all() and full2 == 2 and t2.num_indices == 0
    assert np.array_equal(t2.slot_for_id, before)


@pytest.mark.parametrize("with_bias", [False, True])
def test_sigmoid_group_topk_matches_transformers_deepseek_v3(with_bias):
    """The DSV4 gate's restatement against a published implementation of the same routing:
    transformers 5.5's ``DeepseekV3MoE.route_tokens_to_experts`` (sigmoid, choice = score +
    correction bias, group score = sum of the group's two best choices, ``topk_group``
    groups kept, top-k of the kept experts, weights = unbiased scores renormalised and
    scaled) at configs[3]'s routing shape (256 experts, 8 groups, 4 kept, top-6, scale 2.5).
    That implementation fills dropped groups with 0.0 where this one uses -inf; the two
    agree whenever every kept choice score is positive, as here (sigmoid scores plus a
    non-negative bias)."""
    from types import SimpleNamespace

    moe = pytest.importorskip("transformers.models.deepseek_v3.modeling_deepseek_v3")
    T, E, G, TG, K, scale = 64, 256, 8, 4, 6, 2.5
    g = torch.Generator().manual_seed(11)
    logits = 2.0 * torch.randn(T, E, generator=g)
    bias = 0.02 * torch.rand(E, generator=g) if with_bias else torch.zeros(E)
    ns = SimpleNamespace(n_routed_experts=E, n_group=G, topk_group=TG, top_k=K,
                         norm_topk_prob=True, routed_scaling_factor=scale,
                         gate=SimpleNamespace(e_score_correction_bias=bias))
    ref_ids, ref_w = moe.DeepseekV3MoE.route_tokens_to_experts(ns, logits.clone())
    w, ids = routing.sigmoid_group_topk(logits, K, G, TG, scale, True,
                                        bias if with_bias else None)
    # the reference leaves its picks unsorted: compare per token, ordered by expert id
    o_ref = torch.argsort(ref_ids, dim=-1)
    o = torch.argsort(ids.long(), dim=-1)
    assert torch.equal(torch.gather(ref_ids, 1, o_ref), torch.gather(ids.long(), 1, o))
    torch.testing.assert_close(torch.gather(w, 1, o), torch.gather(ref_w, 1, o_ref),
                               rtol=1e-6, atol=0)


def test_dual_norm_merge_matches_transformers_gemma4_layer():
    """The Gemma merge's restatement against transformers 5.5's Gemma 4 decoder layer, whose
    MoE block ends: h = post_ffn_norm(post_ffn_norm_1(dense) + post_ffn_norm_2(experts));
    out = (residual + h) * layer_scalar, every step in bf16 tensors.  Their RMSNorm raises
    mean + eps to the power -1/2 where this one takes rsqrt, so a few elements may differ by
    one bf16 step."""
    g4 = pytest.importorskip("transformers.models.gemma4.modeling_gemma4")
    T, H, eps, scalar = 6, 2816, 1e-6, 0.5
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(21)
    a, b, x = (torch.randn(T, H, generator=g).to(bf) for _ in range(3))
    ws = [(1 + 0.1 * torch.randn(H, generator=g)).to(bf) for _ in range(3)]
    norms = []
    for w in ws:
        n = g4.Gemma4RMSNorm(H, eps=eps).to(bf)
        with torch.no_grad():
            n.weight.copy_(w)
        norms.append(n)
    with torch.no_grad():
        h = norms[2](norms[0](a) + norms[1](b))
        ref = x + h
        ref *= torch.tensor([scalar], dtype=bf)
    out = ffn.dual_norm_merge(a, b, x, *ws, eps, eps, eps, scalar)
    step = ref.float().abs().clamp(min=2 ** -10) * 2 ** -7  # two bf16 ulps of the value
    diff = (out.float() - ref.float()).abs()
    assert bool((diff <= step).all()), float(diff.max())
    assert float((diff > 0).float().mean()) < 0.01


def test_router_norm_pair_matches_transformers_gemma4_router():
    """The router norm pair's restatement against transformers 5.5's Gemma 4 layer: the
    router input is ``Gemma4TextRouter``'s norm (no weight) times its ``scale`` times
    hidden**-0.5, the routed input ``pre_feedforward_layernorm_2(x)``, each step in bf16
    tensors.  Their RMSNorm takes (mean + eps)**-0.5 where this one takes rsqrt, so a few
    elements may differ by one bf16 step."""
    g4 = pytest.importorskip("transformers.models.gemma4.modeling_gemma4")
    T, H, eps = 5, 2816, 1e-6
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(23)
    x = torch.randn(T, H, generator=g).to(bf)
    scale = (1 + 0.1 * torch.randn(H, generator=g)).to(bf)
    w2 = (1 + 0.1 * torch.randn(H, generator=g)).to(bf)
    plain = g4.Gemma4RMSNorm(H, eps=eps, with_scale=False)
    pre2 = g4.Gemma4RMSNorm(H, eps=eps).to(bf)
    with torch.no_grad():
        pre2.weight.copy_(w2)
        ref_router = plain(x) * scale * H ** -0.5
        ref_routed = pre2(x)
    router, routed = ffn.router_norm_pair(x, torch.ones(H, dtype=bf), w2, scale, eps,
                                          H ** -0.5)
    for got, ref in ((router, ref_router), (routed, ref_routed)):
        diff = (got.float() - ref.float()).abs()
        assert bool((diff <= ref.float().abs() * 2 ** -7 + 1e-30).all()), float(diff.max())
        assert float((diff > 0).float().mean()) < 0.01


def test_nvfp4_dequantize_matches_vllm_emulation():
    """The NVFP4 decoder's restatement (two e2m1 codes per byte, low nibble first; e4m3 scale
    per 16 elements; fp32 global) against vLLM 0.22's CPU emulation of the ModelOpt format
    (``nvfp4_emulation_utils.dequantize_to_dtype``, linear scale layout).  vLLM multiplies
    the scale by the global before the code, this build the code by the scale first (exact)
    and then the global, so values agree to one fp32 rounding and exactly after bf16."""
    ne = pytest.importorskip("vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils")
    from oracle import nvfp4 as onv

    g = torch.Generator().manual_seed(3)
    w = torch.randn(256, 512, generator=g) * 0.02
    w[0, :16] = torch.tensor([0.0, -0.0, 1e-9, -1e-9] * 4)  # zeros and codes that round to 0
    packed, scale, glob = onv.quantize(w)
    assert torch.equal(glob, glob[:1].expand_as(glob))  # one global for the whole tensor
    mine = onv.dequantize(packed, scale, glob)
    theirs = ne.dequantize_to_dtype(packed, scale.view(torch.uint8), glob[:1], torch.float32,
                                    16, swizzle=False)
    torch.testing.assert_close(mine, theirs, rtol=2 ** -23, atol=0)
    assert torch.equal(mine.to(torch.bfloat16), theirs.to(torch.bfloat16))


def test_ds_fp4_dequantize_matches_transformers_mxfp4():
    """The DS-FP4 reading (two e2m1 codes per byte, low nibble first, e8m0 scale 2^(b - 127)
    per 32 elements -- the OCP MX FP4 layout) against transformers 5.5's MXFP4 converter for
    gpt-oss checkpoints (``integrations.mxfp4.convert_moe_packed_tensors``), bit for bit on
    every code and on scales over 2^-17 .. 2^8."""
    mx = pytest.importorskip("transformers.integrations.mxfp4")
    from oracle import nvfp4 as onv

    rows, K = 48, 256
    g = torch.Generator().manual_seed(29)
    packed = torch.randint(0, 256, (rows, K // 2), generator=g, dtype=torch.uint8)
    assert len(torch.unique(packed)) == 256  # every pair of codes occurs
    e8 = torch.randint(110, 136, (rows, K // 32), generator=g, dtype=torch.uint8)
    mine = onv.dequantize_ds_fp4(packed, e8)
    theirs = mx.convert_moe_packed_tensors(packed.view(1, rows, K // 32, 16),
                                           e8.view(1, rows, K // 32), dtype=torch.float32)
    assert torch.equal(mine, theirs.transpose(1, 2)[0])
