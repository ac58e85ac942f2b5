"""GPU parity: every CUDA entry point against the CPU oracle (B200 only).

Tolerances:
* integer work (routing ids, slot tables, permutations): bit-exact.
* router weights: fp32, rtol 1e-5.
* bf16 outputs (norms, expert FFN): max|gpu - oracle| / max|oracle| <= 2e-2 (the
  benchmark's bound against an fp32-accumulated reference); typically ~4e-3 (bf16 ulp).
"""

import numpy as np
import pytest
import torch

from oracle import ffn as off
from oracle import nvfp4 as onv
from oracle import routing as orouting
from oracle import slot_cache as osc
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

DEV = "cuda"
RTOL_BF16 = 2e-2


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


def _canon(w: np.ndarray, ids: np.ndarray):
    order = np.lexsort((ids, -w), axis=-1)
    return np.take_along_axis(w, order, -1), np.take_along_axis(ids, order, -1)


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tideway_b200

    tideway_b200.load()


# ---------------------------------------------------------------- routing

def test_softmax_topk_golden():
    from tideway_b200 import ops

    for name, c in load_golden("fused_topk").items():
        logits = torch.from_numpy(c["logits"])
        if bool(c["is_bf16"]):
            logits = logits.to(torch.bfloat16)
        ntp = int(c["ntp"])
        ntp_t = None if ntp < 0 else torch.tensor([ntp], device=DEV)
        w, ids = ops.softmax_topk(logits.to(DEV), int(c["K"]), bool(c["renorm"]), ntp_t)
        w, ids = w.cpu().numpy(), ids.cpu().numpy()
        if name != "bf16_logits":
            assert np.array_equal(ids, c["ids"]), name
        wg, ig = _canon(w, ids)
        wr, ir = _canon(c["w"], c["ids"])
        assert np.array_equal(ig, ir), name
        np.testing.assert_allclose(wg, wr, rtol=1e-5, atol=1e-7, err_msg=name)


@pytest.mark.parametrize("T,E,K,renorm", [(64, 128, 8, True), (1, 128, 8, True),
                                          (256, 256, 6, False), (4096, 128, 8, True),
                                          (33, 16, 2, True)])
def test_softmax_topk_random(T, E, K, renorm):
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T * 7 + E)
    logits = torch.randn(T, E, generator=g) * 3
    w, ids = ops.softmax_topk(logits.to(DEV), K, renorm)
    wr, ir = orouting.softmax_topk(logits, K, renorm)
    assert np.array_equal(ids.cpu().numpy(), ir.numpy())
    np.testing.assert_allclose(w.cpu().numpy(), wr.numpy(), rtol=1e-5, atol=1e-7)


def test_gemma_topk_golden():
    from tideway_b200 import ops

    for name, c in load_golden("gemma_routing").items():
        w, ids, priv = ops.gemma_topk(torch.from_numpy(c["logits"]).to(DEV),
                                      torch.from_numpy(c["scale"]).to(DEV), int(c["K"]))
        assert np.array_equal(ids.cpu().numpy(), c["ids"]), name
        assert np.array_equal(priv.cpu().numpy(), c["private"]), name
        np.testing.assert_allclose(w.cpu().numpy(), c["w"], rtol=1e-5, atol=1e-7, err_msg=name)


@pytest.mark.parametrize("T", [1, 16, 128, 256])
def test_sigmoid_group_topk(T):
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T)
    logits = torch.randn(T, 256, generator=g)
    bias = torch.randn(256, generator=g) * 0.1
    for b in (None, bias):
        w, ids = ops.sigmoid_group_topk(logits.to(DEV), 6, 8, 4, 2.5, True,
                                        None if b is None else b.to(DEV))
        wr, ir = orouting.sigmoid_group_topk(logits, 6, 8, 4, 2.5, True, b)
        assert np.array_equal(ids.cpu().numpy(), ir.numpy())
        np.testing.assert_allclose(w.cpu().numpy(), wr.numpy(), rtol=1e-5, atol=1e-6)


def test_router_logits():
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(11)
    # T >= 128 runs the tensor-core kernel (E up to 256, any T tail); smaller T the CUDA cores
    for T, H, E in ((4, 1024, 16), (64, 2048, 128), (33, 2816, 128), (128, 4096, 256),
                    (300, 2816, 128), (2048, 2816, 128), (200, 1024, 40), (129, 4096, 256)):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
        out = ops.router_logits(x.to(DEV), w.to(DEV)).cpu()
        ref = x.float() @ w.float().t()
        assert _rel(out, ref) < 1e-5


# ---------------------------------------------------------------- norms

def test_rmsnorm_and_residual():
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(5)
    for T, H in ((4, 1024), (64, 2048), (7, 2816), (3, 4096)):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        r = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
        y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6).cpu()
        assert _rel(y, off.rmsnorm(x, w, 1e-6)) < RTOL_BF16
        res_out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
        y2 = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV),
                         residual_out=res_out).cpu()
        xs = (x.float() + r.float()).to(torch.bfloat16)
        assert torch.equal(res_out.cpu(), xs)
        assert _rel(y2, off.rmsnorm(xs, w, 1e-6)) < RTOL_BF16


@pytest.mark.parametrize("T,H,E,K", [(1, 2048, 128, 8), (8, 2048, 128, 8), (64, 2048, 128, 8),
                                     (5, 1024, 16, 2), (3, 320, 40, 4)])
def test_fused_decode_router_softmax_bit_exact(T, H, E, K):
    """Router projection + softmax top-k in one launch (one cluster per token) gives the
    logits, weights and ids of the warp GEMV followed by the standalone top-k, bit for bit;
    padding rows (num_token_non_padded) get id -1; ids equal the oracle's on those logits."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T * 7 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    rw = (0.02 * torch.randn(E, H, generator=g)).to(torch.bfloat16).to(DEV)
    logits = torch.empty(T, E, dtype=torch.float32, device=DEV)
    w, ids = ops.router_softmax_topk(x, rw, K, True, logits_out=logits)
    ref_logits = ops.router_logits(x, rw)
    wr, ir = ops.softmax_topk(ref_logits, K, True)
    assert torch.equal(logits, ref_logits)
    assert torch.equal(w, wr) and torch.equal(ids, ir)
    wo, io = orouting.softmax_topk(logits.cpu(), K, True)
    assert np.array_equal(_canon(w.cpu().numpy(), ids.cpu().numpy())[1],
                          _canon(wo.numpy(), io.numpy())[1])
    ntp = torch.tensor([max(T - 2, 0)], dtype=torch.int32, device=DEV)
    wp, ip = ops.router_softmax_topk(x, rw, K, False, num_token_non_padded=ntp)
    wq, iq = ops.softmax_topk(ref_logits, K, False, ntp)
    assert torch.equal(wp, wq) and torch.equal(ip, iq)
    # the arrival counters return to 0 after every call: many calls in a row, in a graph too,
    # stay exact, and so do calls with another router size on the same counters
    arr = ops.router_arrivals(DEV)
    for _ in range(5):
        wa, ia = ops.router_softmax_topk(x, rw, K, True, arrivals=arr)
        assert torch.equal(wa, wr) and torch.equal(ia, ir)
    wg, ig = torch.empty_like(wr), torch.empty_like(ir)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.router_softmax_topk(x, rw, K, True, out=(wg, ig), arrivals=arr)
    torch.cuda.current_stream().wait_stream(side)
    with torch.cuda.graph(graph):
        ops.router_softmax_topk(x, rw, K, True, out=(wg, ig), logits_out=logits, arrivals=arr)
    for _ in range(3):
        wg.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(wg, wr) and torch.equal(ig, ir)
    del graph
    # a router of another size on the same counters, then this one again
    rw2 = (0.02 * torch.randn(E + 21, H, generator=g)).to(torch.bfloat16).to(DEV)
    w2, i2 = ops.router_softmax_topk(x, rw2, K, True, arrivals=arr)
    w2r, i2r = ops.softmax_topk(ops.router_logits(x, rw2), K, True)
    assert torch.equal(w2, w2r) and torch.equal(i2, i2r)
    wa, ia = ops.router_softmax_topk(x, rw, K, True, arrivals=arr)
    assert torch.equal(wa, wr) and torch.equal(ia, ir)
    assert int(arr[:T].abs().sum()) == 0


@pytest.mark.parametrize("T,H,E", [(1, 4096, 256), (16, 4096, 256), (64, 4096, 256),
                                   (4, 1024, 64)])
def test_fused_decode_router_sigmoid_group_bit_exact(T, H, E):
    """The DeepSeek-style selection (8 groups, top-4 groups, top-6, x2.5, with a bias) fused
    with its router projection equals the two launches bit for bit."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    rw = (0.02 * torch.randn(E, H, generator=g)).to(torch.bfloat16).to(DEV)
    bias = (0.01 * torch.randn(E, generator=g)).to(DEV)
    w, ids = ops.router_sigmoid_group_topk(x, rw, 6, 8, 4, 2.5, True, bias=bias)
    logits = ops.router_logits(x, rw)
    wr, ir = ops.sigmoid_group_topk(logits, 6, 8, 4, 2.5, True, bias=bias)
    assert torch.equal(w, wr) and torch.equal(ids, ir)
    wo, io = orouting.sigmoid_group_topk(logits.cpu(), 6, 8, 4, 2.5, True, bias=bias.cpu())
    assert np.array_equal(ids.cpu().numpy(), io.numpy())


def test_router_norm_pair():
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(6)
    H = 2816
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    ones = torch.ones(H, dtype=torch.bfloat16)
    rw = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    sc = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    a, b = ops.router_norm_pair(x.to(DEV), ones.to(DEV), rw.to(DEV), sc.to(DEV), 1e-6, 0.0625)
    ar, br = off.router_norm_pair(x, ones, rw, sc, 1e-6, 0.0625)
    assert _rel(a.cpu(), ar) < RTOL_BF16
    assert _rel(b.cpu(), br) < RTOL_BF16


@pytest.mark.parametrize("T,H", [(5, 2816), (3, 4096), (2, 8192)])
def test_router_norm_triple(T, H):
    """The fused three-output norm equals the pair and the plain RMSNorm bit for bit (same
    reduction and rounding), with 128-thread (H <= 4096) and 256-thread rows."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    ones = torch.ones(H, dtype=torch.bfloat16, device=DEV)
    rw, sc, sw = ((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV)
                  for _ in range(3))
    a, b, c = ops.router_norm_triple(x, ones, rw, sc, sw, 1e-6, H ** -0.5)
    a2, b2 = ops.router_norm_pair(x, ones, rw, sc, 1e-6, H ** -0.5)
    assert torch.equal(a, a2) and torch.equal(b, b2)
    assert torch.equal(c, ops.rmsnorm(x, sw, 1e-6))
    ar, br = off.router_norm_pair(x.cpu(), ones.cpu(), rw.cpu(), sc.cpu(), 1e-6, H ** -0.5)
    assert _rel(a, ar) < RTOL_BF16 and _rel(b, br) < RTOL_BF16
    assert _rel(c, off.rmsnorm(x.cpu(), sw.cpu(), 1e-6)) < RTOL_BF16


# ---------------------------------------------------------------- slot table

class _DevTable:
    def __init__(self, L, E, S):
        self.L, self.E, self.S = L, E, S
        self.slot_for_id = torch.full((L * E,), -1, dtype=torch.int32, device=DEV)
        self.id_of_slot = torch.full((S,), -1, dtype=torch.int32, device=DEV)
        self.usage = torch.zeros(S, dtype=torch.int64, device=DEV)
        self.step = torch.zeros(1, dtype=torch.int64, device=DEV)
        self.evict = torch.zeros(E, dtype=torch.int32, device=DEV)
        self.src = torch.zeros(E, dtype=torch.int32, device=DEV)
        self.num = torch.zeros(1, dtype=torch.int64, device=DEV)
        self.stats = torch.zeros(4, dtype=torch.int64, device=DEV)

    def ensure(self, ids: np.ndarray, layer: int, pinned=None) -> np.ndarray:
        from tideway_b200 import ops

        t = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).to(DEV)
        ops.lru_ensure(t, self.slot_for_id, self.id_of_slot, self.usage, self.step, self.E,
                       layer, self.evict, self.src, self.num, stats=self.stats, pinned=pinned)
        return t.cpu().numpy()

    def check_equal(self, ref: osc.SlotTable, msg=""):
        assert np.array_equal(self.slot_for_id.cpu().numpy(), ref.slot_for_id), msg
        assert np.array_equal(self.id_of_slot.cpu().numpy(), ref.id_of_slot), msg
        assert np.array_equal(self.usage.cpu().numpy(), ref.usage), msg
        assert int(self.step.item()) == ref.step, msg
        n = int(self.num.item())
        assert n == ref.num_indices, msg
        assert np.array_equal(self.evict.cpu().numpy()[:n], ref.evict_slots[:n]), msg
        assert np.array_equal(self.src.cpu().numpy()[:n], ref.src_indices[:n]), msg


@pytest.mark.parametrize("stem", ["lru_ensure", "lru_ensure_pinned"])
def test_lru_ensure_golden_sequences(stem):
    """The reference's lru_ensure sequences replayed on the kernel; the second fixture has
    pinned slots (never evicted)."""
    for name, c in load_golden(stem).items():
        L, E, S = int(c["L"]), int(c["E"]), int(c["S"])
        d = _DevTable(L, E, S)
        d.slot_for_id.copy_(torch.from_numpy(c["init_slot_of_id"]))
        d.id_of_slot.copy_(torch.from_numpy(c["init_id_of_slot"]))
        pinned = (torch.from_numpy(c["pinned"].astype(np.int32)).to(DEV) if "pinned" in c
                  else None)
        for i in range(int(c["steps"])):
            out = d.ensure(c[f"s{i}_ids"], int(c[f"s{i}_layer"]), pinned)
            assert np.array_equal(out, c[f"s{i}_out"]), (name, i)
            n = int(c[f"s{i}_num"])
            assert int(d.num.item()) == n, (name, i)
            assert np.array_equal(d.evict.cpu().numpy()[:n], c[f"s{i}_dst"]), (name, i)
            assert np.array_equal(d.src.cpu().numpy()[:n], c[f"s{i}_src"]), (name, i)
            assert np.array_equal(d.slot_for_id.cpu().numpy(), c[f"s{i}_slot_of_id"]), (name, i)
            assert np.array_equal(d.id_of_slot.cpu().numpy(), c[f"s{i}_id_of_slot"]), (name, i)
            assert np.array_equal(d.usage.cpu().numpy(), c[f"s{i}_usage"]), (name, i)
        assert np.array_equal(d.stats.cpu().numpy()[:3], c["stats"][:3]), name


def _hybrid_step(d: "_DevTable", extra: dict, ids: np.ndarray, layer: int, max_fetch: int,
                 frac_q16: int, by_recency: bool) -> np.ndarray:
    from tideway_b200 import ops

    t = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).to(DEV)
    ops.hybrid_ensure(t, d.slot_for_id, d.id_of_slot, d.usage, d.step, d.E, layer,
                      extra["active"], d.evict, d.src, d.num, extra["full"],
                      extra["recency"] if by_recency else None, max_fetch, frac_q16)
    return t.cpu().numpy()


def _hybrid_extra(L, E):
    return dict(active=torch.zeros(E, dtype=torch.int32, device=DEV),
                full=torch.zeros(1, dtype=torch.int64, device=DEV),
                recency=torch.zeros(L, E, dtype=torch.int64, device=DEV))


def test_hybrid_ensure_golden_sequences():
    """The device capped-fetch LRU reproduces the reference's CPU mirror step for step."""
    for name, c in load_golden("hybrid_ensure").items():
        L, E, S = int(c["L"]), int(c["E"]), int(c["S"])
        d, x = _DevTable(L, E, S), _hybrid_extra(L, E)
        d.slot_for_id.copy_(torch.from_numpy(c["init_slot_of_id"]))
        d.id_of_slot.copy_(torch.from_numpy(c["init_id_of_slot"]))
        for i in range(int(c["steps"])):
            out = _hybrid_step(d, x, c[f"s{i}_ids"], int(c[f"s{i}_layer"]), int(c["max_fetch"]),
                               int(c["frac_q16"]), bool(c["by_recency"]))
            n = int(c[f"s{i}_num"])
            assert np.array_equal(out, c[f"s{i}_out"]), (name, i)
            assert int(d.num.item()) == n and int(x["full"].item()) == int(c[f"s{i}_num_full"])
            assert np.array_equal(d.evict.cpu().numpy()[:n], c[f"s{i}_dst"]), (name, i)
            assert np.array_equal(d.src.cpu().numpy()[:n], c[f"s{i}_src"]), (name, i)
            assert np.array_equal(d.slot_for_id.cpu().numpy(), c[f"s{i}_slot_of_id"]), (name, i)
            assert np.array_equal(d.id_of_slot.cpu().numpy(), c[f"s{i}_id_of_slot"]), (name, i)
            assert np.array_equal(d.usage.cpu().numpy(), c[f"s{i}_usage"]), (name, i)
            assert np.array_equal(x["active"].cpu().numpy(), c[f"s{i}_active"]), (name, i)
            if bool(c["by_recency"]):
                assert np.array_equal(x["recency"].cpu().numpy(), c[f"s{i}_recency"]), (name, i)


@pytest.mark.parametrize("L,E,S,T,K,steps,max_fetch,frac_q16,by_rec",
                         [(43, 256, 2752, 16, 6, 60, 4, 0, True),
                          (43, 256, 2752, 128, 6, 30, 1 << 30, 19661, True),
                          (48, 128, 3072, 8, 8, 60, 6, 0, False),
                          (2, 1024, 16384, 256, 8, 6, 100, 0, True)])
def test_hybrid_ensure_random_vs_oracle(L, E, S, T, K, steps, max_fetch, frac_q16, by_rec):
    """Random routing over configs[3]/[1]-sized tables and the largest table, with fixed and
    bandwidth-matched caps, against the oracle, bit for bit."""
    rng = np.random.default_rng(L * 7 + T + max_fetch % 97)
    d, x = _DevTable(L, E, S), _hybrid_extra(L, E)
    ref = osc.SlotTable(L, E, S)
    rec = np.zeros((L, E), np.int64)
    for it in range(steps):
        layer = it % L
        ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
        out = _hybrid_step(d, x, ids, layer, max_fetch, frac_q16, by_rec)
        exp, active, full = osc.hybrid_ensure(ref, rec, ids, layer, max_fetch, frac_q16, by_rec)
        assert np.array_equal(out, exp), it
        assert int(x["full"].item()) == full, it
        assert np.array_equal(x["active"].cpu().numpy(), active), it
        d.check_equal(ref, it)
        if by_rec:
            assert np.array_equal(x["recency"].cpu().numpy(), rec), it


def test_offload_cache_ensure_experts_hybrid():
    """OffloadMoeCache.ensure_experts_hybrid (bandwidth fraction -> Q16, recency order)
    against the oracle over a few steps; overflow misses come back as -1."""
    from tideway_b200.offload_cache import OffloadMoeCache

    L, E, S, T, K = 3, 64, 96, 8, 4
    c = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV,
                        hybrid_fetch_fraction=0.3)
    ref = osc.SlotTable(L, E, S)
    rec = np.zeros((L, E), np.int64)
    rng = np.random.default_rng(12)
    saw_overflow = False
    for it in range(9):
        layer = it % L
        ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
        t = torch.from_numpy(ids).to(DEV)
        c.ensure_experts_hybrid(layer, t)
        exp, active, full = osc.hybrid_ensure(ref, rec, ids, layer, 1 << 30,
                                              round(0.3 * (1 << 16)), True)
        out = t.cpu().numpy()
        assert np.array_equal(out, exp), it
        assert int(c.num_missing_full.item()) == full and int(c.num_indices.item()) == ref.num_indices
        saw_overflow |= bool((out < 0).any())
    assert saw_overflow


@pytest.mark.parametrize("L,E,S,T,K,steps", [(48, 128, 3072, 64, 8, 60), (48, 128, 3072, 1, 8, 100),
                                             (43, 256, 2752, 128, 6, 45), (4, 16, 40, 4, 2, 200),
                                             (2, 1024, 16384, 1024, 8, 6)])
def test_lru_ensure_random_vs_oracle(L, E, S, T, K, steps):
    rng = np.random.default_rng(L * 1000 + T)
    d = _DevTable(L, E, S)
    ref = osc.SlotTable(L, E, S)
    for it in range(steps):
        layer = it % L
        ids = rng.integers(0, E, size=(T, K)).astype(np.int32)
        if it % 7 == 3:
            ids[0, 0] = -1  # padding route
        out = d.ensure(ids, layer)
        exp = osc.lru_ensure(ref, ids, layer)
        assert np.array_equal(out, exp), it
        if it % 10 == 0 or it == steps - 1:
            d.check_equal(ref, it)
    assert np.array_equal(d.stats.cpu().numpy()[:3], ref.stats[:3])


def test_materialize_reset_and_hit_compact():
    from tideway_b200 import ops

    rng = np.random.default_rng(3)
    L, E, S = 6, 32, 100
    d = _DevTable(L, E, S)
    ref = osc.SlotTable(L, E, S)
    for it in range(30):
        ids = rng.integers(0, E, size=(4, 4)).astype(np.int32)
        d.ensure(ids, it % L)
        osc.lru_ensure(ref, ids, it % L)
        if it % 9 == 4:
            ops.materialize_layer(d.slot_for_id, d.id_of_slot, d.usage, d.step, E, it % L,
                                  d.evict, d.src, d.num)
            osc.materialize_layer(ref, it % L)
            d.check_equal(ref, it)
    for layer in range(L):
        dst = torch.zeros(E, dtype=torch.int32, device=DEV)
        srcs = torch.zeros(E, dtype=torch.int32, device=DEV)
        num = torch.zeros(1, dtype=torch.int64, device=DEV)
        ops.prefill_hit_compact(d.slot_for_id[layer * E:(layer + 1) * E], E, layer % 2, dst, srcs,
                                num)
        rd, rs, rn = osc.prefill_hit_compact(ref, layer, layer % 2)
        assert int(num.item()) == rn
        assert np.array_equal(dst.cpu().numpy()[:rn], rd)
        assert np.array_equal(srcs.cpu().numpy()[:rn], rs)
    ops.reset_slots(d.slot_for_id, d.id_of_slot, d.usage, d.step, d.num)
    osc.reset(ref)
    ref.num_indices = 0
    assert np.array_equal(d.slot_for_id.cpu().numpy(), ref.slot_for_id)
    assert int(d.step.item()) == 0 and int(d.num.item()) == 0


def test_copy_rows_from_pinned_host():
    from tideway_b200 import ops

    E, S = 16, 24
    host_a = torch.randn(E, 64, 96).to(torch.bfloat16).pin_memory()
    host_b = torch.randint(0, 255, (E, 4096), dtype=torch.uint8).pin_memory()
    dev_a = torch.zeros(S, 64, 96, dtype=torch.bfloat16, device=DEV)
    dev_b = torch.zeros(S, 4096, dtype=torch.uint8, device=DEV)
    plan = ops.CopyPlan([dev_a, dev_b], [host_a, host_b])
    dst = torch.tensor([3, 17, 5, 0] + [0] * (E - 4), dtype=torch.int32, device=DEV)
    src = torch.tensor([9, 2, 15, 0] + [0] * (E - 4), dtype=torch.int32, device=DEV)
    num = torch.tensor([3], dtype=torch.int64, device=DEV)
    ops.copy_rows(plan, dst, src, num, E)
    torch.cuda.synchronize()
    for d_, s_ in ((3, 9), (17, 2), (5, 15)):
        assert torch.equal(dev_a[d_].cpu(), host_a[s_])
        assert torch.equal(dev_b[d_].cpu(), host_b[s_])
    assert dev_a[0].abs().sum().item() == 0  # the 4th row is beyond num


# ---------------------------------------------------------------- expert FFN

def _bank(S, H, I, g):
    w1 = (torch.randn(S, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(S, H, I, generator=g) * 0.02).to(torch.bfloat16)
    return w1, w2


def _routing(T, K, S, g, skew=False):
    if skew:
        ids = torch.randint(0, max(2, S // 8), (T, K), generator=g)
    else:
        ids = torch.stack([torch.randperm(S, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g)
    w = w / w.sum(-1, keepdim=True)
    return w.float().contiguous(), ids.to(torch.int32).contiguous()


@pytest.mark.parametrize("T,H,I,S,K,skew", [(4, 1024, 512, 8, 2, False),
                                            (1, 2048, 768, 64, 8, False),
                                            (16, 2048, 768, 64, 8, True),
                                            (3, 1024, 512, 16, 8, True),
                                            (8, 2048, 768, 64, 8, False),
                                            (64, 2048, 768, 128, 8, False),
                                            (64, 2048, 768, 128, 8, True),
                                            (17, 2816, 704, 32, 8, False),
                                            (300, 1024, 512, 4, 2, True),
                                            (640, 1024, 512, 4, 2, False),
                                            (40, 2048, 768, 256, 8, False),
                                            (200, 2048, 768, 16, 8, False),
                                            (300, 1024, 512, 32, 2, True),
                                            (600, 1024, 512, 1, 1, False),
                                            (400, 1152, 704, 8, 2, False),
                                            (600, 1024, 512, 4, 2, True),
                                            (600, 1152, 320, 1, 1, False)])
def test_moe_ffn_bf16(T, H, I, S, K, skew):
    """Route tiles: 16 (T <= 16: the up tiles read x's token rows directly, no gathered copy;
    the skewed 16- and 3-token cases repeat ids inside tokens, so a slot gets more routes
    than one tile and its chunks all multiply the same token rows), 64 (T <= 64), 160 (larger T, <= 128 expected routes per
    slot; the skewed 300-token case puts > 160 routes on a slot), 256 (the 640/300-token
    cases over 4 slots).  A slot with more routes than one tile is split into segments of
    one tile each: the skewed cases and the single-slot 600-route case (a shared expert:
    segments of 256, 256 and 88 routes).  160- and 256-route tiles take two weight tiles per
    item; the H=1152 cases have odd up and down tile counts (a single-tile last item).
    1024+ routes over <= 1024 slots take the two-kernel grouping (count, then place), the
    skewed 600-token case with repeated ids inside tokens."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H + S)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(S, H, I, g)
    tw, ti = _routing(T, K, S, g, skew)
    ws = ops.workspace(T * K, H, I, DEV)
    out = ops.moe_ffn_bf16(x.to(DEV), w1.to(DEV), w2.to(DEV), tw.to(DEV), ti.to(DEV),
                           ws=ws).cpu()
    assert ops.workspace_error(ws, T * K, H, I) == 0
    ref = off.moe_decode(x, w1, w2, tw, ti)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)
    # an fp32 end-to-end reference (no intermediate bf16 rounding) is within the same bound
    ref32 = torch.zeros(T, H)
    for t in range(T):
        for k in range(K):
            s = int(ti[t, k])
            h = x[t].float() @ w1[s].float().t()
            a = torch.nn.functional.silu(h[:I]) * h[I:]
            ref32[t] += tw[t, k] * (a @ w2[s].float().t())
    assert _rel(out, ref32) <= RTOL_BF16


@pytest.mark.parametrize("T,H,I", [(1, 1024, 512), (40, 1024, 512), (150, 1024, 512),
                                   (600, 1152, 320), (2048, 2816, 2112)])
def test_ffn_dense_bf16(T, H, I):
    """The dense (shared-expert) entry equals the routed entry with every row routed to slot 0
    at weight 1, bit for bit, over every route-tile size (16, 64, 160, 256 with segments of
    256) including odd tile counts and the configs[2] shared-expert shape; in place too."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H + I)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(1, H, I, g)
    xd, w1d, w2d = x.to(DEV), w1.to(DEV), w2.to(DEV)
    ids = torch.zeros(T, 1, dtype=torch.int32, device=DEV)
    ones = torch.ones(T, 1, dtype=torch.float32, device=DEV)
    routed = ops.moe_ffn_bf16(xd, w1d, w2d, ones, ids)
    ws = ops.workspace(T, H, I, DEV)
    dense = ops.ffn_dense_bf16(xd, w1d[0], w2d[0], ws=ws)
    assert ops.workspace_error(ws, T, H, I) == 0
    assert torch.equal(dense, routed)
    inplace = xd.clone()
    ops.ffn_dense_bf16(inplace, w1d[0], w2d[0], out=inplace, ws=ws)
    assert torch.equal(inplace, routed)
    if T <= 150:
        h = x.float() @ w1[0].float().t()
        ref32 = (torch.nn.functional.silu(h[:, :I]) * h[:, I:]) @ w2[0].float().t()
        assert _rel(dense, ref32) <= RTOL_BF16


def test_moe_ffn_negative_ids_skipped_and_inplace():
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(9)
    T, H, I, S, K = 6, 1024, 512, 16, 2
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(S, H, I, g)
    tw, ti = _routing(T, K, S, g)
    ti[2, 1] = -1
    xd = x.to(DEV)
    out = ops.moe_ffn_bf16(xd, w1.to(DEV), w2.to(DEV), tw.to(DEV), ti.to(DEV), out=xd).cpu()
    ref = off.moe_decode(x, w1, w2, tw, ti)
    assert _rel(out, ref) <= RTOL_BF16


def test_nvfp4_dequantize_bit_exact():
    """The FFN kernel's f16 decoder (code * e4m3 scale) times the row global equals the
    oracle's fp32 dequantisation exactly, over every code, both nibbles and all scales."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(11)
    rows, K = 64, 512
    packed = torch.randint(0, 256, (rows, K // 2), dtype=torch.uint8, generator=g)
    packed[0, :128] = torch.arange(0, 128, dtype=torch.uint8)  # every byte pattern
    packed[1, :128] = torch.arange(128, 256, dtype=torch.uint8)
    sbytes = torch.randint(0, 127, (rows, K // 16), dtype=torch.uint8, generator=g)
    sbytes[2, :] = torch.arange(K // 16, dtype=torch.uint8) + 90  # up to 448 (0x7e)
    scale = sbytes.view(torch.float8_e4m3fn)
    glob = torch.rand(rows, generator=g) * 1e-3 + 1e-5
    out = ops.nvfp4_dequantize(packed.to(DEV), scale.to(DEV), glob.to(DEV)).cpu()
    ref = onv.dequantize(packed, scale, glob)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("T,H,I,S,K,skew", [(1, 4096, 2048, 8, 6, False),
                                            (16, 4096, 2048, 24, 6, False),
                                            (4, 1024, 512, 8, 2, False),
                                            (40, 1024, 512, 16, 4, False),
                                            (128, 1024, 768, 32, 6, False),
                                            (300, 512, 256, 6, 2, True),
                                            (300, 512, 256, 1, 1, False),
                                            (8, 320, 192, 4, 2, False)])
def test_moe_ffn_nvfp4(T, H, I, S, K, skew):
    """Tensor-core path for H, I multiples of 256 (route tiles 16/64/128, >128 routes on one
    slot when skewed); the last case (H=320, I=192) runs the CUDA-core kernels."""
    from tideway_b200 import nvfp4, ops

    g = torch.Generator().manual_seed(T + S)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    packs = [nvfp4.quantize_expert(torch.randn(2 * I, H, generator=g) * 0.02,
                                   torch.randn(H, I, generator=g) * 0.02) for _ in range(S)]
    w1p = torch.stack([p[0][0] for p in packs])
    w1s = torch.stack([p[0][1] for p in packs])
    w1g = torch.stack([p[0][2] for p in packs])
    w2p = torch.stack([p[1][0] for p in packs])
    w2s = torch.stack([p[1][1] for p in packs])
    w2g = torch.stack([p[1][2] for p in packs])
    tw, ti = _routing(T, K, S, g)
    if skew:  # every token's first route on slot 0: 300 routes = 3 route tiles of 128
        ti[:, 0] = 0
        ti[:, 1:] = torch.where(ti[:, 1:] == 0, torch.ones_like(ti[:, 1:]), ti[:, 1:])
    ws = ops.workspace(T * K, H, I, DEV)
    out = ops.moe_ffn_nvfp4(x.to(DEV), (w1p.to(DEV), w1s.to(DEV), w1g.to(DEV)),
                            (w2p.to(DEV), w2s.to(DEV), w2g.to(DEV)), tw.to(DEV), ti.to(DEV),
                            ws=ws).cpu()
    assert ops.workspace_error(ws, T * K, H, I) == 0  # no bounded wait gave up
    # oracle: dequantise then matmul with the bf16 rounding points of the BF16 path
    w1d = torch.stack([onv.dequantize(w1p[s], w1s[s], w1g[s]) for s in range(S)])
    w2d = torch.stack([onv.dequantize(w2p[s], w2s[s], w2g[s]) for s in range(S)])
    ref = off.moe_decode(x, w1d, w2d, tw, ti)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)


@pytest.mark.parametrize("T,H,I,S,K,act,w_in", [(4, 1024, 512, 8, 2, "gelu", False),
                                                (4, 1024, 512, 8, 2, "silu", True),
                                                (1, 2048, 768, 64, 8, "gelu_tanh", False),
                                                (40, 2048, 768, 64, 8, "gelu_tanh", True),
                                                (300, 1024, 512, 16, 2, "gelu", True),
                                                (600, 1152, 320, 1, 1, "gelu_tanh", False)])
def test_moe_ffn_bf16_activation_variants(T, H, I, S, K, act, w_in):
    """GELU and its tanh form on the gate half, and the route weight on the up projection
    (apply_router_weight_on_input), against the oracle's rounding points; decode (16- and
    64-route tiles, the token-row and batch-1 split-K decode paths where w_in is off) and
    prefill tiles (160 routes, paired weight tiles).  Each variant's output differs from the
    default SwiGLU, weight-on-output result, so the flags reach the kernel."""
    from tideway_b200 import fused, ops

    g = torch.Generator().manual_seed(T * 3 + H + S)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(S, H, I, g)
    tw, ti = _routing(T, K, S, g)
    args = (x.to(DEV), w1.to(DEV), w2.to(DEV), tw.to(DEV), ti.to(DEV))
    out = ops.moe_ffn_bf16(*args, activation=act, weight_on_input=w_in).cpu()
    ref = off.moe_decode(x, w1, w2, tw, ti, act, w_in)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)
    assert _rel(off.moe_decode(x, w1, w2, tw, ti), ref) > 5 * _rel(out, ref)
    # the reference's entry points take the same arguments
    dec = fused.fused_experts_decode_impl(*args, act, w_in).cpu()
    assert torch.equal(dec, out)


@pytest.mark.parametrize("T,H,I,S,K,act,w_in", [(16, 1024, 512, 8, 2, "gelu", True),
                                                (128, 1024, 768, 32, 6, "gelu_tanh", False),
                                                (8, 320, 192, 4, 2, "gelu", True)])
def test_moe_ffn_nvfp4_activation_variants(T, H, I, S, K, act, w_in):
    """The NVFP4 FFN's epilogue forms (tensor-core path; H=320 the CUDA-core kernels) against
    dequantise-then-matmul with the same activation and weight placement."""
    from tideway_b200 import nvfp4, ops

    g = torch.Generator().manual_seed(T + S + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    packs = [nvfp4.quantize_expert(torch.randn(2 * I, H, generator=g) * 0.02,
                                   torch.randn(H, I, generator=g) * 0.02) for _ in range(S)]
    b1 = [torch.stack([p[0][j] for p in packs]) for j in range(3)]
    b2 = [torch.stack([p[1][j] for p in packs]) for j in range(3)]
    tw, ti = _routing(T, K, S, g)
    ws = ops.workspace(T * K, H, I, DEV)
    out = ops.moe_ffn_nvfp4(x.to(DEV), tuple(b.to(DEV) for b in b1), tuple(b.to(DEV) for b in b2),
                            tw.to(DEV), ti.to(DEV), ws=ws, activation=act,
                            weight_on_input=w_in).cpu()
    assert ops.workspace_error(ws, T * K, H, I) == 0
    w1d = torch.stack([onv.dequantize(b1[0][s], b1[1][s], b1[2][s]) for s in range(S)])
    w2d = torch.stack([onv.dequantize(b2[0][s], b2[1][s], b2[2][s]) for s in range(S)])
    ref = off.moe_decode(x, w1d, w2d, tw, ti, act, w_in)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)
    assert _rel(off.moe_decode(x, w1d, w2d, tw, ti), ref) > 5 * _rel(out, ref)


@pytest.mark.parametrize("H,I", [(1024, 512), (320, 192)])
def test_reference_schema_nvfp4_cache_through_the_layer(H, I):
    """The reference's nvfp4 bank schema as it stores ModelOpt rows
    (backends/.../moe/offload_cache.py:44-54): packed e2m1, e4m3 per-16 scales and fp16
    per-output-row globals whose gate (w1) and up (w3) rows carry different values.  The
    cache pages those banks (12 slots for 2 x 8 experts: misses every step) and
    OffloadMoELayer's decode and prefill outputs match dequantise-then-matmul; the decoder
    itself is bit-exact against the oracle with fp16 globals.  H=320, I=192 run the
    CUDA-core kernels."""
    from tideway_b200 import OffloadMoeCache, OffloadMoELayer, attach_offload_moe_cache
    from tideway_b200 import batch_context, nvfp4, ops

    L, E, S, K = 2, 8, 12, 2
    g = torch.Generator().manual_seed(H + I)
    names = ("gate_up_packed", "gate_up_scale", "gate_up_global", "down_packed", "down_scale",
             "down_global")
    sources = {n: [] for n in names}
    dense = []
    for _ in range(L):
        packs = []
        for _ in range(E):
            gate = 0.02 * torch.randn(I, H, generator=g)
            up = 0.05 * torch.randn(I, H, generator=g)  # a different range: its own global
            packs.append(nvfp4.quantize_expert(torch.cat([gate, up]),
                                               0.02 * torch.randn(H, I, generator=g),
                                               global_dtype=torch.float16))
        banks = [torch.stack([p[m][j] for p in packs]) for m in range(2) for j in range(3)]
        assert banks[2].dtype == torch.float16 and banks[5].dtype == torch.float16
        assert not torch.equal(banks[2][:, 0], banks[2][:, I])  # distinct gate/up globals
        for n, t in zip(names, banks):
            sources[n].append(t.pin_memory())
        dense.append((torch.stack([onv.dequantize(*p[0]) for p in packs]),
                      torch.stack([onv.dequantize(*p[1]) for p in packs])))
    p0 = sources["gate_up_packed"][0][0]
    got = ops.nvfp4_dequantize(p0.to(DEV), sources["gate_up_scale"][0][0].to(DEV),
                               sources["gate_up_global"][0][0].to(DEV)).cpu()
    assert torch.equal(got, dense[0][0][0])
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV,
                            quant_format="nvfp4")
    cache.set_bank_sources(sources)
    layers = attach_offload_moe_cache([OffloadMoELayer(l, E, K, H, I) for l in range(L)], cache)
    for phase, T in (("decode", 4), ("decode", 3), ("prefill", 40)):
        with batch_context(is_prefill=phase == "prefill"):
            for l in range(L):
                x = torch.randn(T, H, generator=g).to(torch.bfloat16)
                logits = torch.randn(T, E, generator=g)
                out = layers[l].forward(x.to(DEV), logits.to(DEV)).cpu()
                w, ids = orouting.softmax_topk(logits, K, True)
                ref = off.moe_decode(x, dense[l][0], dense[l][1], w, ids)
                assert _rel(out, ref) <= RTOL_BF16, (phase, l, _rel(out, ref))
    cache.verify_tables()


def _ds_fp4_bank(S, rows, cols, g):
    """S DS-FP4 matrices [rows, cols] quantised from N(0, 0.02): (codes, e8m0, fp32 values)."""
    qs = [onv.quantize_ds_fp4(0.02 * torch.randn(rows, cols, generator=g)) for _ in range(S)]
    packed = torch.stack([q[0] for q in qs])
    e8 = torch.stack([q[1] for q in qs])
    dense = torch.stack([onv.dequantize_ds_fp4(q[0], q[1]) for q in qs])
    return packed, e8, dense


@pytest.mark.parametrize("T,H,I,S,K", [(4, 1024, 512, 8, 2), (40, 512, 256, 6, 4),
                                       (8, 320, 192, 4, 2)])
def test_ds_fp4_experts_on_nvfp4_kernels(T, H, I, S, K):
    """DeepSeek-V4 FP4 experts (e2m1 + e8m0 per 32), re-encoded as NVFP4 banks, through the
    NVFP4 FFN (tensor cores; CUDA cores for H=320, I=192) against dequantise-then-matmul of
    the DS-FP4 weights."""
    from tideway_b200 import ds_fp4, ops

    g = torch.Generator().manual_seed(100 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gp, gs, w1d = _ds_fp4_bank(S, 2 * I, H, g)
    dp, dsc, w2d = _ds_fp4_bank(S, H, I, g)
    banks, flushed = ds_fp4.expert_banks(gp, gs, dp, dsc)
    assert flushed == 0
    b = [banks[n].to(DEV) for n in ds_fp4.NVFP4_BANKS]
    tw, ti = _routing(T, K, S, g)
    out = ops.moe_ffn_nvfp4(x.to(DEV), tuple(b[:3]), tuple(b[3:]), tw.to(DEV), ti.to(DEV)).cpu()
    ref = off.moe_decode(x, w1d, w2d, tw, ti)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)


def test_offload_layer_ds_fp4_decode():
    """OffloadMoeCache(quant_format="ds_fp4") takes the reference's four DS-FP4 banks per
    layer, pages experts into NVFP4 slot banks (12 slots for 2 x 8 experts: misses every
    step), and OffloadMoELayer's decode output matches the oracle over the DS-FP4 weights."""
    from tideway_b200 import OffloadMoeCache, OffloadMoELayer, attach_offload_moe_cache, ds_fp4

    L, E, S, T, K, H, I = 2, 8, 12, 4, 2, 512, 256
    g = torch.Generator().manual_seed(21)
    sources = {n: [] for n in ds_fp4.DS_FP4_BANKS}
    dense = []
    for _ in range(L):
        gp, gs, w1d = _ds_fp4_bank(E, 2 * I, H, g)
        dp, dsc, w2d = _ds_fp4_bank(E, H, I, g)
        for name, t in zip(ds_fp4.DS_FP4_BANKS, (gp, gs.view(torch.float8_e8m0fnu), dp, dsc)):
            sources[name].append(t.pin_memory())
        dense.append((w1d, w2d))
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV,
                            quant_format="ds_fp4")
    cache.set_bank_sources(sources)
    assert cache.ds_fp4_flushed_blocks == 0 and len(cache.bank_views()) == 6
    layers = attach_offload_moe_cache([OffloadMoELayer(l, E, K, H, I) for l in range(L)], cache)
    for step in range(3):
        for l in range(L):
            x = torch.randn(T, H, generator=g).to(torch.bfloat16)
            logits = torch.randn(T, E, generator=g)
            out = layers[l].forward(x.to(DEV), logits.to(DEV)).cpu()
            w, ids = orouting.softmax_topk(logits, K, True)
            ref = off.moe_decode(x, dense[l][0], dense[l][1], w, ids)
            assert _rel(out, ref) <= RTOL_BF16, (step, l, _rel(out, ref))
    layers[0].swiglu_limit = 10.0
    with pytest.raises(NotImplementedError):
        layers[0].forward(x.to(DEV), logits.to(DEV))


@pytest.mark.parametrize("installed", [False, True])
def test_prefill_double_buffer_then_decode(installed):
    """Prefill through the whole-layer double buffer (slots [0, 2E), buffer = layer % 2, the
    next layer streamed on the copy stream), then decode on the same cache: every layer's
    output against the oracle.  ``installed`` routes both through the offload manager
    (``runtime.install``: ensure + prefill entry points) instead of the layer's own path."""
    from tideway_b200 import OffloadMoeCache, OffloadMoELayer, attach_offload_moe_cache
    from tideway_b200 import batch_context, runtime

    L, E, K, H, I = 3, 8, 2, 512, 256
    S = 2 * E + 6
    g = torch.Generator().manual_seed(41)
    banks = [_bank(E, H, I, g) for _ in range(L)]
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV,
                            prefill_overlap=True)
    cache.set_bank_sources({"gate_up": [b[0].pin_memory() for b in banks],
                            "down": [b[1].pin_memory() for b in banks]})
    layers = attach_offload_moe_cache([OffloadMoELayer(l, E, K, H, I) for l in range(L)], cache)
    session = runtime.install(cache) if installed else None
    try:
        for phase, T in (("prefill", 40), ("decode", 4), ("prefill", 24), ("decode", 3)):
            with batch_context(is_prefill=phase == "prefill"):
                for l in range(L):
                    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
                    logits = torch.randn(T, E, generator=g)
                    out = layers[l].forward(x.to(DEV), logits.to(DEV)).cpu()
                    w, ids = orouting.softmax_topk(logits, K, True)
                    ref = off.moe_decode(x, banks[l][0], banks[l][1], w, ids)
                    assert _rel(out, ref) <= RTOL_BF16, (phase, l, _rel(out, ref))
        cache.verify_tables()
        if installed:
            st = session.manager.snapshot()
            assert st["prefill_layers"] == 2 * L and st["ensure_calls"] == 2 * L
    finally:
        if session is not None:
            session.uninstall()
    assert "ensure_experts" not in vars(cache)


def test_route_trace_and_histogram_replay_with_the_graph():
    """The decode route trace and routing histogram are device-only: a captured ensure keeps
    recording on every replay (raw expert ids, before the slot rewrite)."""
    from tideway_b200 import OffloadMoeCache

    L, E, S, K = 2, 16, 24, 8
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV)
    cache.enable_route_trace(steps=4, width=K)
    cache.collect_decode_freq = True
    g = torch.Generator().manual_seed(51)
    raws = [torch.randperm(E, generator=g)[:K].to(torch.int32).view(1, K) for _ in range(4)]
    src = raws[0].to(DEV)
    ids = torch.empty_like(src)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ids.copy_(src)
        cache.ensure_experts(1, ids)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ids.copy_(src)
        cache.ensure_experts(1, ids)
    for r in raws[1:]:
        src.copy_(r.to(DEV))
        graph.replay()
    torch.cuda.synchronize()
    layers, rec, total = cache.route_trace.read()
    assert total == 4 and layers.tolist() == [1] * 4
    assert np.array_equal(rec, torch.cat(raws).numpy())
    want = torch.bincount(torch.cat(raws).view(-1).long(), minlength=E)
    assert torch.equal(cache.decode_freq[1].cpu(), want) and int(cache.decode_freq[0].sum()) == 0
    del graph


def test_custom_ops_match_direct_calls_and_compile_without_breaks():
    """torch.ops.tideway_b200 ops give the bits of the direct calls, and a decode step
    built from them (router, in-place slot ensure, FFN) compiles as one graph."""
    from tideway_b200 import ops

    op = torch.ops.tideway_b200
    g = torch.Generator().manual_seed(31)
    T, H, I, E, K = 8, 1024, 512, 16, 2
    S = E + 8
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w1, w2 = (t.to(DEV) for t in _bank(S, H, I, g))
    logits = torch.randn(T, E, generator=g).to(DEV)
    w, ids = op.fused_topk(logits, K, True)
    wr, idr = ops.softmax_topk(logits, K, True)
    assert torch.equal(w, wr) and torch.equal(ids, idr)
    assert torch.equal(op.moe_ffn_bf16(x, w1, w2, w, ids), ops.moe_ffn_bf16(x, w1, w2, w, ids))

    def tables():
        i32, i64 = torch.int32, torch.int64
        return (torch.full((1, E), -1, dtype=i32, device=DEV),
                torch.full((S,), -1, dtype=i32, device=DEV),
                torch.zeros(S, dtype=i64, device=DEV), torch.zeros((), dtype=i64, device=DEV),
                torch.zeros(E, dtype=i32, device=DEV), torch.zeros(E, dtype=i32, device=DEV),
                torch.zeros(1, dtype=i64, device=DEV))

    def step(x, logits, sfi, ios, usage, st, ev, src, num):
        w, ids = op.fused_topk(logits, K, True)
        op.lru_ensure(ids, sfi, ios, usage, st, E, 0, ev, src, num)
        return op.moe_ffn_bf16(x, w1, w2, w, ids), ids

    eager_tables, compiled_tables = tables(), tables()
    y_e, ids_e = step(x, logits, *eager_tables)
    compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
    y_c, ids_c = compiled(x, logits, *compiled_tables)
    assert torch.equal(ids_c, ids_e) and torch.equal(y_c, y_e)
    for a, b in zip(eager_tables, compiled_tables):
        assert torch.equal(a, b)


def test_moe_align_golden_and_random():
    from tideway_b200 import ops

    c = load_golden("moe_align")["docstring"]
    s, e, n = ops.moe_align_block_size(torch.from_numpy(c["topk_ids"]).to(DEV),
                                       int(c["block_size"]), int(c["num_experts"]))
    npad = int(n.item())
    assert npad == 16
    assert np.array_equal(s.cpu().numpy()[:npad], c["sorted_ids"])
    assert e.cpu().numpy()[:4].tolist() == [1, 2, 3, 4]
    rng = np.random.default_rng(0)
    for T, K, E, bs in ((2048, 8, 128, 64), (8192, 6, 256, 128), (3, 2, 16, 16)):
        ids = rng.integers(0, E, size=(T, K)).astype(np.int32)
        s, e, n = ops.moe_align_block_size(torch.from_numpy(ids).to(DEV), bs, E)
        rs, re_, rn = off.moe_align_block_size(ids, bs, E)
        assert int(n.item()) == rn
        assert np.array_equal(s.cpu().numpy()[:rn], rs)
        assert np.array_equal(e.cpu().numpy()[:len(re_)], re_)
        assert (s.cpu().numpy()[rn:] == T * K).all()


def test_dual_norm_merge():
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(17)
    T, H = 9, 2816
    a, b, x = (torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(3))
    w1, w2, w3 = ((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(3))
    out = ops.dual_norm_merge(a.to(DEV), b.to(DEV), x.to(DEV), w1.to(DEV), w2.to(DEV),
                              w3.to(DEV), 1e-6, 1e-6, 1e-6, 0.5).cpu()
    ref = off.dual_norm_merge(a, b, x, w1, w2, w3, 1e-6, 1e-6, 1e-6, 0.5)
    assert _rel(out, ref) < RTOL_BF16


def test_add_shared():
    """routed + shared expert merge (DeepSeek layout): bf16(a + b), exact."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(5)
    a = torch.randn(7, 4096, generator=g).to(torch.bfloat16)
    b = torch.randn(7, 4096, generator=g).to(torch.bfloat16)
    out = ops.add_shared(a.to(DEV), b.to(DEV)).cpu()
    assert torch.equal(out, (a.float() + b.float()).to(torch.bfloat16))


def test_prefill_stack_layer_stages():
    """One layer of the Gemma prefill stack, stage by stage against the oracle, each stage fed
    with the GPU's previous stage: router norm pair, router logits (fp32 tolerance), Gemma
    top-k (ids bit-exact), dense shared expert and routed experts (bf16 bound) and the merge.
    300 tokens run the tensor-core router and the 160-route FFN tiles."""
    from tideway_b200.prefill import GemmaPrefillStack, PrefillConfig

    cfg = PrefillConfig(layers=1, hidden=1024, experts=16, topk=4, inter=256, shared_inter=512,
                        tokens=300, seed=5)
    st = GemmaPrefillStack(cfg, device=DEV)
    g = torch.Generator().manual_seed(6)
    x0 = torch.randn(cfg.tokens, cfg.hidden, generator=g).to(torch.bfloat16)
    st.x.copy_(x0.to(DEV))
    p = st.layers[0]
    st.layer(p)
    torch.cuda.synchronize()
    c = {k: v.cpu() for k, v in p.items()}
    ri, rr = off.router_norm_pair(x0, c["ones"], c["pre_routed"], c["router_scale"], cfg.eps,
                                  st.root)
    assert _rel(st.router_in, ri) <= 1e-2 and _rel(st.routed_in, rr) <= 1e-2
    logits = st.router_in.cpu().float() @ c["router"].float().t()
    assert _rel(st.logits, logits) <= 1e-4
    w, ids, _ = orouting.gemma_topk(st.logits.cpu(), c["expert_scale"], cfg.topk)
    assert np.array_equal(st.ids.cpu().numpy(), ids.numpy())
    np.testing.assert_allclose(st.w.cpu().numpy(), w.numpy(), rtol=1e-5, atol=1e-7)
    sh_in = off.rmsnorm(x0, c["pre_shared"], cfg.eps)
    assert _rel(st.shared_in, sh_in) <= 1e-2
    sh = off.shared_expert(st.shared_in.cpu(), c["sh_w1"][0], c["sh_w2"][0])
    assert _rel(st.shared, sh) <= RTOL_BF16
    # the stack fuses the routed combine into the merge; the routed output on its own:
    from tideway_b200 import ops

    routed_gpu = ops.moe_ffn_bf16(st.routed_in, p["w1"], p["w2"], st.w, st.ids).cpu()
    routed = off.moe_prefill(st.routed_in.cpu(), c["w1"], c["w2"], st.w.cpu(), st.ids.cpu())
    assert _rel(routed_gpu, routed) <= RTOL_BF16
    merged = off.dual_norm_merge(st.shared.cpu(), routed_gpu, x0, c["post_shared"],
                                 c["post_routed"], c["post"], cfg.eps, cfg.eps, cfg.eps,
                                 cfg.layer_scalar)
    assert _rel(st.x, merged) <= 1e-2


@pytest.mark.parametrize("T,K,S,fp4", [(8, 8, 96, False), (1, 8, 64, False), (40, 4, 48, False),
                                      (16, 6, 40, True)])
def test_ensure_group_then_grouped_ffn_bit_exact(T, K, S, fp4):
    """The LRU ensure that also groups the routes (one launch) followed by the FFN that skips
    its grouping gives the slot tables, the staged misses and the FFN output of lru_ensure
    followed by the ungrouped FFN, bit for bit; over several steps with misses."""
    from tideway_b200 import nvfp4, ops

    E, H, I = 32, 1024, 512
    g = torch.Generator().manual_seed(T * 100 + S)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    if fp4:
        packs = [nvfp4.quantize_expert(0.02 * torch.randn(2 * I, H, generator=g),
                                       0.02 * torch.randn(H, I, generator=g)) for _ in range(4)]
        w1 = tuple(torch.stack([packs[s % 4][0][j] for s in range(S)]).to(DEV) for j in range(3))
        w2 = tuple(torch.stack([packs[s % 4][1][j] for s in range(S)]).to(DEV) for j in range(3))
    else:
        w1, w2 = (t.to(DEV) for t in _bank(S, H, I, g))
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV)
    a, b = _DevTable(2, E, S), _DevTable(2, E, S)
    ws_a = torch.empty(ops.workspace_bytes(T * K, H, I), dtype=torch.uint8, device=DEV)
    ws_b = torch.empty_like(ws_a)
    for step in range(4):
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
        tw = torch.rand(T, K, generator=g)
        tw = (tw / tw.sum(-1, keepdim=True)).float().to(DEV)
        ia, ib = ids.to(DEV), ids.to(DEV)
        layer = step % 2
        ops.lru_ensure(ia, a.slot_for_id, a.id_of_slot, a.usage, a.step, E, layer, a.evict,
                       a.src, a.num)
        ops.lru_ensure_group(ib, b.slot_for_id, b.id_of_slot, b.usage, b.step, E, layer,
                             b.evict, b.src, b.num, H, I, ws_b, nvfp4=fp4)
        assert torch.equal(ia, ib) and torch.equal(a.slot_for_id, b.slot_for_id)
        assert torch.equal(a.id_of_slot, b.id_of_slot)
        assert torch.equal(a.num, b.num) and torch.equal(a.usage, b.usage)
        if fp4:
            ya = ops.moe_ffn_nvfp4(x, w1, w2, tw, ia, ws=ws_a)
            yb = ops.moe_ffn_nvfp4(x, w1, w2, tw, ib, ws=ws_b, pregrouped=True)
            assert torch.equal(ya, yb), step
        else:
            ra, rb = res.clone(), res.clone()
            ha, hb = torch.empty_like(x), torch.empty_like(x)
            ops.moe_ffn_bf16_residual_norm(x, w1, w2, tw, ia, ra, ra, nw, 1e-6, ha, ws=ws_a)
            ops.moe_ffn_bf16_residual_norm(x, w1, w2, tw, ib, rb, rb, nw, 1e-6, hb, ws=ws_b,
                                           pregrouped=True)
            assert torch.equal(ha, hb) and torch.equal(ra, rb), step


def test_moe_ffn_residual_norm_bit_exact():
    """The FFN with its combine fused into the next residual RMSNorm equals moe_ffn_bf16
    followed by rmsnorm(residual=...), bit for bit, at a decode size and a larger batch, in
    place as the decode stack calls it."""
    from tideway_b200 import ops

    for T, H, I, S, K in ((8, 2048, 768, 64, 8), (24, 1024, 512, 32, 4)):
        g = torch.Generator().manual_seed(T * 31 + K)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        resid = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        nw = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV)
        w1, w2 = (t.to(DEV) for t in _bank(S, H, I, g))
        tw, ti = (t.to(DEV) for t in _routing(T, K, S, g))
        y = ops.moe_ffn_bf16(x, w1, w2, tw, ti)
        r_ref = torch.empty_like(resid)
        h_ref = ops.rmsnorm(y, nw, 1e-6, residual=resid, residual_out=r_ref)
        r2, h2 = resid.clone(), x.clone()
        ops.moe_ffn_bf16_residual_norm(h2, w1, w2, tw, ti, r2, r2, nw, 1e-6, h2)
        assert torch.equal(r2, r_ref) and torch.equal(h2, h_ref)


@pytest.mark.parametrize("B", [4, 24])
def test_decode_stack_fused_equals_composed(B):
    """A small decode stack (3 layers, slot cache of half the experts, pinned host banks)
    gives bit-identical step outputs with the fused FFN + residual norm and with the composed
    launches, over two steps (the second pages in misses of the first); batch 24 takes the
    gathered-row FFN tiles.  The fused step's graph replay equals its eager step."""
    from tideway_b200.stack import MoEDecodeStack, StackConfig, StackWeights

    cfg = StackConfig("small", layers=3, hidden=1024, experts=16, topk=4, inter=256,
                      slot_fraction=0.5, seed=3)
    wts = StackWeights(cfg, device=DEV)
    try:
        a = MoEDecodeStack(wts, batch=B, fused=True)
        b = MoEDecodeStack(wts, batch=B, fused=False)
        g = torch.Generator().manual_seed(8)
        for _ in range(2):
            x = torch.randn(B, cfg.hidden, generator=g).to(torch.bfloat16).to(DEV)
            for st in (a, b):
                st.x_in.copy_(x)
                st.step_eager()
            torch.cuda.synchronize()
            assert torch.equal(a.out, b.out) and torch.equal(a.h, b.h)
        gather = 0 if B <= 16 else 1
        assert a.launches_per_step() == 3 * (5 + gather) + 1
        assert b.launches_per_step() == 3 * (7 + gather) + 1
        a.capture(verify=True)  # raises if the replay differs from the eager step
    finally:
        wts.release()


def test_fp4_stack_shared_expert_stream_is_race_free():
    """The NVFP4 decode stack runs each layer's shared expert on a side stream next to the
    routed path: over two steps (the second pages in the first one's misses) its output
    equals the same stack run on one stream, bit for bit, eagerly and as a captured graph."""
    from tideway_b200.stack_fp4 import Fp4DecodeStack, Fp4StackConfig, Fp4StackWeights

    cfg = Fp4StackConfig(layers=2, hidden=1024, experts=32, topk=4, inter=512, n_group=4,
                         topk_group=2, slot_fraction=0.5, seed=5)
    wts = Fp4StackWeights(cfg, device=DEV)
    a = Fp4DecodeStack(wts, 8)
    b = Fp4DecodeStack(wts, 8)
    b.side = torch.cuda.current_stream()  # the serial composition
    g = torch.Generator().manual_seed(21)
    for _ in range(2):
        x = torch.randn(8, cfg.hidden, generator=g).to(torch.bfloat16).to(DEV)
        for st in (a, b):
            st.x_in.copy_(x)
            st.step_eager()
        torch.cuda.synchronize()
        assert torch.equal(a.out, b.out) and torch.equal(a.h, b.h)
    graph = a.capture()
    a.x_in.copy_(x)
    graph.replay()
    b.x_in.copy_(x)
    b.step_eager()
    torch.cuda.synchronize()
    assert torch.equal(a.out, b.out) and torch.equal(a.h, b.h)
    assert torch.isfinite(a.out.float()).all()
    del graph


def test_decode_stack_audits_and_fails_closed():
    """The captured step equals the eager step byte for byte (checked at capture); every
    resident slot holds its host source's bytes (payload audit), and a corrupted slot row is
    found; a buffer moved after capture fails the stack, which then refuses every step."""
    from tideway_b200.stack import MoEDecodeStack, StackConfig, StackWeights

    cfg = StackConfig("small", layers=3, hidden=1024, experts=16, topk=4, inter=256,
                      slot_fraction=0.5, seed=5)
    wts = StackWeights(cfg, device=DEV)
    try:
        st = MoEDecodeStack(wts, batch=4)
        g = torch.Generator().manual_seed(9)
        st.x_in.copy_(torch.randn(4, cfg.hidden, generator=g).to(torch.bfloat16))
        st.capture(verify=True)
        assert st.state == "ready"
        for _ in range(3):
            st.x_in.copy_(torch.randn(4, cfg.hidden, generator=g).to(torch.bfloat16))
            st.step()
        st.check()
        audit = st.cache.verify_payload()
        assert audit["rows"] > 0 and audit["mismatches"] == []
        slot = int(torch.nonzero(st.cache.id_of_slot >= 0)[0])
        st.cache.bank_caches["down"][slot].zero_()
        bad = st.cache.verify_payload(raise_on_mismatch=False)["mismatches"]
        assert [m[0] for m in bad] == [slot] and bad[0][3] == "down"
        with pytest.raises(RuntimeError, match="payload"):
            st.cache.verify_payload()
        st.y = torch.zeros_like(st.y)  # a buffer the graph reads is replaced
        with pytest.raises(RuntimeError, match="moved"):
            st.step()
        assert st.state == "failed"
        with pytest.raises(RuntimeError, match="not retried"):
            st.step()
        del st
    finally:
        wts.release()


@pytest.mark.parametrize("change", ["route_trace", "release_host_banks", "topk_ids"])
def test_decode_stack_guard_covers_every_captured_buffer(change):
    """The address guard before each replay also covers the routing-trace ring (a ring
    enabled after capture replaces the one the graph writes), the host banks the miss copies
    read (an unregistered arena), and the per-layer routing outputs: each change fails the
    stack before the graph replays."""
    from tideway_b200.stack import MoEDecodeStack, StackConfig, StackWeights

    cfg = StackConfig("small", layers=2, hidden=1024, experts=16, topk=4, inter=256,
                      slot_fraction=0.5, seed=6)
    wts = StackWeights(cfg, device=DEV)
    released = False
    try:
        st = MoEDecodeStack(wts, batch=4)
        st.x_in.copy_(torch.randn(4, cfg.hidden, generator=torch.Generator().manual_seed(3))
                      .to(torch.bfloat16))
        st.capture()
        st.step()
        torch.cuda.synchronize()
        if change == "route_trace":
            st.cache.enable_route_trace(steps=2, width=16)
        elif change == "release_host_banks":
            wts.release()
            released = True
        else:
            st.topk_ids[1] = torch.zeros_like(st.topk_ids[1])
        with pytest.raises(RuntimeError, match="moved"):
            st.step()
        assert st.state == "failed"
        del st
    finally:
        if not released:
            wts.release()


def test_hybrid_ensure_feeds_the_routing_histogram():
    """ensure_experts_hybrid adds the raw routed ids to decode_freq (before the kernel
    rewrites them in place), like ensure_experts."""
    from tideway_b200 import OffloadMoeCache

    L, E, S, K = 2, 16, 24, 4
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=S, device=DEV,
                            hybrid_max_fetch=2)
    cache.collect_decode_freq = True
    g = torch.Generator().manual_seed(52)
    raws = [torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(3)]).to(torch.int32)
            for _ in range(3)]
    for r in raws:
        ids = r.to(DEV)
        cache.ensure_experts_hybrid(1, ids)
    torch.cuda.synchronize()
    want = torch.bincount(torch.cat(raws).view(-1).long(), minlength=E)
    assert torch.equal(cache.decode_freq[1].cpu(), want) and int(cache.decode_freq[0].sum()) == 0


def test_offload_layer_hybrid_decode_with_an_executor():
    """decode_target='hybrid' through OffloadMoELayer: a fetch cap of 2 per step leaves the
    other misses at -1; a test executor computes those routes from the host banks (the
    oracle over expert ids), and the GPU share plus the executor's share matches the whole
    layer (the oracle over expert ids) within the bf16 bound.  Every route goes to exactly
    one side, and the hybrid counters add up (misses - fetches = the executor's experts)."""
    import tideway_b200 as tw

    H, E, K, I, T, S = 1024, 16, 4, 512, 4, 16
    g = torch.Generator().manual_seed(77)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    cache = tw.OffloadMoeCache(num_layers=1, num_experts=E, cache_size=S, device=DEV,
                               decode_target="hybrid", hybrid_max_fetch=2)
    cache.set_bank_sources({"gate_up": [gate_up.pin_memory()], "down": [down.pin_memory()]})
    cache.collect_stats = True

    class Executor:
        def __init__(self):
            self.routes = []

        def decode_submit(self, layer_id, h, w, ids):
            self.routes.append(ids.clone())
            return h.clone(), w.clone(), ids.clone()

        def decode_sync(self, pending):
            h, w, ids = pending
            return off.moe_decode(h.cpu(), gate_up, down, w.cpu(), ids.cpu()).to(h.device)

    ex = Executor()
    cache.set_cpu_executor(ex)
    layer = tw.OffloadMoELayer(0, E, K, H, I, renormalize=True)
    layer.offload_cache = cache
    cpu_experts = 0
    for step in range(4):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=g)
        with tw.batch_context(is_prefill=False):
            out = layer.forward(x.to(DEV), logits.to(DEV))
        torch.cuda.synchronize()
        w_ref, ids_ref = orouting.softmax_topk(logits, K, True)
        ref = off.moe_decode(x, gate_up, down, w_ref, ids_ref)
        assert _rel(out, ref) <= RTOL_BF16, (step, _rel(out, ref))
        cpu_ids = ex.routes[-1].cpu()
        assert torch.equal(cpu_ids[cpu_ids >= 0], ids_ref[cpu_ids >= 0])
        cpu_experts += len(torch.unique(cpu_ids[cpu_ids >= 0]))
    assert cpu_experts > 0
    st = cache.decode_miss_stats()
    assert st["layer_calls"] == 4 and st["fetched_per_layer"] <= 2
    assert round(st["cpu_per_layer"] * 4) == cpu_experts
    cache.verify_tables()


def test_empty_inputs_are_no_ops():
    """T = 0 through every entry point: no launch error, empty outputs, and the slot
    ensures take a step with nothing to fetch."""
    from tideway_b200 import ops

    H, I, S, E = 1024, 512, 8, 16
    x = torch.empty(0, H, dtype=torch.bfloat16, device=DEV)
    w1 = torch.zeros(S, 2 * I, H, dtype=torch.bfloat16, device=DEV)
    w2 = torch.zeros(S, H, I, dtype=torch.bfloat16, device=DEV)
    tw = torch.empty(0, 2, dtype=torch.float32, device=DEV)
    ti = torch.empty(0, 2, dtype=torch.int32, device=DEV)
    assert ops.moe_ffn_bf16(x, w1, w2, tw, ti).shape == (0, H)
    assert ops.ffn_dense_bf16(x, w1[0], w2[0]).shape == (0, H)
    logits = ops.router_logits(x, torch.zeros(E, H, dtype=torch.bfloat16, device=DEV))
    assert logits.shape == (0, E)
    w, ids = ops.softmax_topk(logits, 2, True)
    assert w.shape == (0, 2) and ids.shape == (0, 2)
    nw = torch.ones(H, dtype=torch.bfloat16, device=DEV)
    assert ops.rmsnorm(x, nw, 1e-6).shape == (0, H)
    d, xh = _DevTable(2, E, S), _hybrid_extra(2, E)
    empty = np.zeros((0, 2), np.int32)
    assert d.ensure(empty, 0).shape == (0, 2)
    assert int(d.num.item()) == 0 and int(d.step.item()) == 1
    assert _hybrid_step(d, xh, empty, 1, 4, 0, True).shape == (0, 2)
    assert int(d.num.item()) == 0 and int(xh["full"].item()) == 0 and int(d.step.item()) == 2
    torch.cuda.synchronize()


def test_moe_ffn_bf16_largest_route_count():
    """65528 routes (T = 8191, K = 8): positions fill the 16-bit range the grouping keeps,
    slots of ~1000 routes split into 256-route segments; against the oracle."""
    from tideway_b200 import ops

    T, H, I, S, K = 8191, 256, 128, 64, 8
    g = torch.Generator().manual_seed(65)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(S, H, I, g)
    tw, ti = _routing(T, K, S, g)
    out = ops.moe_ffn_bf16(x.to(DEV), w1.to(DEV), w2.to(DEV), tw.to(DEV), ti.to(DEV)).cpu()
    ref = off.moe_decode(x, w1, w2, tw, ti)
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)


@pytest.mark.parametrize("T,H,I,S,K", [(300, 1024, 512, 16, 4), (64, 5120, 256, 8, 8)])
def test_moe_ffn_dual_merge_bit_exact(T, H, I, S, K):
    """The routed FFN with its combine fused into the Gemma dual-norm merge equals
    moe_ffn_bf16 followed by dual_norm_merge bit for bit (128- and 256-thread rows), in
    place on the residual as the prefill stack calls it."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    sh = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    wn = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV) for _ in range(3)]
    w1, w2 = (t.to(DEV) for t in _bank(S, H, I, g))
    tw, ti = (t.to(DEV) for t in _routing(T, K, S, g))
    routed = ops.moe_ffn_bf16(x, w1, w2, tw, ti)
    ref = ops.dual_norm_merge(sh, routed, res, *wn, 1e-6, 1e-5, 1e-6, 0.75)
    out = res.clone()
    ops.moe_ffn_bf16_dual_merge(x, w1, w2, tw, ti, sh, out, *wn, 1e-6, 1e-5, 1e-6, 0.75, out=out)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("T,H,I,act", [(40, 1024, 512, "gelu_tanh"), (600, 1152, 320, "gelu")])
def test_ffn_dense_bf16_activation_variants(T, H, I, act):
    """The dense (shared-expert) entry with a GELU gate equals the routed entry with the same
    activation, every row routed to slot 0 at weight 1, bit for bit; and the fp32 form of
    that FFN within the bf16 bound."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H + I + 7)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1, w2 = _bank(1, H, I, g)
    xd, w1d, w2d = x.to(DEV), w1.to(DEV), w2.to(DEV)
    ids = torch.zeros(T, 1, dtype=torch.int32, device=DEV)
    ones = torch.ones(T, 1, dtype=torch.float32, device=DEV)
    routed = ops.moe_ffn_bf16(xd, w1d, w2d, ones, ids, activation=act)
    ws = ops.workspace(T, H, I, DEV)
    dense = ops.ffn_dense_bf16(xd, w1d[0], w2d[0], ws=ws, activation=act)
    assert ops.workspace_error(ws, T, H, I) == 0
    assert torch.equal(dense, routed)
    h = x.float() @ w1[0].float().t()
    ref32 = (off.gate_activation(h[:, :I], act) * h[:, I:]) @ w2[0].float().t()
    assert _rel(dense, ref32) <= RTOL_BF16
    assert not torch.equal(dense, ops.ffn_dense_bf16(xd, w1d[0], w2d[0], ws=ws))


@pytest.mark.parametrize("act,w_in", [("gelu_tanh", False), ("gelu", True)])
def test_moe_ffn_dual_merge_activation_variants(act, w_in):
    """The fused routed FFN + Gemma merge with a GELU gate (and the route weight on the up
    projection) equals moe_ffn_bf16 with the same forms followed by dual_norm_merge, bit for
    bit."""
    from tideway_b200 import ops

    T, H, I, S, K = 300, 1024, 512, 16, 4
    g = torch.Generator().manual_seed(T + H + 3)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    sh = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    wn = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV) for _ in range(3)]
    w1, w2 = (t.to(DEV) for t in _bank(S, H, I, g))
    tw, ti = (t.to(DEV) for t in _routing(T, K, S, g))
    routed = ops.moe_ffn_bf16(x, w1, w2, tw, ti, activation=act, weight_on_input=w_in)
    ref = ops.dual_norm_merge(sh, routed, res, *wn, 1e-6, 1e-5, 1e-6, 0.75)
    out = res.clone()
    ops.moe_ffn_bf16_dual_merge(x, w1, w2, tw, ti, sh, out, *wn, 1e-6, 1e-5, 1e-6, 0.75,
                                out=out, activation=act, weight_on_input=w_in)
    assert torch.equal(out, ref)


def test_cache_rebuild_then_decode_and_prefill():
    """rebuild() resizes the slot cache in place: after decode steps at one size, a rebuild
    to a larger and then a smaller size keeps the layers attached, starts every slot empty
    (the tables match a cold oracle table step for step) and the layers' decode and
    double-buffered prefill outputs still match the oracle."""
    from tideway_b200 import OffloadMoeCache, OffloadMoELayer, attach_offload_moe_cache
    from tideway_b200 import batch_context

    L, E, K, H, I = 2, 8, 2, 512, 256
    g = torch.Generator().manual_seed(43)
    banks = [_bank(E, H, I, g) for _ in range(L)]
    cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=2 * E + 2, device=DEV,
                            prefill_overlap=True)
    cache.set_bank_sources({"gate_up": [b[0].pin_memory() for b in banks],
                            "down": [b[1].pin_memory() for b in banks]})
    layers = attach_offload_moe_cache([OffloadMoELayer(l, E, K, H, I) for l in range(L)], cache)

    def run(phase, T):
        with batch_context(is_prefill=phase == "prefill"):
            for l in range(L):
                x = torch.randn(T, H, generator=g).to(torch.bfloat16)
                logits = torch.randn(T, E, generator=g)
                out = layers[l].forward(x.to(DEV), logits.to(DEV)).cpu()
                w, ids = orouting.softmax_topk(logits, K, True)
                ref = off.moe_decode(x, banks[l][0], banks[l][1], w, ids)
                assert _rel(out, ref) <= RTOL_BF16, (phase, l, _rel(out, ref))

    run("decode", 3)
    for size in (2 * E + 9, E + 3):
        cache.rebuild(size)
        assert cache.cache_size == size and cache.id_of_slot.numel() == size
        assert int((cache.id_of_slot >= 0).sum()) == 0
        assert cache.prefill_overlap == (size >= 2 * E)
        ref = osc.SlotTable(L, E, size)
        for step in range(3):
            ids = torch.randint(0, E, (2, K), generator=g, dtype=torch.int32)
            d = ids.to(DEV)
            cache.ensure_experts(step % L, d)
            cache.copy_missing()
            assert np.array_equal(d.cpu().numpy(), osc.lru_ensure(ref, ids.numpy(), step % L))
        assert np.array_equal(cache.id_of_slot.cpu().numpy(), ref.id_of_slot)
        cache.verify_tables()
        audit = cache.verify_payload(raise_on_mismatch=False)  # copies land in the new banks
        assert audit["rows"] > 0 and not audit["mismatches"]
        run("decode", 2)
        run("prefill", 20)
