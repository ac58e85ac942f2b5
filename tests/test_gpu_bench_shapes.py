"""GPU parity at the exact shapes bench.py times (B200 only).

* one Gemma prefill layer at T=2048, H=2816, 128 experts, top-8, I=704, shared
  I=2112 -- the 160-route paired-tile FFN variant, the tensor-core router, the fused dual-norm
  merge -- stage by stage against the oracle, each stage fed with the GPU's previous one.
* the NVFP4 expert FFN at batch 128, H=4096, I=2048, top-6 sigmoid group routing,
  against dequantise-then-matmul.
* a decode step at batch 64 (H=2048, 128 experts, top-8, I=768) through the slot
  cache with half the experts resident, so every layer pages misses in from the pinned host
  banks before its FFN runs; per layer the routing ids bit-exact and the FFN output against
  the oracle over the host banks (expert ids, not slots).

Tolerances are those of tests/test_gpu_parity.py: ids bit-exact, fp32 router outputs rtol
1e-5 (logits 1e-4 relative to their largest), bf16 outputs max|gpu - oracle| / max|oracle|
<= 2e-2.
"""

import numpy as np
import pytest
import torch

from oracle import ffn as off
from oracle import nvfp4 as onv
from oracle import routing as orouting

pytestmark = pytest.mark.gpu

DEV = "cuda"
RTOL_BF16 = 2e-2


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tideway_b200

    tideway_b200.load()


def test_c3_prefill_layer_at_bench_shape():
    from tideway_b200 import ops
    from tideway_b200.prefill import GemmaPrefillStack, PrefillConfig

    cfg = PrefillConfig(layers=1)  # configs[2] layer shape, 2048 tokens
    assert (cfg.tokens, cfg.hidden, cfg.experts, cfg.topk, cfg.inter, cfg.shared_inter) == (
        2048, 2816, 128, 8, 704, 2112)
    st = GemmaPrefillStack(cfg, device=DEV)
    g = torch.Generator().manual_seed(2)
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
    sh = off.shared_expert(st.shared_in.cpu(), c["sh_w1"][0], c["sh_w2"][0])
    assert _rel(st.shared, sh) <= RTOL_BF16
    routed_gpu = ops.moe_ffn_bf16(st.routed_in, p["w1"], p["w2"], st.w, st.ids).cpu()
    routed = off.moe_prefill(st.routed_in.cpu(), c["w1"], c["w2"], st.w.cpu(), st.ids.cpu())
    assert _rel(routed_gpu, routed) <= RTOL_BF16, _rel(routed_gpu, routed)
    merged = off.dual_norm_merge(st.shared.cpu(), routed, x0, c["post_shared"],
                                 c["post_routed"], c["post"], cfg.eps, cfg.eps, cfg.eps,
                                 cfg.layer_scalar)
    assert _rel(st.x, merged) <= 1e-2


@pytest.mark.parametrize("T,H,I,E,K", [(2048, 2816, 704, 128, 8), (300, 2816, 704, 128, 8),
                                       (2048, 1024, 256, 16, 4)])
def test_paired_tile_ffn_is_deterministic(T, H, I, E, K):
    """The prefill FFN variants (160/256-route tiles, two weight tiles per item, sixteen
    epilogue warps) give the same bits on every call: a down tile starts only after every
    epilogue warp of every up item of its slot has published its activations.  Routed and
    dense (shared-expert) entries, three calls each."""
    from tideway_b200 import ops

    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (0.02 * torch.randn(E, 2 * I, H, generator=g)).to(torch.bfloat16).to(DEV)
    w2 = (0.02 * torch.randn(E, H, I, generator=g)).to(torch.bfloat16).to(DEV)
    logits = torch.randn(T, E, generator=g).to(DEV)
    w, ids = ops.softmax_topk(logits, K, True)
    outs = [ops.moe_ffn_bf16(x, w1, w2, w, ids) for _ in range(3)]
    assert all(torch.isfinite(o.float()).all() for o in outs)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    dense = [ops.ffn_dense_bf16(x, w1[0], w2[0]) for _ in range(3)]
    assert torch.equal(dense[0], dense[1]) and torch.equal(dense[0], dense[2])


def test_c4_nvfp4_ffn_at_bench_shape():
    """Batch 128 at the configs[3] expert shape: 64 slots (8 distinct quantised experts, each
    in 8 slots), routes from the sigmoid group top-k of configs[3] (8 groups, top-4, top-6,
    x2.5)."""
    from tideway_b200 import nvfp4, ops

    T, H, I, S, K = 128, 4096, 2048, 64, 6
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    packs = [nvfp4.quantize_expert(torch.randn(2 * I, H, generator=g) * 0.02,
                                   torch.randn(H, I, generator=g) * 0.02) for _ in range(8)]
    bank = [torch.stack([packs[s % 8][m][j] for s in range(S)]) for m in range(2)
            for j in range(3)]
    logits = torch.randn(T, S, generator=g)
    w, ids = orouting.sigmoid_group_topk(logits, K, 8, 4, 2.5, True)
    wg, idg = ops.sigmoid_group_topk(logits.to(DEV), K, 8, 4, 2.5, True)
    assert np.array_equal(idg.cpu().numpy(), ids.numpy())
    out = ops.moe_ffn_nvfp4(x.to(DEV), tuple(b.to(DEV) for b in bank[:3]),
                            tuple(b.to(DEV) for b in bank[3:]), wg, idg).cpu()
    dense = [(onv.dequantize(*p[0]), onv.dequantize(*p[1])) for p in packs]
    w1d = torch.stack([dense[s % 8][0] for s in range(S)])
    w2d = torch.stack([dense[s % 8][1] for s in range(S)])
    ref = off.moe_decode(x, w1d, w2d, wg.cpu(), idg.cpu())
    assert _rel(out, ref) <= RTOL_BF16, _rel(out, ref)


def test_c2_decode_step_b64_with_paging():
    """Two configs[1]-shaped layers at batch 64 with 128 slots: each layer routes ~126 distinct
    experts and finds half of them missing, so the step pages them in over the host link.
    The stack runs its unfused form (the FFN output is a tensor of its own; the fused form is
    bit-identical to it, tests/test_gpu_parity.py)."""
    from tideway_b200 import ops
    from tideway_b200.stack import MoEDecodeStack, StackConfig, StackWeights

    cfg = StackConfig("c2-b64", layers=2, hidden=2048, experts=128, topk=8, inter=768,
                      slot_fraction=0.5, seed=1)
    B = 64
    wts = StackWeights(cfg, device=DEV)
    rec = {"logits": [], "ids": [], "w": [], "h": [], "y": []}
    real = {n: getattr(ops, n) for n in ("router_softmax_topk", "moe_ffn_bf16")}

    def router_softmax_topk(h, rw, k, renorm, *a, out=None, logits_out=None, **kw):
        logits = torch.empty(h.shape[0], rw.shape[0], dtype=torch.float32, device=h.device)
        r = real["router_softmax_topk"](h, rw, k, renorm, *a, out=out, logits_out=logits, **kw)
        rec["h"].append(h.clone())
        rec["logits"].append(logits)
        rec["w"].append(r[0].clone())
        rec["ids"].append(r[1].clone())
        return r

    def moe_ffn_bf16(*a, **kw):
        r = real["moe_ffn_bf16"](*a, **kw)
        rec["y"].append(r.clone())
        return r

    try:
        st = MoEDecodeStack(wts, batch=B, fused=False)
        st.cache.collect_stats = True
        g = torch.Generator().manual_seed(64)
        st.x_in.copy_(torch.randn(B, cfg.hidden, generator=g).to(torch.bfloat16))
        for n, f in (("router_softmax_topk", router_softmax_topk),
                     ("moe_ffn_bf16", moe_ffn_bf16)):
            setattr(ops, n, f)
        try:
            st.step_eager()
            torch.cuda.synchronize()
        finally:
            for n, f in real.items():
                setattr(ops, n, f)
        assert st.cache.decode_miss_stats()["missing_per_layer"] > 16  # real paging
        for l in range(cfg.layers):
            h = rec["h"][l].cpu()
            logits = h.float() @ st.router_w[l].cpu().float().t()
            assert _rel(rec["logits"][l], logits) <= 1e-4
            w, ids = orouting.softmax_topk(rec["logits"][l].cpu(), cfg.topk, True)
            assert np.array_equal(rec["ids"][l].cpu().numpy(), ids.numpy()), l
            np.testing.assert_allclose(rec["w"][l].cpu().numpy(), w.numpy(), rtol=1e-5,
                                       atol=1e-7)
            ref = off.moe_decode(h, wts.gate_up[l], wts.down[l], w, ids)
            assert _rel(rec["y"][l], ref) <= RTOL_BF16, (l, _rel(rec["y"][l], ref))
        st.cache.verify_tables()
        del st
    finally:
        wts.release()
