"""The torch.library custom ops: registered with their schemas, output shapes from the fake
implementations (no GPU needed), and no CPU kernel behind them."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import tideway_b200  # noqa: F401  (registers torch.ops.tideway_b200)
from tideway_b200 import library

T, E, K, H, I, S = 6, 16, 2, 256, 128, 24


def test_every_op_is_registered():
    for name in library.OPS:
        assert hasattr(torch.ops.tideway_b200, name), name
    mutable = {a.name for a in torch.ops.tideway_b200.lru_ensure.default._schema.arguments
               if a.alias_info is not None and a.alias_info.is_write}
    assert mutable == {"ids", "slot_for_id", "id_of_slot", "usage", "step", "evict_slots",
                       "src_indices", "num_indices"}


def test_fake_shapes():
    op = torch.ops.tideway_b200
    with FakeTensorMode():
        dev = "cuda"
        logits = torch.empty(T, E, device=dev)
        w, ids = op.fused_topk(logits, K, True)
        assert w.shape == (T, K) and w.dtype == torch.float32 and ids.dtype == torch.int32
        w, ids, priv = op.gemma_topk(logits, torch.empty(E, device=dev), K)
        assert priv.shape == (T, K) and priv.dtype == torch.int32
        w, ids = op.sigmoid_group_topk(logits, K, 4, 2, 2.5, True, None)
        assert w.shape == (T, K)
        x = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        assert op.router_logits(x, torch.empty(E, H, device=dev, dtype=torch.bfloat16)).shape \
            == (T, E)
        nw = torch.empty(H, device=dev, dtype=torch.bfloat16)
        assert op.rmsnorm(x, nw, 1e-6, 0.0).shape == x.shape
        a, b = op.router_norm_pair(x, nw, nw, nw, 1e-6, H ** -0.5)
        assert a.shape == b.shape == x.shape
        outs = op.router_norm_triple(x, nw, nw, nw, nw, 1e-6, H ** -0.5)
        assert len(outs) == 3 and all(o.shape == x.shape for o in outs)
        assert op.dual_norm_merge(x, x, x, nw, nw, nw, 1e-6, 1e-6, 1e-6, 1.0).shape == x.shape
        assert op.add_shared(x, x).shape == x.shape
        w1 = torch.empty(S, 2 * I, H, device=dev, dtype=torch.bfloat16)
        w2 = torch.empty(S, H, I, device=dev, dtype=torch.bfloat16)
        tw = torch.empty(T, K, device=dev)
        ti = torch.empty(T, K, device=dev, dtype=torch.int32)
        y = op.moe_ffn_bf16(x, w1, w2, tw, ti)
        assert y.shape == x.shape and y.dtype == torch.bfloat16
        assert op.ffn_dense_bf16(x, w1[0], w2[0]).shape == x.shape
        r, h = op.moe_ffn_bf16_residual_norm(x, w1, w2, tw, ti, x, nw, 1e-6)
        assert r.shape == h.shape == x.shape
        assert op.moe_ffn_bf16_dual_merge(x, w1, w2, tw, ti, x, x, nw, nw, nw, 1e-6, 1e-6,
                                          1e-6, 1.0).shape == x.shape
        u8 = torch.uint8
        y = op.moe_ffn_nvfp4(x, torch.empty(S, 2 * I, H // 2, device=dev, dtype=u8),
                             torch.empty(S, 2 * I, H // 16, device=dev, dtype=u8),
                             torch.empty(S, 2 * I, device=dev),
                             torch.empty(S, H, I // 2, device=dev, dtype=u8),
                             torch.empty(S, H, I // 16, device=dev, dtype=u8),
                             torch.empty(S, H, device=dev), tw, ti)
        assert y.shape == x.shape
        s_ids, e_ids, npad = op.moe_align_block_size(ti, 4, E)
        assert s_ids.shape == (T * K * 4,) and e_ids.shape == (T * K,) and npad.shape == (1,)
        s_ids, e_ids, _ = op.moe_align_block_size(torch.empty(64, 8, device=dev,
                                                               dtype=torch.int32), 16, E)
        assert s_ids.shape == (512 + 17 * 15,) and e_ids.shape == (-(-(512 + 17 * 15) // 16),)
        d = op.nvfp4_dequantize(torch.empty(3, 8, 32, device=dev, dtype=u8),
                                torch.empty(3, 8, 4, device=dev, dtype=u8),
                                torch.empty(3, 8, device=dev))
        assert d.shape == (3, 8, 64) and d.dtype == torch.float32
        i32, i64 = torch.int32, torch.int64
        op.lru_ensure(ti, torch.empty(2, E, device=dev, dtype=i32),
                      torch.empty(S, device=dev, dtype=i32), torch.empty(S, device=dev, dtype=i64),
                      torch.empty((), device=dev, dtype=i64), E, 0,
                      torch.empty(E, device=dev, dtype=i32), torch.empty(E, device=dev, dtype=i32),
                      torch.empty(1, device=dev, dtype=i64))


def test_no_cpu_kernel():
    with pytest.raises(NotImplementedError):
        torch.ops.tideway_b200.fused_topk(torch.zeros(2, 8), 2, True)
