"""The FFN kernels' bounded waits, driven to expiry (B200 only).

Every mbarrier and hand-off wait inside the tensor-core FFN kernels stops after a poll
limit, records error word 1 in the call's workspace, lets the copies and MMAs it already
issued land, frees its tensor memory and returns: the GPU context stays usable.  With the
limit lowered to one poll (tw_set_wait_limit) some wait of a launch gives up before its
data can have arrived, so these tests take that path without any stuck or faulting
kernel: the error word is read back, the decode stack fails closed, and calls made after
the limit is restored give the same bits as before.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tideway_b200

    tideway_b200.load()


def _inputs(T, H, I, S, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (0.02 * torch.randn(S, 2 * I, H, generator=g)).to(torch.bfloat16).to(DEV)
    w2 = (0.02 * torch.randn(S, H, I, generator=g)).to(torch.bfloat16).to(DEV)
    ids = torch.stack([torch.randperm(S, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, K, generator=g)
    return x, w1, w2, (w / w.sum(-1, keepdim=True)).to(DEV), ids.to(DEV)


@pytest.mark.parametrize("T", [1, 8, 300])
def test_bf16_ffn_wait_expiry_sets_the_error_word(T):
    from tideway_b200 import ops

    H, I, S, K = 1024, 512, 16, 4
    x, w1, w2, w, ids = _inputs(T, H, I, S, K, T)
    ws = torch.empty(ops.workspace_bytes(T * K, H, I), dtype=torch.uint8, device=DEV)
    good = ops.moe_ffn_bf16(x, w1, w2, w, ids, ws=ws)
    assert ops.workspace_error(ws, T * K, H, I) == 0
    ops.set_wait_limit(1)
    try:
        ops.moe_ffn_bf16(x, w1, w2, w, ids, ws=ws)
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(0)
    assert ops.workspace_error(ws, T * K, H, I) == 1
    again = ops.moe_ffn_bf16(x, w1, w2, w, ids, ws=ws)
    assert ops.workspace_error(ws, T * K, H, I) == 0
    assert torch.equal(again, good)


def test_nvfp4_ffn_wait_expiry_sets_the_error_word():
    from tideway_b200 import nvfp4, ops

    T, H, I, S, K = 16, 1024, 512, 8, 4
    g = torch.Generator().manual_seed(7)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    packs = [nvfp4.quantize_expert(0.02 * torch.randn(2 * I, H, generator=g),
                                   0.02 * torch.randn(H, I, generator=g)) for _ in range(S)]
    w1 = tuple(torch.stack([p[0][j] for p in packs]).to(DEV) for j in range(3))
    w2 = tuple(torch.stack([p[1][j] for p in packs]).to(DEV) for j in range(3))
    ids = torch.stack([torch.randperm(S, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.full((T, K), 1.0 / K)
    ids, w = ids.to(DEV), w.to(DEV)
    ws = torch.empty(ops.workspace_bytes(T * K, H, I), dtype=torch.uint8, device=DEV)
    good = ops.moe_ffn_nvfp4(x, w1, w2, w, ids, ws=ws)
    assert ops.workspace_error(ws, T * K, H, I) == 0
    ops.set_wait_limit(1)
    try:
        ops.moe_ffn_nvfp4(x, w1, w2, w, ids, ws=ws)
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(0)
    assert ops.workspace_error(ws, T * K, H, I) == 1
    again = ops.moe_ffn_nvfp4(x, w1, w2, w, ids, ws=ws)
    assert ops.workspace_error(ws, T * K, H, I) == 0
    assert torch.equal(again, good)


def test_decode_stack_fails_closed_on_an_expired_wait():
    from tideway_b200 import ops
    from tideway_b200.stack import MoEDecodeStack, StackConfig, StackWeights

    cfg = StackConfig("small", layers=2, hidden=1024, experts=16, topk=4, inter=256,
                      slot_fraction=0.5, seed=8)
    wts = StackWeights(cfg, device=DEV)
    try:
        st = MoEDecodeStack(wts, batch=4)
        st.x_in.copy_(torch.randn(4, cfg.hidden, generator=torch.Generator().manual_seed(1))
                      .to(torch.bfloat16))
        st.step_eager()
        st.check()
        ops.set_wait_limit(1)
        try:
            st.step_eager()  # eager: the limit is read when each FFN is launched
            torch.cuda.synchronize()
        finally:
            ops.set_wait_limit(0)
        with pytest.raises(RuntimeError, match="error word"):
            st.check()
        assert st.state == "failed"
        with pytest.raises(RuntimeError, match="not retried"):
            st.step()
        del st
    finally:
        wts.release()
