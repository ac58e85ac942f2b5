"""The allocation-free expert-FFN entry point against the workspace one (B200 only).

tw_moe_ffn_bf16_noalloc serves callers that cannot hand the library a workspace: a plugin
inside a serving process whose memory pool owns the whole GPU and forbids allocations outside
it, or a foreign-language binding with no device allocator.  Its scratch is a static device
array.  Both entry points run the same kernels on the same inputs, so their outputs must be
bit-identical; a stale scratch left by the previous call would show up as a difference.
This file is collected last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tideway_b200 import _lib

    return _lib.load()


def _inputs(seed, T, H, I, S, K):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(S, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).cuda()
    w2 = (torch.randn(S, H, I, generator=g) * 0.02).to(torch.bfloat16).cuda()
    ids = torch.stack([torch.randperm(S, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, K, generator=g)
    w = (w / w.sum(-1, keepdim=True)).float()
    return x, w1, w2, w.cuda().contiguous(), ids.cuda().contiguous()


def _call_noalloc(lib, x, w1, w2, w, ids, out):
    T, H = x.shape
    S, twoI, _ = w1.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tw_moe_ffn_bf16_noalloc(x.data_ptr(), T, H, twoI // 2, w1.data_ptr(),
                                       w2.data_ptr(), S, w.data_ptr(), ids.data_ptr(),
                                       ids.shape[1], out.data_ptr(), stream)


def _call_workspace(lib, x, w1, w2, w, ids, out):
    T, H = x.shape
    S, twoI, _ = w1.shape
    K = ids.shape[1]
    I = twoI // 2
    ws = torch.empty(lib.tw_moe_workspace_bytes(T * K, H, I), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tw_moe_ffn_bf16(x.data_ptr(), T, H, I, w1.data_ptr(), w2.data_ptr(), S,
                             w.data_ptr(), ids.data_ptr(), K, out.data_ptr(), ws.data_ptr(),
                             ws.numel(), stream)
    return rc, ws


def _noalloc_error_word(lib, n_routes, H, I):
    err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    rc = lib.tw_moe_ffn_noalloc_error(n_routes, H, I, err.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.tw_last_error()
    return int(err.item())


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row(lib):
    # two calls in a row share the static scratch (the second one must reset what the first
    # left there); the second call has other shapes, so a stale segment table would show
    for seed, (T, H, I, S, K) in ((1, (8, 2048, 768, 64, 8)), (2, (37, 1024, 512, 48, 6))):
        x, w1, w2, w, ids = _inputs(seed, T, H, I, S, K)
        out_na = torch.empty_like(x)
        out_ws = torch.empty_like(x)
        rc = _call_noalloc(lib, x, w1, w2, w, ids, out_na)
        assert rc == 0, lib.tw_last_error()
        assert _noalloc_error_word(lib, T * K, H, I) == 0
        rc, _ = _call_workspace(lib, x, w1, w2, w, ids, out_ws)
        assert rc == 0, lib.tw_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out_na.float()).all()
        assert torch.equal(out_na, out_ws)


def test_noalloc_rejects_sizes_beyond_its_scratch(lib):
    H, I, K = 4096, 2048, 8
    cap = lib.tw_moe_ffn_noalloc_scratch_bytes()
    T = 1
    while lib.tw_moe_workspace_bytes(T * K, H, I) <= cap:
        T *= 2
    x = torch.zeros(T, H, dtype=torch.bfloat16, device="cuda")
    w1 = torch.zeros(2, 2 * I, H, dtype=torch.bfloat16, device="cuda")
    w2 = torch.zeros(2, H, I, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(T, K, dtype=torch.float32, device="cuda")
    ids = torch.zeros(T, K, dtype=torch.int32, device="cuda")
    out = torch.full_like(x, 7.0)
    rc = _call_noalloc(lib, x, w1, w2, w, ids, out)
    assert rc == 1  # TW_ERR_INVALID
    assert b"static scratch" in lib.tw_last_error()
    torch.cuda.synchronize()
    assert (out == 7.0).all()  # nothing was launched
