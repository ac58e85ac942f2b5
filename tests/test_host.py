"""CPU-side checks: the C-ABI library loads and exports its header, host utilities."""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4 as onvfp4

ROOT = Path(__file__).resolve().parents[1]


def _header_symbols() -> list[str]:
    text = (ROOT / "include" / "tideway_b200.h").read_text()
    return re.findall(r"^\s*(?:int|const char\*|size_t)\s+(tw_\w+)\s*\(", text, re.M)


def test_library_builds_and_exports_every_header_symbol():
    from tideway_b200 import _lib, build

    build.build()
    lib = _lib.load()
    syms = _header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/tideway_b200.h but not exported"
    # the ctypes binding covers every header entry point
    assert set(syms) <= set(_lib.exported_symbols())
    assert lib.tw_abi_version() == 103


def test_workspace_size_is_monotone():
    from tideway_b200 import _lib

    lib = _lib.load()
    a = lib.tw_moe_workspace_bytes(8, 2048, 768)
    b = lib.tw_moe_workspace_bytes(512, 2048, 768)
    assert 0 < a < b
    assert b >= 512 * (2048 + 768) * 2


def test_ops_refuse_cpu_tensors():
    from tideway_b200 import ops

    try:
        ops.softmax_topk(torch.randn(2, 8), 2, True)
    except RuntimeError as e:
        assert "CUDA" in str(e)
    else:
        raise AssertionError("CPU tensors must be refused (no CPU fallback)")


def test_ensure_refuses_malformed_stats_and_pins():
    """The optional ``stats`` and ``pinned`` tensors are checked before any launch: a CPU
    tensor, a wrong dtype or a pinned mask of the wrong length is refused."""
    from tideway_b200 import ops

    S = 8
    ios = torch.zeros(S, dtype=torch.int32)
    ops._check_ensure_extras(ios, None, None)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops._check_ensure_extras(ios, torch.zeros(4, dtype=torch.int64), None)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops._check_ensure_extras(ios, None, torch.zeros(S, dtype=torch.int32))

    class Dev:  # a CUDA-looking stand-in, so the dtype and shape checks run without a GPU
        def __init__(self, t):
            self.t, self.is_cuda = t, True
            self.dtype = t.dtype

        def is_contiguous(self):
            return self.t.is_contiguous()

        def numel(self):
            return self.t.numel()

    ops._check_ensure_extras(ios, Dev(torch.zeros(3, dtype=torch.int64)),
                             Dev(torch.zeros(S, dtype=torch.int32)))
    for stats, pinned in ((Dev(torch.zeros(2, dtype=torch.int64)), None),
                          (Dev(torch.zeros(4, dtype=torch.int32)), None),
                          (None, Dev(torch.zeros(S, dtype=torch.bool))),
                          (None, Dev(torch.zeros(S - 1, dtype=torch.int32))),
                          (None, Dev(torch.zeros(S, 2, dtype=torch.int32)[:, 0]))):
        with pytest.raises(ValueError):
            ops._check_ensure_extras(ios, stats, pinned)


def test_activation_entries_refuse_unknown_forms_before_any_launch():
    """The C entries check the activation code before touching device memory (no GPU)."""
    from tideway_b200 import _lib

    lib = _lib.load()
    rc = lib.tw_ffn_dense_bf16_act(None, 8, 256, 128, None, None, 7, None, None, 0, None)
    assert rc != 0 and b"activation" in lib.tw_last_error()
    rc = lib.tw_moe_ffn_bf16_act(None, 8, 256, 128, None, None, 4, None, None, 2, 3, 0, None,
                                 None, 0, None)
    assert rc != 0 and b"activation" in lib.tw_last_error()


def test_missing_library_fails_loudly():
    """With the CUDA library absent every op raises; nothing falls back to a CPU path."""
    import os
    import subprocess
    import sys

    code = ("import torch\n"
            "from tideway_b200 import ops\n"
            "try:\n"
            "    ops.workspace_bytes(8, 256, 128)\n"
            "except RuntimeError as e:\n"
            "    assert 'not built' in str(e), e\n"
            "    print('refused')\n")
    env = dict(os.environ, TIDEWAY_B200_LIB=str(ROOT / "no_such_lib.so"))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip() == "refused", r.stdout + r.stderr


def test_activation_names_and_oracle_forms():
    """The FFN's activation names are the reference's (silu, gelu, gelu_tanh); others are
    refused before any launch; the oracle's gate activations follow their formulas."""
    import math

    from oracle import ffn as off
    from tideway_b200 import fused, moe_layer, ops

    assert ops._activation("gelu_tanh", True) == (2, 1)
    for bad in ("relu", "swigluoai"):
        with pytest.raises(ValueError):
            ops._activation(bad, False)
        with pytest.raises(ValueError):
            moe_layer.OffloadMoELayer(0, 8, 2, 64, 64, activation=bad)
    with pytest.raises(ValueError):
        fused._check(torch.zeros(1, 64, dtype=torch.bfloat16),
                     torch.zeros(2, 128, 64, dtype=torch.bfloat16),
                     torch.zeros(2, 64, 64, dtype=torch.bfloat16), torch.zeros(1, 2),
                     torch.zeros(1, 2, dtype=torch.int32), "relu")
    g = torch.tensor([-3.0, -0.5, 0.0, 0.7, 2.5])
    gelu = [0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in g.tolist()]
    tanh = [0.5 * v * (1 + math.tanh(math.sqrt(2 / math.pi) * (v + 0.044715 * v ** 3)))
            for v in g.tolist()]
    silu = [v / (1 + math.exp(-v)) for v in g.tolist()]
    for name, want in (("gelu", gelu), ("gelu_tanh", tanh), ("silu", silu)):
        np.testing.assert_allclose(off.gate_activation(g, name).numpy(), want, rtol=1e-6,
                                   atol=2e-6)


def test_weight_on_input_oracle_rounding_points():
    """weight_on_input scales the first GEMM's fp32 sums before their bf16 rounding and
    leaves the second GEMM unweighted; with every weight 1 both placements agree."""
    from oracle import ffn as off

    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 64, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(64, 64, generator=g) * 0.1).to(torch.bfloat16)
    w2 = (torch.randn(64, 32, generator=g) * 0.1).to(torch.bfloat16)
    w = torch.tensor([0.25, 0.5, 1.0])
    got = off.expert_ffn_routes(x, w1, w2, w, "silu", True)
    c1 = ((x.float() @ w1.float().t()) * w[:, None]).to(torch.bfloat16).float()
    c2 = (c1[:, :32] / (1 + torch.exp(-c1[:, :32])) * c1[:, 32:]).to(torch.bfloat16)
    assert torch.equal(got, (c2.float() @ w2.float().t()).to(torch.bfloat16))
    ones = torch.ones(3)
    assert torch.equal(off.expert_ffn_routes(x, w1, w2, ones, "gelu", True),
                       off.expert_ffn_routes(x, w1, w2, ones, "gelu", False))


def test_nvfp4_packer_matches_oracle_quantiser():
    from tideway_b200 import nvfp4

    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 256, generator=g) * 0.02
    p1, s1, g1 = nvfp4.quantize(w, [32, 32])
    p2, s2, g2 = onvfp4.quantize(w, [32, 32])
    assert torch.equal(p1, p2)
    assert torch.equal(s1.view(torch.uint8), s2.view(torch.uint8))
    assert torch.equal(g1, g2)
    d1 = nvfp4.dequantize(p1, s1, g1)
    d2 = onvfp4.dequantize(p2, s2, g2)
    assert torch.equal(d1, d2)
    # quantisation error of NVFP4 on N(0, 0.02) weights stays at the format's level
    rel = (d1 - w).norm() / w.norm()
    assert rel < 0.15


def test_nvfp4_ties_go_to_even_code():
    from tideway_b200 import nvfp4

    a = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0])
    assert nvfp4._e2m1_code(a).tolist() == [0, 2, 2, 4, 4, 6, 6, 7]
    np.testing.assert_array_equal(onvfp4.E2M1_VALUES[[0, 2, 2, 4, 4, 6, 6, 7]],
                                  [0, 1, 1, 2, 2, 4, 4, 6])


def test_nvfp4_ops_validate_banks_before_any_launch():
    """Wrong NVFP4 bank shapes or dtypes are refused by the shim (ValueError) before the
    kernel could read past a bank; well-formed banks only meet the CUDA-tensor check."""
    from tideway_b200 import ops

    S, H, I, T, K = 4, 256, 128, 3, 2
    u8, e4 = torch.uint8, torch.float8_e4m3fn

    def bank(rows, k):
        return (torch.zeros(S, rows, k // 2, dtype=u8),
                torch.zeros(S, rows, k // 16, dtype=u8).view(e4), torch.zeros(S, rows))

    x = torch.zeros(T, H, dtype=torch.bfloat16)
    tw, ti = torch.zeros(T, K), torch.zeros(T, K, dtype=torch.int32)
    w1, w2 = bank(2 * I, H), bank(H, I)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.moe_ffn_nvfp4(x, w1, w2, tw, ti)
    bad_cases = [
        ((w1[0], w1[1].float(), w1[2]), w2),            # scale dtype
        ((w1[0][:, :-1], w1[1], w1[2]), w2),           # odd row count
        ((w1[0], w1[1], w1[2].half()), w2),             # global dtype
        (w1, (w2[0], w2[1][:, :, :-1], w2[2])),         # scale width
        (w1, (w2[0][:1], w2[1], w2[2])),                # slot count
    ]
    for a, b in bad_cases:
        with pytest.raises(ValueError):
            ops.moe_ffn_nvfp4(x, a, b, tw, ti)
    with pytest.raises(ValueError):
        ops.moe_ffn_nvfp4(x, w1, w2, tw, ti.long())
    with pytest.raises(ValueError):
        ops.moe_ffn_nvfp4(x.float(), w1, w2, tw, ti)
    with pytest.raises(ValueError):
        ops.nvfp4_dequantize(w1[0][0], w1[1][0][:, :-1], w1[2][0])
