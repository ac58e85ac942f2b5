"""DS-FP4 (e2m1 + e8m0 per 32) re-encoded as this build's NVFP4 banks: the NVFP4 reading of
the re-encoded bytes equals the DS-FP4 reading of the original, value for value."""

from __future__ import annotations

import json

import pytest
import torch

from oracle import nvfp4 as onv
from tests.golden import synthetic_checkpoints as sc
from tideway_b200 import ds_fp4, geometry


def _exact(packed, e8m0):
    p, s, g, flushed = ds_fp4.to_nvfp4(packed, e8m0)
    rows = packed.shape[-2]
    nv = onv.dequantize(p.reshape(-1, p.shape[-1]), s.reshape(-1, s.shape[-1]), g.reshape(-1))
    ds = onv.dequantize_ds_fp4(packed.reshape(-1, packed.shape[-1]),
                               e8m0.reshape(-1, e8m0.shape[-1]))
    return nv.reshape(*packed.shape[:-2], rows, -1), ds.reshape(*packed.shape[:-2], rows, -1), \
        flushed, (p, s, g)


def test_quantised_weights_reencode_exactly():
    g = torch.Generator().manual_seed(0)
    w = 0.02 * torch.randn(96, 512, generator=g)
    packed, e8 = onv.quantize_ds_fp4(w)
    assert ((onv.dequantize_ds_fp4(packed, e8) - w).norm() / w.norm()) < 0.2
    nv, ds, flushed, (p, s, gl) = _exact(packed, e8)
    assert flushed == 0 and torch.equal(nv, ds)
    assert p.data_ptr() == packed.data_ptr()  # codes are kept, not copied
    assert s.dtype == torch.float8_e4m3fn and s.shape == (96, 512 // 16)
    assert gl.dtype == torch.float32 and gl.shape == (96,)


def test_every_scale_byte_within_the_span():
    """Each row holds scales b .. b+17 (the widest exact span) for b over 0..235 (up to the
    largest scale whose weights stay finite in fp32); the codes run over all 256 bytes."""
    rows, K = 236, 18 * 32
    e8 = (torch.arange(rows).view(-1, 1) + torch.arange(18).view(1, -1)).to(torch.uint8)
    packed = (torch.arange(rows * K // 2) % 256).to(torch.uint8).view(rows, K // 2)
    nv, ds, flushed, _ = _exact(packed, e8)
    assert flushed == 0 and torch.equal(nv, ds)


def test_blocks_beyond_the_span_flush_to_zero():
    packed = torch.full((2, 64), 0x77, dtype=torch.uint8)  # every weight = 6 * scale
    e8 = torch.tensor([[140, 140 - 17, 140 - 18, 140 - 40],
                       [127, 127, 127, 127]], dtype=torch.uint8)
    nv, ds, flushed, _ = _exact(packed, e8)
    assert flushed == 2
    assert torch.equal(nv[0, :64], ds[0, :64])          # 17 binades down: exact
    assert torch.equal(nv[0, 64:], torch.zeros(64))      # 18 and 40 down: flushed
    assert torch.equal(nv[1], ds[1])


def test_leading_dims_and_e8m0_dtype():
    g = torch.Generator().manual_seed(1)
    E, rows, K = 3, 16, 256
    packed = torch.randint(0, 256, (E, rows, K // 2), dtype=torch.uint8, generator=g)
    e8 = torch.randint(110, 125, (E, rows, K // 32), dtype=torch.uint8, generator=g)
    nv, ds, flushed, (p, s, gl) = _exact(packed, e8.view(torch.float8_e8m0fnu))
    assert flushed == 0 and torch.equal(nv, ds)
    assert s.shape == (E, rows, K // 16) and gl.shape == (E, rows)


def test_rejects_nan_scales_and_mismatched_shapes():
    packed = torch.zeros(2, 32, dtype=torch.uint8)
    with pytest.raises(ValueError, match="NaN"):
        ds_fp4.to_nvfp4(packed, torch.tensor([[1, 255], [1, 1]], dtype=torch.uint8))
    with pytest.raises(ValueError, match="same rows"):
        ds_fp4.to_nvfp4(packed, torch.ones(2, 3, dtype=torch.uint8))
    with pytest.raises(ValueError, match="uint8"):
        ds_fp4.to_nvfp4(packed.to(torch.int16), torch.ones(2, 2, dtype=torch.uint8))


def _ds_checkpoint(root, layers=2, experts=3, H=256, I=128):
    """A DeepSeek-V4-layout checkpoint of quantised N(0, 0.02) experts (realistic scales)."""
    g = torch.Generator().manual_seed(5)
    root.mkdir()
    tensors, dense = [], {}
    for layer in range(layers):
        for e in range(experts):
            for proj, (rows, cols) in (("w1", (I, H)), ("w2", (H, I)), ("w3", (I, H))):
                w = 0.02 * torch.randn(rows, cols, generator=g)
                packed, e8 = onv.quantize_ds_fp4(w)
                dense[layer, e, proj] = onv.dequantize_ds_fp4(packed, e8)
                key = sc.DS_KEY.format(layer=layer, expert=e, proj=proj, kind="{kind}")
                tensors.append((key.format(kind="weight"), "I8", tuple(packed.shape),
                                packed.numpy().tobytes()))
                tensors.append((key.format(kind="scale"), "F8_E8M0", tuple(e8.shape),
                                e8.numpy().tobytes()))
    sc.write_shard(root / "m.safetensors", tensors)
    (root / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {k: "m.safetensors" for k, *_ in tensors}}))
    return root, dense


def test_checkpoint_to_nvfp4_host_banks(tmp_path):
    """A DS-FP4 checkpoint read layer by layer into NVFP4 host banks: gate rows (w1) before
    up rows (w3), every weight the checkpoint's DS-FP4 value."""
    root, dense = _ds_checkpoint(tmp_path / "dsv4")
    geo = geometry.from_checkpoint(root)
    assert geo.quant == "ds_fp4" and (geo.layers, geo.experts) == (2, 3)
    sources, flushed = ds_fp4.host_bank_sources(geo, pin=False, workers=2)
    assert flushed == 0 and tuple(sources) == ds_fp4.NVFP4_BANKS
    for layer in range(2):
        for e in range(3):
            gp, gs, gg, dp, dsc, dg = (sources[n][layer][e] for n in ds_fp4.NVFP4_BANKS)
            w13 = onv.dequantize(gp, gs, gg)
            assert torch.equal(w13, torch.cat([dense[layer, e, "w1"], dense[layer, e, "w3"]]))
            assert torch.equal(onv.dequantize(dp, dsc, dg), dense[layer, e, "w2"])
    with pytest.raises(ValueError, match="not ds_fp4"):
        ds_fp4.host_bank_sources(geometry.from_checkpoint(sc.write_fused(tmp_path, "plain")))


def test_random_synthetic_checkpoint_scales_are_rejected_or_flushed(tmp_path):
    """The miniature golden checkpoint holds uniformly random bytes: its scales include the
    NaN byte or spans far beyond 17 binades, and the re-encoding says so."""
    geo = geometry.from_checkpoint(sc.write_ds(tmp_path))
    with geometry.CheckpointReader(geo) as r:
        banks = r.layer_banks(0)
    raw = torch.cat([banks["gate_up_scale"].view(torch.uint8).reshape(-1),
                     banks["down_scale"].view(torch.uint8).reshape(-1)])
    if bool((raw == 255).any()):
        with pytest.raises(ValueError, match="NaN"):
            ds_fp4.expert_banks(*(banks[n] for n in ds_fp4.DS_FP4_BANKS))
    else:
        _, flushed = ds_fp4.expert_banks(*(banks[n] for n in ds_fp4.DS_FP4_BANKS))
        assert flushed > 0
