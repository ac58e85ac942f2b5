"""DeepSeek-V4 FP4 experts on the NVFP4 tensor-core path.

DS-FP4 (the reference's ``ds_fp4`` bank schema, backends/.../moe/offload_cache.py:71-73;
checkpoint layout in src/tideway/offload/geometry.py:196-258) stores each weight row as
packed e2m1 codes ``[rows, K/2]`` and one e8m0 power-of-two scale per 32 elements
``[rows, K/32]``, with no global scale: W = e2m1 * 2^(b - 127).

This build's NVFP4 banks hold the same e2m1 codes with an e4m3 scale per 16 elements and
an fp32 scale per row: W = e2m1 * e4m3 * global.  A DS-FP4 row is re-encoded exactly,
once, when its banks are loaded:

* global = 2^(m - 135), m = the largest scale byte of the row;
* each 32-element scale 2^(b - 127) becomes two equal e4m3 scales 2^(b - m + 8).

e4m3 represents the powers of two 2^-9 .. 2^8 exactly, so every block whose scale lies
within 17 binades of the row's largest is reproduced bit for bit (the kernel's f16 code x
f16 scale products and the fp32 row scale are exact).  A block further below the row's
largest scale holds weights under 2^-17 of that block's; it is flushed to zero and counted.
The codes are copied unchanged (two per byte, element 2j in the low nibble, as the NVFP4
banks store them).  The scale bytes grow from 1/32 to 1/16 byte per weight plus 4 bytes a
row: 4.5 instead of 4.25 bits per weight.

The reference's DS-FP4 kernels take a ``swiglu_limit`` (backends/.../layers/moe.py:606-637)
whose arithmetic lives in the absent FreeToken; this path computes the unclamped SwiGLU
and is used only with ``swiglu_limit`` None.
"""

from __future__ import annotations

import torch

NVFP4_BANKS = ("gate_up_packed", "gate_up_scale", "gate_up_global",
               "down_packed", "down_scale", "down_global")
DS_FP4_BANKS = ("gate_up_packed", "gate_up_scale", "down_packed", "down_scale")
E8M0_NAN = 255
MAX_SPAN = 17   # binades an e4m3 power-of-two scale spans exactly (2^-9 .. 2^8)


def _pow2_f32(e: torch.Tensor) -> torch.Tensor:
    """Exact float32 2^e for integer e in [-149, 127] (subnormals included)."""
    e = e.to(torch.int32)
    normal = (e + 127).clamp(min=0) << 23
    sub = torch.ones_like(e) << (e + 149).clamp(min=0, max=22)
    return torch.where(e >= -126, normal, sub).view(torch.float32)


def _pow2_e4m3(d: torch.Tensor) -> torch.Tensor:
    """e4m3 bytes of 2^d for d in [-9, 8] (normal from 2^-6, subnormal below)."""
    d = d.to(torch.int32)
    normal = (d + 7).clamp(min=0) << 3
    sub = torch.ones_like(d) << (d + 9).clamp(min=0, max=2)
    return torch.where(d >= -6, normal, sub).to(torch.uint8)


def to_nvfp4(packed: torch.Tensor, scale: torch.Tensor):
    """Re-encode DS-FP4 rows ``packed [..., rows, K/2]`` (uint8) with e8m0 scales
    ``scale [..., rows, K/32]`` (uint8 or float8_e8m0fnu) as NVFP4.

    Returns ``(packed, scale_e4m3 [..., rows, K/16], global_f32 [..., rows], flushed)``;
    ``flushed`` counts the 32-element blocks set to zero (scale more than 17 binades below
    the row's largest).  Raises ``ValueError`` on a NaN scale byte or mismatched shapes.
    """
    if packed.dtype != torch.uint8:
        raise ValueError(f"packed codes must be uint8, got {packed.dtype}")
    b = scale.view(torch.uint8) if scale.dtype != torch.uint8 else scale
    if packed.shape[:-1] != b.shape[:-1] or packed.shape[-1] != 16 * b.shape[-1]:
        raise ValueError(f"codes {tuple(packed.shape)} and e8m0 scales {tuple(b.shape)} do "
                         "not describe the same rows (K/2 codes, K/32 scales)")
    b = b.to(torch.int32)
    if bool((b == E8M0_NAN).any()):
        raise ValueError("e8m0 scale byte 0xff (NaN) in a DS-FP4 bank")
    m = b.amax(dim=-1, keepdim=True) if b.shape[-1] else torch.zeros_like(b[..., :1])
    d = b - m + 8
    keep = d >= 8 - MAX_SPAN   # 2^-9, the smallest exact e4m3 power of two
    e4 = torch.where(keep, _pow2_e4m3(d), torch.zeros_like(d, dtype=torch.uint8))
    e4 = e4.repeat_interleave(2, dim=-1).contiguous().view(torch.float8_e4m3fn)
    glob = _pow2_f32(m.squeeze(-1) - 135).contiguous()
    return packed.contiguous(), e4, glob, int((~keep).sum())


def expert_banks(gate_up_packed, gate_up_scale, down_packed, down_scale):
    """DS-FP4 expert banks (any leading dims, gate rows before up rows as the checkpoint
    stacks w1 before w3) -> the six NVFP4 banks in schema order, plus the flushed count."""
    gp, gs, gg, f1 = to_nvfp4(gate_up_packed, gate_up_scale)
    dp, ds, dg, f2 = to_nvfp4(down_packed, down_scale)
    return dict(zip(NVFP4_BANKS, (gp, gs, gg, dp, ds, dg))), f1 + f2


def host_bank_sources(geo, layers=None, pin: bool = True, workers: int = 8):
    """NVFP4 host banks (``bank name -> [layer] -> [E, ...]``, the form
    ``OffloadMoeCache.set_bank_sources`` takes with ``quant_format="nvfp4"``) read from a
    DS-FP4 checkpoint one layer at a time and re-encoded.  Returns (sources, flushed)."""
    from .geometry import CheckpointReader

    if geo.quant != "ds_fp4":
        raise ValueError(f"{geo.name} is a {geo.quant!r} checkpoint, not ds_fp4")
    layers = range(geo.layers) if layers is None else layers
    out = {name: [] for name in NVFP4_BANKS}
    flushed = 0
    with CheckpointReader(geo, workers=workers) as reader:
        for layer in layers:
            ds = reader.layer_banks(layer)
            banks, f = expert_banks(*(ds[n] for n in DS_FP4_BANKS))
            flushed += f
            for name, t in banks.items():
                out[name].append(t.pin_memory() if pin else t)
    return out, flushed
