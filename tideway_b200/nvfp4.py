"""NVFP4 weight packing for the slot banks (host/setup utility, not on the hot path).

Layout consumed by ``tw_moe_ffn_nvfp4``:

* ``packed``  uint8 [rows, K/2]: element 2j in the low nibble, 2j+1 in the high nibble;
  nibble = sign (bit 3) | e2m1 magnitude code over {0, .5, 1, 1.5, 2, 3, 4, 6}.
* ``scale``   float8_e4m3fn [rows, K/16], one per 16-element block.
* ``global_`` float32 or float16 [rows]: the per-tensor scale broadcast to each of its rows
  (float16 per-output-row globals are the reference's ModelOpt row format).

W = e2m1 * e4m3 * global.  Quantisation: global = amax / (6 * 448) per tensor;
block scale = e4m3(block_amax / 6 / global); code = nearest e2m1 of w / (scale * global)
with ties to the even code.
"""

from __future__ import annotations

import torch

_MAGS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
# decision boundaries between consecutive magnitudes and which side wins a tie
_BOUNDS = ((0.25, 0), (0.75, 2), (1.25, 2), (1.75, 4), (2.5, 4), (3.5, 6), (5.0, 6))


def _e2m1_code(a: torch.Tensor) -> torch.Tensor:
    """Nearest e2m1 magnitude code (0..7) of |values| a, ties to the even code."""
    code = torch.zeros_like(a, dtype=torch.uint8)
    for i, (b, even) in enumerate(_BOUNDS):
        above = (a > b) | ((a == b) & (even == i + 1))
        code = code + above.to(torch.uint8)
    return code


def quantize(w: torch.Tensor, row_groups: list[int] | None = None,
             global_dtype: torch.dtype = torch.float32):
    """[rows, K] float -> (packed u8 [rows, K/2], scale e4m3 [rows, K/16], global [rows]).

    ``global_dtype`` float16 gives the reference's ModelOpt row format (fp16 per-row globals):
    the global is rounded to fp16 first and the block scales are taken against the rounded
    value, so the three factors still multiply back to the quantised weight exactly."""
    w = w.float()
    rows, K = w.shape
    if K % 32:
        raise ValueError("K must be a multiple of 32")
    groups = row_groups or [rows]
    glob = torch.empty(rows, dtype=torch.float32, device=w.device)
    r0 = 0
    for n in groups:
        amax = w[r0:r0 + n].abs().max().clamp(min=1e-12)
        glob[r0:r0 + n] = amax / (6.0 * 448.0)
        r0 += n
    glob = glob.to(global_dtype).float()
    blocks = w.view(rows, K // 16, 16)
    bamax = blocks.abs().amax(dim=-1)
    scale = (bamax / 6.0 / glob.view(-1, 1)).clamp(max=448.0).to(torch.float8_e4m3fn)
    denom = scale.float() * glob.view(-1, 1)
    denom = torch.where(denom > 0, denom, torch.ones_like(denom))
    q = (blocks / denom.unsqueeze(-1)).reshape(rows, K)
    code = _e2m1_code(q.abs())
    code = torch.where((q < 0) & (code > 0), code | 8, code)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), scale.contiguous(), glob.to(global_dtype)


def quantize_expert(w1: torch.Tensor, w2: torch.Tensor,
                    global_dtype: torch.dtype = torch.float32):
    """One expert: w1 [2I, H] (gate rows then up rows, separate tensor scales), w2 [H, I]."""
    I = w1.shape[0] // 2
    return quantize(w1, [I, I], global_dtype), quantize(w2, None, global_dtype)


def dequantize(packed: torch.Tensor, scale: torch.Tensor, global_: torch.Tensor) -> torch.Tensor:
    """Exact fp32 values of a packed tensor (for setup checks)."""
    lut = torch.tensor(_MAGS + tuple(-m for m in _MAGS), dtype=torch.float32, device=packed.device)
    lo = (packed & 0xF).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], dim=-1).reshape(packed.shape[0], -1)
    return lut[codes] * scale.float().repeat_interleave(16, dim=1) * global_.float().view(-1, 1)
