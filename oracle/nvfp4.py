"""NVFP4 weight format restatement (CPU, test infrastructure only; parity unpinned).

Format named by the benchmark configuration: W = e2m1 * e4m3_scale[16-element block] *
fp32 global scale.  The reference reads this family of formats through kernels that are
absent here (backends/freetoken_tideway/freetoken/layers/moe.py:499-538, bank schema at
backends/.../moe/offload_cache.py:44-54), so the layout below is this build's own:

* ``packed``  uint8 [rows, K/2]: element 2j in the low nibble, 2j+1 in the high nibble;
  nibble = sign(bit 3) | magnitude code (bits 0-2) over {0, .5, 1, 1.5, 2, 3, 4, 6}.
* ``scale``   float8_e4m3fn [rows, K/16].
* ``global_`` float32 or float16 [rows]: the per-tensor scale broadcast to each row (gate
  and up rows of one expert may carry different tensor scales); float16 per-output-row
  globals are the reference's ModelOpt row format (offload_cache.py:44-54).
"""

from __future__ import annotations

import numpy as np
import torch

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


def dequantize(packed: torch.Tensor, scale: torch.Tensor, global_: torch.Tensor) -> torch.Tensor:
    """Exact fp32 dequantisation: e2m1 * float(e4m3) * global (per row)."""
    p = packed.numpy().astype(np.uint8)
    rows, half = p.shape
    codes = np.empty((rows, half * 2), np.uint8)
    codes[:, 0::2] = p & 0xF
    codes[:, 1::2] = p >> 4
    vals = torch.from_numpy(E2M1_VALUES[codes])
    s = scale.float().repeat_interleave(16, dim=1)
    return vals * s * global_.float().view(-1, 1)


def quantize(w: torch.Tensor, row_groups: list[int] | None = None):
    """Reference NVFP4 quantiser for tests: returns (packed, scale, global_).

    ``row_groups`` splits the rows into tensors that each get their own global scale
    (e.g. [I, I] for stacked gate/up).  Global dequant scale = amax / (6 * 448); block scale
    = e4m3(block_amax / 6 / global); code = nearest e2m1 of w / (scale * global), ties to
    the even code.
    """
    w = w.float()
    rows, K = w.shape
    groups = row_groups or [rows]
    glob = torch.empty(rows)
    r0 = 0
    for n in groups:
        amax = w[r0:r0 + n].abs().max().clamp(min=1e-12)
        glob[r0:r0 + n] = amax / (6.0 * 448.0)
        r0 += n
    blocks = w.view(rows, K // 16, 16)
    bamax = blocks.abs().amax(dim=-1)
    scale = (bamax / 6.0 / glob.view(-1, 1)).clamp(max=448.0).to(torch.float8_e4m3fn)
    denom = scale.float() * glob.view(-1, 1)
    denom = torch.where(denom > 0, denom, torch.ones_like(denom))
    q = (blocks / denom.unsqueeze(-1)).reshape(rows, K).numpy()
    mags = E2M1_VALUES[:8]
    a = np.abs(q)
    dist = np.abs(a[..., None] - mags)
    best = dist.min(axis=-1, keepdims=True)
    cand = dist == best
    # ties -> even code (lowest set bit clear); codes are 0..7 in magnitude order
    even_first = np.where(cand[..., ::2].any(axis=-1),
                          np.argmax(np.where(np.arange(8) % 2 == 0, cand, False), axis=-1),
                          np.argmax(cand, axis=-1))
    code = even_first.astype(np.uint8) | np.where(q < 0, 8, 0).astype(np.uint8)
    code = np.where(even_first == 0, 0, code).astype(np.uint8)  # no negative zero
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return torch.from_numpy(packed), scale, glob


# ------------------------------------------------------------------ DS-FP4
# DeepSeek-V4 FP4 (bank schema backends/.../moe/offload_cache.py:71-73): the same packed
# e2m1 codes with one e8m0 power-of-two scale per 32 elements and no global scale.  The
# kernels that read it live in the absent FreeToken (backends/.../layers/moe.py:606-637), so
# this restatement follows the format alone (parity unpinned); the nibble order is taken
# to be the NVFP4 banks' (element 2j in the low nibble).

def dequantize_ds_fp4(packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Exact fp32 DS-FP4 weights: e2m1 * 2^(b - 127) per 32-element block."""
    p = packed.numpy().astype(np.uint8)
    rows, half = p.shape
    codes = np.empty((rows, half * 2), np.uint8)
    codes[:, 0::2] = p & 0xF
    codes[:, 1::2] = p >> 4
    b = scale.view(torch.uint8).numpy().astype(np.int32)
    s = np.ldexp(np.float32(1.0), b - 127).astype(np.float32)
    return torch.from_numpy(E2M1_VALUES[codes] * np.repeat(s, 32, axis=1))


def quantize_ds_fp4(w: torch.Tensor):
    """Test quantiser: (packed u8 [rows, K/2], e8m0 scale u8 [rows, K/32]).  Block scale =
    the smallest power of two with |w| / scale <= 6; code = nearest e2m1, ties to even."""
    w = w.float()
    rows, K = w.shape
    blocks = w.view(rows, K // 32, 32)
    bamax = blocks.abs().amax(dim=-1).clamp(min=2.0 ** -120)
    e = torch.ceil(torch.log2(bamax / 6.0)).to(torch.int32).clamp(-127, 127)
    # log2 rounding: make sure the block fits under 6 * 2^e
    e = torch.where(bamax > 6.0 * torch.pow(2.0, e.float()), e + 1, e)
    q = (blocks / torch.pow(2.0, e.float()).unsqueeze(-1)).reshape(rows, K).numpy()
    mags = E2M1_VALUES[:8]
    a = np.abs(q)
    dist = np.abs(a[..., None] - mags)
    cand = dist == dist.min(axis=-1, keepdims=True)
    code = np.where(cand[..., ::2].any(axis=-1),
                    np.argmax(np.where(np.arange(8) % 2 == 0, cand, False), axis=-1),
                    np.argmax(cand, axis=-1)).astype(np.uint8)
    code = np.where((q < 0) & (code > 0), code | 8, code).astype(np.uint8)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return torch.from_numpy(packed), (e + 127).to(torch.uint8)
