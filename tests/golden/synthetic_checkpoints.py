"""Seeded miniature safetensors checkpoints in the reference's expert key layouts.

Used twice: by ``make_golden.py`` (which runs the reference's checkpoint geometry and
row reader over them to record the golden summary) and by the tests (which rebuild the
same files in a temporary directory and check tideway_b200's geometry against that
summary).  Every byte is a function of the spec below, so both sides see the same files.

Layouts (the three fused BF16 key templates and the per-expert DeepSeek-V4 FP4 keys) are
the ones the reference recognises in ``src/tideway/offload/geometry.py:129-136``.  The
writer is plain Python: 8-byte little-endian header length, a JSON header of
``{key: {dtype, shape, data_offsets}}`` and the raw tensor bytes, which is the safetensors
file format.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

# name -> (template, layers, experts, H, I, shards); shards split the layers in order
FUSED = {
    "qwen": ("model.language_model.layers.{layer}.mlp.experts.{proj}", 3, 4, 16, 8, 2),
    "gemma": ("model.language_model.layers.{layer}.experts.{proj}", 2, 3, 24, 8, 1),
    "plain": ("model.layers.{layer}.mlp.experts.{proj}", 2, 2, 8, 16, 2),
}
# name -> (layers, experts, H, I, shards); FP4 weights pack two values per byte, E8M0
# scales cover 32 values
DS = {
    "dsv4": (2, 3, 64, 32, 2),
}
DS_KEY = "layers.{layer}.ffn.experts.{expert}.{proj}.{kind}"

_ITEMSIZE = {"BF16": 2, "F16": 2, "F32": 4, "F64": 8, "I8": 1, "U8": 1, "F8_E4M3": 1,
             "F8_E8M0": 1}


def _bytes(seed: int, n: int) -> bytes:
    return np.random.default_rng(seed).integers(0, 256, size=n, dtype=np.uint8).tobytes()


def write_shard(path: Path, tensors: list[tuple[str, str, tuple, bytes | None]]) -> None:
    """Write one safetensors file.  ``data=None`` writes a header-only file whose
    offsets run past the end (enough for code that reads headers alone)."""
    header, at, blobs = {}, 0, []
    for key, dtype, shape, data in tensors:
        n = int(np.prod(shape)) * _ITEMSIZE[dtype]
        if data is not None:
            assert len(data) == n, (key, len(data), n)
            blobs.append(data)
        header[key] = {"dtype": dtype, "shape": list(shape), "data_offsets": [at, at + n]}
        at += n
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    with path.open("wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)


def _write_index(root: Path, weight_map: dict) -> None:
    (root / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {}, "weight_map": weight_map}))


def _split(layers: int, shards: int) -> list[list[int]]:
    per = -(-layers // shards)
    return [list(range(s * per, min(layers, (s + 1) * per))) for s in range(shards)]


def fused_tensor_bytes(name: str, layer: int, proj: str) -> bytes:
    _, _, experts, H, I, _ = FUSED[name]
    shape = (experts, 2 * I, H) if proj == "gate_up_proj" else (experts, H, I)
    seed = 1000 * layer + (1 if proj == "gate_up_proj" else 2)
    seed += {"qwen": 0, "gemma": 100_000, "plain": 200_000}[name]
    return _bytes(seed, int(np.prod(shape)) * 2)


def write_fused(root: Path, name: str, gate_dtype: str = "BF16",
                down_experts: int | None = None) -> Path:
    """A fused BF16 checkpoint: per layer ``gate_up_proj [E, 2I, H]`` and
    ``down_proj [E, H, I]``, plus a non-expert tensor in the first shard."""
    template, layers, experts, H, I, shards = FUSED[name]
    root = Path(root) / name
    root.mkdir(parents=True, exist_ok=True)
    weight_map = {}
    for s, lay in enumerate(_split(layers, shards)):
        shard = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        tensors = []
        if s == 0:
            tensors.append(("model.embed_tokens.weight", "BF16", (4, H), _bytes(7, 8 * H)))
        for layer in lay:
            gu = template.format(layer=layer, proj="gate_up_proj")
            dn = template.format(layer=layer, proj="down_proj")
            tensors.append((gu, gate_dtype, (experts, 2 * I, H),
                            fused_tensor_bytes(name, layer, "gate_up_proj")
                            if gate_dtype == "BF16" else _bytes(layer, experts * 2 * I * H * 2)))
            de = experts if down_experts is None else down_experts
            tensors.append((dn, "BF16", (de, H, I),
                            fused_tensor_bytes(name, layer, "down_proj")
                            if de == experts else _bytes(layer + 1, de * H * I * 2)))
        for key, *_ in tensors:
            weight_map[key] = shard
        write_shard(root / shard, tensors)
    _write_index(root, weight_map)
    return root


def ds_tensor(name: str, layer: int, expert: int, proj: str, kind: str) -> tuple:
    _, _, H, I, _ = DS[name]
    rows, cols = (I, H) if proj in ("w1", "w3") else (H, I)
    if kind == "weight":
        shape, dtype = (rows, cols // 2), "I8"
    else:
        shape, dtype = (rows, cols // 32), "F8_E8M0"
    seed = 10_000 * layer + 10 * expert + {"w1": 2, "w2": 4, "w3": 6}[proj] + (kind == "scale")
    return shape, dtype, _bytes(300_000 + seed, int(np.prod(shape)))


def write_ds(root: Path, name: str = "dsv4", w3_rows: int | None = None,
             scale_dtype: str | None = None) -> Path:
    """A DeepSeek-V4-style checkpoint: per layer and expert, ``w1``/``w2``/``w3``
    ``weight`` (I8, two FP4 values per byte) and ``scale`` (E8M0, one per 32 values)."""
    layers, experts, H, I, shards = DS[name]
    root = Path(root) / name
    root.mkdir(parents=True, exist_ok=True)
    weight_map = {}
    for s, lay in enumerate(_split(layers, shards)):
        shard = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        tensors = [("embed.weight", "BF16", (4, H), _bytes(8, 8 * H))] if s == 0 else []
        for layer in lay:
            for expert in range(experts):
                for proj in ("w1", "w2", "w3"):
                    for kind in ("weight", "scale"):
                        shape, dtype, data = ds_tensor(name, layer, expert, proj, kind)
                        if proj == "w3" and w3_rows is not None:
                            shape = (w3_rows, shape[1])
                            data = _bytes(9, int(np.prod(shape)))
                        if kind == "scale" and scale_dtype is not None:
                            dtype = scale_dtype
                            data = _bytes(9, int(np.prod(shape)) * _ITEMSIZE[dtype])
                        tensors.append((DS_KEY.format(layer=layer, expert=expert, proj=proj,
                                                      kind=kind), dtype, shape, data))
        for key, *_ in tensors:
            weight_map[key] = shard
        write_shard(root / shard, tensors)
    _write_index(root, weight_map)
    return root


def write_headers_only(root: Path, name: str, layers: int, experts: int,
                       tensors0: list[tuple[str, str, tuple]], keys_per_layer) -> Path:
    """An index naming every expert key plus one header-only shard that describes the
    layer-0 tensors: enough for geometry derivation at full model size without data."""
    root = Path(root) / name
    root.mkdir(parents=True, exist_ok=True)
    shard = "model-00001-of-00001.safetensors"
    write_shard(root / shard, [(k, d, s, None) for k, d, s in tensors0])
    weight_map = {k: shard for layer in range(layers) for k in keys_per_layer(layer)}
    _write_index(root, weight_map)
    return root


def write_qwen36_headers(root: Path) -> Path:
    """Qwen3.6 at full size (40 layers x 256 experts, H=2048, I=512), headers only."""
    t = FUSED["qwen"][0]
    return write_headers_only(
        root, "qwen36_full", 40, 256,
        [(t.format(layer=0, proj="gate_up_proj"), "BF16", (256, 1024, 2048)),
         (t.format(layer=0, proj="down_proj"), "BF16", (256, 2048, 512))],
        lambda layer: [t.format(layer=layer, proj=p) for p in ("gate_up_proj", "down_proj")])


def write_dsv4_headers(root: Path) -> Path:
    """DeepSeek-V4-Flash at full size (43 layers x 256 experts, H=4096, I=2048),
    headers only."""
    H, I = 4096, 2048

    def key(layer, expert, proj, kind):
        return DS_KEY.format(layer=layer, expert=expert, proj=proj, kind=kind)

    t0 = []
    for proj in ("w1", "w2", "w3"):
        rows, cols = (I, H) if proj != "w2" else (H, I)
        t0.append((key(0, 0, proj, "weight"), "I8", (rows, cols // 2)))
        t0.append((key(0, 0, proj, "scale"), "F8_E8M0", (rows, cols // 32)))
    return write_headers_only(
        root, "dsv4_full", 43, 256, t0,
        lambda layer: [key(layer, e, p, k) for e in range(256) for p in ("w1", "w2", "w3")
                       for k in ("weight", "scale")])
