"""Checkpoint geometry: which safetensors tensors fill which expert bank, and where.

Mirrors ``src/tideway/offload/geometry.py`` (``Bank``, ``Piece``, ``Geometry``,
``from_checkpoint``, the pinned ``QWEN36``/``DSV4`` layouts and their checks) and adds the
reader that moves expert bytes from the checkpoint into host banks:

* a fused BF16 checkpoint (Qwen3.6, Gemma-4 and plain ``model.layers`` keys,
  ``geometry.py:129-134``) stores each layer's experts as one ``[E, ...]`` tensor per
  projection, so a layer's bank is ONE contiguous byte range of the shard and lands in
  the ``[E, 2I, H]`` / ``[E, H, I]`` host bank that ``OffloadMoeCache.set_bank_sources``
  takes, with no reshuffle (gate rows first, as the checkpoint stores them);
* a DeepSeek-V4 FP4 checkpoint (``geometry.py:136``, ``:196-258``) stores one tensor per
  expert and projection; ``w1`` (gate) and ``w3`` (up) stack into one ``gate_up`` bank with
  ``w1`` first, and the packed weights and block scales are separate banks.

An expert's RAM row is every bank's per-expert bytes, contiguous, in bank order
(``geometry.py:79-93``); ``CheckpointReader.read`` builds that row the way the reference's
raw reader does (``src/tideway/baselines/expert_paging/pack.py:46-61``), and
``CheckpointReader.read_layer`` fills whole ``[E, ...]`` banks with large positioned reads
(one per fused tensor, split into chunks that a thread pool reads in parallel).

Errors follow the reference: ``RuntimeError`` for an unknown or inconsistent layout,
``ValueError`` for an expert outside the model, ``IOError`` for a short read.  The reader
also checks each tensor's header (dtype and byte length) before reading it, so a layer
whose tensors differ from layer 0's raises instead of filling a bank with wrong bytes.
"""

from __future__ import annotations

import json
import math
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

# safetensors dtype -> (torch dtype name, bytes per element); geometry.py:14-23
SAFETENSORS_DTYPES = {
    "BF16": ("bfloat16", 2),
    "F16": ("float16", 2),
    "F32": ("float32", 4),
    "I8": ("uint8", 1),
    "U8": ("uint8", 1),
    "F8_E4M3": ("float8_e4m3fn", 1),
    "F8_E8M0": ("float8_e8m0fnu", 1),
}

# Where the fused expert tensors live, tried in this order (geometry.py:129-134).
FUSED_TEMPLATES = (
    "model.language_model.layers.{layer}.mlp.experts.{proj}",  # Qwen3.6
    "model.language_model.layers.{layer}.experts.{proj}",      # Gemma-4
    "model.layers.{layer}.mlp.experts.{proj}",
)
FUSED_PROJS = ("gate_up_proj", "down_proj")


def ds_key(proj: str, kind: str) -> str:
    """DeepSeek-V4 per-expert key template (``{layer}``/``{expert}`` left open)."""
    return "layers.{layer}.ffn.experts.{expert}." + f"{proj}.{kind}"


@dataclass(frozen=True)
class Bank:
    """One offload-cache bank, described per expert (``geometry.py:26-38``)."""

    name: str
    shape: tuple
    dtype: str      # torch dtype name
    itemsize: int

    @property
    def nbytes(self) -> int:
        return math.prod(self.shape) * self.itemsize

    @property
    def torch_dtype(self) -> torch.dtype:
        return getattr(torch, self.dtype)


@dataclass(frozen=True)
class Piece:
    """One checkpoint tensor and where its bytes land in an expert's row
    (``geometry.py:41-59``).  A fused source is an ``[E, ...]`` tensor holding expert e
    at row e; an unfused source is that expert's own tensor.  ``offset`` is the byte
    offset inside the bank's per-expert buffer (non-zero only for the second of two
    tensors stacked into one bank)."""

    bank: str
    key: str        # template with {layer} and {expert}
    fused: bool
    offset: int
    nbytes: int

    def resolve(self, layer: int, expert: int) -> str:
        return self.key.format(layer=layer, expert=expert)


@dataclass(frozen=True)
class Geometry:
    """Expert banks of one checkpoint (``geometry.py:62-126``)."""

    name: str
    path: Path
    layers: int      # layers that carry routed experts
    experts: int     # experts per layer
    banks: tuple     # Bank, in bank order
    pieces: tuple    # Piece
    quant: str = "bf16"
    gate_up_shape: tuple = ()
    down_shape: tuple = ()
    key_template: str = ""

    @property
    def bank_names(self) -> tuple:
        return tuple(b.name for b in self.banks)

    @property
    def bank_offsets(self) -> dict:
        """Byte offset of each bank inside one contiguous expert row."""
        offsets = np.cumsum([0] + [b.nbytes for b in self.banks[:-1]]).tolist()
        return {b.name: int(o) for b, o in zip(self.banks, offsets)}

    @property
    def row_bytes(self) -> int:
        return sum(b.nbytes for b in self.banks)

    @property
    def gate_up_bytes(self) -> int:
        return self.banks[0].nbytes

    @property
    def down_bytes(self) -> int:
        return self.banks[1].nbytes

    @property
    def total_experts(self) -> int:
        return self.layers * self.experts

    @property
    def double_buffer(self) -> int:
        """Slots the prefill double buffer borrows: two whole layers."""
        return 2 * self.experts

    def key(self, layer: int, proj: str) -> str:
        return self.key_template.format(layer=layer, proj=proj)

    def host_rows_for(self, ram_gib: float, runtime_gib: float) -> int:
        """Expert rows that fit in ``ram_gib`` after ``runtime_gib`` is set aside."""
        return int((ram_gib - runtime_gib) * 2**30) // self.row_bytes

    def host_views(self, row: torch.Tensor) -> dict:
        """Split one expert's uint8 RAM row into per-bank tensors (views, no copy)."""
        assert row.dtype == torch.uint8 and row.numel() >= self.row_bytes, (
            row.dtype, row.numel(), self.row_bytes)
        out = {}
        for b in self.banks:
            at = self.bank_offsets[b.name]
            out[b.name] = row[at:at + b.nbytes].view(b.torch_dtype).view(*b.shape)
        return out


class _Headers:
    """safetensors headers of one checkpoint, read once per shard."""

    def __init__(self, path: Path, index: dict):
        self.path, self.index, self._cache = path, index, {}

    def shard(self, key: str) -> tuple[str, int, dict]:
        shard = self.index[key]
        if shard not in self._cache:
            with (self.path / shard).open("rb") as f:
                n = struct.unpack("<Q", f.read(8))[0]
                self._cache[shard] = (8 + n, json.loads(f.read(n)))
        start, header = self._cache[shard]
        return shard, start, header

    def entry(self, key: str) -> dict:
        return self.shard(key)[2][key]


def _read_index(path: Path) -> dict:
    return json.loads((path / "model.safetensors.index.json").read_text())["weight_map"]


def _count(probe) -> int:
    n = 0
    while probe(n):
        n += 1
    return n


def _fused_bf16(path: Path, index: dict, heads: _Headers) -> Geometry | None:
    """Fused BF16 banks ``gate_up [2I, H]`` and ``down [H, I]`` (geometry.py:152-193)."""
    template = next((t for t in FUSED_TEMPLATES
                     if t.format(layer=0, proj="gate_up_proj") in index), None)
    if template is None:
        return None
    layers = _count(lambda l: template.format(layer=l, proj="gate_up_proj") in index)
    shapes = {}
    for proj in FUSED_PROJS:
        key = template.format(layer=0, proj=proj)
        entry = heads.entry(key)
        if entry["dtype"] != "BF16":
            raise RuntimeError(f"{key} is {entry['dtype']}, the fused arms assume BF16")
        shapes[proj] = tuple(entry["shape"])
    experts = shapes["gate_up_proj"][0]
    if shapes["down_proj"][0] != experts:
        raise RuntimeError("gate_up and down disagree on the expert count")
    gu, dn = shapes["gate_up_proj"][1:], shapes["down_proj"][1:]
    banks = (Bank("gate_up", gu, "bfloat16", 2), Bank("down", dn, "bfloat16", 2))
    pieces = tuple(Piece(b.name, template.replace("{proj}", proj), True, 0, b.nbytes)
                   for b, proj in zip(banks, FUSED_PROJS))
    return Geometry(name=path.name, path=path, layers=layers, experts=experts, banks=banks,
                    pieces=pieces, quant="bf16", gate_up_shape=gu, down_shape=dn,
                    key_template=template)


def _ds_fp4(path: Path, index: dict, heads: _Headers) -> Geometry | None:
    """DeepSeek-V4 FP4 banks from per-expert w1/w2/w3 (geometry.py:196-258): gate rows
    (w1) stacked before up rows (w3) in both the packed and the scale bank."""
    w1 = ds_key("w1", "weight")
    if w1.format(layer=0, expert=0) not in index:
        return None
    layers = _count(lambda l: w1.format(layer=l, expert=0) in index)
    experts = _count(lambda e: w1.format(layer=0, expert=e) in index)
    got = {}
    for proj in ("w1", "w2", "w3"):
        for kind in ("weight", "scale"):
            key = ds_key(proj, kind).format(layer=0, expert=0)
            entry = heads.entry(key)
            if entry["dtype"] not in SAFETENSORS_DTYPES:
                raise RuntimeError(f"{key}: unhandled dtype {entry['dtype']}")
            got[proj, kind] = (tuple(entry["shape"]), *SAFETENSORS_DTYPES[entry["dtype"]])
    if got["w1", "weight"] != got["w3", "weight"] or got["w1", "scale"] != got["w3", "scale"]:
        raise RuntimeError("w1 and w3 differ in shape; the gate_up stacking assumes they match")

    def stacked(proj_kind):
        shape, dt, size = got[proj_kind]
        return (2 * shape[0], *shape[1:]), dt, size

    banks = (
        Bank("gate_up_packed", *stacked(("w1", "weight"))),
        Bank("gate_up_scale", *stacked(("w1", "scale"))),
        Bank("down_packed", *got["w2", "weight"]),
        Bank("down_scale", *got["w2", "scale"]),
    )
    half = {kind: math.prod(got["w1", kind][0]) * got["w1", kind][2]
            for kind in ("weight", "scale")}
    pieces = (
        Piece("gate_up_packed", ds_key("w1", "weight"), False, 0, half["weight"]),
        Piece("gate_up_packed", ds_key("w3", "weight"), False, half["weight"], half["weight"]),
        Piece("gate_up_scale", ds_key("w1", "scale"), False, 0, half["scale"]),
        Piece("gate_up_scale", ds_key("w3", "scale"), False, half["scale"], half["scale"]),
        Piece("down_packed", ds_key("w2", "weight"), False, 0, banks[2].nbytes),
        Piece("down_scale", ds_key("w2", "scale"), False, 0, banks[3].nbytes),
    )
    return Geometry(name=path.name, path=path, layers=layers, experts=experts, banks=banks,
                    pieces=pieces, quant="ds_fp4")


def from_checkpoint(path) -> Geometry:
    """Derive the expert banks of a safetensors checkpoint directory
    (``geometry.py:261-268``): fused BF16 layouts first, then DeepSeek-V4 FP4."""
    path = Path(path).expanduser().resolve()
    index = _read_index(path)
    heads = _Headers(path, index)
    for builder in (_fused_bf16, _ds_fp4):
        geo = builder(path, index, heads)
        if geo is not None:
            return geo
    raise RuntimeError(f"no known expert key layout in {path}")


# Known layouts, pinned for explicit validation (geometry.py:271-291).
QWEN36 = dict(layers=40, experts=256, row_bytes=6 * 2**20, total_experts=10240,
              double_buffer=512, gate_up_shape=(1024, 2048), down_shape=(2048, 512))
DSV4 = dict(layers=43, experts=256, row_bytes=int(12.75 * 2**20), total_experts=11008,
            double_buffer=512, quant="ds_fp4")


def _check(geo: Geometry, expected: dict) -> None:
    for field, want in expected.items():
        have = getattr(geo, field)
        assert have == want, f"{field}: {have} != {want}"


def check_qwen(geo: Geometry) -> None:
    _check(geo, QWEN36)


def check_dsv4(geo: Geometry) -> None:
    """The pinned DeepSeek-V4-Flash layout, bank order, and gate-before-up stacking
    (``geometry.py:300-311``): a swapped w1/w3 would run and give wrong tokens."""
    _check(geo, DSV4)
    assert geo.bank_names == ("gate_up_packed", "gate_up_scale", "down_packed",
                              "down_scale"), geo.bank_names
    order = [(p.bank, p.key.split(".")[-2], p.offset) for p in geo.pieces]
    assert order[0] == ("gate_up_packed", "w1", 0), order
    assert order[1] == ("gate_up_packed", "w3", geo.banks[0].nbytes // 2), order


# ----------------------------------------------------------------- reading
_CHUNK = 64 << 20   # bytes per positioned read in a layer load


def _byte_view(t) -> memoryview:
    """Writable flat byte view of a contiguous CPU tensor or numpy array."""
    if isinstance(t, torch.Tensor):
        if t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError("host banks must be contiguous CPU tensors")
        if t.numel() == 0:
            return memoryview(bytearray())
        t = t.view(torch.uint8).reshape(-1).numpy()
    if not t.flags.c_contiguous or not t.flags.writeable:
        raise ValueError("rows must be contiguous, writable arrays")
    return memoryview(t.reshape(-1).view(np.uint8))


def _pread_into(fd: int, view: memoryview, offset: int) -> None:
    done = 0
    while done < len(view):
        got = os.preadv(fd, [view[done:]], offset + done)
        if got <= 0:
            raise IOError("Short checkpoint read")
        done += got


class CheckpointReader:
    """Reads expert bytes of a checkpoint described by a ``Geometry``.

    ``read(expert)`` returns one expert's contiguous RAM row (flat expert index
    ``layer * experts + local``, as ``pack.py:46-61`` numbers them);
    ``read_layer(layer, banks)`` fills per-layer ``[E, ...]`` bank tensors, the layout
    the slot cache's host sources use.  Files stay open until ``close()``.
    """

    def __init__(self, geo: Geometry, workers: int = 8):
        self.geo = geo
        self.index = _read_index(Path(geo.path))
        self.heads = _Headers(Path(geo.path), self.index)
        self.fds: dict[str, int] = {}
        self.workers = max(1, int(workers))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        for fd in self.fds.values():
            os.close(fd)
        self.fds.clear()

    def _locate(self, piece: Piece, key: str, nbytes: int) -> tuple[int, int]:
        """(fd, file offset of the tensor's first byte) after checking its header."""
        shard, start, header = self.heads.shard(key)
        entry = header[key]
        bank = next(b for b in self.geo.banks if b.name == piece.bank)
        dtype = SAFETENSORS_DTYPES.get(entry["dtype"], (None, 0))[0]
        lo, hi = entry["data_offsets"]
        if dtype != bank.dtype or hi - lo != nbytes:
            raise RuntimeError(f"{key}: {entry['dtype']} {entry['shape']} does not match "
                               f"bank {bank.name!r} ({bank.dtype}, {nbytes} bytes)")
        if shard not in self.fds:
            self.fds[shard] = os.open(Path(self.geo.path) / shard, os.O_RDONLY)
        return self.fds[shard], start + lo

    def read_into(self, expert: int, row) -> None:
        """Fill ``row`` (uint8, ``row_bytes`` long) with one expert's bytes."""
        g = self.geo
        layer, local = divmod(int(expert), g.experts)
        if not 0 <= layer < g.layers:
            raise ValueError("Expert index outside model")
        view = _byte_view(row)
        if len(view) < g.row_bytes:
            raise ValueError(f"row holds {len(view)} bytes, the expert needs {g.row_bytes}")
        offsets = g.bank_offsets
        for p in g.pieces:
            key = p.resolve(layer, local)
            fd, at = self._locate(p, key, g.experts * p.nbytes if p.fused else p.nbytes)
            if p.fused:
                at += local * p.nbytes
            dst = offsets[p.bank] + p.offset
            _pread_into(fd, view[dst:dst + p.nbytes], at)

    def read(self, expert: int) -> np.ndarray:
        row = np.empty(self.geo.row_bytes, dtype=np.uint8)
        self.read_into(expert, row)
        return row

    def read_layer(self, layer: int, banks: dict) -> None:
        """Fill ``banks[name]`` (contiguous CPU tensors ``[E, *bank.shape]`` of the
        bank's dtype, pinned or not) with every expert of ``layer``."""
        g = self.geo
        if not 0 <= layer < g.layers:
            raise ValueError("Layer index outside model")
        views = {}
        for b in g.banks:
            t = banks[b.name]
            if tuple(t.shape) != (g.experts, *b.shape) or t.dtype != b.torch_dtype:
                raise ValueError(f"bank {b.name!r}: {tuple(t.shape)} {t.dtype}, expected "
                                 f"{(g.experts, *b.shape)} {b.torch_dtype}")
            views[b.name] = _byte_view(t)
        jobs = []
        for p in g.pieces:
            bank_bytes = next(b.nbytes for b in g.banks if b.name == p.bank)
            if p.fused:
                fd, at = self._locate(p, p.resolve(layer, 0), g.experts * p.nbytes)
                whole = views[p.bank]
                for lo in range(0, len(whole), _CHUNK):
                    jobs.append((fd, whole[lo:lo + _CHUNK], at + lo))
            else:
                for e in range(g.experts):
                    fd, at = self._locate(p, p.resolve(layer, e), p.nbytes)
                    dst = e * bank_bytes + p.offset
                    jobs.append((fd, views[p.bank][dst:dst + p.nbytes], at))
        if self.workers == 1 or len(jobs) == 1:
            for job in jobs:
                _pread_into(*job)
            return
        with ThreadPoolExecutor(min(self.workers, len(jobs))) as pool:
            for _ in pool.map(lambda j: _pread_into(*j), jobs):
                pass

    def layer_banks(self, layer: int, pin: bool = False) -> dict:
        """Allocate and fill one layer's ``[E, ...]`` host banks."""
        g = self.geo
        banks = {b.name: torch.empty((g.experts, *b.shape), dtype=b.torch_dtype,
                                     pin_memory=pin) for b in g.banks}
        self.read_layer(layer, banks)
        return banks


def host_bank_sources(geo: Geometry, layers=None, pin: bool = True,
                      workers: int = 8) -> dict[str, list[torch.Tensor]]:
    """Per-bank lists of per-layer host banks, read from the checkpoint, in the form
    ``OffloadMoeCache.set_bank_sources`` takes (``bank name -> [layer] -> [E, ...]``)."""
    layers = range(geo.layers) if layers is None else layers
    out = {b.name: [] for b in geo.banks}
    with CheckpointReader(geo, workers=workers) as reader:
        for layer in layers:
            for name, t in reader.layer_banks(layer, pin=pin).items():
                out[name].append(t)
    return out
