"""Checkpoint geometry: which safetensors tensors fill which expert bank, and where.

Produces the same ``Bank``/``Piece``/``Geometry`` descriptions as
``src/tideway/offload/geometry.py`` (the checkpoint and host-row formats a drop-in must read
the same way, with its pinned ``QWEN36``/``DSV4`` layouts), derived here from a table of
layout families walked by one generic derivation, and adds the reader that moves expert
bytes from the checkpoint into host banks:

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

Error types follow the reference: ``RuntimeError`` for an unknown or inconsistent layout,
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


# ----------------------------------------------------------------- layout families
#
# A checkpoint family is described as data: where its expert tensors are named, which
# tensors fill which bank (several tensors of one bank are stacked along their first
# dimension, in the order given), and which dtypes it may hold.  One generic derivation
# (``_derive``) walks these descriptions; adding a family is adding an entry.

@dataclass(frozen=True)
class _BankSpec:
    bank: str
    sources: tuple      # source names filled into the family's key template, stacked in order


@dataclass(frozen=True)
class _Family:
    quant: str
    templates: tuple    # key templates tried in order; {layer}, {expert}, {source} open
    fused: bool         # one [E, ...] tensor per layer and source (else one per expert)
    banks: tuple        # _BankSpec, in bank order
    dtypes: frozenset | None   # allowed safetensors dtypes (None: any known one)
    records_shapes: bool       # fused BF16 families keep gate_up/down shapes and the template


_FAMILIES = (
    _Family("bf16", tuple(t.replace("{proj}", "{source}") for t in FUSED_TEMPLATES), True,
            (_BankSpec("gate_up", ("gate_up_proj",)), _BankSpec("down", ("down_proj",))),
            frozenset({"BF16"}), True),
    _Family("ds_fp4", ("layers.{layer}.ffn.experts.{expert}.{source}",), False,
            (_BankSpec("gate_up_packed", ("w1.weight", "w3.weight")),
             _BankSpec("gate_up_scale", ("w1.scale", "w3.scale")),
             _BankSpec("down_packed", ("w2.weight",)),
             _BankSpec("down_scale", ("w2.scale",))),
            None, False),
)


def _key(template: str, source: str, layer="{layer}", expert="{expert}") -> str:
    return template.replace("{source}", source).replace("{layer}", str(layer)).replace(
        "{expert}", str(expert))


def _run_length(present) -> int:
    """Smallest n >= 0 with present(n) false (layers or experts numbered from 0)."""
    n = 0
    while present(n):
        n += 1
    return n


def _derive(fam: _Family, path: Path, index: dict, heads: _Headers) -> Geometry | None:
    anchor = fam.banks[0].sources[0]
    template = next((t for t in fam.templates if _key(t, anchor, 0, 0) in index), None)
    if template is None:
        return None
    layers = _run_length(lambda l: _key(template, anchor, l, 0) in index)
    # every source's layer-0 header: (per-expert shape, torch dtype, itemsize, experts)
    info = {}
    for spec in fam.banks:
        for src in spec.sources:
            key = _key(template, src, 0, 0)
            entry = heads.entry(key)
            dt = entry["dtype"]
            if dt not in SAFETENSORS_DTYPES or (fam.dtypes is not None and dt not in fam.dtypes):
                allowed = sorted(fam.dtypes or SAFETENSORS_DTYPES)
                raise RuntimeError(f"{key}: dtype {dt} is not one the {fam.quant} layout "
                                   f"reads ({', '.join(allowed)})")
            shape = tuple(entry["shape"])
            per_expert, count = (shape[1:], shape[0]) if fam.fused else (shape, None)
            info[src] = (per_expert, *SAFETENSORS_DTYPES[dt], count)
    if fam.fused:
        counts = {src: v[3] for src, v in info.items()}
        if len(set(counts.values())) != 1:
            raise RuntimeError(f"{path.name}: layer-0 expert tensors hold different expert "
                               f"counts {counts}")
        experts = next(iter(counts.values()))
    else:
        experts = _run_length(lambda e: _key(template, anchor, 0, e) in index)
    banks, pieces = [], []
    for spec in fam.banks:
        parts = [info[src] for src in spec.sources]
        if len({p[:3] for p in parts}) != 1:
            raise RuntimeError(f"bank {spec.bank!r} stacks {', '.join(spec.sources)} along "
                               f"rows, but their per-expert tensors differ: "
                               f"{[p[:3] for p in parts]}")
        shape, dtype, size, _ = parts[0]
        stacked = (len(parts) * shape[0], *shape[1:]) if len(parts) > 1 else shape
        bank = Bank(spec.bank, stacked, dtype, size)
        banks.append(bank)
        part_bytes = bank.nbytes // len(parts)
        for i, src in enumerate(spec.sources):
            pieces.append(Piece(spec.bank, _key(template, src), fam.fused, i * part_bytes,
                                part_bytes))
    extra = {}
    if fam.records_shapes:
        extra = dict(gate_up_shape=banks[0].shape, down_shape=banks[1].shape,
                     key_template=template.replace("{source}", "{proj}"))
    return Geometry(name=path.name, path=path, layers=layers, experts=experts,
                    banks=tuple(banks), pieces=tuple(pieces), quant=fam.quant, **extra)


def from_checkpoint(path) -> Geometry:
    """Derive the expert banks of a safetensors checkpoint directory, trying each known
    layout family in turn (the fused BF16 families, then DeepSeek-V4 FP4) -- the layouts
    src/tideway/offload/geometry.py:129-136 recognises."""
    path = Path(path).expanduser().resolve()
    index = _read_index(path)
    heads = _Headers(path, index)
    for fam in _FAMILIES:
        geo = _derive(fam, path, index, heads)
        if geo is not None:
            return geo
    raise RuntimeError(f"no known expert key layout in {path}: none of the "
                       f"{', '.join(f.quant for f in _FAMILIES)} layouts names its tensors")


# Known layouts, pinned for explicit validation (geometry.py:271-291).
QWEN36 = dict(layers=40, experts=256, row_bytes=6 * 2**20, total_experts=10240,
              double_buffer=512, gate_up_shape=(1024, 2048), down_shape=(2048, 512))
DSV4 = dict(layers=43, experts=256, row_bytes=int(12.75 * 2**20), total_experts=11008,
            double_buffer=512, quant="ds_fp4")


def _pinned(geo: Geometry, expected: dict) -> None:
    wrong = {f: (getattr(geo, f), v) for f, v in expected.items() if getattr(geo, f) != v}
    assert not wrong, f"{geo.name} differs from the pinned layout: {wrong}"


def check_qwen(geo: Geometry) -> None:
    _pinned(geo, QWEN36)


def check_dsv4(geo: Geometry) -> None:
    """The pinned DeepSeek-V4-Flash layout, its bank order and gate-before-up stacking: in
    each stacked bank the w1 (gate) piece sits at offset 0 and the w3 (up) piece after it.
    A swapped pair would load and run, and give wrong tokens."""
    _pinned(geo, DSV4)
    want = tuple(spec.bank for spec in _FAMILIES[1].banks)
    assert geo.bank_names == want, f"bank order {geo.bank_names}, expected {want}"
    for bank in ("gate_up_packed", "gate_up_scale"):
        by_offset = sorted((p.offset, p.key.rsplit(".", 2)[-2]) for p in geo.pieces
                           if p.bank == bank)
        assert [src for _, src in by_offset] == ["w1", "w3"], (bank, by_offset)


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
            raise IOError(f"checkpoint ended {len(view) - done} bytes early at offset {offset + done}")
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
            raise ValueError(f"expert {expert} is not in the model's {g.total_experts} experts")
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
            raise ValueError(f"layer {layer} is not in the model's {g.layers} layers")
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
