"""Checkpoint geometry and expert-row reading against the reference's own output.

``tests/golden/geometry.json`` holds what the reference's ``geometry.from_checkpoint``
and raw row reader (``SourceExperts.read``) produced over the seeded miniature
checkpoints of ``tests/golden/synthetic_checkpoints.py``; each test rebuilds the same
files in a temporary directory and checks tideway_b200's geometry and reader against it.
"""

from __future__ import annotations

import builtins
import dataclasses
import hashlib
import json

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN
from tests.golden import synthetic_checkpoints as sc
from tideway_b200 import geometry as G
from tideway_b200.offload_cache import BANK_SCHEMAS

REF = json.loads((GOLDEN / "geometry.json").read_text())


def summary(geo: G.Geometry) -> dict:
    return {
        "layers": geo.layers, "experts": geo.experts, "quant": geo.quant,
        "banks": [[b.name, list(b.shape), b.dtype, b.itemsize] for b in geo.banks],
        "pieces": [[p.bank, p.key, p.fused, p.offset, p.nbytes] for p in geo.pieces],
        "bank_offsets": geo.bank_offsets, "row_bytes": geo.row_bytes,
        "gate_up_shape": list(geo.gate_up_shape), "down_shape": list(geo.down_shape),
        "key_template": geo.key_template, "total_experts": geo.total_experts,
        "double_buffer": geo.double_buffer, "host_rows_for_1_0.25": geo.host_rows_for(1, 0.25),
    }


def build(tmp_path, name: str):
    return sc.write_ds(tmp_path) if name in sc.DS else sc.write_fused(tmp_path, name)


@pytest.mark.parametrize("name", sorted(REF["layouts"]))
def test_layout_matches_reference(tmp_path, name):
    geo = G.from_checkpoint(build(tmp_path, name))
    want = {k: v for k, v in REF["layouts"][name].items()
            if k not in ("row_sha256", "read_past_end")}
    assert summary(geo) == want


@pytest.mark.parametrize("name", sorted(REF["layouts"]))
def test_expert_rows_match_reference_reader(tmp_path, name):
    geo = G.from_checkpoint(build(tmp_path, name))
    ref = REF["layouts"][name]
    with G.CheckpointReader(geo) as reader:
        got = [hashlib.sha256(reader.read(e).tobytes()).hexdigest()
               for e in range(geo.total_experts)]
        assert got == ref["row_sha256"]
        assert ref["read_past_end"] == "ValueError"
        with pytest.raises(ValueError):
            reader.read(geo.total_experts)
        with pytest.raises(ValueError):
            reader.read(-1)


@pytest.mark.parametrize("name", sorted(REF["layouts"]))
@pytest.mark.parametrize("workers,chunk", [(1, 64 << 20), (4, 40)])
def test_layer_banks_equal_expert_rows(tmp_path, monkeypatch, name, workers, chunk):
    """A whole-layer load (large positioned reads, optionally split into small chunks
    over a thread pool) puts every expert's bytes where its row has them."""
    monkeypatch.setattr(G, "_CHUNK", chunk)
    geo = G.from_checkpoint(build(tmp_path, name))
    offsets = geo.bank_offsets
    with G.CheckpointReader(geo, workers=workers) as reader:
        for layer in range(geo.layers):
            banks = reader.layer_banks(layer)
            for b in geo.banks:
                t = banks[b.name]
                assert tuple(t.shape) == (geo.experts, *b.shape) and t.dtype == b.torch_dtype
            for e in range(geo.experts):
                row = reader.read(layer * geo.experts + e)
                for b in geo.banks:
                    got = banks[b.name][e].contiguous().view(torch.uint8).numpy().reshape(-1)
                    lo = offsets[b.name]
                    assert np.array_equal(got, row[lo:lo + b.nbytes]), (layer, e, b.name)


def test_fused_banks_are_the_checkpoint_tensors(tmp_path):
    """A fused layer's host bank is byte-for-byte the checkpoint's ``[E, ...]`` tensor,
    gate rows first, in the layout the slot cache's bf16 schema registers."""
    geo = G.from_checkpoint(sc.write_fused(tmp_path, "qwen"))
    assert geo.bank_names == BANK_SCHEMAS["bf16"]
    sources = G.host_bank_sources(geo, pin=False)
    _, L, E, H, I, _ = sc.FUSED["qwen"]
    assert set(sources) == set(BANK_SCHEMAS["bf16"])
    for layer in range(L):
        for proj, bank in (("gate_up_proj", "gate_up"), ("down_proj", "down")):
            t = sources[bank][layer]
            assert t.dtype == torch.bfloat16
            assert tuple(t.shape) == ((E, 2 * I, H) if bank == "gate_up" else (E, H, I))
            raw = np.frombuffer(sc.fused_tensor_bytes("qwen", layer, proj), np.uint8)
            assert np.array_equal(t.view(torch.uint8).numpy().reshape(-1), raw)


def test_rows_match_safetensors_library(tmp_path):
    """Independent check with the safetensors package: each expert's slice of the
    fused tensors equals the row's bank bytes (the reference's independent_expected)."""
    safetensors = pytest.importorskip("safetensors")
    geo = G.from_checkpoint(sc.write_fused(tmp_path, "qwen"))
    index = json.loads((geo.path / "model.safetensors.index.json").read_text())["weight_map"]
    with G.CheckpointReader(geo) as reader:
        for expert in (0, 5, geo.total_experts - 1):
            layer, local = divmod(expert, geo.experts)
            views = geo.host_views(torch.from_numpy(reader.read(expert)))
            for p in geo.pieces:
                key = p.resolve(layer, local)
                with safetensors.safe_open(geo.path / index[key], framework="pt") as f:
                    want = f.get_slice(key)[local]
                assert torch.equal(views[p.bank].view(torch.int16), want.view(torch.int16))


def test_ds_fp4_stacks_gate_before_up(tmp_path):
    geo = G.from_checkpoint(sc.write_ds(tmp_path))
    assert geo.quant == "ds_fp4"
    with G.CheckpointReader(geo) as reader:
        banks = reader.layer_banks(1)
    for e in range(geo.experts):
        for kind, bank in (("weight", "gate_up_packed"), ("scale", "gate_up_scale")):
            w1 = np.frombuffer(sc.ds_tensor("dsv4", 1, e, "w1", kind)[2], np.uint8)
            w3 = np.frombuffer(sc.ds_tensor("dsv4", 1, e, "w3", kind)[2], np.uint8)
            got = banks[bank][e].view(torch.uint8).numpy().reshape(-1)
            assert np.array_equal(got, np.concatenate([w1, w3])), (e, kind)


@pytest.mark.parametrize("case", sorted(REF["errors"]))
def test_malformed_checkpoints_raise_like_reference(tmp_path, case):
    make = {
        "fused_f16": lambda d: sc.write_fused(d, "qwen", gate_dtype="F16"),
        "fused_expert_mismatch": lambda d: sc.write_fused(d, "gemma", down_experts=2),
        "ds_w3_rows": lambda d: sc.write_ds(d, w3_rows=16),
        "ds_unhandled_dtype": lambda d: sc.write_ds(d, scale_dtype="F64"),
    }
    if case == "no_layout":
        root = tmp_path / "none"
        root.mkdir()
        sc.write_shard(root / "a.safetensors", [("x.weight", "BF16", (2, 2), bytes(8))])
        (root / "model.safetensors.index.json").write_text(
            json.dumps({"weight_map": {"x.weight": "a.safetensors"}}))
    else:
        root = make[case](tmp_path)
    exc_name, _ = REF["errors"][case]  # the reference's exception type; messages are ours
    with pytest.raises(getattr(builtins, exc_name)) as info:
        G.from_checkpoint(root)
    assert type(info.value).__name__ == exc_name
    names = {"fused_f16": "gate_up_proj: dtype F16", "fused_expert_mismatch": "expert counts",
             "ds_w3_rows": "stacks w1.weight, w3.weight", "ds_unhandled_dtype": "dtype F64",
             "no_layout": "no known expert key layout"}
    assert names[case] in str(info.value), str(info.value)


def test_reader_rejects_a_layer_unlike_layer0(tmp_path):
    """The reference derives the layout from layer 0 only; reading a later layer whose
    tensor differs raises instead of filling the bank with the wrong bytes."""
    t = sc.FUSED["plain"][0]
    root = tmp_path / "odd"
    root.mkdir()
    tensors = []
    for layer, experts in ((0, 2), (1, 3)):
        tensors.append((t.format(layer=layer, proj="gate_up_proj"), "BF16", (experts, 4, 2),
                        bytes(experts * 16)))
        tensors.append((t.format(layer=layer, proj="down_proj"), "BF16", (experts, 2, 2),
                        bytes(experts * 8)))
    sc.write_shard(root / "m.safetensors", tensors)
    (root / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {k: "m.safetensors" for k, *_ in tensors}}))
    geo = G.from_checkpoint(root)
    assert (geo.layers, geo.experts) == (2, 2)
    with G.CheckpointReader(geo) as reader:
        reader.layer_banks(0)
        reader.read(1)
        with pytest.raises(RuntimeError, match="does not match"):
            reader.layer_banks(1)
        with pytest.raises(RuntimeError, match="does not match"):
            reader.read(2)


def test_read_layer_rejects_wrong_bank_tensors(tmp_path):
    geo = G.from_checkpoint(sc.write_fused(tmp_path, "gemma"))
    with G.CheckpointReader(geo) as reader:
        banks = {b.name: torch.empty((geo.experts, *b.shape), dtype=b.torch_dtype)
                 for b in geo.banks}
        bad = dict(banks, down=banks["down"].float())
        with pytest.raises(ValueError):
            reader.read_layer(0, bad)
        bad = dict(banks, gate_up=banks["gate_up"].transpose(1, 2))
        with pytest.raises(ValueError):
            reader.read_layer(0, bad)
        with pytest.raises(ValueError):
            reader.read_layer(geo.layers, banks)
        with pytest.raises(ValueError):
            reader.read_into(0, np.empty(geo.row_bytes - 1, np.uint8))


@pytest.mark.parametrize("name", ["qwen36", "dsv4"])
def test_pinned_full_size_layouts(tmp_path, name):
    make = {"qwen36": sc.write_qwen36_headers, "dsv4": sc.write_dsv4_headers}[name]
    geo = G.from_checkpoint(make(tmp_path))
    assert summary(geo) == REF["pinned"][name]
    (G.check_qwen if name == "qwen36" else G.check_dsv4)(geo)


def test_dsv4_check_catches_swapped_gate_and_up(tmp_path):
    geo = G.from_checkpoint(sc.write_dsv4_headers(tmp_path))
    p = list(geo.pieces)
    p[0], p[1] = (dataclasses.replace(p[0], key=p[1].key),
                  dataclasses.replace(p[1], key=p[0].key))
    with pytest.raises(AssertionError):
        G.check_dsv4(dataclasses.replace(geo, pieces=tuple(p)))
    with pytest.raises(AssertionError):
        G.check_qwen(geo)


def test_host_views_split_a_row_without_copies(tmp_path):
    geo = G.from_checkpoint(sc.write_ds(tmp_path))
    with G.CheckpointReader(geo) as reader:
        row = torch.from_numpy(reader.read(4))
    views = geo.host_views(row)
    assert list(views) == list(geo.bank_names)
    for b in geo.banks:
        v = views[b.name]
        assert tuple(v.shape) == b.shape and v.dtype == b.torch_dtype
        assert v.data_ptr() == row.data_ptr() + geo.bank_offsets[b.name]
