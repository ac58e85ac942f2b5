"""Generate the golden fixtures in this directory from the reference's own code.

Run from the repository root in a container that has the reference checkout:

    TIDEWAY_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py [geometry]

The reference is Python; only the pieces of its hot path that run without FreeToken
are executed, exactly as shipped:

* ``fused_topk`` (backends/freetoken_tideway/freetoken/moe/fused.py:38-85) imported with
  a minimal stub of the ``freetoken`` package (base class, logger, ``div_ceil`` and
  ``is_triton_kernels_installed() -> False``), so its torch router (fused.py:16-35) runs;
* the vendored slot-cache ``lru_ensure`` (backends/.../moe/shift.py:698-777) and the
  Gemma ``_routing_with_copy`` kernel (src/tideway/gemma_route_copy_kernel.py:28-70),
  both Triton, run on CPU tensors under ``TRITON_INTERPRET=1``;
* ``offload/cache.py:Cache.access`` (numpy) as a cross-check of the slot mapping;
* the hybrid backend's capped-fetch LRU CPU mirror
  (backends/.../moe/offload_kernels.py:135-195), with flashlib's import stubbed;
* the checkpoint geometry (src/tideway/offload/geometry.py) and raw expert-row reader
  (src/tideway/baselines/expert_paging/pack.py, its codec import stubbed) over the seeded
  miniature checkpoints of ``synthetic_checkpoints.py`` -> ``geometry.json``.

The fixtures are small ``.npz`` files committed next to this script; the tests read
them without the reference.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
if "TIDEWAY_REFERENCE" not in os.environ:
    raise SystemExit("set TIDEWAY_REFERENCE to the reference checkout")
REF = Path(os.environ["TIDEWAY_REFERENCE"])


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _stub_freetoken() -> None:
    """Minimal stand-ins for the FreeToken symbols fused.py imports at module level."""
    ft = types.ModuleType("freetoken")
    moe = types.ModuleType("freetoken.moe")
    utils = types.ModuleType("freetoken.utils")
    kernel = types.ModuleType("freetoken.kernel")
    backend = types.ModuleType("freetoken.kernel.backend")

    class BaseMoeBackend:  # noqa: D401 - stub
        pass

    class _Log:
        def __getattr__(self, _name):
            return lambda *a, **k: None

    moe.BaseMoeBackend = BaseMoeBackend
    utils.div_ceil = lambda a, b: -(-a // b)
    utils.init_logger = lambda _n: _Log()
    backend.is_triton_kernels_installed = lambda: False
    for m in (ft, moe, utils, kernel, backend):
        sys.modules[m.__name__] = m
    ft.moe, ft.utils, ft.kernel, kernel.backend = moe, utils, kernel, backend


def gen_fused_topk(fused) -> None:
    cases = {}
    g = torch.Generator().manual_seed(100)
    specs = [
        ("c1", 4, 16, 2, True, torch.float32, None),
        ("c2_b64", 64, 128, 8, True, torch.float32, None),
        ("c2_b1", 1, 128, 8, True, torch.float32, None),
        ("norenorm", 32, 128, 8, False, torch.float32, None),
        ("bf16_logits", 16, 128, 8, True, torch.bfloat16, None),
        ("padded", 8, 64, 4, True, torch.float32, 5),
        ("e256_k6", 16, 256, 6, True, torch.float32, None),
    ]
    for name, T, E, K, renorm, dt, ntp in specs:
        logits = (torch.randn(T, E, generator=g) * 2.0).to(dt)
        hidden = torch.zeros(T, 8)
        ntp_t = None if ntp is None else torch.tensor(ntp)
        w, ids = fused.fused_topk(hidden, logits, K, renorm, ntp_t)
        cases[name] = dict(logits=logits.float().numpy(), is_bf16=dt == torch.bfloat16,
                           K=K, renorm=renorm, ntp=-1 if ntp is None else ntp,
                           w=w.numpy(), ids=ids.numpy())
    _save("fused_topk", cases)


def gen_gemma(gemma) -> None:
    cases = {}
    g = torch.Generator().manual_seed(101)
    for name, T, E, K, ties in (("c3", 64, 128, 8, False), ("ties", 16, 128, 8, True),
                                ("small", 4, 16, 2, False)):
        logits = torch.randn(T, E, generator=g) * 2.0
        if ties:  # quantise to force exact ties between different experts
            logits = torch.round(logits * 2.0) / 2.0
        scale = 1.0 + 0.1 * torch.randn(E, generator=g)
        w = torch.empty(T, K)
        ids = torch.empty(T, K, dtype=torch.int32)
        priv = torch.empty(T, K, dtype=torch.int32)
        bl = 1 << (E - 1).bit_length()
        gemma._routing_with_copy[(T,)](logits, scale, w, ids, priv, logits.stride(0),
                                       E=E, K=K, BLOCK_E=bl)
        cases[name] = dict(logits=logits.numpy(), scale=scale.numpy(), K=K,
                           w=w.numpy(), ids=ids.numpy(), private=priv.numpy())
    _save("gemma_routing", cases)


def _lru_case(shift, cache_mod, L, E, S, T, K, steps, seed, frac, pins=()) -> dict:
    """One replayed sequence of the reference's ``lru_ensure_pinned``; ``pins`` are slots
    whose pinned flag is set (never evicted).  Without pins every step is cross-checked
    against ``Cache.access``, which has no pinned slots."""
    g = torch.Generator().manual_seed(seed)
    slot_of_id = torch.full((L * E,), -1, dtype=torch.int32)
    id_of_slot = torch.full((S,), -1, dtype=torch.int32)
    usage = torch.zeros(S, dtype=torch.int64)
    step = torch.zeros((), dtype=torch.int64)
    pinned = torch.zeros(S, dtype=torch.int32)
    pinned[list(pins)] = 1
    src = torch.zeros(E, dtype=torch.int32)
    dst = torch.zeros(E, dtype=torch.int32)
    num = torch.zeros(1, dtype=torch.int64)
    stats = torch.zeros(4, dtype=torch.int64)
    # seeded initial residency: a random permutation of all flat ids, the first
    # round(frac * S) of them placed in slots 0.. in that order
    n_seed = int(round(frac * S))
    perm = torch.randperm(L * E, generator=g)[:n_seed]
    for s, fid in enumerate(perm.tolist()):
        id_of_slot[s] = fid
        slot_of_id[fid] = s
    init = dict(slot_of_id=slot_of_id.numpy().copy(), id_of_slot=id_of_slot.numpy().copy())
    host = cache_mod.Cache(S, L * E)
    host.slots[:] = id_of_slot.numpy()
    host.where[:] = slot_of_id.numpy()
    seq = []
    for it in range(steps):
        layer = it % L
        ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
        q = ids.clone()
        shift.lru_ensure_pinned(q, slot_of_id, id_of_slot, usage, step, pinned, q, src,
                                dst, num, stats=stats, id_base=layer * E)
        if not pins:
            host.access(ids.numpy().reshape(-1).astype(np.int64) + layer * E)
            assert np.array_equal(host.where[ids.numpy().reshape(-1) + layer * E],
                                  q.numpy().reshape(-1)), "Cache.access disagrees"
        else:  # a pinned slot keeps its expert
            assert np.array_equal(id_of_slot.numpy()[list(pins)],
                                  init["id_of_slot"][list(pins)])
        n = int(num.item())
        seq.append(dict(layer=layer, ids=ids.numpy(), out=q.numpy(), num=n,
                        src=src.numpy()[:n].copy(), dst=dst.numpy()[:n].copy(),
                        slot_of_id=slot_of_id.numpy().copy(),
                        id_of_slot=id_of_slot.numpy().copy(),
                        usage=usage.numpy().copy(), step=int(step.item())))
    flat = dict(L=L, E=E, S=S, steps=steps, init_slot_of_id=init["slot_of_id"],
                init_id_of_slot=init["id_of_slot"], stats=stats.numpy())
    if pins:
        flat["pinned"] = pinned.numpy()
    for i, rec in enumerate(seq):
        for k, v in rec.items():
            flat[f"s{i}_{k}"] = v
    return flat


def gen_lru(shift, cache_mod) -> None:
    specs = [
        # name, L, E, S, T, K, steps, seed, seeded-resident fraction
        ("small", 3, 8, 16, 2, 3, 12, 0, 0.0),
        ("c1", 1, 16, 8, 4, 2, 10, 0, 0.5),
        ("c2_like", 4, 128, 256, 64, 8, 6, 1, 0.5),
        ("b1_many_layers", 8, 64, 128, 1, 8, 24, 2, 0.25),
    ]
    _save("lru_ensure", {spec[0]: _lru_case(shift, cache_mod, *spec[1:]) for spec in specs})


def gen_lru_pinned(shift, cache_mod) -> None:
    """Sequences with pinned slots (resident experts that are never evicted): the pins sit
    on seeded slots, with enough unpinned slots for every step's misses."""
    specs = [
        # name, L, E, S, T, K, steps, seed, seeded-resident fraction, pinned slots
        ("pins_low", 2, 16, 12, 1, 4, 16, 3, 0.5, (0, 1, 2, 3)),
        ("pins_spread", 3, 32, 40, 2, 4, 20, 4, 0.5, (1, 5, 9, 13, 17)),
        ("pins_one_layer", 1, 64, 24, 4, 2, 18, 5, 0.75, tuple(range(0, 16, 2))),
    ]
    _save("lru_ensure_pinned",
          {spec[0]: _lru_case(shift, cache_mod, *spec[1:]) for spec in specs})


def _stub_flashlib() -> None:
    """offload_kernels.py imports flashlib's lru_ensure at module level; the hybrid CPU
    mirror does not use it."""
    fl = types.ModuleType("flashlib")
    kn = types.ModuleType("flashlib.kernels")
    sc = types.ModuleType("flashlib.kernels.slot_cache")
    sc.lru_ensure = lambda *a, **k: None
    for m in (fl, kn, sc):
        sys.modules[m.__name__] = m
    fl.kernels, kn.slot_cache = kn, sc


def gen_hybrid(kern) -> None:
    """Capped-fetch LRU (``_ensure_experts_hybrid_cpu``, offload_kernels.py:135-195): the
    reference's CPU mirror of its hybrid-backend kernel, run as shipped."""
    cases = {}
    specs = [
        # name, L, E, S, T, K, steps, seed, resident fraction, max_fetch, frac_q16, by_recency
        ("cap2_recency", 3, 16, 24, 4, 2, 18, 5, 0.5, 2, 0, True),
        ("frac_recency", 4, 64, 128, 8, 6, 16, 6, 0.25, 1000, 26214, True),
        ("cap3_lowest_id", 3, 16, 24, 4, 2, 18, 7, 0.5, 3, 0, False),
        ("frac_lowest_id", 2, 128, 160, 16, 8, 10, 8, 0.5, 1000, 45875, False),
        ("uncapped", 3, 32, 48, 4, 4, 12, 9, 0.0, 1000, 0, True),
    ]
    for name, L, E, S, T, K, steps, seed, frac, max_fetch, fq, by_rec in specs:
        kern._HYBRID_FETCH_BY_RECENCY = by_rec
        g = torch.Generator().manual_seed(seed)
        cache = types.SimpleNamespace(
            num_experts=E, cache_size=S,
            slot_for_id=torch.full((L, E), -1, dtype=torch.int32),
            id_of_slot=torch.full((S,), -1, dtype=torch.int32),
            usage=torch.zeros(S, dtype=torch.int64),
            step=torch.zeros((), dtype=torch.int64),
            active_mask=torch.zeros(E, dtype=torch.int32),
            evict_slots=torch.zeros(E, dtype=torch.int32),
            src_indices=torch.zeros(E, dtype=torch.int32),
            num_indices=torch.zeros(1, dtype=torch.int64),
            num_missing_full=torch.zeros(1, dtype=torch.int64),
            expert_recency=torch.zeros((L, E), dtype=torch.int64))
        n_seed = int(round(frac * S))
        perm = torch.randperm(L * E, generator=g)[:n_seed]
        for s, fid in enumerate(perm.tolist()):
            cache.id_of_slot[s] = fid
            cache.slot_for_id.view(-1)[fid] = s
        flat = dict(L=L, E=E, S=S, steps=steps, max_fetch=max_fetch, frac_q16=fq,
                    by_recency=by_rec,
                    init_slot_of_id=cache.slot_for_id.view(-1).numpy().copy(),
                    init_id_of_slot=cache.id_of_slot.numpy().copy())
        for it in range(steps):
            layer = it % L
            ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
            q = ids.clone()
            kern._ensure_experts_hybrid_cpu(cache, layer, q, max_fetch, fq)
            n = int(cache.num_indices.item())
            rec = dict(layer=layer, ids=ids.numpy(), out=q.numpy(), num=n,
                       num_full=int(cache.num_missing_full.item()),
                       src=cache.src_indices.numpy()[:n].copy(),
                       dst=cache.evict_slots.numpy()[:n].copy(),
                       slot_of_id=cache.slot_for_id.view(-1).numpy().copy(),
                       id_of_slot=cache.id_of_slot.numpy().copy(),
                       usage=cache.usage.numpy().copy(), step=int(cache.step.item()),
                       recency=cache.expert_recency.numpy().copy(),
                       active=cache.active_mask.numpy().copy())
            for k, v in rec.items():
                flat[f"s{it}_{k}"] = v
        cases[name] = flat
    _save("hybrid_ensure", cases)


def gen_align() -> None:
    # Worked example of moe_align_block_size (backends/.../moe/fused.py:113-126), as
    # written in the reference docstring: experts 1..4, block 4.
    cases = {"docstring": dict(
        topk_ids=np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], np.int32),
        block_size=4, num_experts=5,
        sorted_ids=np.array([3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12], np.int32),
    )}
    _save("moe_align", cases)


def _stub_pack_package() -> str:
    """``expert_paging/pack.py`` imports four names from its sibling ``codec`` (a native
    entropy codec this reader does not use); a stub package provides them so the raw
    checkpoint reader ``SourceExperts`` loads on its own."""
    import struct as _struct

    pkg = types.ModuleType("ref_paging")
    pkg.__path__ = []
    codec = types.ModuleType("ref_paging.codec")
    codec.Codec = object
    codec.HEADER = _struct.Struct("<8sQIIII")
    codec.RAW = b"PRAW001\0"
    codec.CHUNK = 1024
    sys.modules["ref_paging"] = pkg
    sys.modules["ref_paging.codec"] = codec
    return "ref_paging"


def _geo_summary(geo) -> dict:
    return {
        "layers": geo.layers, "experts": geo.experts, "quant": geo.quant,
        "banks": [[b.name, list(b.shape), b.dtype, b.itemsize] for b in geo.banks],
        "pieces": [[p.bank, p.key, p.fused, p.offset, p.nbytes] for p in geo.pieces],
        "bank_offsets": geo.bank_offsets, "row_bytes": geo.row_bytes,
        "gate_up_shape": list(geo.gate_up_shape), "down_shape": list(geo.down_shape),
        "key_template": geo.key_template, "total_experts": geo.total_experts,
        "double_buffer": geo.double_buffer, "host_rows_for_1_0.25": geo.host_rows_for(1, 0.25),
    }


def gen_geometry() -> None:
    """Checkpoint geometry (src/tideway/offload/geometry.py:261-311) and the raw expert
    row reader (src/tideway/baselines/expert_paging/pack.py:46-61) over the seeded
    miniature checkpoints of synthetic_checkpoints.py: the derived banks and pieces, the
    sha256 of every expert row, the exception each malformed checkpoint raises, and the
    pinned full-size Qwen3.6 / DeepSeek-V4 layouts from header-only checkpoints."""
    import hashlib
    import json
    import tempfile

    sys.path.insert(0, str(HERE))
    import synthetic_checkpoints as sc

    geom = _load("ref_geometry", REF / "src/tideway/offload/geometry.py")
    pkg = _stub_pack_package()
    spec = importlib.util.spec_from_file_location(
        f"{pkg}.pack", REF / "src/tideway/baselines/expert_paging/pack.py")
    pack = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = pack
    spec.loader.exec_module(pack)

    out = {"layouts": {}, "errors": {}, "pinned": {}}
    with tempfile.TemporaryDirectory() as tmp:
        roots = {n: sc.write_fused(tmp, n) for n in sc.FUSED}
        roots["dsv4"] = sc.write_ds(tmp)
        for name, root in roots.items():
            geo = geom.from_checkpoint(root)
            summary = _geo_summary(geo)
            reader = pack.SourceExperts(geo)
            summary["row_sha256"] = [hashlib.sha256(reader.read(e).tobytes()).hexdigest()
                                     for e in range(geo.total_experts)]
            try:
                reader.read(geo.total_experts)
                summary["read_past_end"] = None
            except Exception as exc:  # noqa: BLE001 - recorded as the expected error
                summary["read_past_end"] = type(exc).__name__
            reader.close()
            out["layouts"][name] = summary

        bad = {
            "fused_f16": lambda d: sc.write_fused(d, "qwen", gate_dtype="F16"),
            "fused_expert_mismatch": lambda d: sc.write_fused(d, "gemma", down_experts=2),
            "ds_w3_rows": lambda d: sc.write_ds(d, w3_rows=16),
            "ds_unhandled_dtype": lambda d: sc.write_ds(d, scale_dtype="F64"),
        }
        for name, make in bad.items():
            with tempfile.TemporaryDirectory() as d:
                try:
                    geom.from_checkpoint(make(d))
                    out["errors"][name] = None
                except Exception as exc:  # noqa: BLE001
                    out["errors"][name] = [type(exc).__name__, str(exc)]
        with tempfile.TemporaryDirectory() as d:
            root = Path(d) / "none"
            root.mkdir()
            sc.write_shard(root / "a.safetensors", [("x.weight", "BF16", (2, 2), bytes(8))])
            (root / "model.safetensors.index.json").write_text(
                json.dumps({"weight_map": {"x.weight": "a.safetensors"}}))
            try:
                geom.from_checkpoint(root)
                out["errors"]["no_layout"] = None
            except Exception as exc:  # noqa: BLE001
                out["errors"]["no_layout"] = [type(exc).__name__, "no known expert key layout"]

        for name, make, check in (("qwen36", sc.write_qwen36_headers, geom.check_qwen),
                                  ("dsv4", sc.write_dsv4_headers, geom.check_dsv4)):
            geo = geom.from_checkpoint(make(tmp))
            check(geo)
            out["pinned"][name] = _geo_summary(geo)
    (HERE / "geometry.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("geometry:", {k: len(v) for k, v in out.items()})


def _save(stem: str, cases: dict) -> None:
    flat = {}
    for case, d in cases.items():
        for k, v in d.items():
            flat[f"{case}.{k}"] = np.asarray(v)
    np.savez_compressed(HERE / f"{stem}.npz", **flat)
    print("wrote", stem, sorted(cases))


def main(only: list[str]) -> None:
    """Regenerate every fixture, or only the named generators (``geometry``, ``lru``)."""
    if only == ["geometry"]:
        gen_geometry()
        return
    _stub_freetoken()
    shift = _load("ref_shift", REF / "backends/freetoken_tideway/freetoken/moe/shift.py")
    cache_mod = _load("ref_cache", REF / "src/tideway/offload/cache.py")
    if only == ["lru"]:
        gen_lru(shift, cache_mod)
        gen_lru_pinned(shift, cache_mod)
        return
    fused = _load("ref_fused", REF / "backends/freetoken_tideway/freetoken/moe/fused.py")
    gemma = _load("ref_gemma", REF / "src/tideway/gemma_route_copy_kernel.py")
    torch.manual_seed(0)
    gen_fused_topk(fused)
    gen_gemma(gemma)
    gen_lru(shift, cache_mod)
    gen_lru_pinned(shift, cache_mod)
    gen_align()
    _stub_flashlib()
    kern = _load("ref_offload_kernels",
                 REF / "backends/freetoken_tideway/freetoken/moe/offload_kernels.py")
    gen_hybrid(kern)
    gen_geometry()


if __name__ == "__main__":
    main(sys.argv[1:])
