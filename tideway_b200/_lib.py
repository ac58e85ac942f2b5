"""ctypes binding of the tideway_b200 C ABI (include/tideway_b200.h).

The library is loaded from ``tideway_b200/_lib/libtideway_b200.so``.  There is no CPU
fallback: if the library is missing or no CUDA device is present, every op raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import os

# TIDEWAY_B200_LIB points at an alternative build of the same library (tuning builds).
LIB_PATH = Path(os.environ.get("TIDEWAY_B200_LIB") or
                Path(__file__).resolve().parent / "_lib" / "libtideway_b200.so")

_i32, _i64, _f32, _vp, _sz = C.c_int, C.c_int64, C.c_float, C.c_void_p, C.c_size_t

# name -> argtypes (restype int unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "tw_last_error": [],
    "tw_abi_version": [],
    "tw_set_wait_limit": [C.c_uint32],
    "tw_router_softmax_topk": [_vp, _i32, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp],
    "tw_router_gemma_topk": [_vp, _i32, _i64, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp],
    "tw_router_sigmoid_group_topk": [_vp, _i32, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _i32,
                                     _f32, _vp, _vp, _vp],
    "tw_router_logits": [_vp, _vp, _i64, _i32, _i32, _vp, _vp],
    "tw_router_softmax_topk_fused": [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                                     _vp, _vp],
    "tw_router_sigmoid_group_topk_fused": [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp,
                                           _i32, _f32, _vp, _vp, _vp, _vp, _vp],
    "tw_rmsnorm": [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _f32, _vp, _vp],
    "tw_router_norm_pair": [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _f32, _vp, _vp, _vp],
    "tw_router_norm_triple": [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _f32, _vp, _vp, _vp,
                              _vp],
    "tw_add_shared": [_vp, _vp, _vp, _i64, _i32, _vp],
    "tw_dual_norm_merge": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _f32, _f32, _f32, _vp,
                           _vp],
    "tw_lru_ensure": [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                      _vp],
    "tw_hybrid_ensure": [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp,
                         _vp, _vp, _i32, _i32, _vp],
    "tw_materialize_layer": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp],
    "tw_reset_slots": [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp],
    "tw_prefill_hit_compact": [_vp, _i32, _i32, _vp, _vp, _vp, _vp],
    "tw_copy_rows": [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp],
    "tw_moe_workspace_bytes": [_i64, _i32, _i32],
    "tw_moe_workspace_error_offset": [_i64, _i32, _i32],
    "tw_host_register": [_vp, _sz],
    "tw_host_unregister": [_vp],
    "tw_moe_ffn_bf16": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32, _vp, _vp, _sz,
                        _vp],
    "tw_moe_ffn_bf16_residual_norm": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32,
                                      _vp, _vp, _vp, _f32, _vp, _vp, _sz, _vp],
    "tw_moe_ffn_bf16_dual_merge": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32, _vp,
                                   _vp, _vp, _vp, _vp, _f32, _f32, _f32, _f32, _vp, _vp, _sz,
                                   _vp],
    "tw_ffn_dense_bf16": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp],
    "tw_moe_ffn_nvfp4": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64, _vp,
                         _vp, _i32, _vp, _vp, _sz, _vp],
    "tw_nvfp4_dequantize": [_vp, _vp, _vp, _i32, _i64, _i32, _vp, _vp],
    "tw_moe_ffn_bf16_act": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32, _i32, _i32,
                            _vp, _vp, _sz, _vp],
    "tw_moe_ffn_nvfp4_act": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64,
                             _vp, _vp, _i32, _i32, _i32, _vp, _vp, _sz, _vp],
    "tw_ffn_dense_bf16_act": [_vp, _i64, _i32, _i32, _vp, _vp, _i32, _vp, _vp, _sz, _vp],
    "tw_moe_ffn_bf16_dual_merge_act": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32,
                                       _vp, _vp, _vp, _vp, _vp, _f32, _f32, _f32, _f32, _i32,
                                       _i32, _vp, _vp, _sz, _vp],
    "tw_moe_align_block_size": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _i64, _vp],
    "tw_moe_ffn_bf16_noalloc": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32, _vp, _vp],
    "tw_moe_ffn_noalloc_scratch_bytes": [],
    "tw_moe_ffn_noalloc_error": [_i64, _i32, _i32, _vp, _vp],
    "tw_ep_row_bytes": [_i32, _i32],
    "tw_ep_dispatch": [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp],
    "tw_ep_receive": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp],
    "tw_ep_combine": [_vp, _i64, _i32, _i32, _vp, _vp],
    "tw_moe_ffn_bf16_routes": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32, _vp, _sz,
                               _vp],
    "tw_moe_ffn_nvfp4_routes": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64,
                                _vp, _vp, _i32, _vp, _sz, _vp],
    "tw_lru_ensure_group": [_vp, _i64, _i32, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp,
                            _vp, _vp, _vp, _i32, _i32, _i32, _vp, _sz, _vp],
    "tw_moe_ffn_bf16_residual_norm_grouped": [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp,
                                              _i32, _vp, _vp, _vp, _f32, _vp, _vp, _sz, _vp],
    "tw_moe_ffn_nvfp4_grouped": [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                                 _i64, _vp, _vp, _i32, _vp, _vp, _sz, _vp],
    "tw_ep_p2p_bytes": [_i32, _i64, _i32, _i32],
    "tw_ep_p2p_offsets": [_i32, _i64, _i32, _i32, _vp],
    "tw_ep_p2p_handle_bytes": [],
    "tw_ep_p2p_export": [_vp, _vp, _vp],
    "tw_ep_p2p_open": [_vp, C.c_uint64, _vp, _vp],
    "tw_ep_p2p_close": [_vp],
    "tw_ep_p2p_dispatch": [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp],
    "tw_ep_p2p_combine": [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _vp, _vp, _vp,
                          _vp, _f32, _vp, _vp, _vp],
    "tw_ep_p2p_error": [_vp, _vp, _vp],
}
_RESTYPES = {"tw_last_error": C.c_char_p, "tw_moe_workspace_bytes": _sz,
             "tw_moe_workspace_error_offset": _sz, "tw_moe_ffn_noalloc_scratch_bytes": _sz,
             "tw_ep_row_bytes": _sz, "tw_ep_p2p_bytes": _sz, "tw_ep_p2p_handle_bytes": _sz}

_lib: C.CDLL | None = None


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def load() -> C.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"tideway_b200 CUDA library not built ({LIB_PATH}); run "
                "`python -m tideway_b200.build` (nvcc, sm_100a)")
        lib = C.CDLL(str(LIB_PATH))
        for name, args in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point and raise RuntimeError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.tw_last_error().decode(errors="replace")
        kind = {1: ValueError, 3: NotImplementedError}.get(rc, RuntimeError)
        raise kind(f"{name}: {msg} (status {rc})")
