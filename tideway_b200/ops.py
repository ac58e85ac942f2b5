"""Torch-tensor wrappers over the C ABI.  CUDA tensors only; no CPU fallback.

Each op enqueues on ``torch.cuda.current_stream()`` and never synchronises, so a
sequence of ops can be captured into a CUDA graph.
"""

from __future__ import annotations

import torch

from . import _lib

F32, BF16 = 0, 1
_DT = {torch.float32: F32, torch.bfloat16: BF16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tideway_b200 ops run on CUDA tensors only (no CPU fallback)")


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


# ---------------------------------------------------------------- routing

def softmax_topk(logits: torch.Tensor, topk: int, renormalize: bool,
                 num_token_non_padded: torch.Tensor | None = None,
                 out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """fp32 softmax over experts, top-k (ties -> lower id), optional renormalisation."""
    _need_cuda(logits, num_token_non_padded)
    _need(logits.dim() == 2 and logits.stride(1) == 1, "logits must be [T, E] row-major")
    _need(logits.dtype in _DT, "logits must be float32 or bfloat16")
    T, E = logits.shape
    w, ids = out if out is not None else (
        torch.empty(T, topk, dtype=torch.float32, device=logits.device),
        torch.empty(T, topk, dtype=torch.int32, device=logits.device))
    ntp = None
    if num_token_non_padded is not None:
        ntp = num_token_non_padded.to(torch.int32).reshape(1)
    _lib.call("tw_router_softmax_topk", _ptr(logits), _DT[logits.dtype], logits.stride(0), T, E,
              topk, int(bool(renormalize)), _ptr(ntp), _ptr(w), _ptr(ids), _stream())
    return w, ids


def gemma_topk(logits: torch.Tensor, per_expert_scale: torch.Tensor, topk: int,
               out: tuple | None = None):
    """Gemma routing: (weights fp32, ids int32, private ids int32); ``out`` = preallocated
    (weights [T, topk] fp32, ids [T, topk] int32, private ids [T, topk] int32)."""
    _need_cuda(logits, per_expert_scale)
    _need(logits.dim() == 2 and logits.stride(1) == 1, "logits must be [T, E] row-major")
    _need(logits.dtype in _DT and per_expert_scale.dtype in _DT, "float32/bfloat16 inputs only")
    T, E = logits.shape
    _need(per_expert_scale.numel() == E, "per_expert_scale must have E entries")
    scale = per_expert_scale.contiguous()
    if out is not None:
        w, ids, priv = out
        _need(w.dtype == torch.float32 and ids.dtype == torch.int32 and priv.dtype == torch.int32
              and all(t.shape == (T, topk) and t.is_contiguous() for t in out),
              "out: (fp32, int32, int32) contiguous [T, topk]")
    else:
        w = torch.empty(T, topk, dtype=torch.float32, device=logits.device)
        ids = torch.empty(T, topk, dtype=torch.int32, device=logits.device)
        priv = torch.empty_like(ids)
    _lib.call("tw_router_gemma_topk", _ptr(logits), _DT[logits.dtype], logits.stride(0), T, E,
              topk, _ptr(scale), _DT[scale.dtype], _ptr(w), _ptr(ids), _ptr(priv), _stream())
    return w, ids, priv


def sigmoid_group_topk(logits: torch.Tensor, topk: int, n_group: int, topk_group: int,
                       routed_scaling_factor: float, renormalize: bool = True,
                       bias: torch.Tensor | None = None,
                       out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """DeepSeek-style sigmoid group-limited routing: (weights fp32, ids int32)."""
    _need_cuda(logits, bias)
    _need(logits.dim() == 2 and logits.stride(1) == 1, "logits must be [T, E] row-major")
    T, E = logits.shape
    b = None if bias is None else bias.float().contiguous()
    w, ids = out if out is not None else (
        torch.empty(T, topk, dtype=torch.float32, device=logits.device),
        torch.empty(T, topk, dtype=torch.int32, device=logits.device))
    _lib.call("tw_router_sigmoid_group_topk", _ptr(logits), _DT[logits.dtype], logits.stride(0),
              T, E, topk, n_group, topk_group, _ptr(b), int(bool(renormalize)),
              float(routed_scaling_factor), _ptr(w), _ptr(ids), _stream())
    return w, ids


def router_logits(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 logits [T, E] = x[T, H] . w[E, H]^T (bf16 inputs)."""
    _need_cuda(x, w)
    _need(x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, "bf16 inputs only")
    x, w = x.contiguous(), w.contiguous()
    T, H = x.shape
    E = w.shape[0]
    out = out if out is not None else torch.empty(T, E, dtype=torch.float32, device=x.device)
    _lib.call("tw_router_logits", _ptr(x), _ptr(w), T, H, E, _ptr(out), _stream())
    return out


_FUSED_MAX_T = 64
_ARRIVALS: dict[int, torch.Tensor] = {}


def router_arrivals(device) -> torch.Tensor:
    """A fresh zeroed block of arrival counters for the fused routers (one per token of a
    decode batch); callers whose router calls may overlap on the GPU each keep their own."""
    return torch.zeros(_FUSED_MAX_T, dtype=torch.int32, device=device)


def _default_arrivals(device) -> torch.Tensor:
    dev = torch.device(device).index or 0
    if dev not in _ARRIVALS:
        _ARRIVALS[dev] = router_arrivals(device)
    return _ARRIVALS[dev]


def _fused_router_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    T, H = x.shape
    E = w.shape[0]
    return E <= 1024 and H % 8 == 0 and H <= 4096 and 0 < T <= _FUSED_MAX_T


def _router_outputs(T: int, E: int, topk: int, device, out, logits_out):
    w, ids = out if out is not None else (
        torch.empty(T, topk, dtype=torch.float32, device=device),
        torch.empty(T, topk, dtype=torch.int32, device=device))
    _need(w.dtype == torch.float32 and ids.dtype == torch.int32 and w.is_contiguous()
          and ids.is_contiguous() and tuple(w.shape) == (T, topk) == tuple(ids.shape),
          "out: (fp32, int32) contiguous [T, topk]")
    logits = logits_out if logits_out is not None else torch.empty(
        T, E, dtype=torch.float32, device=device)
    _need(logits.dtype == torch.float32 and logits.is_contiguous()
          and tuple(logits.shape) == (T, E), "logits_out: contiguous fp32 [T, E]")
    return w, ids, logits


def router_softmax_topk(x: torch.Tensor, router_w: torch.Tensor, topk: int, renormalize: bool,
                        num_token_non_padded: torch.Tensor | None = None,
                        out: tuple[torch.Tensor, torch.Tensor] | None = None,
                        logits_out: torch.Tensor | None = None,
                        arrivals: torch.Tensor | None = None):
    """Router projection and softmax top-k in one launch (decode batches): the logits
    x . Wr^T (into ``logits_out`` when given), then the selection of ``softmax_topk``; the same
    bits as ``router_logits`` (warp GEMV) followed by ``softmax_topk``.  ``arrivals``: the
    kernel's per-token counters (``router_arrivals``; a shared per-device block by default).
    Larger batches run those two launches."""
    _need_cuda(x, router_w, num_token_non_padded)
    _need(x.dtype == torch.bfloat16 and router_w.dtype == torch.bfloat16, "bf16 inputs only")
    _need(x.dim() == 2 and x.is_contiguous() and router_w.is_contiguous(),
          "contiguous x [T, H] and router weight [E, H]")
    T, H = x.shape
    E = router_w.shape[0]
    w, ids, logits = _router_outputs(T, E, topk, x.device, out, logits_out)
    if not _fused_router_ok(x, router_w):
        router_logits(x, router_w, out=logits)
        return softmax_topk(logits, topk, renormalize, num_token_non_padded, out=(w, ids))
    ntp = None
    if num_token_non_padded is not None:
        ntp = num_token_non_padded.to(torch.int32).reshape(1)
    arr = arrivals if arrivals is not None else _default_arrivals(x.device)
    _need(arr.numel() >= T and arr.element_size() == 4, "arrivals: >= T 32-bit counters")
    _lib.call("tw_router_softmax_topk_fused", _ptr(x), _ptr(router_w), T, H, E, topk,
              int(bool(renormalize)), _ptr(ntp), _ptr(logits), _ptr(arr), _ptr(w), _ptr(ids),
              _stream())
    return w, ids


def router_sigmoid_group_topk(x: torch.Tensor, router_w: torch.Tensor, topk: int, n_group: int,
                              topk_group: int, routed_scaling_factor: float,
                              renormalize: bool = True, bias: torch.Tensor | None = None,
                              out: tuple[torch.Tensor, torch.Tensor] | None = None,
                              logits_out: torch.Tensor | None = None,
                              arrivals: torch.Tensor | None = None):
    """Router projection and sigmoid group-limited top-k in one launch (decode batches); the
    same bits as ``router_logits`` followed by ``sigmoid_group_topk``."""
    _need_cuda(x, router_w, bias)
    _need(x.dtype == torch.bfloat16 and router_w.dtype == torch.bfloat16, "bf16 inputs only")
    _need(x.dim() == 2 and x.is_contiguous() and router_w.is_contiguous(),
          "contiguous x [T, H] and router weight [E, H]")
    T, H = x.shape
    E = router_w.shape[0]
    w, ids, logits = _router_outputs(T, E, topk, x.device, out, logits_out)
    if not _fused_router_ok(x, router_w):
        router_logits(x, router_w, out=logits)
        return sigmoid_group_topk(logits, topk, n_group, topk_group, routed_scaling_factor,
                                  renormalize, bias, out=(w, ids))
    b = None if bias is None else bias.float().contiguous()
    arr = arrivals if arrivals is not None else _default_arrivals(x.device)
    _need(arr.numel() >= T and arr.element_size() == 4, "arrivals: >= T 32-bit counters")
    _lib.call("tw_router_sigmoid_group_topk_fused", _ptr(x), _ptr(router_w), T, H, E, topk,
              n_group, topk_group, _ptr(b), int(bool(renormalize)),
              float(routed_scaling_factor), _ptr(logits), _ptr(arr), _ptr(w), _ptr(ids),
              _stream())
    return w, ids


# ---------------------------------------------------------------- norms

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, weight_bias: float = 0.0,
            residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 RMSNorm; with ``residual`` the input is bf16(x + residual) (written to
    ``residual_out`` when given)."""
    _need_cuda(x, w, residual, residual_out)
    _need(x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, "bf16 inputs only")
    _need(x.is_contiguous(), "x must be contiguous")
    T, H = x.shape
    out = out if out is not None else torch.empty_like(x)
    _lib.call("tw_rmsnorm", _ptr(x), _ptr(residual), _ptr(residual_out), _ptr(w), T, H,
              float(eps), float(weight_bias), _ptr(out), _stream())
    return out


def router_norm_pair(x, ones, routed_weight, scale, eps: float, root: float,
                     out: tuple | None = None):
    """(router input, routed input) from one RMSNorm reduction (bf16); ``out`` = the two
    preallocated [T, H] outputs."""
    _need_cuda(x, ones, routed_weight, scale)
    T, H = x.shape
    if out is not None:
        a, b = out
        _need(all(t.shape == x.shape and t.dtype == x.dtype and t.is_contiguous() for t in out),
              "out: two contiguous tensors shaped like x")
    else:
        a, b = torch.empty_like(x), torch.empty_like(x)
    _lib.call("tw_router_norm_pair", _ptr(x), _ptr(ones), _ptr(routed_weight), _ptr(scale), T,
              H, float(eps), float(root), _ptr(a), _ptr(b), _stream())
    return a, b


def router_norm_triple(x, ones, routed_weight, scale, shared_weight, eps: float, root: float,
                       out: tuple | None = None):
    """(router input, routed input, shared-expert input) from one RMSNorm reduction of x;
    ``out`` = the three preallocated [T, H] outputs."""
    _need_cuda(x, ones, routed_weight, scale, shared_weight)
    T, H = x.shape
    if out is not None:
        _need(len(out) == 3 and all(t.shape == x.shape and t.dtype == x.dtype and
                                    t.is_contiguous() for t in out),
              "out: three contiguous tensors shaped like x")
        a, b, c = out
    else:
        a, b, c = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    _lib.call("tw_router_norm_triple", _ptr(x), _ptr(ones), _ptr(routed_weight), _ptr(scale),
              _ptr(shared_weight), T, H, float(eps), float(root), _ptr(a), _ptr(b), _ptr(c),
              _stream())
    return a, b, c


def add_shared(routed: torch.Tensor, shared: torch.Tensor, out: torch.Tensor | None = None
               ) -> torch.Tensor:
    """bf16(routed + shared) for [T, H] bf16 tensors (DeepSeek routed + shared expert)."""
    _need_cuda(routed, shared)
    _need(routed.shape == shared.shape and routed.dtype == torch.bfloat16 and
          shared.dtype == torch.bfloat16, "routed/shared must be matching bf16 [T, H]")
    out = out if out is not None else torch.empty_like(routed)
    T, H = routed.shape
    _lib.call("tw_add_shared", _ptr(routed), _ptr(shared), _ptr(out), T, H, _stream())
    return out


def dual_norm_merge(a, b, x, w1, w2, w3, eps1: float, eps2: float, eps3: float,
                    scalar: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(bf16(x + N3(bf16(N1(a) + N2(b)))) * scalar): shared + routed post-FFN merge, the
    layer scalar on the residual sum (the Gemma 4 decoder layer's order)."""
    _need_cuda(a, b, x, w1, w2, w3)
    T, H = x.shape
    out = out if out is not None else torch.empty_like(x)
    _lib.call("tw_dual_norm_merge", _ptr(a), _ptr(b), _ptr(x), _ptr(w1), _ptr(w2), _ptr(w3), T,
              H, float(eps1), float(eps2), float(eps3), float(scalar), _ptr(out), _stream())
    return out


# ---------------------------------------------------------------- slot table

def _check_ensure_extras(id_of_slot: torch.Tensor, stats, pinned) -> None:
    """The optional ensure outputs/inputs the kernels index: ``stats`` (int64, the first
    three entries += unique, misses, calls) and ``pinned`` (int32 per slot, non-zero = never
    evicted, shift.py:758-760)."""
    if stats is not None:
        _need_cuda(stats)
        _need(stats.dtype == torch.int64 and stats.is_contiguous() and stats.numel() >= 3,
              "stats must be a contiguous int64 tensor of at least 3 entries")
    if pinned is not None:
        _need_cuda(pinned)
        _need(pinned.dtype == torch.int32 and pinned.is_contiguous() and
              pinned.numel() == id_of_slot.numel(), "pinned must be contiguous int32 [num_slots]")


def lru_ensure(ids: torch.Tensor, slot_for_id, id_of_slot, usage, step, num_experts: int,
               layer_id: int, evict_slots, src_indices, num_indices, stats=None,
               pinned=None) -> None:
    """Rewrite ``ids`` (expert ids of one layer, int32) into slot ids in place."""
    _need_cuda(ids, slot_for_id, id_of_slot, usage, step)
    _need(ids.dtype == torch.int32 and ids.is_contiguous(), "ids must be contiguous int32")
    _check_ensure_extras(id_of_slot, stats, pinned)
    _lib.call("tw_lru_ensure", _ptr(ids), ids.numel(), _ptr(slot_for_id), _ptr(id_of_slot),
              _ptr(usage), _ptr(step), id_of_slot.numel(), num_experts, layer_id,
              _ptr(evict_slots), _ptr(src_indices), _ptr(num_indices), _ptr(stats), _ptr(pinned),
              _stream())


def lru_ensure_group(ids: torch.Tensor, slot_for_id, id_of_slot, usage, step, num_experts: int,
                     layer_id: int, evict_slots, src_indices, num_indices, H: int, I: int,
                     ws: torch.Tensor, stats=None, pinned=None, nvfp4: bool = False) -> None:
    """``lru_ensure`` on ids [T, K] (decode: T*K < 1024) plus, in the same launch, the expert
    FFN's grouping of the rewritten routes into ``ws`` (the workspace of T*K routes at H, I);
    the FFN then runs with ``pregrouped=True`` on the same workspace."""
    _need_cuda(ids, slot_for_id, id_of_slot, usage, step, ws)
    _need(ids.dtype == torch.int32 and ids.is_contiguous() and ids.dim() == 2,
          "ids must be contiguous int32 [T, K]")
    _check_ensure_extras(id_of_slot, stats, pinned)
    T, K = ids.shape
    _lib.call("tw_lru_ensure_group", _ptr(ids), T, K, _ptr(slot_for_id), _ptr(id_of_slot),
              _ptr(usage), _ptr(step), id_of_slot.numel(), num_experts, layer_id,
              _ptr(evict_slots), _ptr(src_indices), _ptr(num_indices), _ptr(stats),
              _ptr(pinned), H, I, int(bool(nvfp4)), _ptr(ws), ws.numel(), _stream())


def hybrid_ensure(ids: torch.Tensor, slot_for_id, id_of_slot, usage, step, num_experts: int,
                  layer_id: int, active_mask, evict_slots, src_indices, num_indices,
                  num_missing_full, recency, max_fetch: int, fetch_frac_q16: int) -> None:
    """Capped-fetch LRU: rewrite ``ids`` in place to slots, or -1 for the misses beyond the
    fetch cap.  ``recency`` ([L, E] int64, or None for the lowest-id fetch order)."""
    _need_cuda(ids, slot_for_id, id_of_slot, usage, step, active_mask, num_missing_full)
    _need(ids.dtype == torch.int32 and ids.is_contiguous(), "ids must be contiguous int32")
    _need(recency is None or (recency.dtype == torch.int64 and recency.is_contiguous()),
          "recency must be contiguous int64 [L, E]")
    _lib.call("tw_hybrid_ensure", _ptr(ids), ids.numel(), _ptr(slot_for_id), _ptr(id_of_slot),
              _ptr(usage), _ptr(step), id_of_slot.numel(), num_experts, layer_id,
              _ptr(active_mask), _ptr(evict_slots), _ptr(src_indices), _ptr(num_indices),
              _ptr(num_missing_full), _ptr(recency), int(max_fetch), int(fetch_frac_q16),
              _stream())


def materialize_layer(slot_for_id, id_of_slot, usage, step, num_experts: int, layer_id: int,
                      evict_slots, src_indices, num_indices) -> None:
    _lib.call("tw_materialize_layer", _ptr(slot_for_id), _ptr(id_of_slot), _ptr(usage),
              _ptr(step), id_of_slot.numel(), num_experts, layer_id, _ptr(evict_slots),
              _ptr(src_indices), _ptr(num_indices), _stream())


def reset_slots(slot_for_id, id_of_slot, usage, step, num_indices) -> None:
    _lib.call("tw_reset_slots", _ptr(slot_for_id), slot_for_id.numel(), _ptr(id_of_slot),
              _ptr(usage), id_of_slot.numel(), _ptr(step), _ptr(num_indices), _stream())


def prefill_hit_compact(slot_row, num_experts: int, buffer_id: int, dst_rows, src_slots,
                        num_hits) -> None:
    _lib.call("tw_prefill_hit_compact", _ptr(slot_row), num_experts, buffer_id, _ptr(dst_rows),
              _ptr(src_slots), _ptr(num_hits), _stream())


class CopyPlan:
    """Host-side pointer table for ``copy_rows`` over a fixed set of banks."""

    def __init__(self, dst_banks: list[torch.Tensor], src_banks: list[torch.Tensor]):
        import ctypes as C
        _need(len(dst_banks) == len(src_banks) and 0 < len(dst_banks) <= 8, "1..8 banks")
        n = len(dst_banks)
        self.n = n
        self.dst = (C.c_void_p * n)(*[t.data_ptr() for t in dst_banks])
        self.src = (C.c_void_p * n)(*[t.data_ptr() for t in src_banks])
        rb = []
        for d, s in zip(dst_banks, src_banks):
            row = d[0].numel() * d.element_size()
            _need(row == s[0].numel() * s.element_size(), "bank row sizes differ")
            rb.append(row)
        self.row_bytes = (C.c_int64 * n)(*rb)
        self._keep = (dst_banks, src_banks)


def copy_rows(plan: CopyPlan, dst_rows: torch.Tensor, src_rows: torch.Tensor,
              num_rows: torch.Tensor, max_rows: int) -> None:
    import ctypes as C
    _lib.call("tw_copy_rows", plan.n, C.cast(plan.dst, C.c_void_p), C.cast(plan.src, C.c_void_p),
              C.cast(plan.row_bytes, C.c_void_p), _ptr(dst_rows), _ptr(src_rows),
              _ptr(num_rows), max_rows, _stream())


# ---------------------------------------------------------------- expert FFN

_WS: dict[int, torch.Tensor] = {}


def workspace_bytes(n_routes: int, H: int, I: int) -> int:
    return int(_lib.load().tw_moe_workspace_bytes(n_routes, H, I))


def workspace(n_routes: int, H: int, I: int, device) -> torch.Tensor:
    """A cached per-device workspace large enough for n_routes routes."""
    need = workspace_bytes(n_routes, H, I)
    dev = torch.device(device).index or 0
    ws = _WS.get(dev)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _WS[dev] = ws
    return ws


def workspace_error(ws: torch.Tensor, n_routes: int, H: int, I: int) -> int:
    """Read (synchronously) the error word of an FFN workspace: 0 = ok."""
    off = int(_lib.load().tw_moe_workspace_error_offset(n_routes, H, I))
    return int(ws[off:off + 4].view(torch.int32).item())


def set_wait_limit(polls: int) -> None:
    """Polls after which a bounded wait of the tensor-core FFN kernels launched from now on
    gives up and sets the call's error word (0 restores the default, 2^24)."""
    _lib.call("tw_set_wait_limit", int(polls))


def host_register(ptr: int, nbytes: int) -> None:
    """Page-lock (portable, mapped) a host range in place; raises RuntimeError on failure and
    leaves no pending CUDA error behind, so the caller may retry."""
    _lib.call("tw_host_register", ptr, nbytes)


def host_unregister(ptr: int) -> None:
    _lib.call("tw_host_unregister", ptr)


ACTIVATIONS = {"silu": 0, "gelu": 1, "gelu_tanh": 2}


def _activation(activation: str, weight_on_input: bool) -> tuple[int, int]:
    if activation not in ACTIVATIONS:
        raise ValueError(f"Unsupported activation: {activation}")
    return ACTIVATIONS[activation], int(bool(weight_on_input))


def moe_ffn_bf16(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_weights: torch.Tensor,
                 topk_ids: torch.Tensor, out: torch.Tensor | None = None,
                 ws: torch.Tensor | None = None, activation: str = "silu",
                 weight_on_input: bool = False) -> torch.Tensor:
    """out[t] = sum_k bf16(gated expert FFN of x[t] through bank row topk_ids[t,k]).
    ``activation``: silu (SwiGLU), gelu or gelu_tanh on the gate half; ``weight_on_input``:
    the route weight scales the up projection instead of the down projection's output."""
    _need_cuda(x, w1, w2, topk_weights, topk_ids)
    _need(x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16,
          "bf16 activations and weights")
    _need(topk_weights.dtype == torch.float32 and topk_ids.dtype == torch.int32,
          "topk_weights fp32, topk_ids int32")
    _need(x.is_contiguous() and w1.is_contiguous() and w2.is_contiguous()
          and topk_weights.is_contiguous() and topk_ids.is_contiguous(), "contiguous inputs")
    T, H = x.shape
    S, twoI, H1 = w1.shape
    I = twoI // 2
    _need(H1 == H and w2.shape == (S, H, I), "bank shapes: w1 [S,2I,H], w2 [S,H,I]")
    K = topk_ids.shape[1]
    out = out if out is not None else torch.empty_like(x)
    ws = ws if ws is not None else workspace(T * K, H, I, x.device)
    act, w_in = _activation(activation, weight_on_input)
    if act or w_in:
        _lib.call("tw_moe_ffn_bf16_act", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), S,
                  _ptr(topk_weights), _ptr(topk_ids), K, act, w_in, _ptr(out), _ptr(ws),
                  ws.numel(), _stream())
        return out
    _lib.call("tw_moe_ffn_bf16", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), S, _ptr(topk_weights),
              _ptr(topk_ids), K, _ptr(out), _ptr(ws), ws.numel(), _stream())
    return out


def moe_ffn_bf16_residual_norm(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                               topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                               residual: torch.Tensor, residual_out: torch.Tensor,
                               norm_w: torch.Tensor, eps: float, h_out: torch.Tensor,
                               ws: torch.Tensor | None = None,
                               pregrouped: bool = False) -> torch.Tensor:
    """moe_ffn_bf16 then the next residual RMSNorm, the combine fused into the norm:
    residual_out = bf16(y + residual), h_out = rmsnorm(residual_out, norm_w, eps).  Returns
    h_out.  Bit-identical to moe_ffn_bf16 followed by rmsnorm(y, norm_w, eps, residual=...,
    residual_out=...).  ``pregrouped``: ``lru_ensure_group`` already grouped these routes into
    ``ws`` (same shapes), so the FFN skips its grouping launch."""
    _need_cuda(x, w1, w2, topk_weights, topk_ids, residual, residual_out, norm_w, h_out)
    _need(x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16,
          "bf16 activations and weights")
    _need(topk_weights.dtype == torch.float32 and topk_ids.dtype == torch.int32,
          "topk_weights fp32, topk_ids int32")
    T, H = x.shape
    S, twoI, H1 = w1.shape
    I = twoI // 2
    _need(H1 == H and w2.shape == (S, H, I), "bank shapes: w1 [S,2I,H], w2 [S,H,I]")
    _need(all(t.shape == x.shape and t.dtype == torch.bfloat16 and t.is_contiguous()
              for t in (residual, residual_out, h_out)), "residual/outputs shaped like x")
    K = topk_ids.shape[1]
    _need(ws is not None or not pregrouped, "pregrouped calls take the grouped workspace")
    ws = ws if ws is not None else workspace(T * K, H, I, x.device)
    name = ("tw_moe_ffn_bf16_residual_norm_grouped" if pregrouped
            else "tw_moe_ffn_bf16_residual_norm")
    _lib.call(name, _ptr(x), T, H, I, _ptr(w1), _ptr(w2), S,
              _ptr(topk_weights), _ptr(topk_ids), K, _ptr(residual), _ptr(residual_out),
              _ptr(norm_w), float(eps), _ptr(h_out), _ptr(ws), ws.numel(), _stream())
    return h_out


def moe_ffn_bf16_dual_merge(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                            topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                            shared: torch.Tensor, residual: torch.Tensor, w1n, w2n, w3n,
                            eps1: float, eps2: float, eps3: float, scalar: float,
                            out: torch.Tensor | None = None,
                            ws: torch.Tensor | None = None, activation: str = "silu",
                            weight_on_input: bool = False) -> torch.Tensor:
    """moe_ffn_bf16 then dual_norm_merge(shared, routed, residual, ...), the combine fused
    into the merge: out = bf16(bf16(residual + N3(bf16(N1(shared) + N2(routed)))) * scalar).
    Bit-identical to the two calls (``activation`` and ``weight_on_input`` as moe_ffn_bf16
    takes them); out may alias residual."""
    _need_cuda(x, w1, w2, topk_weights, topk_ids, shared, residual, w1n, w2n, w3n)
    _need(x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16,
          "bf16 activations and weights")
    _need(topk_weights.dtype == torch.float32 and topk_ids.dtype == torch.int32,
          "topk_weights fp32, topk_ids int32")
    T, H = x.shape
    S, twoI, H1 = w1.shape
    I = twoI // 2
    _need(H1 == H and w2.shape == (S, H, I), "bank shapes: w1 [S,2I,H], w2 [S,H,I]")
    _need(all(t.shape == x.shape and t.dtype == torch.bfloat16 and t.is_contiguous()
              for t in (shared, residual)), "shared/residual shaped like x")
    K = topk_ids.shape[1]
    act, w_in = _activation(activation, weight_on_input)
    out = out if out is not None else torch.empty_like(residual)
    ws = ws if ws is not None else workspace(T * K, H, I, x.device)
    if act or w_in:
        _lib.call("tw_moe_ffn_bf16_dual_merge_act", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), S,
                  _ptr(topk_weights), _ptr(topk_ids), K, _ptr(shared), _ptr(residual),
                  _ptr(w1n), _ptr(w2n), _ptr(w3n), float(eps1), float(eps2), float(eps3),
                  float(scalar), act, w_in, _ptr(out), _ptr(ws), ws.numel(), _stream())
        return out
    _lib.call("tw_moe_ffn_bf16_dual_merge", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), S,
              _ptr(topk_weights), _ptr(topk_ids), K, _ptr(shared), _ptr(residual), _ptr(w1n),
              _ptr(w2n), _ptr(w3n), float(eps1), float(eps2), float(eps3), float(scalar),
              _ptr(out), _ptr(ws), ws.numel(), _stream())
    return out


def ffn_dense_bf16(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                   out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
                   activation: str = "silu") -> torch.Tensor:
    """Dense gated FFN of one expert (w1 [2I,H], w2 [H,I]) over every row of x: the shared
    expert, SwiGLU by default (``activation`` as moe_ffn_bf16 takes it).  Bit-identical to
    moe_ffn_bf16 with one slot, K = 1 and weight 1."""
    _need_cuda(x, w1, w2)
    _need(x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16,
          "bf16 activations and weights")
    _need(x.is_contiguous() and w1.is_contiguous() and w2.is_contiguous(), "contiguous inputs")
    T, H = x.shape
    twoI, H1 = w1.shape[-2:]
    I = twoI // 2
    _need(H1 == H and w2.shape[-2:] == (H, I) and w1.numel() == twoI * H and w2.numel() == H * I,
          "weights: w1 [2I,H], w2 [H,I]")
    act, _ = _activation(activation, False)
    out = out if out is not None else torch.empty_like(x)
    ws = ws if ws is not None else workspace(T, H, I, x.device)
    if act:
        _lib.call("tw_ffn_dense_bf16_act", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), act, _ptr(out),
                  _ptr(ws), ws.numel(), _stream())
        return out
    _lib.call("tw_ffn_dense_bf16", _ptr(x), T, H, I, _ptr(w1), _ptr(w2), _ptr(out), _ptr(ws),
              ws.numel(), _stream())
    return out


_GLOBAL_DTYPES = {torch.float32: 0, torch.float16: 2}  # TW_F32, TW_F16


def _fp4_bank(name: str, packed, scale, global_, shape) -> None:
    """One NVFP4 bank of ``shape`` [S, rows, K]: packed u8 [S, rows, K/2], e4m3 (or its
    u8 bytes) [S, rows, K/16], fp32 or fp16 per-output-row globals [S, rows] (the reference's
    ModelOpt rows carry fp16 ones), all contiguous."""
    S, rows, K = shape
    _need(packed.dtype == torch.uint8 and tuple(packed.shape) == (S, rows, K // 2),
          f"{name} packed must be uint8 [S, rows, K/2] = {(S, rows, K // 2)}")
    _need(scale.dtype in (torch.float8_e4m3fn, torch.uint8)
          and tuple(scale.shape) == (S, rows, K // 16),
          f"{name} scale must be e4m3 [S, rows, K/16] = {(S, rows, K // 16)}")
    _need(global_.dtype in _GLOBAL_DTYPES and tuple(global_.shape) == (S, rows),
          f"{name} global must be float32 or float16 [S, rows] = {(S, rows)}")
    _need(packed.is_contiguous() and scale.is_contiguous() and global_.is_contiguous(),
          f"{name} banks must be contiguous")


def moe_ffn_nvfp4(x: torch.Tensor, w1: tuple, w2: tuple, topk_weights: torch.Tensor,
                  topk_ids: torch.Tensor, out: torch.Tensor | None = None,
                  ws: torch.Tensor | None = None, pregrouped: bool = False,
                  activation: str = "silu", weight_on_input: bool = False) -> torch.Tensor:
    """NVFP4 banks: w1 = (packed [S,2I,H/2] u8, scale [S,2I,H/16] e4m3, global [S,2I] f32 or
    f16), w2 = (packed [S,H,I/2], scale [S,H,I/16], global [S,H], the same global dtype).
    ``activation`` / ``weight_on_input`` as for moe_ffn_bf16."""
    w1p, w1s, w1g = w1
    w2p, w2s, w2g = w2
    _need(x.dim() == 2 and x.dtype == torch.bfloat16 and x.is_contiguous(),
          "x must be contiguous bf16 [T, H]")
    T, H = x.shape
    _need(w1p.dim() == 3 and w1p.shape[2] * 2 == H and w1p.shape[1] % 2 == 0,
          "w1 packed must be [S, 2I, H/2]")
    S, twoI, _ = w1p.shape
    I = twoI // 2
    _need(H % 16 == 0 and I % 16 == 0, "H and I must be multiples of 16 (e4m3 blocks)")
    _fp4_bank("w1", w1p, w1s, w1g, (S, twoI, H))
    _fp4_bank("w2", w2p, w2s, w2g, (S, H, I))
    _need(w1g.dtype == w2g.dtype, "w1 and w2 globals must share one dtype")
    _need(topk_weights.dtype == torch.float32 and topk_ids.dtype == torch.int32,
          "topk_weights fp32, topk_ids int32")
    _need(topk_ids.dim() == 2 and topk_ids.shape[0] == T and topk_weights.shape == topk_ids.shape
          and topk_ids.is_contiguous() and topk_weights.is_contiguous(),
          "topk_weights / topk_ids must be contiguous [T, K]")
    _need_cuda(x, w1p, w1s, w1g, w2p, w2s, w2g, topk_weights, topk_ids)
    K = topk_ids.shape[1]
    out = out if out is not None else torch.empty_like(x)
    ws = ws if ws is not None else workspace(T * K, H, I, x.device)
    _need(not pregrouped or ws is not None, "pregrouped calls take the grouped workspace")
    act, w_in = _activation(activation, weight_on_input)
    if act or w_in:
        _need(not pregrouped, "the activation variants group their own routes")
        _lib.call("tw_moe_ffn_nvfp4_act", _ptr(x), T, H, I, _ptr(w1p), _ptr(w1s), _ptr(w1g),
                  _ptr(w2p), _ptr(w2s), _ptr(w2g), _GLOBAL_DTYPES[w1g.dtype], S,
                  _ptr(topk_weights), _ptr(topk_ids), K, act, w_in, _ptr(out), _ptr(ws),
                  ws.numel(), _stream())
        return out
    _lib.call("tw_moe_ffn_nvfp4_grouped" if pregrouped else "tw_moe_ffn_nvfp4", _ptr(x), T, H,
              I, _ptr(w1p), _ptr(w1s), _ptr(w1g), _ptr(w2p),
              _ptr(w2s), _ptr(w2g), _GLOBAL_DTYPES[w1g.dtype], S, _ptr(topk_weights),
              _ptr(topk_ids), K, _ptr(out), _ptr(ws), ws.numel(), _stream())
    return out


def nvfp4_dequantize(packed: torch.Tensor, scale: torch.Tensor, global_: torch.Tensor
                     ) -> torch.Tensor:
    """fp32 [..., K] = e2m1 * e4m3 block scale * row global, decoded on the GPU."""
    half = packed.shape[-1]
    rows = packed.numel() // max(half, 1)
    _need(packed.dtype == torch.uint8 and half % 8 == 0, "packed must be uint8 [..., K/2], K % 16 == 0")
    _need(scale.dtype in (torch.float8_e4m3fn, torch.uint8) and scale.numel() == rows * half // 8
          and global_.dtype in _GLOBAL_DTYPES and global_.numel() == rows,
          "scale e4m3 [..., K/16] and global float32/float16 [...] must match packed")
    _need(packed.is_contiguous() and scale.is_contiguous() and global_.is_contiguous(),
          "contiguous inputs")
    _need_cuda(packed, scale, global_)
    out = torch.empty(rows, 2 * half, dtype=torch.float32, device=packed.device)
    _lib.call("tw_nvfp4_dequantize", _ptr(packed), _ptr(scale), _ptr(global_),
              _GLOBAL_DTYPES[global_.dtype], rows, 2 * half, _ptr(out), _stream())
    return out.view(*packed.shape[:-1], 2 * half)


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int):
    """(sorted_ids, expert_ids, num_tokens_post_padded) with the reference's sizing."""
    _need_cuda(topk_ids)
    ids = topk_ids.contiguous().to(torch.int32)
    numel = ids.numel()
    if numel < num_experts + 1:
        max_padded = numel * block_size
    else:
        max_padded = numel + (num_experts + 1) * (block_size - 1)
    max_padded = max(max_padded, 1)
    sorted_ids = torch.empty(max_padded, dtype=torch.int32, device=ids.device)
    expert_ids = torch.empty(-(-max_padded // block_size), dtype=torch.int32, device=ids.device)
    npad = torch.empty(1, dtype=torch.int32, device=ids.device)
    _lib.call("tw_moe_align_block_size", _ptr(ids), numel, num_experts, block_size,
              _ptr(sorted_ids), _ptr(expert_ids), _ptr(npad), max_padded, _stream())
    return sorted_ids, expert_ids, npad
