"""CPU oracle for the MoE expert-execution path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of Tideway's MoE expert-execution
step (router top-k, expert-slot table, slot-indirect SwiGLU expert FFN, weighted
combine, RMSNorm, NVFP4 dequantisation, expert-parallel dispatch/combine).  It is the
checker the CUDA product path is compared against.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it.  The product package ``tideway_b200`` never imports it and has no CPU
fallback: it fails loudly when its CUDA library is missing.

Parity status per module (how each restatement is pinned):

* ``routing.softmax_topk``      -- pinned: golden vectors produced by the reference's
  own ``fused_topk`` torch path (backends/freetoken_tideway/freetoken/moe/fused.py:16-85).
* ``routing.gemma_topk``        -- pinned: golden vectors produced by the reference's
  ``_routing_with_copy`` Triton kernel run under TRITON_INTERPRET=1
  (src/tideway/gemma_route_copy_kernel.py:28-70).
* ``routing.sigmoid_group_topk`` -- parity unpinned: the DeepSeek gate is absent from the
  reference; this restates the published DeepSeek-V3 group-limited routing.
* ``slot_cache.lru_ensure``     -- pinned: golden vectors produced by the reference's
  vendored ``lru_ensure`` (backends/.../moe/shift.py:698-777, pinned mask 0) under
  TRITON_INTERPRET=1, and cross-checked against ``offload/cache.py:Cache.access``.
* ``ffn.*``                     -- parity unpinned for the expert FFN arithmetic (the
  reference's Triton FFN kernels live in the absent FreeToken 0.1.2); the rounding points
  follow the reference orchestration (fused.py:261-450).  ``moe_align_block_size`` is
  pinned by the worked example in its docstring (fused.py:113-126).
* ``nvfp4``                     -- parity unpinned (reference kernels absent); restates the
  NVFP4 format named by the benchmark configuration.
"""
