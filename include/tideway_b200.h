/*
 * tideway_b200 C ABI -- the drop-in boundary of the B200 MoE expert-execution path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t (passed as
 * void*), enqueues its kernels on that stream and returns an int status: 0 on success,
 * otherwise a TW_ERR_* code with a message available from tw_last_error().  Nothing
 * here allocates memory, synchronises the host or reads a device value back, so the
 * routing, slot-table, FFN, norm and expert-parallel calls can be captured into a CUDA
 * graph (the allocation-free entry point below states its own rules).  Counts that only
 * exist on the device (misses, unique experts) are read by the kernels themselves.
 *
 * Dtype codes: TW_F32 = 0, TW_BF16 = 1, TW_F16 = 2.  Index tensors are int32 unless noted.
 *
 * Each declaration names the reference interface it replaces (path:line inside the
 * Tideway checkout).
 */
#ifndef TIDEWAY_B200_H
#define TIDEWAY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TW_OK 0
#define TW_ERR_INVALID 1     /* bad argument (shape, dtype, alignment, limit) */
#define TW_ERR_CUDA 2        /* a CUDA runtime call failed */
#define TW_ERR_UNSUPPORTED 3 /* shape outside what the kernels implement */

#define TW_F32 0
#define TW_BF16 1
#define TW_F16 2

/* Gate activations of the expert FFN (the *_act entry points). */
#define TW_ACT_SILU 0
#define TW_ACT_GELU 1      /* g/2 (1 + erf(g / sqrt 2)) */
#define TW_ACT_GELU_TANH 2 /* g/2 (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))) */

/* Last error message of the calling thread ("" if none). */
const char* tw_last_error(void);

/* Polls after which a bounded device wait of the tensor-core FFN kernels (an mbarrier, a
 * hand-off between up and down tiles) gives up, for the FFN launches issued after this call
 * in this process; 0 restores the default 2^24.  A wait that gives up sets the call's error
 * word to 1 (tw_moe_workspace_error_offset), lets the copies and MMAs already issued land,
 * frees its tensor memory and returns; its output is then invalid.  Lowering it makes a
 * stuck launch return sooner (and lets a test drive that path without a stuck GPU).  No
 * reference counterpart: the reference's Triton kernels have no device error channel. */
int tw_set_wait_limit(uint32_t polls);
/* ABI version (major * 100 + minor). */
int tw_abi_version(void);

/* ---------------------------------------------------------------- routing (a1-a3) */

/* Softmax router: fp32 softmax over E, top-K (ties -> lower id), optional renormalise,
 * rows >= *num_token_non_padded (device int32, may be NULL) get id -1.
 * Replaces fused_topk / _torch_fused_topk,
 * backends/freetoken_tideway/freetoken/moe/fused.py:16-85. */
int tw_router_softmax_topk(const void* logits, int logits_dtype, int64_t ld_logits,
                           int64_t T, int E, int K, int renormalize,
                           const int32_t* num_token_non_padded,
                           float* topk_weights, int32_t* topk_ids, void* stream);

/* Gemma routing: top-K logits (ties -> lower id), softmax over the K, x scale[id];
 * ids written to topk_ids and private_ids (either may be NULL).
 * Replaces routing_with_private_ids / _routing_with_copy,
 * src/tideway/gemma_route_copy_kernel.py:28-102. */
int tw_router_gemma_topk(const void* logits, int logits_dtype, int64_t ld_logits,
                         int64_t T, int E, int K, const void* per_expert_scale,
                         int scale_dtype, float* topk_weights, int32_t* topk_ids,
                         int32_t* private_ids, void* stream);

/* Sigmoid scoring with group-limited top-k (DeepSeek style): groups scored by the sum of
 * their two best (sigmoid + bias) scores, top_group groups kept, top-K experts of those,
 * weights = sigmoid (no bias), renormalised if asked, x routed_scaling.  bias may be NULL.
 * Replaces the gate consumed at src/tideway/offload/ffn_front_graph.py:24-30. */
int tw_router_sigmoid_group_topk(const void* logits, int logits_dtype, int64_t ld_logits,
                                 int64_t T, int E, int K, int n_group, int topk_group,
                                 const float* bias, int renormalize, float routed_scaling,
                                 float* topk_weights, int32_t* topk_ids, void* stream);

/* Router logits GEMM: logits[T,E] (fp32) = x[T,H] . w[E,H]^T, both bf16.
 * Replaces the model router projection feeding OffloadMoELayer.forward,
 * backends/freetoken_tideway/freetoken/layers/moe.py:229-239. */
int tw_router_logits(const void* x, const void* w, int64_t T, int H, int E,
                     float* logits, void* stream);

/* Decode router in one launch: logits = x[T,H] . w[E,H]^T (fp32, into `logits` [T,E], which
 * is required) and the softmax top-k of tw_router_softmax_topk on them.  The GEMV keeps its
 * parallelism (CTA (b, t): 16 router rows of token t, a warp per row); the CTA that
 * completes token t's arrival count runs the selection and sets the count back to 0.
 * `arrivals` is uint32 [T] device memory set to 0 once before the first call; every call
 * leaves it at 0 again (a call that does not complete, an aborted launch, must be followed
 * by zeroing it).  Logits, weights and ids are
 * bit-identical to tw_router_logits' warp GEMV (T < 128) followed by tw_router_softmax_topk.
 * E <= 1024, H % 8 == 0, H <= 4096, T <= 64 (decode batches); calls that share `arrivals`
 * must not overlap on the GPU.  Replaces the router projection feeding
 * OffloadMoELayer.forward (backends/freetoken_tideway/freetoken/layers/moe.py:229-239)
 * together with fused_topk (backends/freetoken_tideway/freetoken/moe/fused.py:16-85). */
int tw_router_softmax_topk_fused(const void* x, const void* w, int64_t T, int H, int E, int K,
                                 int renormalize, const int32_t* num_token_non_padded,
                                 float* logits, uint32_t* arrivals, float* topk_weights,
                                 int32_t* topk_ids, void* stream);

/* The same with the sigmoid group-limited selection of tw_router_sigmoid_group_topk
 * (bit-identical to tw_router_logits' warp GEMV followed by it; same limits and counters).
 * Replaces the router projection and the gate consumed at
 * src/tideway/offload/ffn_front_graph.py:24-30. */
int tw_router_sigmoid_group_topk_fused(const void* x, const void* w, int64_t T, int H, int E,
                                       int K, int n_group, int topk_group, const float* bias,
                                       int renormalize, float routed_scaling, float* logits,
                                       uint32_t* arrivals, float* topk_weights,
                                       int32_t* topk_ids, void* stream);

/* ---------------------------------------------------------------- RMSNorm (a4, a14) */

/* y = bf16(x * rsqrt(mean(x^2) + eps) * (w + weight_bias)), fp32 reduction.
 * If residual != NULL, first x = bf16(x + residual) is formed, written back to
 * residual_out (may alias x), and normalised.  Replaces the RMSNorm of
 * src/tideway/cute_router_norm_pair.py:252-306 (FlashInfer RMSNormKernel). */
int tw_rmsnorm(const void* x, const void* residual, void* residual_out, const void* w,
               int64_t T, int H, float eps, float weight_bias, void* y, void* stream);

/* Router/routed RMSNorm pair with the router's bf16 cast chain:
 * router = bf16(bf16(bf16(x*rstd*ones)*scale)*root), routed = bf16(x*rstd*routed_w).
 * Replaces router_norm_pair, src/tideway/cute_router_norm_pair.py:353-395. */
int tw_router_norm_pair(const void* x, const void* ones, const void* routed_weight,
                        const void* scale, int64_t T, int H, float eps, float root,
                        void* router_out, void* routed_out, void* stream);

/* The pair plus the shared expert's pre-norm from the same reduction of x (same eps):
 * shared = bf16(x*rstd*shared_w); with shared_w == shared_out == NULL it is the pair.  One
 * pass over x for the three RMSNorms of a Gemma MoE block's input (the router norm pair and
 * the pre-feedforward norm whose output feeds layer.shared_forward,
 * src/tideway/overlap_shared_expert.py:253). */
int tw_router_norm_triple(const void* x, const void* ones, const void* routed_weight,
                          const void* scale, const void* shared_weight, int64_t T, int H,
                          float eps, float root, void* router_out, void* routed_out,
                          void* shared_out, void* stream);

/* DeepSeek-layout merge of the routed and the always-active shared expert outputs:
 * out = bf16(routed + shared), [T, H] bf16.  Replaces the routed + shared sum of
 * src/tideway/offload/ffn_back_graph.py:29-37. */
int tw_add_shared(const void* routed, const void* shared, void* out, int64_t T, int H,
                  void* stream);

/* Post-FFN merge of a shared-expert output a and a routed output b (Gemma layout):
 * out = bf16(bf16(x + N3(bf16(N1(a) + N2(b)))) * scalar), Nk = bf16 RMSNorm with weight wk and
 * eps_k: the layer scalar scales the residual sum, as in the Gemma 4 decoder layer.  Replaces
 * the merge consumed at src/tideway/overlap_shared_expert.py:253-276 (its kernel, FreeToken's
 * gemma_dual_rmsnorm_residual_scalar, is not in the reference). */
int tw_dual_norm_merge(const void* a, const void* b, const void* x, const void* w1,
                       const void* w2, const void* w3, int64_t T, int H, float eps1,
                       float eps2, float eps3, float scalar, void* out, void* stream);

/* ---------------------------------------------------------------- slot table (a5-a8) */

/* Sequential-argmin LRU ensure over the fixed-address slot table, bit-exact with the
 * reference: ids [n] (expert ids of one layer, in place -> slot ids), slot_for_id
 * [L*E], id_of_slot [S], usage int64 [S], step int64 [1], evict_slots/src_indices [E],
 * num_indices int64 [1], stats int64 [3] (may be NULL), pinned int32 [S] (may be NULL).
 * n <= 8192, E <= 1024, S <= 16384.
 * Replaces ensure_experts / lru_ensure, backends/.../moe/offload_kernels.py:19-51 and
 * backends/.../moe/shift.py:698-777. */
int tw_lru_ensure(int32_t* ids, int64_t n, int32_t* slot_for_id, int32_t* id_of_slot,
                  int64_t* usage, int64_t* step, int64_t num_slots, int num_experts,
                  int layer_id, int32_t* evict_slots, int32_t* src_indices,
                  int64_t* num_indices, int64_t* stats, const int32_t* pinned,
                  void* stream);

/* Map one layer onto slots [0, E) for a whole-layer copy.
 * Replaces materialize_layer, backends/.../moe/offload_kernels.py:256-292. */
/* Capped-fetch LRU of the hybrid backend: as tw_lru_ensure, but only the first
 * min(misses, cap) misses -- ordered by (recency descending, id ascending), or by id when
 * recency == NULL -- get a victim slot and a pending copy; the other misses keep no slot
 * and their ids become -1.  cap = max_fetch, or with fetch_frac_q16 > 0 (Q16 fraction) the
 * integer F near frac * misses minimising max(F*(1-frac), (misses-F)*frac).  Writes
 * active_mask [E] (routed this step), num_indices (fetches), num_missing_full (misses) and
 * recency[layer, e] = step for the routed experts (recency: [L, E] int64).  Replaces
 * ensure_experts_hybrid / _ensure_experts_hybrid_kernel,
 * backends/.../moe/offload_kernels.py:54-79, :296-415 (CPU mirror :135-195). */
int tw_hybrid_ensure(int32_t* ids, int64_t n, int32_t* slot_for_id, int32_t* id_of_slot,
                     int64_t* usage, int64_t* step, int64_t num_slots, int num_experts,
                     int layer_id, int32_t* active_mask, int32_t* evict_slots,
                     int32_t* src_indices, int64_t* num_indices, int64_t* num_missing_full,
                     int64_t* recency, int max_fetch, int fetch_frac_q16, void* stream);

int tw_materialize_layer(int32_t* slot_for_id, int32_t* id_of_slot, int64_t* usage,
                         int64_t* step, int64_t num_slots, int num_experts, int layer_id,
                         int32_t* evict_slots, int32_t* src_indices, int64_t* num_indices,
                         void* stream);

/* Clear the slot table.  Replaces reset_cache, backends/.../moe/offload_kernels.py:233-253. */
int tw_reset_slots(int32_t* slot_for_id, int64_t num_ids, int32_t* id_of_slot,
                   int64_t* usage, int64_t num_slots, int64_t* step, int64_t* num_indices,
                   void* stream);

/* Compact the experts of one layer resident at slot >= 2E into gather lists.
 * Replaces prefill_hit_compact, backends/.../moe/offload_kernels.py:74-93, :418-436. */
int tw_prefill_hit_compact(const int32_t* slot_for_id_row, int num_experts, int buffer_id,
                           int32_t* dst_rows, int32_t* src_slots, int64_t* num_hits,
                           void* stream);

/* Copy *num_rows rows per bank: dst_base[b] + dst_rows[i]*row_bytes[b] <-
 * src_base[b] + src_rows[i]*row_bytes[b], for i < min(*num_rows, max_rows).
 * Sources may be pinned host memory (read over the host link) or device memory.
 * All bases and row sizes 16-byte aligned; n_banks <= 8.
 * Replaces copy_missing / fast_index_copy_multi_jit,
 * backends/.../moe/offload_cache.py:1024-1054. */
/* Page-lock (portable, mapped) / release a host range that backs host-tier expert banks, in
 * place.  A failed registration returns TW_ERR_CUDA and leaves no pending CUDA error behind,
 * so a caller may retry (a process that has just exited can still be releasing its own
 * page-locked memory).  Replaces the pinned host tier's allocation in
 * src/tideway/offload/runtime.py (pinned RAM banks read by copy_missing). */
int tw_host_register(void* ptr, size_t bytes);
int tw_host_unregister(void* ptr);

int tw_copy_rows(int n_banks, void* const* dst_base, const void* const* src_base,
                 const int64_t* row_bytes, const int32_t* dst_rows, const int32_t* src_rows,
                 const int64_t* num_rows, int64_t max_rows, void* stream);

/* ---------------------------------------------------------------- expert FFN (a9-a12) */

/* Workspace bytes the expert-FFN entry points need for n_routes = T*K routes. */
size_t tw_moe_workspace_bytes(int64_t n_routes, int H, int I);

/* Byte offset, inside that workspace, of the int32 error word the tensor-core kernels set
 * (0 = ok, 1 = a bounded wait gave up) and every FFN call clears on entry.  New in this
 * build (the reference's Triton kernels have no device error channel). */
size_t tw_moe_workspace_error_offset(int64_t n_routes, int H, int I);

/* Slot-indirect SwiGLU expert FFN plus combine over a bf16 slot bank:
 * out[t] = bf16(sum_k bf16(bf16(silu(c1_g)*c1_u) . w2[s]^T * w[t,k])), c1 = bf16(x . w1[s]^T),
 * s = topk_ids[t,k] (slot id; negative -> route skipped).  w1 [S,2I,H] (gate rows first),
 * w2 [S,H,I].  Each distinct slot's weights are read once for all its routes.
 * out may alias x.  Replaces fused_experts_decode_impl / fused_experts_impl,
 * backends/.../moe/fused.py:261-450. */
int tw_moe_ffn_bf16(const void* x, int64_t T, int H, int I, const void* w1, const void* w2,
                    int64_t num_slots, const float* topk_weights, const int32_t* topk_ids,
                    int K, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free form of tw_moe_ffn_bf16, for callers that may not allocate device
 * memory at call time: plugins inside a serving process whose memory pool owns all of the
 * GPU's memory and forbids allocations outside it, and foreign-language bindings (a C,
 * Go or Java host) that have no device allocator to hand a workspace over.
 * It has no counterpart in the reference.  Its scratch is one static device array of
 * tw_moe_ffn_noalloc_scratch_bytes() (32 MiB) that every GPU loading this library holds
 * until exit; calls needing more (n = T*K routes: tw_moe_workspace_bytes(n, H, I) bytes)
 * fail with TW_ERR_INVALID and launch nothing.  The first call on a device looks the array's
 * device address up (cudaGetSymbolAddress) with that device current: make that first call
 * before any stream capture.  All calls share the array and it keeps the previous call's
 * contents (each call clears the counters that must start at zero), so calls that may
 * overlap on the GPU -- on different streams without ordering -- race; serialise them.
 * Nothing is allocated or freed by this call. */
int tw_moe_ffn_bf16_noalloc(const void* x, int64_t T, int H, int I, const void* w1,
                            const void* w2, int64_t num_slots, const float* topk_weights,
                            const int32_t* topk_ids, int K, void* out, void* stream);

/* Dense SwiGLU FFN of one expert over every row (a shared expert):
 * out[t] = bf16(bf16(bf16(silu(c1_g)*c1_u) . w2^T)), c1 = bf16(x[t] . w1^T), w1 [2I,H] (gate
 * rows first), w2 [H,I]; bit-identical to tw_moe_ffn_bf16 with one slot, K = 1 and every
 * weight 1, without its grouping, gather and combine.  Workspace: tw_moe_workspace_bytes(T,
 * H, I).  H % 128 == 0, I % 64 == 0, T <= 65535; out may alias x.  Replaces the shared
 * expert's GatedMLP forward (layer.shared_forward, gate_up_proj then down_proj) of
 * src/tideway/overlap_shared_expert.py:114-115,253. */
int tw_ffn_dense_bf16(const void* x, int64_t T, int H, int I, const void* w1, const void* w2,
                      void* out, void* workspace, size_t workspace_bytes, void* stream);

/* tw_moe_ffn_bf16 followed by the next residual add and RMSNorm, with the combine fused
 * into that norm: y = the routes' combined output (as tw_moe_ffn_bf16 would write it),
 * residual_out = bf16(y + residual), h_out = RMSNorm(residual_out) * norm_w (eps) --
 * bit-identical to tw_moe_ffn_bf16 then tw_rmsnorm(y, residual, residual_out, norm_w, eps, 0,
 * h_out), one launch shorter.  residual_out may alias residual, h_out may alias x; K <= 64.
 * Replaces the combine (moe_sum_reduce, backends/.../moe/fused.py:360-363) and the decoder's
 * residual RMSNorm that follows it (the FlashInfer RMSNorm of
 * src/tideway/cute_router_norm_pair.py:252-306 on the residual sum). */
int tw_moe_ffn_bf16_residual_norm(const void* x, int64_t T, int H, int I, const void* w1,
                                  const void* w2, int64_t num_slots,
                                  const float* topk_weights, const int32_t* topk_ids, int K,
                                  const void* residual, void* residual_out, const void* norm_w,
                                  float eps, void* h_out, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* tw_moe_ffn_bf16 followed by tw_dual_norm_merge(shared, routed, residual, ...), the
 * combine fused into the merge: out = bf16(bf16(residual + N3(bf16(N1(shared) +
 * N2(routed)))) * scalar) with routed the routes' combined output -- bit-identical to the
 * two calls, one launch and one [T, H] round trip fewer.  out may alias residual; K <= 64.  Replaces
 * the routed FFN's combine (backends/.../moe/fused.py:360-363) and the Gemma merge of
 * src/tideway/overlap_shared_expert.py:253-276. */
int tw_moe_ffn_bf16_dual_merge(const void* x, int64_t T, int H, int I, const void* w1,
                               const void* w2, int64_t num_slots, const float* topk_weights,
                               const int32_t* topk_ids, int K, const void* shared,
                               const void* residual, const void* w1n, const void* w2n,
                               const void* w3n, float eps1, float eps2, float eps3,
                               float scalar, void* out, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Size in bytes of the static scratch behind tw_moe_ffn_bf16_noalloc. */
size_t tw_moe_ffn_noalloc_scratch_bytes(void);

/* Enqueue on `stream` a 4-byte copy of the error word that the last tw_moe_ffn_bf16_noalloc
 * call of n_routes = T*K routes at (H, I) left in the static scratch, into err_out (device
 * memory or page-locked host memory): 0 = ok, 1 = a bounded wait inside the FFN kernel gave
 * up (its output is then not valid although the call returned 0).  Allocates nothing.  The
 * allocation-free path's counterpart of reading tw_moe_workspace_error_offset in a caller
 * workspace; no reference counterpart. */
int tw_moe_ffn_noalloc_error(int64_t n_routes, int H, int I, int32_t* err_out, void* stream);

/* The same over an NVFP4 slot bank: w1 packed uint8 [S,2I,H/2], w1 scale e4m3
 * [S,2I,H/16], w1 global [S,2I]; w2 packed [S,H,I/2], scale [S,H,I/16], global [S,H].
 * The per-output-row globals are fp32 or fp16 (global_dtype TW_F32 / TW_F16); the reference's
 * ModelOpt rows carry fp16 globals with distinct values for the gate (w1) and up (w3) rows
 * (backends/.../moe/offload_cache.py:44-54).  Weights are dequantised in-kernel:
 * f16(e2m1) * f16(e4m3) is exact, the tensor cores multiply it with f16 activations in fp32
 * and the row global (exact in fp32) scales the result, i.e. dequant-then-matmul up to
 * summation order.  Activations are taken as f16
 * (bf16 values beyond +-65504 saturate).  H and I multiples of 256 run on tcgen05 (scale
 * banks 16-byte aligned); other multiples of 64 on the CUDA cores.  Replaces the nvfp4
 * branch of _expert_gemm, backends/freetoken_tideway/freetoken/layers/moe.py:499-538. */
int tw_moe_ffn_nvfp4(const void* x, int64_t T, int H, int I,
                     const void* w1_packed, const void* w1_scale, const void* w1_global,
                     const void* w2_packed, const void* w2_scale, const void* w2_global,
                     int global_dtype, int64_t num_slots, const float* topk_weights, const int32_t* topk_ids,
                     int K, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* tw_moe_ffn_bf16 / tw_moe_ffn_nvfp4 with the reference's other epilogue forms: `activation`
 * (TW_ACT_SILU, TW_ACT_GELU, TW_ACT_GELU_TANH) is applied to the gate half, c2 = bf16(act(c1
 * gate) * c1 up); with weight_on_input = 1 the route weight multiplies the up projection's
 * fp32 accumulators before their bf16 rounding, c1 = bf16(w * x . w1^T), and the down
 * projection's output is not weighted.  Replaces the activation / apply_router_weight_on_input
 * arguments of fused_experts_impl and fused_experts_decode_impl
 * (backends/freetoken_tideway/freetoken/moe/fused.py:261-364, :367-450: FN_MAP at :343, :428;
 * the first GEMM's weight flag at :410-420) and the nvfp4 branch's same arguments
 * (backends/freetoken_tideway/freetoken/layers/moe.py:499-538).  Other arguments, limits and
 * errors as the two entries above; activation outside 0..2 -> TW_ERR_INVALID. */
int tw_moe_ffn_bf16_act(const void* x, int64_t T, int H, int I, const void* w1, const void* w2,
                        int64_t num_slots, const float* topk_weights, const int32_t* topk_ids,
                        int K, int activation, int weight_on_input, void* out, void* workspace,
                        size_t workspace_bytes, void* stream);
int tw_moe_ffn_nvfp4_act(const void* x, int64_t T, int H, int I,
                         const void* w1_packed, const void* w1_scale, const void* w1_global,
                         const void* w2_packed, const void* w2_scale, const void* w2_global,
                         int global_dtype, int64_t num_slots, const float* topk_weights,
                         const int32_t* topk_ids, int K, int activation, int weight_on_input,
                         void* out, void* workspace, size_t workspace_bytes, void* stream);

/* The same epilogue forms for the shared expert's dense FFN and for the routed FFN fused
 * into the Gemma merge: tw_ffn_dense_bf16 / tw_moe_ffn_bf16_dual_merge with `activation`
 * (TW_ACT_*) on the gate half (Gemma 4 checkpoints gate with GELU-tanh), and for the merge
 * entry weight_on_input as in tw_moe_ffn_bf16_act (the dense FFN's weights are all 1).
 * Other arguments, limits and errors as those entries; activation outside 0..2 ->
 * TW_ERR_INVALID. */
int tw_ffn_dense_bf16_act(const void* x, int64_t T, int H, int I, const void* w1,
                          const void* w2, int activation, void* out, void* workspace,
                          size_t workspace_bytes, void* stream);
int tw_moe_ffn_bf16_dual_merge_act(const void* x, int64_t T, int H, int I, const void* w1,
                                   const void* w2, int64_t num_slots,
                                   const float* topk_weights, const int32_t* topk_ids, int K,
                                   const void* shared, const void* residual, const void* w1n,
                                   const void* w2n, const void* w3n, float eps1, float eps2,
                                   float eps3, float scalar, int activation,
                                   int weight_on_input, void* out, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Dequantise NVFP4 rows (packed [rows, K/2], e4m3 scale [rows, K/16], global [rows] fp32 or
 * fp16 as global_dtype says)
 * to fp32 [rows, K] with the FFN kernel's decoder: the dequant half of the reference's
 * dequant-then-matmul nvfp4 path (backends/freetoken_tideway/freetoken/layers/moe.py:499-538).
 * K % 32 == 0. */
int tw_nvfp4_dequantize(const void* packed, const void* scale, const void* global_scale,
                        int global_dtype, int64_t rows, int K, float* out, void* stream);

/* Stable by-expert permutation of T*K routes padded per expert to block_size, sentinel
 * numel; sorted_ids [max_padded], expert_ids [max_padded/block_size], num_post_pad [1].
 * Replaces moe_align_block_size, backends/.../moe/fused.py:88-158. */
int tw_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int num_experts,
                            int block_size, int32_t* sorted_ids, int32_t* expert_ids,
                            int32_t* num_tokens_post_pad, int64_t max_padded, void* stream);

/* The LRU ensure of tw_lru_ensure (ids [T*K] rewritten in place to slots, misses staged for
 * tw_copy_rows) followed, in the same launch, by the expert FFN's grouping of those routes
 * by slot into `workspace` (the layout of tw_moe_workspace_bytes(T*K, H, I)); the FFN then
 * runs with tw_moe_ffn_bf16_residual_norm_grouped / tw_moe_ffn_nvfp4_grouped (nvfp4 = 1),
 * which skip their own grouping launch -- same results as tw_lru_ensure followed by the
 * ungrouped entry, one launch fewer per layer.  Decode batches: T*K < 1024.  The grouped
 * FFN calls must take the same T, K, H, I, slot count and workspace.  Replaces
 * ensure_experts (backends/.../moe/offload_kernels.py:19-51) together with the start of the
 * expert FFN (the routes' sort by expert of fused.py:411-446). */
int tw_lru_ensure_group(int32_t* ids, int64_t T, int K, int32_t* slot_for_id,
                        int32_t* id_of_slot, int64_t* usage, int64_t* step, int64_t num_slots,
                        int num_experts, int layer_id, int32_t* evict_slots,
                        int32_t* src_indices, int64_t* num_indices, int64_t* stats,
                        const int32_t* pinned, int H, int I, int nvfp4, void* workspace,
                        size_t workspace_bytes, void* stream);
int tw_moe_ffn_bf16_residual_norm_grouped(const void* x, int64_t T, int H, int I,
                                          const void* w1, const void* w2, int64_t num_slots,
                                          const float* topk_weights, const int32_t* topk_ids,
                                          int K, const void* residual, void* residual_out,
                                          const void* norm_w, float eps, void* h_out,
                                          void* workspace, size_t workspace_bytes,
                                          void* stream);
int tw_moe_ffn_nvfp4_grouped(const void* x, int64_t T, int H, int I,
                             const void* w1_packed, const void* w1_scale, const void* w1_global,
                             const void* w2_packed, const void* w2_scale, const void* w2_global,
                             int global_dtype, int64_t num_slots, const float* topk_weights,
                             const int32_t* topk_ids, int K, void* out, void* workspace,
                             size_t workspace_bytes, void* stream);

/* tw_moe_ffn_bf16 without the combine: the weighted output of every route stays in the
 * workspace (position-ordered rows, c3, and the route -> position map, pos, at the offsets of
 * the workspace layout for T*K routes), for a combine that sends them elsewhere -- the
 * expert-parallel combine below.  No reference counterpart (the reference's MoE path is
 * single-GPU, src/tideway/offload/paged_decode_graph.py:62-63). */
int tw_moe_ffn_bf16_routes(const void* x, int64_t T, int H, int I, const void* w1,
                           const void* w2, int64_t num_slots, const float* topk_weights,
                           const int32_t* topk_ids, int K, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The same over an NVFP4 slot bank (arguments of tw_moe_ffn_nvfp4 without out). */
int tw_moe_ffn_nvfp4_routes(const void* x, int64_t T, int H, int I,
                            const void* w1_packed, const void* w1_scale, const void* w1_global,
                            const void* w2_packed, const void* w2_scale, const void* w2_global,
                            int global_dtype, int64_t num_slots, const float* topk_weights,
                            const int32_t* topk_ids, int K, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- expert parallelism */

/* The reference's MoE path is single-GPU (src/tideway/offload/paged_decode_graph.py:62-63);
 * these three entry points add the expert-parallel sharding the benchmark configuration asks
 * for.  Experts are sharded evenly: GPU d owns experts [d*Eg, (d+1)*Eg).  A dispatch row is
 * [H bf16 input | K int32 local expert ids (-1 = route on another GPU) | K fp32 router
 * weights], padded to tw_ep_row_bytes(H, K). */
size_t tw_ep_row_bytes(int H, int K);

/* Write row d*T + t of send_rows ([world*T] rows) for every destination d and token t. */
int tw_ep_dispatch(const void* x, const float* topk_weights, const int32_t* topk_ids,
                   int64_t T, int K, int H, int experts_per_rank, int world, void* send_rows,
                   void* stream);

/* Unpack received rows into the expert-FFN operands x [rows, H] bf16, ids [rows, K] int32
 * (local expert ids, -1 = none) and w [rows, K] fp32. */
int tw_ep_receive(const void* recv_rows, int64_t rows, int K, int H, void* x, int32_t* ids,
                  float* w, void* stream);

/* out[t] = bf16(sum over d of parts[d*T + t]) in GPU order: the per-GPU partial expert
 * outputs returned by the second all-to-all. */
int tw_ep_combine(const void* parts, int64_t T, int H, int world, void* out, void* stream);

/* The same exchange over NVLink peer memory, without NCCL: every GPU of the group holds one
 * zeroed exchange buffer of tw_ep_p2p_bytes(world, T, H, K) bytes in device memory from
 * cudaMalloc (a caching allocator's block is fine), exports it (tw_ep_p2p_export: a CUDA
 * IPC handle of tw_ep_p2p_handle_bytes() bytes for its allocation and the buffer's offset in
 * it), the handles are exchanged over the host (any process-group all-gather) and each GPU
 * maps its peers' (tw_ep_p2p_open, undone by tw_ep_p2p_close on the returned mapping);
 * `peers` then lists the world buffers in rank order (its own at `rank`).
 * tw_ep_p2p_offsets gives the byte offsets of the received operands in a buffer: x [world*T,
 * H] bf16, local ids [world*T, K] int32, weights [world*T, K] fp32, and the returned
 * partials [world*T, H] bf16.
 * tw_ep_p2p_dispatch writes every token's K local ids and weights into each peer's buffer
 * and its input row only where it has a route, raises this GPU's flag on every peer and
 * returns once every peer's rows for this GPU have landed (a bounded wait; see
 * tw_set_wait_limit).  The received rows run through the slot cache (ensure/copy) and
 * tw_moe_ffn_bf16_routes; tw_ep_p2p_combine then sends each received row's partial output
 * back into its source GPU's buffer and, per local token, adds the partials of the GPUs its
 * routes went to in GPU order into y, or with residual/norm_w given applies
 * residual_out = bf16(sum + residual), h_out = RMSNorm(residual_out) * norm_w (eps) -- the
 * arithmetic of tw_ep_combine followed by tw_rmsnorm.  Flags carry a step count, so nothing
 * is cleared between steps and a captured graph replays unchanged; calls on one GPU must
 * follow the order dispatch, routes FFN, combine.  world <= 8, K <= 64, T <= 4096, combine
 * H <= 4096 and world*T <= 4 x SMs.  No reference counterpart (see above). */
size_t tw_ep_p2p_bytes(int world, int64_t T, int H, int K);
int tw_ep_p2p_offsets(int world, int64_t T, int H, int K, size_t* offsets4);
size_t tw_ep_p2p_handle_bytes(void);
int tw_ep_p2p_export(const void* buffer, void* ipc_handle, uint64_t* offset);
int tw_ep_p2p_open(const void* ipc_handle, uint64_t offset, void** peer_buffer, void** mapping);
int tw_ep_p2p_close(void* mapping);
int tw_ep_p2p_dispatch(const void* x, const float* topk_weights, const int32_t* topk_ids,
                       int64_t T, int K, int H, int experts_per_rank, int world, int rank,
                       void* const* peers, void* stream);
int tw_ep_p2p_combine(const void* workspace, int64_t T, int K, int H, int I,
                      int experts_per_rank, const int32_t* topk_ids, int world, int rank,
                      void* const* peers, const void* residual, void* residual_out,
                      const void* norm_w, float eps, void* h_out, void* y, void* stream);
/* The exchange buffer's error word: 0 = ok, 1 = a bounded wait for a peer gave up (copied
 * into err_out, device or page-locked host memory, in stream order). */
int tw_ep_p2p_error(const void* buffer, int32_t* err_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TIDEWAY_B200_H */
