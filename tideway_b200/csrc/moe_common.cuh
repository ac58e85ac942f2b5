// Workspace shared by the expert-FFN kernels (route grouping, up/down GEMMs, combine).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace tw {

// Per-output-row global scale of an NVFP4 bank, fp32 or fp16 (the reference's ModelOpt rows
// carry fp16 globals, distinct for the gate and up rows).
struct RowScale {
  const void* p = nullptr;
  int f16 = 0;
  __device__ __forceinline__ float at(int64_t i) const {
    return f16 ? __half2float(static_cast<const __half*>(p)[i]) : static_cast<const float*>(p)[i];
  }
};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Routes are grouped by slot into positions p = 0..n_used-1; every per-route buffer is
// indexed by position.
struct Workspace {
  int32_t* num_unique;  // [1]      distinct slots routed
  int32_t* seg_start;   // [n + 1]  first position of each distinct slot's routes
  int32_t* seg_slot;    // [n]      slot id of each segment
  int32_t* perm;        // [n]      position -> route (t * K + k)
  int32_t* pos;         // [n]      route -> position (-1 when the route is skipped)
  int* err;             // [1]      error word of the tensor-core kernels (0 = ok)
  int* up_ctr;          // [1]      next unclaimed up tile of the FFN kernel
  int* down_ctr;        // [1]      next unclaimed down tile of the FFN kernel
  int* up_done;         // [n * 32] per-segment finished up-tile arrivals (128-byte stride)
  int* ready_tail;      // [1]      slots whose activations are complete
  uint16_t* woff;       // [ceil(n/128) * 1024] two-kernel grouping: slice offsets per slot
  int* ready_slots;     // [n]      those slots, in completion order (-1 = not yet)
  __nv_bfloat16* xg;    // [n, H]   gathered input rows, position order
  __nv_bfloat16* act;   // [n, I]   SwiGLU activations, position order
  __nv_bfloat16* c3;    // [n, H]   weighted expert outputs, position order
};

inline size_t workspace_layout(int64_t n, int H, int I, char* base, Workspace* ws) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  char* a = take(sizeof(int32_t));
  char* b = take(sizeof(int32_t) * (n + 1));
  char* c = take(sizeof(int32_t) * n);
  char* d = take(sizeof(int32_t) * n);
  char* e = take(sizeof(int32_t) * n);
  char* f = take(sizeof(int));
  char* f2 = take(sizeof(int) * 4);
  char* f4 = take(sizeof(int) * n);
  char* f3 = take(sizeof(int) * 32 * n);
  char* f5 = take(sizeof(uint16_t) * (size_t)((n + 127) / 128) * 1024);
  char* g = take(sizeof(__nv_bfloat16) * (size_t)n * H);
  char* h = take(sizeof(__nv_bfloat16) * (size_t)n * I);
  char* i = take(sizeof(__nv_bfloat16) * (size_t)n * H);
  if (ws) {
    ws->num_unique = reinterpret_cast<int32_t*>(a);
    ws->seg_start = reinterpret_cast<int32_t*>(b);
    ws->seg_slot = reinterpret_cast<int32_t*>(c);
    ws->perm = reinterpret_cast<int32_t*>(d);
    ws->pos = reinterpret_cast<int32_t*>(e);
    ws->err = reinterpret_cast<int*>(f);
    ws->up_ctr = reinterpret_cast<int*>(f2);
    ws->down_ctr = reinterpret_cast<int*>(f2) + 1;
    ws->ready_tail = reinterpret_cast<int*>(f2) + 2;
    ws->ready_slots = reinterpret_cast<int*>(f4);
    ws->up_done = reinterpret_cast<int*>(f3);
    ws->woff = reinterpret_cast<uint16_t*>(f5);
    ws->xg = reinterpret_cast<__nv_bfloat16*>(g);
    ws->act = reinterpret_cast<__nv_bfloat16*>(h);
    ws->c3 = reinterpret_cast<__nv_bfloat16*>(i);
  }
  return off;
}

// The expert FFN's epilogue variant: the gate activation (0 SiLU, 1 GELU, 2 GELU tanh form)
// and where the route weight multiplies -- the down projection's output (w_in 0) or the up
// projection's fp32 accumulators before their bf16 rounding (w_in 1, the reference's
// apply_router_weight_on_input).
struct FfnAct {
  int act = 0;
  int w_in = 0;
};

// Tensor-core expert GEMMs over grouped routes (expert_gemm_tc.cu).  w1: [S, 2I, H] bf16,
// w2: [S, H, I] bf16.  Enqueues gather -> up (SwiGLU) -> down (x route weight).
int launch_expert_ffn_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                         const __nv_bfloat16* w1, const __nv_bfloat16* w2, int64_t S,
                         const float* topk_w, const Workspace& ws, int64_t n,
                         cudaStream_t st, FfnAct fx = FfnAct{});

// The combine fused with the next residual add and RMSNorm (norm.cu): per token
// y = bf16(sum_k c3[pos[t, k]]) (k order), resid_out = bf16(y + resid), h = RMSNorm(resid_out)
// * w -- bit-identical to combine_kernel followed by the residual RMSNorm.
struct CombineNorm {
  const void* resid;
  void* resid_out;  // may alias resid
  const void* w;
  float eps;
  void* h;
};
int launch_combine_norm(const Workspace& ws, int64_t T, int K, int H, const CombineNorm& cn,
                        cudaStream_t st);

// The combine fused into the Gemma post-FFN merge (norm.cu): per token
// out = bf16(bf16(x + N3(bf16(N1(a) + N2(b)))) * scalar) with b = the routes' combine --
// bit-identical to combine_kernel followed by the dual-norm merge.
struct CombineMerge {
  const void* a;  // shared expert output [T, H]
  const void* x;  // residual [T, H]
  const void* w1;
  const void* w2;
  const void* w3;
  float eps1, eps2, eps3, scalar;
  void* out;      // may alias x
};
int launch_combine_merge(const Workspace& ws, int64_t T, int K, int H, const CombineMerge& cm,
                         cudaStream_t st);

// Dense SwiGLU FFN of one expert (w1 [2I, H], w2 [H, I]) over all T rows of x into out
// (a shared expert): no grouping, gather or combine; bit-identical to the routed path with
// every row routed to that expert at weight 1.
int launch_expert_ffn_dense_tc(const __nv_bfloat16* x, int64_t T, int H, int I,
                               const __nv_bfloat16* w1, const __nv_bfloat16* w2,
                               const Workspace& ws, __nv_bfloat16* out, cudaStream_t st,
                               FfnAct fx = FfnAct{});

// NVFP4 weights (expert_gemm_fp4_tc.cu): packed e2m1 [S, rows, K/2], e4m3 scales
// [S, rows, K/16], fp32 or fp16 row globals [S, rows]; needs H % 256 == 0 and I % 256 == 0.
int launch_expert_ffn_fp4_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                             const uint8_t* w1p, const uint8_t* w1s, RowScale w1g,
                             const uint8_t* w2p, const uint8_t* w2s, RowScale w2g,
                             int64_t S, const float* topk_w, const Workspace& ws, int64_t n,
                             cudaStream_t st, FfnAct fx = FfnAct{});

// Routes per MMA chunk of the tensor-core FFN kernels for a launch of T tokens, n routes
// and S slots; the grouping kernel splits larger slots into segments of this many routes.
int expert_ffn_tc_route_cap(int64_t T, int64_t n, int64_t S);
int expert_ffn_fp4_tc_route_cap(int64_t T);

int num_sms();

// Polls before a bounded wait of the tensor-core FFN kernels gives up (tw_set_wait_limit;
// read at each launch).
uint32_t ffn_wait_limit();

}  // namespace tw
