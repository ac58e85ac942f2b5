// Token permutation for the grouped prefill GEMM: a stable by-expert permutation of the
// T*K routes, each expert padded to a multiple of block_size with the sentinel numel.
// Same contract as moe_align_block_size (backends/freetoken_tideway/freetoken/moe/
// fused.py:88-158): experts without routes get no block; unused tail entries keep the
// sentinel; unused tail blocks get expert -1.
//
// One CTA of 32 warps.  Warp w owns a contiguous range of routes; per-warp per-expert
// counts give every warp its starting offset inside each expert's segment, then each
// warp places its routes in order with __match_any_sync, so the result is stable.
#include "common.cuh"

namespace tw {
namespace {

constexpr int kAlignWarps = 32;
constexpr int kAlignThreads = kAlignWarps * 32;
constexpr int kAlignMaxE = 1024;

__global__ void __launch_bounds__(kAlignThreads)
moe_align_kernel(const int32_t* __restrict__ ids, int numel, int E, int bs,
                 int32_t* __restrict__ sorted_ids, int32_t* __restrict__ expert_ids,
                 int32_t* __restrict__ npad_out, int max_padded) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int wcnt[];  // [kAlignWarps][E]: counts, then per-warp cursors
  __shared__ int eoff[kAlignMaxE + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kAlignWarps * E; i += kAlignThreads) wcnt[i] = 0;
  for (int i = tid; i < max_padded; i += kAlignThreads) sorted_ids[i] = numel;
  const int max_blocks = max_padded / bs;
  for (int i = tid; i < max_blocks; i += kAlignThreads) expert_ids[i] = -1;
  __syncthreads();
  const int per = (numel + kAlignWarps - 1) / kAlignWarps;
  const int r0 = warp * per, r1 = min(numel, r0 + per);
  for (int r = r0 + lane; r < r1; r += 32) {
    const int e = ids[r];
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + e], 1);
  }
  __syncthreads();
  // per expert: exclusive scan over warps -> warp cursors; padded segment sizes
  for (int e = tid; e < E; e += kAlignThreads) {
    int run = 0;
    for (int w = 0; w < kAlignWarps; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += c;
    }
    eoff[e] = ((run + bs - 1) / bs) * bs;  // padded size for now
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      const int sz = eoff[e];
      eoff[e] = acc;
      acc += sz;
    }
    eoff[E] = acc;
    npad_out[0] = acc;
  }
  __syncthreads();
  for (int e = tid; e < E; e += kAlignThreads) {
    for (int b = eoff[e] / bs; b < eoff[e + 1] / bs; ++b) expert_ids[b] = e;
  }
  // stable placement within each warp's range
  for (int base = r0; base < r1; base += 32) {
    const int r = base + lane;
    const int e = r < r1 ? ids[r] : -1;
    const bool ok = r < r1 && e >= 0 && e < E;
    const int key = ok ? e : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(peers) - 1;
    int start = 0;
    if (ok && lane == leader) {
      start = wcnt[warp * E + e];
      wcnt[warp * E + e] = start + __popc(peers);
    }
    start = __shfl_sync(0xffffffffu, start, leader);
    if (ok) sorted_ids[eoff[e] + start + __popc(peers & ((1u << lane) - 1))] = r;
    __syncwarp();
  }
}

}  // namespace
}  // namespace tw

using namespace tw;

extern "C" int tw_moe_align_block_size(const int32_t* ids, int64_t numel, int E, int bs,
                                       int32_t* sorted_ids, int32_t* expert_ids,
                                       int32_t* npad, int64_t max_padded, void* stream) {
  TW_CHECK_ARG(E > 0 && E <= kAlignMaxE, "moe_align: need 0 < num_experts <= %d", kAlignMaxE);
  TW_CHECK_ARG(bs > 0 && numel >= 0 && numel < (1 << 24), "moe_align: bad block_size/numel");
  const int64_t need = numel + (int64_t)E * (bs - 1);
  TW_CHECK_ARG(max_padded >= need || max_padded >= numel * bs,
               "moe_align: max_padded %lld too small (need %lld)", (long long)max_padded,
               (long long)need);
  const size_t smem = sizeof(int) * (size_t)kAlignWarps * E;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(moe_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  TW_LAUNCH(moe_align_kernel, dim3(1), dim3(kAlignThreads), smem, as_stream(stream), 
      ids, (int)numel, E, bs, sorted_ids, expert_ids, npad, (int)max_padded);
  TW_CHECK_LAUNCH("moe_align_kernel");
  return TW_OK;
}
