// Slot-indirect SwiGLU expert FFN with weighted combine: the host entry points, route
// grouping, the combine and the CUDA-core fallback kernels.
//
// Pipeline (all graph-safe, counts stay on the device):
//   1. route grouping -- a stable counting sort of the T*K routes by slot id, so every
//      distinct slot's weights are streamed from HBM once for all its routes (the reference
//      streams them once per route, backends/.../moe/fused.py:411-446); slots with more
//      routes than one MMA route tile become several segments.  Decode sizes: one CTA
//      (group_routes_kernel); >= 1024 routes over <= 1024 slots: group_count_kernel (one
//      CTA) + group_place_kernel (one warp per 128-route slice).
//   2. the expert GEMMs -- tensor cores (expert_gemm_tc.cu, expert_gemm_fp4_tc.cu):
//      c1 = bf16(x . w1^T), act = bf16(silu(c1_gate) * c1_up), c3 = bf16((act . w2^T) *
//      route weight), per route.  NVFP4 shapes that are not multiples of 256 run the
//      CUDA-core ffn_up_kernel / ffn_down_kernel below instead.
//   3. combine_kernel -- out[t] = bf16(sum_k c3[t,k]) in k order (moe_sum_reduce), or the
//      combine fused into the next residual RMSNorm or the Gemma merge (norm.cu).
//
// Weights are BF16 or NVFP4 (e2m1 codes, e4m3 scale per 16, fp32 or fp16 global per row); NVFP4
// is dequantised exactly (f16 code x f16 scale) before the fp32-accumulating multiply, so
// it matches dequant-then-matmul up to the order of the fp32 sums.
#include <cuda_fp8.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "moe_common.cuh"
#include "moe_group.cuh"

namespace tw {
namespace {

constexpr int kMaxRoutes = 65535;
constexpr int kMaxGroupSlots = 32768;
constexpr int kFfnThreads = 256;
constexpr int kFfnWarps = kFfnThreads / 32;
constexpr int kUpPairsPerCta = kFfnWarps;       // one gate/up row pair per warp
constexpr int kDownRowsPerWarp = 2;
constexpr int kDownRowsPerCta = kFfnWarps * kDownRowsPerWarp;
constexpr int kRouteTile = 8;                    // routes accumulated per weight pass
constexpr int kSegElems = 2048;                  // row elements per lane-segment pass (64/lane)

// ---------------------------------------------------------------- 1. grouping

__global__ void __launch_bounds__(kGroupThreads, 1)
group_routes_kernel(const int32_t* __restrict__ ids, int n, int S, int per_warp, int split,
                    Workspace ws) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int cnt[];
  group_routes<true>(ids, n, S, per_warp, split, ws, cnt);
}

// Two-kernel grouping for many routes over at most 1024 slots (prefill).  The routes are cut
// into slices of kSliceRoutes in route order.  group_count_kernel (one CTA) counts every
// slice per slot with shared-memory atomics, takes per slot the exclusive prefix over the
// slices (route order), runs the slot scan above and writes each slice's first position per
// slot; group_place_kernel (one warp per slice, many CTAs) then places its slice's routes in
// order.  Same (stable) result as group_routes_kernel; the counting no longer runs on one SM
// 32 routes at a time.
constexpr int kSliceRoutes = 128;
constexpr int kPlaceWarps = 8;
constexpr int kTwoPassHistInts = 48 * 1024;  // [slices][S] int counts in shared memory

__global__ void __launch_bounds__(kGroupThreads, 1)
group_count_kernel(const int32_t* __restrict__ ids, int n, int S, int split, Workspace ws) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sm[];
  int* cnt = sm;       // [S]: counts, then the slots' first positions
  int* hist = sm + S;  // [slices][S]: counts, then the slice's offset within the slot
  __shared__ unsigned warp_tot[32];
  __shared__ unsigned s_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nsl = (n + kSliceRoutes - 1) / kSliceRoutes;
  if (tid == 0) {
    ws.err[0] = 0;
    ws.up_ctr[0] = 0;
    ws.down_ctr[0] = 0;
    ws.ready_tail[0] = 0;
  }
  for (int i = tid; i < nsl * S; i += kGroupThreads) hist[i] = 0;
  __syncthreads();
  // warp w counts slices w, w + 32, ...: all of a slice's ids in flight, then the atomics
  for (int sl = warp; sl < nsl; sl += kGroupThreads / 32) {
    int v[kSliceRoutes / 32];
#pragma unroll
    for (int j = 0; j < kSliceRoutes / 32; ++j) {
      const int r = sl * kSliceRoutes + 32 * j + lane;
      v[j] = r < n ? ids[r] : -1;
    }
#pragma unroll
    for (int j = 0; j < kSliceRoutes / 32; ++j)
      if (v[j] >= 0 && v[j] < S) atomicAdd(&hist[sl * S + v[j]], 1);
  }
  __syncthreads();
  for (int s = tid; s < S; s += kGroupThreads) {
    int run = 0;
    for (int sl = 0; sl < nsl; ++sl) {
      const int c = hist[sl * S + s];
      hist[sl * S + s] = run;
      run += c;
    }
    cnt[s] = run;
  }
  __syncthreads();
  scan_slots(cnt, S, split, ws, warp_tot, &s_total);
  for (int i = tid; i < nsl * S; i += kGroupThreads) {
    const int s = i % S;
    ws.woff[i] = (uint16_t)(cnt[s] + hist[i]);
  }
}

__global__ void __launch_bounds__(32 * kPlaceWarps)
group_place_kernel(const int32_t* __restrict__ ids, int n, int S, Workspace ws) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint16_t cur[];  // [kPlaceWarps][S]: next position of each slot
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nsl = (n + kSliceRoutes - 1) / kSliceRoutes;
  const int sl = blockIdx.x * kPlaceWarps + warp;
  if (sl >= nsl) return;  // whole warps only; no block-wide barrier follows
  uint16_t* c = cur + warp * S;
  for (int s = lane; s < S; s += 32) c[s] = ws.woff[sl * S + s];
  __syncwarp();
  const int kbits = 32 - __clz(S);  // keys 0..S (S marks a skipped route)
  int v[kSliceRoutes / 32];
#pragma unroll
  for (int j = 0; j < kSliceRoutes / 32; ++j) {
    const int r = sl * kSliceRoutes + 32 * j + lane;
    v[j] = r < n ? ids[r] : -1;
  }
#pragma unroll
  for (int j = 0; j < kSliceRoutes / 32; ++j) {
    const int r = sl * kSliceRoutes + 32 * j + lane;
    const int s = v[j];
    const bool ok = r < n && s >= 0 && s < S;
    const unsigned peers = match_by_ballots(ok ? s : S, kbits);
    const int leader = __ffs(peers) - 1;
    int start = 0;
    if (ok && lane == leader) {
      start = c[s];
      c[s] = (uint16_t)(start + __popc(peers));
    }
    start = __shfl_sync(0xffffffffu, start, leader);
    if (ok) {
      const int p = start + __popc(peers & ((1u << lane) - 1));
      ws.perm[p] = r;
      ws.pos[r] = p;
    } else if (r < n) {
      ws.pos[r] = -1;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- weight row access

// A weight row segment as seen by one lane: 64 consecutive elements starting at
// element (seg * kSegElems + lane * 64).
struct Bf16Rows {
  const __nv_bfloat16* w;  // [S, rows, K]
  int64_t rows, K;
};

struct Fp4Rows {
  const uint8_t* packed;  // [S, rows, K/2]
  const uint8_t* scale;   // [S, rows, K/16] e4m3
  RowScale global_;       // [S, rows] fp32 or fp16
  int64_t rows, K;
};

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __nv_fp8_e4m3 v;
  v.__x = b;
  return float(v);
}

// One lane's 64-element segment of an NVFP4 weight row (elements seg*kSegElems + lane*64
// ...), kept packed in registers and decoded on the fly by dot().  (BF16 weights always run
// on the tensor cores, so only the NVFP4 CUDA-core kernels use it.)
template <bool FP4>
struct Seg;

template <>
struct Seg<true> {
  uint4 v[2];
  float s[4];  // e4m3 block scale * fp32 row global, per 16-element block
  __device__ __forceinline__ void load(const Fp4Rows& R, int64_t slot, int64_t row, int seg,
                                       int lane) {
    const int64_t e0 = (int64_t)seg * kSegElems + lane * 64;
    const int64_t r = slot * R.rows + row;
    uint32_t sc = 0;
    float g = 0.f;
    v[0] = v[1] = make_uint4(0, 0, 0, 0);
    if (e0 < R.K) {
      const uint8_t* p = R.packed + r * (R.K / 2) + e0 / 2;
      v[0] = ld_stream16(p);
      if (e0 + 32 < R.K) v[1] = ld_stream16(p + 16);
      const uint8_t* sp = R.scale + r * (R.K / 16) + e0 / 16;
      sc = (e0 + 32 < R.K) ? *reinterpret_cast<const uint32_t*>(sp)
                           : (uint32_t)*reinterpret_cast<const uint16_t*>(sp);
      g = R.global_.at(r);
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) s[b] = e4m3_to_f32((sc >> (8 * b)) & 0xff) * g;
  }
  __device__ __forceinline__ float dot(const __nv_bfloat16* arow, int64_t K, int seg, int lane,
                                       const float2* lut) const {
    const int64_t e0 = (int64_t)seg * kSegElems + lane * 64;
    const uint32_t words[8] = {v[0].x, v[0].y, v[0].z, v[0].w, v[1].x, v[1].y, v[1].z, v[1].w};
    float acc = 0.f;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      if (e0 + blk * 16 < K) {
        float part = 0.f;
#pragma unroll
        for (int wq = 0; wq < 2; ++wq) {
          float a[8];
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(arow + e0 + blk * 16 + wq * 8)), a);
          const uint32_t w = words[blk * 2 + wq];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const float2 pr = lut[(w >> (8 * b)) & 0xff];
            part = fmaf(a[2 * b], pr.x, part);
            part = fmaf(a[2 * b + 1], pr.y, part);
          }
        }
        acc = fmaf(part, s[blk], acc);
      }
    }
    return acc;
  }
};

template <bool FP4>
using RowsOf = typename std::conditional<FP4, Fp4Rows, Bf16Rows>::type;

__device__ __forceinline__ void init_lut(float2* lut) {
  // byte -> (low nibble value, high nibble value); e2m1 magnitudes {0,.5,1,1.5,2,3,4,6}
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    const int lo = b & 15, hi = b >> 4;
    const float vl = (lo & 8) ? -mag[lo & 7] : mag[lo & 7];
    const float vh = (hi & 8) ? -mag[hi & 7] : mag[hi & 7];
    lut[b] = make_float2(vl, vh);
  }
}

// ---------------------------------------------------------------- 2. up projection

template <bool FP4>
__global__ void __launch_bounds__(kFfnThreads, 2)
ffn_up_kernel(const __nv_bfloat16* __restrict__ x, int H, int I, int K, RowsOf<FP4> W1,
              Workspace ws, const float* __restrict__ topk_w, FfnAct fx) {
  pdl_wait();
  pdl_trigger();
  __shared__ float2 lut[256];
  if (FP4) {
    init_lut(lut);
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (I + kUpPairsPerCta - 1) / kUpPairsPerCta;
  const int U = ws.num_unique[0];
  const int nseg = (H + kSegElems - 1) / kSegElems;
  for (int item = blockIdx.x; item < U * chunks; item += gridDim.x) {
    const int u = item / chunks;
    const int j = (item % chunks) * kUpPairsPerCta + warp;
    if (j >= I) continue;
    const int64_t slot = ws.seg_slot[u];
    const int p0 = ws.seg_start[u], p1 = ws.seg_start[u + 1];
    for (int pb = p0; pb < p1; pb += kRouteTile) {
      const int nr = min(kRouteTile, p1 - pb);
      float ag[kRouteTile], au[kRouteTile];
#pragma unroll
      for (int q = 0; q < kRouteTile; ++q) ag[q] = au[q] = 0.f;
      for (int seg = 0; seg < nseg; ++seg) {
        Seg<FP4> wg, wu;
        wg.load(W1, slot, j, seg, lane);
        wu.load(W1, slot, I + j, seg, lane);
#pragma unroll
        for (int q = 0; q < kRouteTile; ++q) {
          if (q < nr) {
            const int r = ws.perm[pb + q];
            const __nv_bfloat16* xr = x + (int64_t)(r / K) * H;
            ag[q] += wg.dot(xr, H, seg, lane, lut);
            au[q] += wu.dot(xr, H, seg, lane, lut);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kRouteTile; ++q) {
        if (q < nr) {
          // with w_in the route's weight multiplies both fp32 sums before their rounding
          const float wr = fx.w_in ? topk_w[ws.perm[pb + q]] : 1.0f;
          const float g = bf16_round(warp_sum(ag[q]) * wr);
          const float uu = bf16_round(warp_sum(au[q]) * wr);
          const float act = fx.act == 0 ? silu_f(g) : gelu_act(fx.act, g);
          if (lane == 0) ws.act[(int64_t)(pb + q) * I + j] = __float2bfloat16_rn(act * uu);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- 3. down projection

template <bool FP4>
__global__ void __launch_bounds__(kFfnThreads, 2)
ffn_down_kernel(int H, int I, const float* __restrict__ topk_w, RowsOf<FP4> W2, Workspace ws,
                FfnAct fx) {
  pdl_wait();
  pdl_trigger();
  __shared__ float2 lut[256];
  if (FP4) {
    init_lut(lut);
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (H + kDownRowsPerCta - 1) / kDownRowsPerCta;
  const int U = ws.num_unique[0];
  const int nseg = (I + kSegElems - 1) / kSegElems;
  for (int item = blockIdx.x; item < U * chunks; item += gridDim.x) {
    const int u = item / chunks;
    const int h0 = (item % chunks) * kDownRowsPerCta + warp * kDownRowsPerWarp;
    if (h0 >= H) continue;
    const int64_t slot = ws.seg_slot[u];
    const int p0 = ws.seg_start[u], p1 = ws.seg_start[u + 1];
    for (int pb = p0; pb < p1; pb += kRouteTile) {
      const int nr = min(kRouteTile, p1 - pb);
      float acc[kDownRowsPerWarp][kRouteTile];
#pragma unroll
      for (int rr = 0; rr < kDownRowsPerWarp; ++rr)
#pragma unroll
        for (int q = 0; q < kRouteTile; ++q) acc[rr][q] = 0.f;
      for (int seg = 0; seg < nseg; ++seg) {
#pragma unroll
        for (int rr = 0; rr < kDownRowsPerWarp; ++rr) {
          if (h0 + rr < H) {
            Seg<FP4> wv;
            wv.load(W2, slot, h0 + rr, seg, lane);
#pragma unroll
            for (int q = 0; q < kRouteTile; ++q)
              if (q < nr) acc[rr][q] += wv.dot(ws.act + (int64_t)(pb + q) * I, I, seg, lane, lut);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kRouteTile; ++q) {
        if (q < nr) {
          const int r = ws.perm[pb + q];
          const float w = fx.w_in ? 1.0f : topk_w[r];
#pragma unroll
          for (int rr = 0; rr < kDownRowsPerWarp; ++rr) {
            if (h0 + rr < H) {
              const float v = warp_sum(acc[rr][q]);
              if (lane == 0)
                ws.c3[(int64_t)(pb + q) * H + h0 + rr] = __float2bfloat16_rn(v * w);
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- 4. combine

// out[t] = bf16(sum_k c3[pos[t,k]]) with the sum in k order.  Routes are taken eight at a
// time: their positions, then their rows, are loaded together (two round trips per eight
// routes instead of two per route).
constexpr int kCombineThreads = 64;

__global__ void __launch_bounds__(kCombineThreads)
combine_kernel(int H, int K, Workspace ws, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= H) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 8) {
    int p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = k0 + j < K ? ws.pos[t * K + k0 + j] : -1;
    uint4 r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      r[j] = p[j] >= 0 ? *reinterpret_cast<const uint4*>(ws.c3 + (int64_t)p[j] * H + v * 8)
                       : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (p[j] < 0) continue;
      float c[8];
      bf16x8_to_f32(r[j], c);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += c[i];
    }
  }
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    ow[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i])) |
            ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i + 1])) << 16);
  *reinterpret_cast<uint4*>(out + t * H + v * 8) = o;
}

// With cn == cm == nullptr the routes' outputs are combined into out; otherwise out is unused
// and the combine is fused with the next residual add and RMSNorm (launch_combine_norm) or
// with the Gemma dual-norm merge (launch_combine_merge).
template <bool FP4>
int run_ffn(const void* x, int64_t T, int H, int I, RowsOf<FP4> W1, RowsOf<FP4> W2, int64_t S,
            const float* topk_w, const int32_t* topk_ids, int K, void* out, void* workspace,
            size_t ws_bytes, cudaStream_t st, const CombineNorm* cn = nullptr,
            const CombineMerge* cm = nullptr, bool routes_only = false,
            bool pregrouped = false, FfnAct fx = FfnAct{}) {
  const int64_t n = T * K;
  TW_CHECK_ARG(T >= 0 && K > 0 && n <= kMaxRoutes, "moe_ffn: need T*K <= %d", kMaxRoutes);
  TW_CHECK_ARG(fx.act >= TW_ACT_SILU && fx.act <= TW_ACT_GELU_TANH && (fx.w_in == 0 || fx.w_in == 1),
               "moe_ffn: activation must be silu/gelu/gelu_tanh (0..2), weight_on_input 0 or 1");
  TW_CHECK_ARG(H > 0 && I > 0 && H % 64 == 0 && I % 64 == 0,
               "moe_ffn: H and I must be multiples of 64 (got H=%d I=%d)", H, I);
  TW_CHECK_ARG(S > 0 && S <= kMaxGroupSlots, "moe_ffn: need 0 < num_slots <= %d",
               kMaxGroupSlots);
  TW_CHECK_ARG(aligned16(x) && (cn != nullptr || cm != nullptr || routes_only || aligned16(out)),
               "moe_ffn: x/out must be 16-byte aligned");
  if (n == 0) return TW_OK;
  Workspace ws;
  const size_t need = workspace_layout(n, H, I, static_cast<char*>(workspace), &ws);
  TW_CHECK_ARG(workspace != nullptr && ws_bytes >= need,
               "moe_ffn: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  TW_CHECK_ARG(aligned16(workspace), "moe_ffn: workspace must be 16-byte aligned");
  const bool fp4_tc = FP4 && H % 256 == 0 && I % 256 == 0;
  const int per_warp = (n >= 1024 && S <= 1024) ? 1 : 0;
  const int64_t nsl = (n + kSliceRoutes - 1) / kSliceRoutes;
  const bool two_pass = per_warp && nsl * S <= kTwoPassHistInts;
  const size_t smem = sizeof(int) * (size_t)S + (per_warp ? 32 * sizeof(unsigned short) * S : 0);
  if (!two_pass && smem > 48 * 1024) {
    cudaFuncSetAttribute(group_routes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  }
  // slots with more routes than one MMA chunk of the tensor-core FFN are split into
  // segments of one chunk each (the CUDA-core kernels take whole slots)
  const int cap = !FP4 ? expert_ffn_tc_route_cap(T, n, S)
                  : fp4_tc ? expert_ffn_fp4_tc_route_cap(T) : 0;
  // with distinct ids per token a slot has at most T routes: no split is needed when T fits
  // one chunk (a repeated id then only makes the kernels walk a second chunk)
  const int split = cap > 0 && T > cap ? cap : 0;
  if (pregrouped) {
    // the LRU ensure grouped these routes already (tw_lru_ensure_group, same T, K, H, I, S)
    TW_CHECK_ARG(n < 1024, "moe_ffn: pregrouped calls are decode batches (T*K < 1024)");
  } else if (two_pass) {
    const size_t csmem = sizeof(int) * (size_t)(S + nsl * S);
    if (csmem > 48 * 1024) {
      cudaFuncSetAttribute(group_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)csmem);
    }
    TW_LAUNCH(group_count_kernel, dim3(1), dim3(kGroupThreads), csmem, st, topk_ids, (int)n,
              (int)S, split, ws);
    TW_CHECK_LAUNCH("group_count_kernel");
    TW_LAUNCH(group_place_kernel, dim3((unsigned)((nsl + kPlaceWarps - 1) / kPlaceWarps)),
              dim3(32 * kPlaceWarps), sizeof(uint16_t) * kPlaceWarps * (size_t)S, st, topk_ids,
              (int)n, (int)S, ws);
    TW_CHECK_LAUNCH("group_place_kernel");
  } else {
    TW_LAUNCH(group_routes_kernel, dim3(1), dim3(kGroupThreads), smem, st, topk_ids, (int)n,
              (int)S, per_warp, split, ws);
    TW_CHECK_LAUNCH("group_routes_kernel");
  }
  if constexpr (FP4) {
    if (fp4_tc) {  // tensor cores; CUDA cores for other shapes
      if (int rc = launch_expert_ffn_fp4_tc(reinterpret_cast<const __nv_bfloat16*>(x), T, K, H, I,
                                            W1.packed, W1.scale, W1.global_, W2.packed,
                                            W2.scale, W2.global_, S, topk_w, ws, n, st, fx))
        return rc;
    } else {
      const int grid = num_sms() * 2;
      TW_LAUNCH(ffn_up_kernel<FP4>, dim3(grid), dim3(kFfnThreads), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(x), H, I, K, W1, ws, topk_w, fx);
      TW_CHECK_LAUNCH("ffn_up_kernel");
      TW_LAUNCH(ffn_down_kernel<FP4>, dim3(grid), dim3(kFfnThreads), 0, st, H, I, topk_w, W2, ws,
                fx);
      TW_CHECK_LAUNCH("ffn_down_kernel");
    }
  } else {
    if (int rc = launch_expert_ffn_tc(reinterpret_cast<const __nv_bfloat16*>(x), T, K, H, I,
                                      W1.w, W2.w, S, topk_w, ws, n, st, fx))
      return rc;
  }
  if (routes_only) return TW_OK;  // the routes' outputs stay in the workspace (c3, pos)
  if (cn != nullptr) return launch_combine_norm(ws, T, K, H, *cn, st);
  if (cm != nullptr) return launch_combine_merge(ws, T, K, H, *cm, st);
  dim3 cg((H / 8 + kCombineThreads - 1) / kCombineThreads, (unsigned)T);
  TW_LAUNCH(combine_kernel, dim3(cg), dim3(kCombineThreads), 0, st, H, K, ws,
            reinterpret_cast<__nv_bfloat16*>(out));
  TW_CHECK_LAUNCH("combine_kernel");
  return TW_OK;
}

}  // namespace

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

}  // namespace tw

using namespace tw;

extern "C" size_t tw_moe_workspace_bytes(int64_t n_routes, int H, int I) {
  return workspace_layout(n_routes, H, I, nullptr, nullptr);
}

extern "C" size_t tw_moe_workspace_error_offset(int64_t n_routes, int H, int I) {
  Workspace ws;
  workspace_layout(n_routes, H, I, reinterpret_cast<char*>(1024), &ws);
  return reinterpret_cast<char*>(ws.err) - reinterpret_cast<char*>(1024);
}

extern "C" int tw_moe_ffn_bf16(const void* x, int64_t T, int H, int I, const void* w1,
                               const void* w2, int64_t S, const float* topk_w,
                               const int32_t* topk_ids, int K, void* out, void* workspace,
                               size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, out, workspace,
                                  ws_bytes, as_stream(stream));
}

extern "C" int tw_moe_ffn_bf16_routes(const void* x, int64_t T, int H, int I, const void* w1,
                                      const void* w2, int64_t S, const float* topk_w,
                                      const int32_t* topk_ids, int K, void* workspace,
                                      size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace,
                        ws_bytes, as_stream(stream), nullptr, nullptr, true);
}

extern "C" int tw_moe_ffn_bf16_residual_norm(const void* x, int64_t T, int H, int I,
                                             const void* w1, const void* w2, int64_t S,
                                             const float* topk_w, const int32_t* topk_ids,
                                             int K, const void* residual, void* residual_out,
                                             const void* norm_w, float eps, void* h_out,
                                             void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  TW_CHECK_ARG(residual && residual_out && norm_w && h_out && aligned16(residual) &&
                   aligned16(residual_out) && aligned16(norm_w) && aligned16(h_out),
               "moe_ffn_bf16_residual_norm: residual, norm weight and outputs are required "
               "and must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  const CombineNorm cn{residual, residual_out, norm_w, eps, h_out};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace,
                        ws_bytes, as_stream(stream), &cn);
}

extern "C" int tw_moe_ffn_bf16_residual_norm_grouped(
    const void* x, int64_t T, int H, int I, const void* w1, const void* w2, int64_t S,
    const float* topk_w, const int32_t* topk_ids, int K, const void* residual,
    void* residual_out, const void* norm_w, float eps, void* h_out, void* workspace,
    size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  TW_CHECK_ARG(residual && residual_out && norm_w && h_out && aligned16(residual) &&
                   aligned16(residual_out) && aligned16(norm_w) && aligned16(h_out),
               "moe_ffn_bf16_residual_norm: residual, norm weight and outputs are required "
               "and must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  const CombineNorm cn{residual, residual_out, norm_w, eps, h_out};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace,
                        ws_bytes, as_stream(stream), &cn, nullptr, false, true);
}

extern "C" int tw_moe_ffn_nvfp4_grouped(const void* x, int64_t T, int H, int I, const void* w1p,
                                        const void* w1s, const void* w1g, const void* w2p,
                                        const void* w2s, const void* w2g, int global_dtype,
                                        int64_t S, const float* topk_w,
                                        const int32_t* topk_ids, int K, void* out,
                                        void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(global_dtype == TW_F32 || global_dtype == TW_F16,
               "moe_ffn_nvfp4: row globals must be fp32 or fp16");
  TW_CHECK_ARG(aligned16(w1p) && aligned16(w2p), "moe_ffn_nvfp4: packed banks must be 16-byte aligned");
  TW_CHECK_ARG((reinterpret_cast<uintptr_t>(w1s) & 3) == 0 && (reinterpret_cast<uintptr_t>(w2s) & 3) == 0,
               "moe_ffn_nvfp4: scale banks must be 4-byte aligned");
  const int g16 = global_dtype == TW_F16;
  Fp4Rows W1{reinterpret_cast<const uint8_t*>(w1p), reinterpret_cast<const uint8_t*>(w1s),
             RowScale{w1g, g16}, 2 * (int64_t)I, H};
  Fp4Rows W2{reinterpret_cast<const uint8_t*>(w2p), reinterpret_cast<const uint8_t*>(w2s),
             RowScale{w2g, g16}, H, I};
  return run_ffn<true>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, out, workspace, ws_bytes,
                       as_stream(stream), nullptr, nullptr, false, true);
}

extern "C" int tw_moe_ffn_bf16_dual_merge(const void* x, int64_t T, int H, int I,
                                          const void* w1, const void* w2, int64_t S,
                                          const float* topk_w, const int32_t* topk_ids, int K,
                                          const void* shared, const void* residual,
                                          const void* w1n, const void* w2n, const void* w3n,
                                          float eps1, float eps2, float eps3, float scalar,
                                          void* out, void* workspace, size_t ws_bytes,
                                          void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  TW_CHECK_ARG(shared && residual && w1n && w2n && w3n && out && aligned16(shared) &&
                   aligned16(residual) && aligned16(w1n) && aligned16(w2n) && aligned16(w3n) &&
                   aligned16(out),
               "moe_ffn_bf16_dual_merge: shared, residual, norm weights and out are required "
               "and must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  const CombineMerge cm{shared, residual, w1n, w2n, w3n, eps1, eps2, eps3, scalar, out};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace,
                        ws_bytes, as_stream(stream), nullptr, &cm);
}

extern "C" int tw_moe_ffn_bf16_dual_merge_act(
    const void* x, int64_t T, int H, int I, const void* w1, const void* w2, int64_t S,
    const float* topk_w, const int32_t* topk_ids, int K, const void* shared,
    const void* residual, const void* w1n, const void* w2n, const void* w3n, float eps1,
    float eps2, float eps3, float scalar, int activation, int weight_on_input, void* out,
    void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  TW_CHECK_ARG(shared && residual && w1n && w2n && w3n && out && aligned16(shared) &&
                   aligned16(residual) && aligned16(w1n) && aligned16(w2n) && aligned16(w3n) &&
                   aligned16(out),
               "moe_ffn_bf16_dual_merge: shared, residual, norm weights and out are required "
               "and must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  const CombineMerge cm{shared, residual, w1n, w2n, w3n, eps1, eps2, eps3, scalar, out};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace,
                        ws_bytes, as_stream(stream), nullptr, &cm, false, false,
                        FfnAct{activation, weight_on_input});
}

namespace {

int ffn_dense_bf16(const void* x, int64_t T, int H, int I, const void* w1, const void* w2,
                   void* out, void* workspace, size_t ws_bytes, void* stream, FfnAct fx) {
  TW_CHECK_ARG(fx.act >= TW_ACT_SILU && fx.act <= TW_ACT_GELU_TANH,
               "ffn_dense_bf16: activation must be silu/gelu/gelu_tanh (0..2)");
  TW_CHECK_ARG(T >= 0 && T <= kMaxRoutes, "ffn_dense_bf16: need T <= %d", kMaxRoutes);
  TW_CHECK_ARG(H > 0 && I > 0 && H % 128 == 0 && I % 64 == 0,
               "ffn_dense_bf16: need H %% 128 == 0 and I %% 64 == 0 (got H=%d I=%d)", H, I);
  TW_CHECK_ARG(aligned16(x) && aligned16(out) && aligned16(w1) && aligned16(w2),
               "ffn_dense_bf16: x, out and weights must be 16-byte aligned");
  if (T == 0) return TW_OK;
  Workspace ws;
  const size_t need = workspace_layout(T, H, I, static_cast<char*>(workspace), &ws);
  TW_CHECK_ARG(workspace != nullptr && ws_bytes >= need,
               "ffn_dense_bf16: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  TW_CHECK_ARG(aligned16(workspace), "ffn_dense_bf16: workspace must be 16-byte aligned");
  return launch_expert_ffn_dense_tc(reinterpret_cast<const __nv_bfloat16*>(x), T, H, I,
                                    reinterpret_cast<const __nv_bfloat16*>(w1),
                                    reinterpret_cast<const __nv_bfloat16*>(w2), ws,
                                    reinterpret_cast<__nv_bfloat16*>(out), as_stream(stream),
                                    fx);
}

}  // namespace

extern "C" int tw_ffn_dense_bf16(const void* x, int64_t T, int H, int I, const void* w1,
                                 const void* w2, void* out, void* workspace, size_t ws_bytes,
                                 void* stream) {
  return ffn_dense_bf16(x, T, H, I, w1, w2, out, workspace, ws_bytes, stream, FfnAct{});
}

extern "C" int tw_ffn_dense_bf16_act(const void* x, int64_t T, int H, int I, const void* w1,
                                     const void* w2, int activation, void* out,
                                     void* workspace, size_t ws_bytes, void* stream) {
  return ffn_dense_bf16(x, T, H, I, w1, w2, out, workspace, ws_bytes, stream,
                        FfnAct{activation, 0});
}

extern "C" int tw_moe_ffn_nvfp4(const void* x, int64_t T, int H, int I, const void* w1p,
                                const void* w1s, const void* w1g, const void* w2p,
                                const void* w2s, const void* w2g, int global_dtype, int64_t S,
                                const float* topk_w, const int32_t* topk_ids, int K, void* out,
                                void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(global_dtype == TW_F32 || global_dtype == TW_F16,
               "moe_ffn_nvfp4: row globals must be fp32 or fp16");
  const int g16 = global_dtype == TW_F16;
  TW_CHECK_ARG(aligned16(w1p) && aligned16(w2p), "moe_ffn_nvfp4: packed banks must be 16-byte aligned");
  TW_CHECK_ARG((reinterpret_cast<uintptr_t>(w1s) & 3) == 0 && (reinterpret_cast<uintptr_t>(w2s) & 3) == 0,
               "moe_ffn_nvfp4: scale banks must be 4-byte aligned");
  Fp4Rows W1{reinterpret_cast<const uint8_t*>(w1p), reinterpret_cast<const uint8_t*>(w1s),
             RowScale{w1g, g16}, 2 * (int64_t)I, H};
  Fp4Rows W2{reinterpret_cast<const uint8_t*>(w2p), reinterpret_cast<const uint8_t*>(w2s),
             RowScale{w2g, g16}, H, I};
  return run_ffn<true>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, out, workspace,
                                ws_bytes, as_stream(stream));
}

extern "C" int tw_moe_ffn_bf16_act(const void* x, int64_t T, int H, int I, const void* w1,
                                   const void* w2, int64_t S, const float* topk_w,
                                   const int32_t* topk_ids, int K, int activation,
                                   int weight_on_input, void* out, void* workspace,
                                   size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(aligned16(w1) && aligned16(w2), "moe_ffn_bf16: banks must be 16-byte aligned");
  Bf16Rows W1{reinterpret_cast<const __nv_bfloat16*>(w1), 2 * (int64_t)I, H};
  Bf16Rows W2{reinterpret_cast<const __nv_bfloat16*>(w2), H, I};
  return run_ffn<false>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, out, workspace, ws_bytes,
                        as_stream(stream), nullptr, nullptr, false, false,
                        FfnAct{activation, weight_on_input});
}

extern "C" int tw_moe_ffn_nvfp4_act(const void* x, int64_t T, int H, int I, const void* w1p,
                                    const void* w1s, const void* w1g, const void* w2p,
                                    const void* w2s, const void* w2g, int global_dtype,
                                    int64_t S, const float* topk_w, const int32_t* topk_ids,
                                    int K, int activation, int weight_on_input, void* out,
                                    void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(global_dtype == TW_F32 || global_dtype == TW_F16,
               "moe_ffn_nvfp4: row globals must be fp32 or fp16");
  const int g16 = global_dtype == TW_F16;
  TW_CHECK_ARG(aligned16(w1p) && aligned16(w2p), "moe_ffn_nvfp4: packed banks must be 16-byte aligned");
  TW_CHECK_ARG((reinterpret_cast<uintptr_t>(w1s) & 3) == 0 && (reinterpret_cast<uintptr_t>(w2s) & 3) == 0,
               "moe_ffn_nvfp4: scale banks must be 4-byte aligned");
  Fp4Rows W1{reinterpret_cast<const uint8_t*>(w1p), reinterpret_cast<const uint8_t*>(w1s),
             RowScale{w1g, g16}, 2 * (int64_t)I, H};
  Fp4Rows W2{reinterpret_cast<const uint8_t*>(w2p), reinterpret_cast<const uint8_t*>(w2s),
             RowScale{w2g, g16}, H, I};
  return run_ffn<true>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, out, workspace, ws_bytes,
                       as_stream(stream), nullptr, nullptr, false, false,
                       FfnAct{activation, weight_on_input});
}

extern "C" int tw_moe_ffn_nvfp4_routes(const void* x, int64_t T, int H, int I, const void* w1p,
                                       const void* w1s, const void* w1g, const void* w2p,
                                       const void* w2s, const void* w2g, int global_dtype,
                                       int64_t S, const float* topk_w, const int32_t* topk_ids,
                                       int K, void* workspace, size_t ws_bytes, void* stream) {
  TW_CHECK_ARG(global_dtype == TW_F32 || global_dtype == TW_F16,
               "moe_ffn_nvfp4: row globals must be fp32 or fp16");
  TW_CHECK_ARG(aligned16(w1p) && aligned16(w2p), "moe_ffn_nvfp4: packed banks must be 16-byte aligned");
  TW_CHECK_ARG((reinterpret_cast<uintptr_t>(w1s) & 3) == 0 && (reinterpret_cast<uintptr_t>(w2s) & 3) == 0,
               "moe_ffn_nvfp4: scale banks must be 4-byte aligned");
  const int g16 = global_dtype == TW_F16;
  Fp4Rows W1{reinterpret_cast<const uint8_t*>(w1p), reinterpret_cast<const uint8_t*>(w1s),
             RowScale{w1g, g16}, 2 * (int64_t)I, H};
  Fp4Rows W2{reinterpret_cast<const uint8_t*>(w2p), reinterpret_cast<const uint8_t*>(w2s),
             RowScale{w2g, g16}, H, I};
  return run_ffn<true>(x, T, H, I, W1, W2, S, topk_w, topk_ids, K, nullptr, workspace, ws_bytes,
                       as_stream(stream), nullptr, nullptr, true);
}

// ---------------------------------------------------------------- allocation-free entry

// Scratch for tw_moe_ffn_bf16_noalloc: one fixed block of device memory per GPU that loads
// this library, reserved at module load and held until the process exits.
constexpr size_t kStaticScratchBytes = size_t(32) << 20;  // 32 MiB
static __device__ __align__(256) unsigned char g_ffn_static_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxScratchDevices = 64;
void* g_scratch_ptr[kMaxScratchDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the static scratch on the current device (looked up once per device;
// the host-side symbol itself is not a device address and must never reach a kernel).
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("tw_moe_ffn_bf16_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxScratchDevices) {
    set_error("tw_moe_ffn_bf16_noalloc: device ordinal %d beyond %d", dev, kMaxScratchDevices);
    return TW_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ffn_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("tw_moe_ffn_bf16_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return TW_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TW_OK;
}
}  // namespace

extern "C" size_t tw_moe_ffn_noalloc_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int tw_moe_ffn_bf16_noalloc(const void* x, int64_t T, int H, int I, const void* w1,
                                       const void* w2, int64_t S, const float* topk_w,
                                       const int32_t* topk_ids, int K, void* out,
                                       void* stream) {
  TW_CHECK_ARG(T >= 0 && K > 0 && H > 0 && I > 0, "tw_moe_ffn_bf16_noalloc: bad shape");
  const size_t need = tw_moe_workspace_bytes(T * K, H, I);
  TW_CHECK_ARG(need <= kStaticScratchBytes,
               "tw_moe_ffn_bf16_noalloc: %lld routes at H=%d, I=%d need %zu bytes of scratch, "
               "more than the %zu-byte static scratch; use tw_moe_ffn_bf16 with a workspace",
               (long long)(T * K), H, I, need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  return tw_moe_ffn_bf16(x, T, H, I, w1, w2, S, topk_w, topk_ids, K, out, scratch,
                         kStaticScratchBytes, stream);
}

extern "C" int tw_moe_ffn_noalloc_error(int64_t n_routes, int H, int I, int32_t* err_out,
                                        void* stream) {
  TW_CHECK_ARG(n_routes >= 0 && H > 0 && I > 0 && err_out != nullptr,
               "tw_moe_ffn_noalloc_error: bad arguments");
  TW_CHECK_ARG(tw_moe_workspace_bytes(n_routes, H, I) <= kStaticScratchBytes,
               "tw_moe_ffn_noalloc_error: %lld routes do not fit the static scratch",
               (long long)n_routes);
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  const size_t off = tw_moe_workspace_error_offset(n_routes, H, I);
  const cudaError_t e = cudaMemcpyAsync(err_out, static_cast<char*>(scratch) + off,
                                        sizeof(int32_t), cudaMemcpyDefault, as_stream(stream));
  if (e != cudaSuccess) {
    set_error("tw_moe_ffn_noalloc_error: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  return TW_OK;
}
