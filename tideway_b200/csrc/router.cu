// Router kernels: logits GEMM, softmax top-k, Gemma top-k, sigmoid group-limited top-k.
//
// One warp owns one token for the top-k family.  The token's E scores live in shared
// memory; selection is K rounds of a warp-wide argmax with ties broken toward the lower
// expert id (the Gemma kernel's documented order, src/tideway/gemma_route_copy_kernel.py:47-54).
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace tw {

bool router_logits_tc_ok(int64_t T, int H, int E);
int launch_router_logits_tc(const void* x, const void* w, int64_t T, int H, int E, float* logits,
                            cudaStream_t st);

namespace {

constexpr int kWarpsPerBlock = 4;
constexpr int kMaxE = 1024;
constexpr int kMaxK = 32;

// Warp argmax over vals[0..n) excluding entries flagged in the per-lane bitmask `taken`
// (bit j of lane l <-> index l + 32 j).  Returns the winning index (or -1 if none).
__device__ __forceinline__ int warp_argmax(const float* vals, int n, uint32_t taken,
                                           float* best_out) {
  const int lane = threadIdx.x & 31;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = 0, i = lane; i < n; ++j, i += 32) {
    if (taken & (1u << j)) continue;
    const float v = vals[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  *best_out = bv;
  return bi == 0x7fffffff ? -1 : bi;
}

__device__ __forceinline__ void mark_taken(uint32_t& taken, int idx) {
  if (idx >= 0 && (idx & 31) == (int)(threadIdx.x & 31)) taken |= 1u << (idx >> 5);
}

__device__ __forceinline__ float load_score(const void* p, int dtype, int64_t off) {
  return dtype == TW_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off])
                          : reinterpret_cast<const float*>(p)[off];
}

// Softmax over the E scores in v (this warp's shared-memory row), top-K, optional
// renormalisation; lane 0 writes the K weights and ids (-1 when pad).  The one selection
// used by the standalone top-k kernel and the fused router, so both give the same bits.
__device__ __forceinline__ void softmax_select(float* v, int E, int K, int renorm, bool pad,
                                               float* __restrict__ w_row,
                                               int32_t* __restrict__ id_row) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int i = lane; i < E; i += 32) mx = fmaxf(mx, v[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int i = lane; i < E; i += 32) {
    const float e = expf(v[i] - mx);
    v[i] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  const float inv = 1.0f / sum;
  for (int i = lane; i < E; i += 32) v[i] = v[i] * inv;  // == torch softmax up to ulps
  __syncwarp();
  uint32_t taken = 0;
  float wk[kMaxK];
  int ik[kMaxK];
  float wsum = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv;
    const int bi = warp_argmax(v, E, taken, &bv);
    mark_taken(taken, bi);
    wk[k] = bv;
    ik[k] = bi;
    wsum += bv;
  }
  if (lane == 0) {
    for (int k = 0; k < K; ++k) {
      w_row[k] = renorm ? wk[k] / wsum : wk[k];
      id_row[k] = pad ? -1 : ik[k];
    }
  }
}

__global__ void softmax_topk_kernel(const void* __restrict__ logits, int dtype, int64_t ld,
                                    int64_t T, int E, int K, int renorm,
                                    const int32_t* __restrict__ ntp, float* __restrict__ w_out,
                                    int32_t* __restrict__ id_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[kWarpsPerBlock][kMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (t >= T) return;
  float* v = sv[warp];
  for (int i = lane; i < E; i += 32) v[i] = load_score(logits, dtype, t * ld + i);
  __syncwarp();
  const bool pad = ntp != nullptr && t >= (int64_t)(*ntp);
  softmax_select(v, E, K, renorm, pad, w_out + t * K, id_out + t * K);
}

__global__ void gemma_topk_kernel(const void* __restrict__ logits, int dtype, int64_t ld,
                                  int64_t T, int E, int K, const void* __restrict__ scale,
                                  int sdtype, float* __restrict__ w_out,
                                  int32_t* __restrict__ id_out, int32_t* __restrict__ priv_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[kWarpsPerBlock][kMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (t >= T) return;
  float* v = sv[warp];
  for (int i = lane; i < E; i += 32) v[i] = load_score(logits, dtype, t * ld + i);
  __syncwarp();
  uint32_t taken = 0;
  float lk[kMaxK];
  int ik[kMaxK];
  for (int k = 0; k < K; ++k) {
    float bv;
    const int bi = warp_argmax(v, E, taken, &bv);
    mark_taken(taken, bi);
    lk[k] = bv;
    ik[k] = bi;
  }
  if (lane == 0) {
    const float mx = lk[0];
    float e[kMaxK];
    float den = 0.f;
    for (int k = 0; k < K; ++k) {
      e[k] = expf(lk[k] - mx);
      den += e[k];
    }
    const float d = den > 0.f ? den : 1.f;
    for (int k = 0; k < K; ++k) {
      w_out[t * K + k] = (e[k] / d) * load_score(scale, sdtype, ik[k]);
      if (id_out) id_out[t * K + k] = ik[k];
      if (priv_out) priv_out[t * K + k] = ik[k];
    }
  }
}

// DeepSeek-style selection over E logits in s (this warp's shared-memory rows s, c and
// sg[32]): sigmoid scores, groups ranked by the sum of their two best (score + bias), the
// KG best groups kept, top-K experts of those; lane 0 writes weights (sigmoid, renormalised
// if asked, x scaling) and ids.  Shared by the standalone kernel and the fused router.
__device__ __forceinline__ void sigmoid_group_select(float* s, float* c, float* sg, int E,
                                                     int K, int G, int KG,
                                                     const float* __restrict__ bias,
                                                     int renorm, float scaling,
                                                     float* __restrict__ w_row,
                                                     int32_t* __restrict__ id_row) {
  const int lane = threadIdx.x & 31;
  for (int i = lane; i < E; i += 32) {
    const float x = s[i];
    const float sig = 1.0f / (1.0f + expf(-x));
    s[i] = sig;
    c[i] = bias ? sig + bias[i] : sig;
  }
  __syncwarp();
  const int gsz = E / G;
  if (lane < G) {
    float b0 = -INFINITY, b1 = -INFINITY;
    for (int j = 0; j < gsz; ++j) {
      const float x = c[lane * gsz + j];
      if (x > b0) {
        b1 = b0;
        b0 = x;
      } else if (x > b1) {
        b1 = x;
      }
    }
    sg[lane] = b0 + b1;
  }
  __syncwarp();
  // keep the KG best groups (ties -> lower group index)
  uint32_t gtaken = 0;
  uint32_t keep = 0;  // bit g set -> group kept (identical on every lane)
  for (int k = 0; k < KG; ++k) {
    float bv;
    const int bi = warp_argmax(sg, G, gtaken, &bv);
    mark_taken(gtaken, bi);
    if (bi >= 0) keep |= 1u << bi;
  }
  // exclude experts of dropped groups from the expert selection
  uint32_t taken = 0;
  for (int j = 0, i = lane; i < E; ++j, i += 32)
    if (!((keep >> (i / gsz)) & 1u)) taken |= 1u << j;
  float wk[kMaxK];
  int ik[kMaxK];
  float wsum = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv;
    const int bi = warp_argmax(c, E, taken, &bv);
    mark_taken(taken, bi);
    ik[k] = bi;
    wk[k] = bi >= 0 ? s[bi] : 0.f;
    wsum += wk[k];
  }
  if (lane == 0) {
    for (int k = 0; k < K; ++k) {
      const float w = renorm ? wk[k] / wsum : wk[k];
      w_row[k] = w * scaling;
      id_row[k] = ik[k];
    }
  }
}

__global__ void sigmoid_group_topk_kernel(const void* __restrict__ logits, int dtype,
                                          int64_t ld, int64_t T, int E, int K, int G, int KG,
                                          const float* __restrict__ bias, int renorm,
                                          float scaling, float* __restrict__ w_out,
                                          int32_t* __restrict__ id_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float ss[kWarpsPerBlock][kMaxE];
  __shared__ float sc[kWarpsPerBlock][kMaxE];
  __shared__ float sg[kWarpsPerBlock][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (t >= T) return;
  for (int i = lane; i < E; i += 32) ss[warp][i] = load_score(logits, dtype, t * ld + i);
  __syncwarp();
  sigmoid_group_select(ss[warp], sc[warp], sg[warp], E, K, G, KG, bias, renorm, scaling,
                       w_out + t * K, id_out + t * K);
}

// logits[t, e] = x[t, :] . w[e, :]: H % 8 == 0, H <= 32 * 8 * kMaxVec.
constexpr int kRouterWarps = 8;
constexpr int kMaxVec = 16;

// x_row . w_row in fp32 by one warp: lane l takes the 16-byte vectors l, l + 32, ...
// (H % 8 == 0, H <= 32 * 8 * kMaxVec), both rows loaded in one round trip, then a butterfly
// sum.  The GEMV below and the fused router use this one function, so their logits agree
// bit for bit.
__device__ __forceinline__ float router_dot(const __nv_bfloat16* __restrict__ xr,
                                            const __nv_bfloat16* __restrict__ wr, int H) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const uint4* wrow = reinterpret_cast<const uint4*>(wr);
  const uint4* xrow = reinterpret_cast<const uint4*>(xr);
  uint4 wv[kMaxVec], xv[kMaxVec];
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int v = lane + 32 * j;
    wv[j] = v < nvec ? __ldg(wrow + v) : make_uint4(0, 0, 0, 0);
    xv[j] = v < nvec ? __ldg(xrow + v) : make_uint4(0, 0, 0, 0);
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    float a[8], b[8];
    bf16x8_to_f32(xv[j], a);
    bf16x8_to_f32(wv[j], b);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc = fmaf(a[q], b[q], acc);
  }
  return warp_sum(acc);
}

// router_dot with the router row already in registers (loaded by load_router_row): the same
// arithmetic, so that a kernel can fetch its rows before waiting for its predecessor.
__device__ __forceinline__ void load_router_row(const __nv_bfloat16* __restrict__ wr, int H,
                                                uint4 (&wv)[kMaxVec]) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const uint4* wrow = reinterpret_cast<const uint4*>(wr);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int v = lane + 32 * j;
    wv[j] = v < nvec ? __ldg(wrow + v) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ float router_dot_row(const __nv_bfloat16* __restrict__ xr,
                                                const uint4 (&wv)[kMaxVec], int H) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const uint4* xrow = reinterpret_cast<const uint4*>(xr);
  uint4 xv[kMaxVec];
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int v = lane + 32 * j;
    xv[j] = v < nvec ? __ldg(xrow + v) : make_uint4(0, 0, 0, 0);
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    float a[8], b[8];
    bf16x8_to_f32(xv[j], a);
    bf16x8_to_f32(wv[j], b);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc = fmaf(a[q], b[q], acc);
  }
  return warp_sum(acc);
}

// One warp per (token, router row) dot product (decode batches have few tokens, so
// parallelism comes from the E x T pairs).
__global__ void __launch_bounds__(kRouterWarps * 32)
router_logits_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                     int64_t T, int H, int E, float* __restrict__ logits) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * kRouterWarps + warp;
  if (g >= T * E) return;
  const int64_t t = g / E;
  const int e = (int)(g % E);
  const float acc = router_dot(x + t * H, w + (int64_t)e * H, H);
  if (lane == 0) logits[t * E + e] = acc;
}

// ---------------------------------------------------------------- fused decode router
//
// Logits GEMV and top-k selection in one launch.  The GEMV keeps its parallelism: CTA
// (b, t) computes router rows [16 b, 16 b + 16) of token t, one warp per row with
// router_dot (so every logit has the bits of the standalone GEMV), and writes them to the
// logits buffer.  Each CTA then counts itself done on the token's arrival counter; the CTA
// that completes the count (the last of the token's E/16) reads the token's E logits back
// and runs the standalone kernels' selection with one warp.  That CTA also sets the counter
// back to 0 (every other CTA of the call has arrived), so each call starts from 0 whatever
// its E: the counters are zeroed once, at allocation.  (Counters that only grew, completing
// at every multiple of E/16, broke when calls with different E shared them: a token could be
// declared complete before all its router rows were written.)
constexpr int kFusedRows = 16;   // router rows (= warps) per CTA
constexpr int kFusedMaxT = 64;   // tokens per launch (decode batches)

enum class Select { kSoftmax = 0, kSigmoidGroup = 1 };

struct SelectArgs {
  int K, renorm;
  const int32_t* ntp;  // softmax: rows >= *ntp get id -1 (may be null)
  int G, KG;           // sigmoid group
  const float* bias;   // sigmoid group (may be null)
  float scaling;
};

template <Select kSel>
__global__ void __launch_bounds__(kFusedRows * 32)
router_topk_fused_kernel(const __nv_bfloat16* __restrict__ x,
                         const __nv_bfloat16* __restrict__ w, int H, int E,
                         float* __restrict__ logits, unsigned* __restrict__ arrivals,
                         SelectArgs sa, float* __restrict__ w_out,
                         int32_t* __restrict__ id_out) {
  __shared__ float v[kMaxE];
  __shared__ float c[kSel == Select::kSigmoidGroup ? kMaxE : 1];
  __shared__ float sg[32];
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.y;
  const int e = blockIdx.x * kFusedRows + warp;
  // the router rows are weights (no kernel writes them): they are fetched before waiting for
  // the predecessor, so their latency overlaps its tail; x is read after the wait
  uint4 wv[kMaxVec];
  if (e < E) load_router_row(w + (int64_t)e * H, H, wv);
  pdl_wait();
  pdl_trigger();
  if (e < E) {
    const float acc = router_dot_row(x + t * H, wv, H);
    if (lane == 0) logits[t * E + e] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this CTA's logits before its arrival
    const unsigned done = atomicAdd(arrivals + t, 1u) + 1u;
    last = done == gridDim.x;
    if (last) {
      arrivals[t] = 0u;  // every CTA of this call has arrived: ready for the next call
      __threadfence();   // every other CTA's logits before reading them
    }
  }
  __syncthreads();
  if (!last || warp != 0) return;
  const volatile float* lt = logits + t * E;  // written by other CTAs: bypass L1
  for (int i = lane; i < E; i += 32) v[i] = lt[i];
  __syncwarp();
  if (kSel == Select::kSoftmax) {
    const bool pad = sa.ntp != nullptr && t >= (int64_t)(*sa.ntp);
    softmax_select(v, E, sa.K, sa.renorm, pad, w_out + t * sa.K, id_out + t * sa.K);
  } else {
    sigmoid_group_select(v, c, sg, E, sa.K, sa.G, sa.KG, sa.bias, sa.renorm, sa.scaling,
                         w_out + t * sa.K, id_out + t * sa.K);
  }
}

int launch_router_fused(Select sel, const void* x, const void* w, int64_t T, int H, int E,
                        float* logits, unsigned* arrivals, const SelectArgs& sa, float* w_out,
                        int32_t* id_out, cudaStream_t st) {
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= 32 * 8 * kMaxVec,
               "fused router: need H %% 8 == 0 and H <= %d", 32 * 8 * kMaxVec);
  TW_CHECK_ARG(E > 0 && E <= kMaxE, "fused router: need 0 < E <= %d", kMaxE);
  TW_CHECK_ARG(T <= kFusedMaxT, "fused router: decode batches only (T <= %d)", kFusedMaxT);
  TW_CHECK_ARG(logits != nullptr && arrivals != nullptr,
               "fused router: the logits buffer and the arrival counters are required");
  TW_CHECK_ARG(aligned16(x) && aligned16(w), "fused router: x and w must be 16-byte aligned");
  if (T == 0) return TW_OK;
  const dim3 grid((unsigned)((E + kFusedRows - 1) / kFusedRows), (unsigned)T);
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* wb = reinterpret_cast<const __nv_bfloat16*>(w);
  if (sel == Select::kSoftmax) {
    TW_LAUNCH(router_topk_fused_kernel<Select::kSoftmax>, grid, dim3(kFusedRows * 32), 0, st,
              xb, wb, H, E, logits, arrivals, sa, w_out, id_out);
  } else {
    TW_LAUNCH(router_topk_fused_kernel<Select::kSigmoidGroup>, grid, dim3(kFusedRows * 32), 0,
              st, xb, wb, H, E, logits, arrivals, sa, w_out, id_out);
  }
  TW_CHECK_LAUNCH("router_topk_fused_kernel");
  return TW_OK;
}

int check_common(int64_t T, int E, int K, int64_t ld) {
  TW_CHECK_ARG(T >= 0, "router: T must be >= 0");
  TW_CHECK_ARG(E > 0 && E <= kMaxE, "router: need 0 < E <= %d (got %d)", kMaxE, E);
  TW_CHECK_ARG(K > 0 && K <= E && K <= kMaxK, "router: need 0 < K <= min(E, %d) (got %d)",
               kMaxK, K);
  TW_CHECK_ARG(ld >= E, "router: ld_logits %lld < E", (long long)ld);
  return TW_OK;
}

}  // namespace
}  // namespace tw

using namespace tw;

extern "C" int tw_router_softmax_topk(const void* logits, int dtype, int64_t ld, int64_t T,
                                      int E, int K, int renorm, const int32_t* ntp,
                                      float* w, int32_t* ids, void* stream) {
  if (int rc = check_common(T, E, K, ld)) return rc;
  TW_CHECK_ARG(dtype == TW_F32 || dtype == TW_BF16, "router: logits dtype must be f32/bf16");
  if (T == 0) return TW_OK;
  const int64_t blocks = (T + kWarpsPerBlock - 1) / kWarpsPerBlock;
  TW_LAUNCH(softmax_topk_kernel, dim3((unsigned)blocks), dim3(kWarpsPerBlock * 32), 0, as_stream(stream), 
      logits, dtype, ld, T, E, K, renorm, ntp, w, ids);
  TW_CHECK_LAUNCH("softmax_topk_kernel");
  return TW_OK;
}

extern "C" int tw_router_gemma_topk(const void* logits, int dtype, int64_t ld, int64_t T,
                                    int E, int K, const void* scale, int sdtype, float* w,
                                    int32_t* ids, int32_t* priv, void* stream) {
  if (int rc = check_common(T, E, K, ld)) return rc;
  TW_CHECK_ARG(scale != nullptr, "gemma router: per_expert_scale is required");
  if (T == 0) return TW_OK;
  const int64_t blocks = (T + kWarpsPerBlock - 1) / kWarpsPerBlock;
  TW_LAUNCH(gemma_topk_kernel, dim3((unsigned)blocks), dim3(kWarpsPerBlock * 32), 0, as_stream(stream), 
      logits, dtype, ld, T, E, K, scale, sdtype, w, ids, priv);
  TW_CHECK_LAUNCH("gemma_topk_kernel");
  return TW_OK;
}

extern "C" int tw_router_sigmoid_group_topk(const void* logits, int dtype, int64_t ld,
                                            int64_t T, int E, int K, int G, int KG,
                                            const float* bias, int renorm, float scaling,
                                            float* w, int32_t* ids, void* stream) {
  if (int rc = check_common(T, E, K, ld)) return rc;
  TW_CHECK_ARG(G > 0 && G <= 32 && E % G == 0, "group router: need 0 < n_group <= 32, E %% n_group == 0");
  TW_CHECK_ARG(KG > 0 && KG <= G, "group router: need 0 < topk_group <= n_group");
  TW_CHECK_ARG(E / G >= 2, "group router: groups need at least 2 experts");
  TW_CHECK_ARG(K <= KG * (E / G), "group router: K exceeds the experts of the kept groups");
  if (T == 0) return TW_OK;
  const int64_t blocks = (T + kWarpsPerBlock - 1) / kWarpsPerBlock;
  TW_LAUNCH(sigmoid_group_topk_kernel, dim3((unsigned)blocks), dim3(kWarpsPerBlock * 32), 0, as_stream(stream), 
      logits, dtype, ld, T, E, K, G, KG, bias, renorm, scaling, w, ids);
  TW_CHECK_LAUNCH("sigmoid_group_topk_kernel");
  return TW_OK;
}

extern "C" int tw_router_logits(const void* x, const void* w, int64_t T, int H, int E,
                                float* logits, void* stream) {
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= 32 * 8 * kMaxVec,
               "router_logits: need H %% 8 == 0 and H <= %d", 32 * 8 * kMaxVec);
  TW_CHECK_ARG(E > 0, "router_logits: E must be > 0");
  TW_CHECK_ARG(aligned16(x) && aligned16(w), "router_logits: x and w must be 16-byte aligned");
  if (T == 0) return TW_OK;
  // many tokens: tensor cores (router_tc.cu); decode-sized batches: one warp per router row
  if (router_logits_tc_ok(T, H, E))
    return launch_router_logits_tc(x, w, T, H, E, logits, as_stream(stream));
  const int64_t pairs = T * (int64_t)E;
  dim3 grid((unsigned)((pairs + kRouterWarps - 1) / kRouterWarps));
  TW_LAUNCH(router_logits_kernel, dim3(grid), dim3(kRouterWarps * 32), 0, as_stream(stream), 
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w), T,
      H, E, logits);
  TW_CHECK_LAUNCH("router_logits_kernel");
  return TW_OK;
}

extern "C" int tw_router_softmax_topk_fused(const void* x, const void* w, int64_t T, int H,
                                            int E, int K, int renorm, const int32_t* ntp,
                                            float* logits, uint32_t* arrivals, float* topk_w,
                                            int32_t* topk_ids, void* stream) {
  if (int rc = check_common(T, E, K, E)) return rc;
  SelectArgs sa{K, renorm, ntp, 0, 0, nullptr, 1.0f};
  return launch_router_fused(Select::kSoftmax, x, w, T, H, E, logits, arrivals, sa, topk_w,
                             topk_ids, as_stream(stream));
}

extern "C" int tw_router_sigmoid_group_topk_fused(const void* x, const void* w, int64_t T,
                                                  int H, int E, int K, int G, int KG,
                                                  const float* bias, int renorm, float scaling,
                                                  float* logits, uint32_t* arrivals,
                                                  float* topk_w, int32_t* topk_ids,
                                                  void* stream) {
  if (int rc = check_common(T, E, K, E)) return rc;
  TW_CHECK_ARG(G > 0 && G <= 32 && E % G == 0, "group router: need 0 < n_group <= 32, E %% n_group == 0");
  TW_CHECK_ARG(KG > 0 && KG <= G, "group router: need 0 < topk_group <= n_group");
  TW_CHECK_ARG(E / G >= 2, "group router: groups need at least 2 experts");
  TW_CHECK_ARG(K <= KG * (E / G), "group router: K exceeds the experts of the kept groups");
  SelectArgs sa{K, renorm, nullptr, G, KG, bias, scaling};
  return launch_router_fused(Select::kSigmoidGroup, x, w, T, H, E, logits, arrivals, sa, topk_w,
                             topk_ids, as_stream(stream));
}
