// RMSNorm kernels: plain (optionally fused with the residual add), the router/routed pair
// (optionally with the shared expert's pre-norm), the Gemma dual-norm merge (optionally
// with the expert FFN's combine fused in), the combine fused with the next residual
// RMSNorm, and the DeepSeek routed + shared add.  One block per row (128 threads up to
// H = 4096, 256 beyond); 16-byte vectors; fp32 sums of squares.
#include <algorithm>

#include "common.cuh"
#include "moe_common.cuh"

namespace tw {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4;  // H <= 256 * 8 * 4 = 8192

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < (kThreads / 32) ? red[lane] : 0.f;
  r = warp_sum(r);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]));
    w[i] = lo | (hi << 16);
  }
  return r;
}

// Threads per row: 128 up to H = 4096 (more rows resident per SM, a 4-warp reduction),
// 256 beyond (H <= 8192).
inline int norm_threads(int H) { return H <= 128 * 8 * kNormMaxVec ? 128 : 256; }

template <int kThreads>
__global__ void __launch_bounds__(kThreads)
rmsnorm_kernel(const uint4* __restrict__ x, const uint4* __restrict__ res, uint4* res_out,
               const uint4* __restrict__ w, int H, float eps, float wb, uint4* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = H / 8;
  float v[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      bf16x8_to_f32(x[row * nvec + c], v[j]);
      if (res) {
        float r[8];
        bf16x8_to_f32(res[row * nvec + c], r);
#pragma unroll
        for (int q = 0; q < 8; ++q) v[j][q] = bf16_round(v[j][q] + r[q]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += v[j][q] * v[j][q];
    }
  }
  const float tot = block_sum<kThreads>(ss, red);
  const float rstd = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      if (res_out) res_out[row * nvec + c] = pack_bf16x8(v[j]);
      float wf[8], o[8];
      bf16x8_to_f32(w[c], wf);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = v[j][q] * rstd * (wf[q] + wb);
      y[row * nvec + c] = pack_bf16x8(o);
    }
  }
}

// Router input and routed input from one RMSNorm reduction of x; with sw != nullptr also a
// third output bf16(x * rstd * sw) (the shared expert's pre-norm, same x and eps).
template <int kThreads>
__global__ void __launch_bounds__(kThreads)
norm_pair_kernel(const uint4* __restrict__ x, const uint4* __restrict__ ones,
                 const uint4* __restrict__ rw, const uint4* __restrict__ scale,
                 const uint4* __restrict__ sw, int H, float eps, float root,
                 uint4* __restrict__ router_out, uint4* __restrict__ routed_out,
                 uint4* __restrict__ shared_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = H / 8;
  float v[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      bf16x8_to_f32(x[row * nvec + c], v[j]);
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += v[j][q] * v[j][q];
    }
  }
  const float tot = block_sum<kThreads>(ss, red);
  const float rstd = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      float on[8], sc[8], w2[8], a[8], b[8];
      bf16x8_to_f32(ones[c], on);
      bf16x8_to_f32(scale[c], sc);
      bf16x8_to_f32(rw[c], w2);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float h0 = bf16_round(v[j][q] * rstd * on[q]);
        const float h1 = bf16_round(h0 * sc[q]);
        a[q] = h1 * root;
        b[q] = v[j][q] * rstd * w2[q];
      }
      router_out[row * nvec + c] = pack_bf16x8(a);
      routed_out[row * nvec + c] = pack_bf16x8(b);
      if (sw != nullptr) {
        float w3[8], o[8];
        bf16x8_to_f32(sw[c], w3);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = v[j][q] * rstd * w3[q];
        shared_out[row * nvec + c] = pack_bf16x8(o);
      }
    }
  }
}

constexpr int kMaxCombineK = 64;

// The routed input of a merge, straight from an expert FFN's workspace: b[t] = bf16(sum_k
// c3[pos[t, k]]) in k order (skipped routes add nothing) -- the FFN's combine.
struct RouteSum {
  const int32_t* pos;
  const __nv_bfloat16* c3;
  int K;
};

// out = bf16(bf16(x + N3(bf16(N1(a) + N2(b)))) * scalar), Nk = bf16 RMSNorm with weight wk:
// the post-FFN merge of a shared expert output a and a routed output b with the residual x,
// the layer scalar applied to the residual sum as the Gemma 4 decoder layer applies it
// (loaded with a and b, so that the row costs one round trip to memory).  kCombine: b is
// the expert FFN's combine, computed here from its route rows (rs) -- bit-identical to
// combine_kernel followed by this merge, one launch and the b round trip fewer.
template <int kThreads, bool kCombine>
__global__ void __launch_bounds__(kThreads)
dual_norm_merge_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                       const uint4* __restrict__ x, const uint4* __restrict__ w1,
                       const uint4* __restrict__ w2, const uint4* __restrict__ w3, int H,
                       float eps1, float eps2, float eps3, float scalar,
                       uint4* __restrict__ out, RouteSum rs) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int sp[kMaxCombineK];
  const int64_t row = blockIdx.x;
  const int nvec = H / 8;
  float va[kNormMaxVec][8], vb[kNormMaxVec][8];
  uint4 xr[kNormMaxVec], rav[kNormMaxVec], rbv[kNormMaxVec];
  float sa = 0.f, sb = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      rav[j] = a[row * nvec + c];
      xr[j] = x[row * nvec + c];
      if (!kCombine) rbv[j] = b[row * nvec + c];
    }
  }
  if (kCombine) {
    for (int k = threadIdx.x; k < rs.K; k += kThreads) sp[k] = rs.pos[row * rs.K + k];
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      bf16x8_to_f32(rav[j], va[j]);
      if (kCombine) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k0 = 0; k0 < rs.K; k0 += 8) {
          int p[8];
          uint4 r[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            p[q] = k0 + q < rs.K ? sp[k0 + q] : -1;
            r[q] = p[q] >= 0 ? *reinterpret_cast<const uint4*>(rs.c3 + (int64_t)p[q] * H + c * 8)
                             : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (p[q] < 0) continue;
            float f[8];
            bf16x8_to_f32(r[q], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += f[e];
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) vb[j][q] = bf16_round(acc[q]);
      } else {
        bf16x8_to_f32(rbv[j], vb[j]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        sa += va[j][q] * va[j][q];
        sb += vb[j][q] * vb[j][q];
      }
    }
  }
  const float ra = rsqrtf(block_sum<kThreads>(sa, red) / (float)H + eps1);
  const float rb = rsqrtf(block_sum<kThreads>(sb, red) / (float)H + eps2);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      float f1[8], f2[8];
      bf16x8_to_f32(w1[c], f1);
      bf16x8_to_f32(w2[c], f2);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float m = bf16_round(bf16_round(va[j][q] * ra * f1[q]) +
                                   bf16_round(vb[j][q] * rb * f2[q]));
        va[j][q] = m;
        ss += m * m;
      }
    }
  }
  const float r3 = rsqrtf(block_sum<kThreads>(ss, red) / (float)H + eps3);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      float f3[8], xv[8], o[8];
      bf16x8_to_f32(w3[c], f3);
      bf16x8_to_f32(xr[j], xv);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        o[q] = bf16_round(xv[q] + bf16_round(va[j][q] * r3 * f3[q])) * scalar;
      out[row * nvec + c] = pack_bf16x8(o);
    }
  }
}

// The expert FFN's combine fused with the next residual add and RMSNorm, one block per
// token: y = bf16(sum_k c3[pos[t, k]]) in k order (skipped routes add nothing), then exactly
// rmsnorm_kernel's residual path on y (same threads, order and reduction).
template <int kThreads>
__global__ void __launch_bounds__(kThreads)
combine_norm_kernel(int H, int K, const int32_t* __restrict__ pos,
                    const __nv_bfloat16* __restrict__ c3, const uint4* __restrict__ res,
                    uint4* res_out, const uint4* __restrict__ w, float eps,
                    uint4* __restrict__ y) {
  __shared__ float red[32];
  __shared__ int sp[kMaxCombineK];
  const int64_t row = blockIdx.x;
  const int nvec = H / 8;
  // the norm weight is a parameter (no kernel writes it): fetched before waiting for the
  // predecessor, so the last phase does not wait for it
  uint4 wreg[kNormMaxVec];
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) wreg[j] = w[c];
  }
  pdl_wait();
  pdl_trigger();
  // the residual rows do not depend on the positions: their loads go out first
  uint4 rres[kNormMaxVec];
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) rres[j] = res[row * nvec + c];
  }
  for (int k = threadIdx.x; k < K; k += kThreads) sp[k] = pos[row * K + k];
  __syncthreads();
  float v[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int k0 = 0; k0 < K; k0 += 8) {
        int p[8];
        uint4 r[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          p[q] = k0 + q < K ? sp[k0 + q] : -1;
          r[q] = p[q] >= 0 ? *reinterpret_cast<const uint4*>(c3 + (int64_t)p[q] * H + c * 8)
                           : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (p[q] < 0) continue;
          float f[8];
          bf16x8_to_f32(r[q], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += f[e];
        }
      }
      float rr[8];
      bf16x8_to_f32(rres[j], rr);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[j][q] = bf16_round(bf16_round(acc[q]) + rr[q]);
        ss += v[j][q] * v[j][q];
      }
    }
  }
  const float tot = block_sum<kThreads>(ss, red);
  const float rstd = rsqrtf(tot / (float)H + eps);
  const float wb = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c < nvec) {
      res_out[row * nvec + c] = pack_bf16x8(v[j]);
      float wf[8], o[8];
      bf16x8_to_f32(wreg[j], wf);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = v[j][q] * rstd * (wf[q] + wb);
      y[row * nvec + c] = pack_bf16x8(o);
    }
  }
}

}  // namespace

int launch_combine_merge(const Workspace& ws, int64_t T, int K, int H, const CombineMerge& cm,
                         cudaStream_t st) {
  TW_CHECK_ARG(K > 0 && K <= kMaxCombineK, "combine_merge: need 0 < K <= %d", kMaxCombineK);
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kNormThreads * 8 * kNormMaxVec,
               "combine_merge: need H %% 8 == 0 and H <= %d", kNormThreads * 8 * kNormMaxVec);
  if (T == 0) return TW_OK;
  const RouteSum rs{ws.pos, ws.c3, K};
  if (norm_threads(H) == 128) {
    TW_LAUNCH((dual_norm_merge_kernel<128, true>), dim3((unsigned)T), dim3(128), 0, st,
              (const uint4*)cm.a, (const uint4*)nullptr, (const uint4*)cm.x,
              (const uint4*)cm.w1, (const uint4*)cm.w2, (const uint4*)cm.w3, H, cm.eps1,
              cm.eps2, cm.eps3, cm.scalar, (uint4*)cm.out, rs);
  } else {
    TW_LAUNCH((dual_norm_merge_kernel<256, true>), dim3((unsigned)T), dim3(256), 0, st,
              (const uint4*)cm.a, (const uint4*)nullptr, (const uint4*)cm.x,
              (const uint4*)cm.w1, (const uint4*)cm.w2, (const uint4*)cm.w3, H, cm.eps1,
              cm.eps2, cm.eps3, cm.scalar, (uint4*)cm.out, rs);
  }
  TW_CHECK_LAUNCH("dual_norm_merge_kernel");
  return TW_OK;
}

int launch_combine_norm(const Workspace& ws, int64_t T, int K, int H, const CombineNorm& cn,
                        cudaStream_t st) {
  TW_CHECK_ARG(K > 0 && K <= kMaxCombineK, "combine_norm: need 0 < K <= %d", kMaxCombineK);
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kNormThreads * 8 * kNormMaxVec,
               "combine_norm: need H %% 8 == 0 and H <= %d", kNormThreads * 8 * kNormMaxVec);
  if (T == 0) return TW_OK;
  if (norm_threads(H) == 128) {
    TW_LAUNCH(combine_norm_kernel<128>, dim3((unsigned)T), dim3(128), 0, st, H, K,
              (const int32_t*)ws.pos, (const __nv_bfloat16*)ws.c3, (const uint4*)cn.resid,
              (uint4*)cn.resid_out, (const uint4*)cn.w, cn.eps, (uint4*)cn.h);
  } else {
    TW_LAUNCH(combine_norm_kernel<256>, dim3((unsigned)T), dim3(256), 0, st, H, K,
              (const int32_t*)ws.pos, (const __nv_bfloat16*)ws.c3, (const uint4*)cn.resid,
              (uint4*)cn.resid_out, (const uint4*)cn.w, cn.eps, (uint4*)cn.h);
  }
  TW_CHECK_LAUNCH("combine_norm_kernel");
  return TW_OK;
}

}  // namespace tw

using namespace tw;

extern "C" int tw_dual_norm_merge(const void* a, const void* b, const void* x, const void* w1,
                                  const void* w2, const void* w3, int64_t T, int H, float eps1,
                                  float eps2, float eps3, float scalar, void* out,
                                  void* stream) {
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kNormThreads * 8 * kNormMaxVec,
               "dual_norm_merge: need H %% 8 == 0 and H <= %d", kNormThreads * 8 * kNormMaxVec);
  TW_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(x) && aligned16(w1) && aligned16(w2) &&
                   aligned16(w3) && aligned16(out),
               "dual_norm_merge: pointers must be 16-byte aligned");
  if (T == 0) return TW_OK;
  const RouteSum none{nullptr, nullptr, 0};
  if (norm_threads(H) == 128) {
    TW_LAUNCH((dual_norm_merge_kernel<128, false>), dim3((unsigned)T), dim3(128), 0,
              as_stream(stream), (const uint4*)a, (const uint4*)b, (const uint4*)x,
              (const uint4*)w1, (const uint4*)w2, (const uint4*)w3, H, eps1, eps2, eps3, scalar,
              (uint4*)out, none);
  } else {
    TW_LAUNCH((dual_norm_merge_kernel<256, false>), dim3((unsigned)T), dim3(256), 0,
              as_stream(stream), (const uint4*)a, (const uint4*)b, (const uint4*)x,
              (const uint4*)w1, (const uint4*)w2, (const uint4*)w3, H, eps1, eps2, eps3, scalar,
              (uint4*)out, none);
  }
  return TW_OK;
}

extern "C" int tw_rmsnorm(const void* x, const void* residual, void* residual_out,
                          const void* w, int64_t T, int H, float eps, float wb, void* y,
                          void* stream) {
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kNormThreads * 8 * kNormMaxVec,
               "rmsnorm: need H %% 8 == 0 and H <= %d", kNormThreads * 8 * kNormMaxVec);
  TW_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(y) &&
                   (!residual || aligned16(residual)) && (!residual_out || aligned16(residual_out)),
               "rmsnorm: pointers must be 16-byte aligned");
  TW_CHECK_ARG(!(residual_out && !residual), "rmsnorm: residual_out needs residual");
  if (T == 0) return TW_OK;
  if (norm_threads(H) == 128) {
    TW_LAUNCH(rmsnorm_kernel<128>, dim3((unsigned)T), dim3(128), 0, as_stream(stream),
              (const uint4*)x, (const uint4*)residual, (uint4*)residual_out, (const uint4*)w, H,
              eps, wb, (uint4*)y);
  } else {
    TW_LAUNCH(rmsnorm_kernel<256>, dim3((unsigned)T), dim3(256), 0, as_stream(stream),
              (const uint4*)x, (const uint4*)residual, (uint4*)residual_out, (const uint4*)w, H,
              eps, wb, (uint4*)y);
  }
  TW_CHECK_LAUNCH("rmsnorm_kernel");
  return TW_OK;
}

extern "C" int tw_router_norm_triple(const void* x, const void* ones, const void* rw,
                                     const void* scale, const void* sw, int64_t T, int H,
                                     float eps, float root, void* router_out, void* routed_out,
                                     void* shared_out, void* stream) {
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kNormThreads * 8 * kNormMaxVec,
               "router_norm_pair: need H %% 8 == 0 and H <= %d", kNormThreads * 8 * kNormMaxVec);
  TW_CHECK_ARG(aligned16(x) && aligned16(ones) && aligned16(rw) && aligned16(scale) &&
                   aligned16(router_out) && aligned16(routed_out),
               "router_norm_pair: pointers must be 16-byte aligned");
  TW_CHECK_ARG((sw == nullptr) == (shared_out == nullptr) &&
                   (sw == nullptr || (aligned16(sw) && aligned16(shared_out))),
               "router_norm_triple: shared weight and output come together, 16-byte aligned");
  TW_CHECK_ARG(eps > 0.f, "router_norm_pair: eps must be > 0");
  if (T == 0) return TW_OK;
  if (norm_threads(H) == 128) {
    TW_LAUNCH(norm_pair_kernel<128>, dim3((unsigned)T), dim3(128), 0, as_stream(stream),
              (const uint4*)x, (const uint4*)ones, (const uint4*)rw, (const uint4*)scale,
              (const uint4*)sw, H, eps, root, (uint4*)router_out, (uint4*)routed_out,
              (uint4*)shared_out);
  } else {
    TW_LAUNCH(norm_pair_kernel<256>, dim3((unsigned)T), dim3(256), 0, as_stream(stream),
              (const uint4*)x, (const uint4*)ones, (const uint4*)rw, (const uint4*)scale,
              (const uint4*)sw, H, eps, root, (uint4*)router_out, (uint4*)routed_out,
              (uint4*)shared_out);
  }
  TW_CHECK_LAUNCH("norm_pair_kernel");
  return TW_OK;
}

extern "C" int tw_router_norm_pair(const void* x, const void* ones, const void* rw,
                                   const void* scale, int64_t T, int H, float eps, float root,
                                   void* router_out, void* routed_out, void* stream) {
  return tw_router_norm_triple(x, ones, rw, scale, nullptr, T, H, eps, root, router_out,
                               routed_out, nullptr, stream);
}

// ---------------------------------------------------------------- shared-expert merge

// out = bf16(routed + shared), eight elements per thread.
__global__ void __launch_bounds__(256)
add_shared_kernel(const uint4* __restrict__ routed, const uint4* __restrict__ shared,
                  uint4* __restrict__ out, int64_t n8) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    float a[8], b[8];
    bf16x8_to_f32(routed[i], a);
    bf16x8_to_f32(shared[i], b);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      ow[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a[2 * k] + b[2 * k])) |
              ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a[2 * k + 1] + b[2 * k + 1]))
               << 16);
    out[i] = o;
  }
}

extern "C" int tw_add_shared(const void* routed, const void* shared, void* out, int64_t T, int H,
                             void* stream) {
  TW_CHECK_ARG(T >= 0 && H > 0 && H % 8 == 0, "add_shared: need H %% 8 == 0");
  TW_CHECK_ARG(aligned16(routed) && aligned16(shared) && aligned16(out),
               "add_shared: pointers must be 16-byte aligned");
  const int64_t n8 = T * (int64_t)H / 8;
  if (n8 == 0) return TW_OK;
  const int blocks = (int)std::min<int64_t>((n8 + 255) / 256, 1184);
  TW_LAUNCH(add_shared_kernel, dim3(blocks), dim3(256), 0, as_stream(stream),
            (const uint4*)routed, (const uint4*)shared, (uint4*)out, n8);
  TW_CHECK_LAUNCH("add_shared_kernel");
  return TW_OK;
}
