// Shared helpers for the tideway_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "tideway_b200.h"

namespace tw {

// ---------------------------------------------------------------- error reporting

void set_error(const char* fmt, ...);

#define TW_CHECK_ARG(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      ::tw::set_error(__VA_ARGS__);             \
      return TW_ERR_INVALID;                    \
    }                                           \
  } while (0)

#define TW_CHECK_LAUNCH(what)                                                     \
  do {                                                                            \
    cudaError_t e_ = cudaGetLastError();                                          \
    if (e_ != cudaSuccess) {                                                      \
      ::tw::set_error("%s: %s", what, cudaGetErrorString(e_));                    \
      return TW_ERR_CUDA;                                                         \
    }                                                                             \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---------------------------------------------------------------- numerics

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Unpack 8 bf16 held in a uint4 into fp32.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// SiLU with the fast exponential and divide (a few ulp of fp32; the result is rounded to
// bf16 right after, which is coarser by four orders of magnitude).
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// The other gate activations of the expert FFN, fp32 (activation codes 1 and 2; 0 is SiLU):
// GELU, g/2 (1 + erf(g / sqrt 2)), and its tanh form, g/2 (1 + tanh(sqrt(2/pi) (g +
// 0.044715 g^3))) -- the published forms of Hendrycks and Gimpel (2016).
__device__ __forceinline__ float gelu_act(int act, float g) {
  if (act == 1) return 0.5f * g * (1.0f + erff(g * 0.7071067811865476f));
  return 0.5f * g * (1.0f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g)));
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------- programmatic launch

// Kernels of a decode step are launched with programmatic stream serialization: a kernel
// may be scheduled while its predecessor drains, runs its prologue, and blocks in
// pdl_wait() until the predecessor has completed and its writes are visible.  Every kernel
// calls pdl_wait() before its first global-memory access and then pdl_trigger() so that its
// own successor can be scheduled early.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// The same with thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t st, unsigned cluster_x, Args... args) {
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Devices whose per-function attributes the launchers track.
constexpr int kMaxAttrDevices = 64;

// Launch with programmatic stream serialization; returns TW_ERR_CUDA on a launch error.
#define TW_LAUNCH(...)                                                         \
  do {                                                                         \
    cudaError_t le_ = ::tw::launch_pdl(__VA_ARGS__);                           \
    if (le_ != cudaSuccess) {                                                  \
      ::tw::set_error("kernel launch failed: %s", cudaGetErrorString(le_));    \
      return TW_ERR_CUDA;                                                      \
    }                                                                          \
  } while (0)

#define TW_LAUNCH_CLUSTER(...)                                                 \
  do {                                                                         \
    cudaError_t le_ = ::tw::launch_pdl_cluster(__VA_ARGS__);                   \
    if (le_ != cudaSuccess) {                                                  \
      ::tw::set_error("kernel launch failed: %s", cudaGetErrorString(le_));    \
      return TW_ERR_CUDA;                                                      \
    }                                                                          \
  } while (0)

}  // namespace tw
