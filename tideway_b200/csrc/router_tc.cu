// Router logits for many tokens on the tensor cores: logits[T, E] (fp32) = x[T, H] . W[E, H]^T.
//
// One CTA per 128-token tile: the tile's token rows are the M = 128 operand, all E <= 256
// router rows the N operand, fp32 accumulation in TMEM (bf16 products are exact, so this is
// the fp32 dot product up to summation order).  Warp 0 streams 64-element K boxes of both
// operands by TMA into a ring of stages, warp 1 issues the MMAs, then all four warps read the
// accumulator back (lane = token) and store the logits.  Every wait is bounded.
#include <algorithm>

#include "tc_common.cuh"

namespace tw {
namespace {

using namespace tc;

constexpr int kRtThreads = 128;
constexpr int kRtBK = 64;
constexpr int kRtStages = 4;

template <int kN>
struct RouterSmem {
  static constexpr int kA = 128 * 128;        // 128 token rows x 64 bf16
  static constexpr int kB = kN * 128;         // kN router rows x 64 bf16
  static constexpr int kStage = kA + kB;
  static constexpr int kBarOffset = kRtStages * kStage;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
  static constexpr int kTmemCols = kN <= 32 ? 32 : kN <= 64 ? 64 : kN <= 128 ? 128 : 256;
  static_assert(kStage % 1024 == 0 && kBytes <= 227 * 1024, "router smem");
};

template <int kN>
__global__ void __launch_bounds__(kRtThreads, 1)
router_logits_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_w, int64_t T, int H, int E,
                        float* __restrict__ logits, int* err) {
  using L = RouterSmem<kN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kRtStages;
  uint64_t* done = empty + kRtStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();
  const int nk = H / kRtBK;
  const int t0 = blockIdx.x * 128;
  if (warp == 0 && lane == 0) {
    int kb = 0;
    for (; kb < nk; ++kb) {
      const int s = kb % kRtStages;
      if (!mbar_wait(&empty[s], ((kb / kRtStages) & 1) ^ 1, err)) break;
      uint8_t* A = smem + s * L::kStage;
      mbar_arrive_expect_tx(&full[s], L::kStage);
      tma_load_2d(A, &tm_x, &full[s], kb * kRtBK, t0);
      tma_load_2d(A + L::kA, &tm_w, &full[s], kb * kRtBK, 0);
    }
    if (kb < nk) {  // let every load already issued land before the CTA can exit
      for (int j = std::max(0, kb - kRtStages); j < kb; ++j)
        mbar_wait(&full[j % kRtStages], (j / kRtStages) & 1, err);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_bf16(128, kN);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kRtStages;
      if (!mbar_wait(&full[s], (kb / kRtStages) & 1, err)) break;
      tc_fence_after();
      const uint64_t a_desc = umma_desc_sw128(smem_u32(smem + s * L::kStage));
      const uint64_t b_desc = a_desc + (uint64_t)(L::kA >> 4);
#pragma unroll
      for (int kk = 0; kk < kRtBK / 16; ++kk)
        mma_bf16(tmem, a_desc + (uint64_t)((kk * 32) >> 4), b_desc + (uint64_t)((kk * 32) >> 4),
                 idesc, (kb | kk) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(done);  // also when stopped early: the epilogue waits on it, bounded
  }
  // epilogue: lane = token row of this warp's TMEM quarter
  if (mbar_wait(done, 0, err) && *reinterpret_cast<volatile int*>(err) == 0) {
    tc_fence_after();
    const int64_t t = t0 + warp * 32 + lane;
    const uint32_t tb = tmem + ((uint32_t)(warp * 32) << 16);
    const bool vec = (E & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    for (int c = 0; c < kN; c += 16) {
      float v[16];
      tmem_ld16(tb + c, v);
      if (t < T) {
        float* dst = logits + t * E + c;
        if (c + 16 <= E && vec) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
          for (int i = 0; i < 16 && c + i < E; ++i) dst[i] = v[i];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// Error word of the router kernel: one per device, zeroed before each launch (a timed-out
// wait sets it; the launch's other waits then return early).
__device__ int g_router_err;

int router_err_word(int** out) {
  static int* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("router_logits: no usable current device");
    return TW_ERR_CUDA;
  }
  if (addr[dev] == nullptr &&
      cudaGetSymbolAddress(reinterpret_cast<void**>(&addr[dev]), g_router_err) != cudaSuccess) {
    set_error("router_logits: cudaGetSymbolAddress failed");
    return TW_ERR_CUDA;
  }
  *out = addr[dev];
  return TW_OK;
}

template <int kN>
int launch_router_tc(const void* x, const void* w, int64_t T, int H, int E, float* logits,
                     cudaStream_t st) {
  using L = RouterSmem<kN>;
  CUtensorMap mx, mw;
  {
    const uint64_t d[2] = {(uint64_t)H, (uint64_t)T};
    const uint64_t s[1] = {(uint64_t)H * 2};
    const uint32_t b[2] = {kRtBK, 128};
    if (int rc = make_tmap_bf16(&mx, x, 2, d, s, b)) return rc;
  }
  {  // kN rows per box: router rows past E read as zeros
    const uint64_t d[2] = {(uint64_t)H, (uint64_t)E};
    const uint64_t s[1] = {(uint64_t)H * 2};
    const uint32_t b[2] = {kRtBK, (uint32_t)kN};
    if (int rc = make_tmap_bf16(&mw, w, 2, d, s, b)) return rc;
  }
  int* err = nullptr;
  if (int rc = router_err_word(&err)) return rc;
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) {
    set_error("router_logits: cudaMemsetAsync failed");
    return TW_ERR_CUDA;
  }
  auto kern = router_logits_tc_kernel<kN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    attr_set = true;
  }
  const unsigned tiles = (unsigned)((T + 127) / 128);
  TW_LAUNCH(kern, dim3(tiles), dim3(kRtThreads), L::kBytes, st, mx, mw, T, H, E, logits, err);
  TW_CHECK_LAUNCH("router_logits_tc_kernel");
  return TW_OK;
}

}  // namespace

// Enqueues the tensor-core router GEMM; the caller checks the shape first
// (router_logits_tc_ok).
bool router_logits_tc_ok(int64_t T, int H, int E) {
  return T >= 128 && H % kRtBK == 0 && E >= 1 && E <= 256 && T < ((int64_t)1 << 31) - 256;
}

int launch_router_logits_tc(const void* x, const void* w, int64_t T, int H, int E, float* logits,
                            cudaStream_t st) {
  const int n = (E + 15) & ~15;
  if (n <= 64) return launch_router_tc<64>(x, w, T, H, E, logits, st);
  if (n <= 128) return launch_router_tc<128>(x, w, T, H, E, logits, st);
  return launch_router_tc<256>(x, w, T, H, E, logits, st);
}

}  // namespace tw
