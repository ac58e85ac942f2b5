// Router logits for many tokens on the tensor cores: logits[T, E] (fp32) = x[T, H] . W[E, H]^T.
//
// Per 128-token tile, a thread-block cluster of ksplit CTAs (1, 2, 4 or 8, so that a few
// tiles still fill the GPU), each over a contiguous slice of the K boxes: the tile's token
// rows are the M = 128 operand, all E <= 256 router rows the N operand, fp32 accumulation in
// TMEM (bf16 products are exact, so this is the fp32 dot product up to summation order).
// Warp 0 streams 64-element K boxes of both operands by TMA into a ring of stages, warp 1
// issues the MMAs, then all four warps read the accumulator back (lane = token).  With one
// CTA per tile they store the logits; with a cluster each CTA parks its fp32 partial in its
// own shared memory and, after a cluster barrier, CTA r sums rows [r * 128 / ksplit, ...) of
// every CTA's partial in rank order (fixed order: deterministic) through distributed shared
// memory and stores them.  Every mbarrier wait is bounded; both cluster barriers are reached
// by every thread unconditionally, so none can wait on a CTA that left early.
#include <algorithm>

#include "tc_common.cuh"

namespace tw {

int num_sms();  // moe_ffn.cu

namespace {

using namespace tc;

constexpr int kRtThreads = 128;
constexpr int kRtBK = 64;
constexpr int kRtStages = 3;  // 96 KB of stages at kN = 128: two CTAs fit on an SM

template <int kN>
struct RouterSmem {
  static constexpr int kA = 128 * 128;        // 128 token rows x 64 bf16
  static constexpr int kB = kN * 128;         // kN router rows x 64 bf16
  static constexpr int kStage = kA + kB;
  static constexpr int kBarOffset = kRtStages * kStage;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
  static constexpr int kTmemCols = kN <= 32 ? 32 : kN <= 64 ? 64 : kN <= 128 ? 128 : 256;
  // a split-K partial, [128][kN + 4] fp32 (rows padded against bank conflicts), reuses the
  // stage ring once every MMA has completed
  static constexpr int kRedStride = kN + 4;
  static_assert(kStage % 1024 == 0 && kBytes <= 227 * 1024, "router smem");
  static_assert(128 * kRedStride * 4 <= kBarOffset, "router split-K partial");
};

template <int kN>
__global__ void __launch_bounds__(kRtThreads, 1)
router_logits_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_w, int64_t T, int H, int E,
                        float* __restrict__ logits, int* err, int ksplit) {
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
  const int rank = (int)(blockIdx.x % (unsigned)ksplit);  // cluster rank: clusters run along x
  const int t0 = (int)(blockIdx.x / (unsigned)ksplit) * 128;
  const int kb0 = rank * nk / ksplit, nkb = (rank + 1) * nk / ksplit - kb0;  // >= 1 K box
  if (warp == 0 && lane == 0) {
    int j = 0;
    for (; j < nkb; ++j) {
      const int s = j % kRtStages;
      if (!mbar_wait(&empty[s], ((j / kRtStages) & 1) ^ 1, err)) break;
      uint8_t* A = smem + s * L::kStage;
      mbar_arrive_expect_tx(&full[s], L::kStage);
      tma_load_2d(A, &tm_x, &full[s], (kb0 + j) * kRtBK, t0);
      tma_load_2d(A + L::kA, &tm_w, &full[s], (kb0 + j) * kRtBK, 0);
    }
    if (j < nkb) {  // let every load already issued land before the CTA can exit
      for (int i = std::max(0, j - kRtStages); i < j; ++i)
        mbar_drain(&full[i % kRtStages], (i / kRtStages) & 1, err);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_bf16(128, kN);
    for (int j = 0; j < nkb; ++j) {
      const int s = j % kRtStages;
      if (!mbar_wait(&full[s], (j / kRtStages) & 1, err)) break;
      tc_fence_after();
      const uint64_t a_desc = umma_desc_sw128(smem_u32(smem + s * L::kStage));
      const uint64_t b_desc = a_desc + (uint64_t)(L::kA >> 4);
#pragma unroll
      for (int kk = 0; kk < kRtBK / 16; ++kk)
        mma_bf16(tmem, a_desc + (uint64_t)((kk * 32) >> 4), b_desc + (uint64_t)((kk * 32) >> 4),
                 idesc, (j | kk) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(done);  // also when stopped early: the epilogue waits on it, bounded
  }
  __syncwarp();
  // epilogue: lane = token row of this warp's TMEM quarter
  // a drain: the MMAs issued (all of them, or those before an early stop) complete before
  // TMEM is read or freed
  const bool good =
      warp_all(mbar_drain(done, 0, err) && *reinterpret_cast<volatile int*>(err) == 0);
  const bool vec = (E & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  const uint32_t tb = tmem + ((uint32_t)(warp * 32) << 16);
  if (ksplit == 1) {
    if (good) {
      tc_fence_after();
      const int64_t t = t0 + warp * 32 + lane;
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
  } else {
    // every MMA has completed (done), so every stage's loads have landed: the ring is free
    float* red = reinterpret_cast<float*>(smem);
    if (good) {
      tc_fence_after();
      float* row = red + (warp * 32 + lane) * L::kRedStride;
      for (int c = 0; c < kN; c += 16) {
        float v[16];
        tmem_ld16(tb + c, v);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(row + c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
    cluster_sync();  // every partial is in place
    if (good && *reinterpret_cast<volatile int*>(err) == 0) {
      const int rows = 128 / ksplit, r0 = rank * rows;
      const uint32_t base = smem_u32(red);
      for (int idx = threadIdx.x; idx < rows * (kN / 4); idx += kRtThreads) {
        const int r = r0 + idx / (kN / 4), c = (idx % (kN / 4)) * 4;
        const uint32_t off = (uint32_t)((r * L::kRedStride + c) * 4);
        // every rank's partial first (all remote loads in flight), then the fixed-order sum
        float4 p[8];
#pragma unroll
        for (int src = 0; src < 8; ++src)
          if (src < ksplit) p[src] = ld_cluster_f4(cluster_map(base + off, (uint32_t)src));
        float4 acc = p[0];
#pragma unroll
        for (int src = 1; src < 8; ++src) {
          if (src < ksplit) {
            acc.x += p[src].x;
            acc.y += p[src].y;
            acc.z += p[src].z;
            acc.w += p[src].w;
          }
        }
        const int64_t t = t0 + r;
        if (t < T && c < E) {
          float* dst = logits + t * E + c;
          if (c + 4 <= E && vec) {
            *reinterpret_cast<float4*>(dst) = acc;
          } else {
            dst[0] = acc.x;
            if (c + 1 < E) dst[1] = acc.y;
            if (c + 2 < E) dst[2] = acc.z;
            if (c + 3 < E) dst[3] = acc.w;
          }
        }
      }
    }
    cluster_sync();  // no CTA leaves while a peer may still read its partial
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
  // the dynamic shared-memory limit is a per-device attribute: raise it once per device
  static bool attr_set[kMaxAttrDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxAttrDevices || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (dev >= 0 && dev < kMaxAttrDevices) attr_set[dev] = true;
  }
  const unsigned tiles = (unsigned)((T + 127) / 128);
  // split K over a cluster when few tiles would leave most SMs idle, and only as far as all
  // of the launch's clusters can be resident at once (clusters are placed within a GPC)
  const int nk = H / kRtBK;
  static int resident[9] = {0};  // cluster size -> clusters resident at once (0 = unknown)
  auto clusters_resident = [&](int c) -> int {
    if (resident[c] == 0) {
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)c;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(c * 16));
      cfg.blockDim = dim3(kRtThreads);
      cfg.dynamicSmemBytes = L::kBytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();  // not fatal: no split at this size
        nc = -1;
      }
      resident[c] = nc;
    }
    return resident[c];
  };
  int ksplit = 1;
  for (int c : {8, 4, 2}) {
    if ((int64_t)tiles * c <= 2 * (int64_t)num_sms() && c <= nk &&
        (int64_t)tiles <= clusters_resident(c)) {
      ksplit = c;
      break;
    }
  }
  if (ksplit == 1) {
    TW_LAUNCH(kern, dim3(tiles), dim3(kRtThreads), L::kBytes, st, mx, mw, T, H, E, logits, err,
              1);
  } else {
    TW_LAUNCH_CLUSTER(kern, dim3(tiles * ksplit), dim3(kRtThreads), L::kBytes, st,
                      (unsigned)ksplit, mx, mw, T, H, E, logits, err, ksplit);
  }
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
