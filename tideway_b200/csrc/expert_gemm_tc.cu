// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// Both projections of the SwiGLU expert run as one persistent kernel shape:
//   D[routes, weight rows] = A[routes, K] . B[weight rows, K]^T
// A is the slot's routes (gathered input rows for the up projection, SwiGLU activations
// for the down projection), up to 2 x 128 routes per MMA pass; B is a 128-row tile of the
// slot's weights, loaded through a 3-D tensor map whose outer coordinate is the slot id
// read from the device-side route grouping, so the kernel streams straight out of the
// fixed-address slot bank and stays valid inside a captured graph.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: weight tile + route rows per 64-element K stage into a
//               ring of shared-memory stages (128-byte swizzle), mbarrier tx counts.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=128, K=16) into a
//               double-buffered TMEM accumulator and frees stages with tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld the accumulator rows (one route per TMEM lane) and
//               write bf16(silu(bf16 gate) * bf16 up) (up projection, gate and up rows
//               interleaved in the tile) or bf16(acc * route weight) (down projection).
//
// Every wait is bounded; on a timeout the kernel records an error word, drains and exits.
#include <algorithm>

#include "moe_common.cuh"
#include "tc_common.cuh"

namespace tw {
namespace {

using namespace tc;

constexpr int kTcThreads = 192;
constexpr int kBK = 64;                  // K elements per stage (128-byte rows)
constexpr int kTileRows = 128;           // weight rows per tile (MMA N)
constexpr int kRouteBox = 16;            // route rows per TMA box
constexpr int kRoutesPerMma = 128;       // MMA M
constexpr int kWStageBytes = kTileRows * 128;
constexpr int kRStageBytes = kRoutesPerMma * 128;

struct TcArgs {
  int mode;                 // 0: up projection (SwiGLU), 1: down projection (x route weight)
  int K;                    // reduction length
  int I, H;
  int tiles_per_expert;     // weight tiles per slot
  const int32_t* num_unique;
  const int32_t* seg_start;
  const int32_t* seg_slot;
  const int32_t* perm;
  const float* topk_w;
  __nv_bfloat16* out;       // act [n, I] (up) or c3 [n, H] (down), position order
  int* err;
};

template <int kMTiles, int kStages>
struct Smem {
  static constexpr int kStageBytes = kWStageBytes + kMTiles * kRStageBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
  static_assert(2 * kStages + 5 <= 30, "barrier area");
};

// Persistent work schedule shared by all roles: (item over slots x tiles, route chunk).
struct Sched {
  int total, tpe;
  __device__ Sched(const TcArgs& a) : total(a.num_unique[0] * a.tiles_per_expert),
                                      tpe(a.tiles_per_expert) {}
};

template <int kMTiles, int kStages>
__global__ void __launch_bounds__(kTcThreads, 1)
expert_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmR, TcArgs a) {
  using L = Smem<kMTiles, kStages>;
  constexpr int kChunk = kMTiles * kRoutesPerMma;  // routes per weight pass
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;   // [2] accumulator ready
  uint64_t* tempty = tfull + 2;        // [2] accumulator drained
  uint64_t* drain = tempty + 2;         // MMA completion before TMEM release
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmR);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const Sched sch(a);
  const int kst = a.K / kBK;
  int* err = a.err;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < sch.total; item += gridDim.x) {
        const int u = item / sch.tpe, tile = item % sch.tpe;
        const int slot = a.seg_slot[u];
        const int p0 = a.seg_start[u], p1 = a.seg_start[u + 1];
        for (int pc = p0; ok && pc < p1; pc += kChunk) {
          const int n = min(kChunk, p1 - pc);
          const int nbox = (n + kRouteBox - 1) / kRouteBox;
          for (int ks = 0; ks < kst; ++ks, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err)) {
              ok = false;
              break;
            }
            uint8_t* W = smem + s * L::kStageBytes;
            uint8_t* R = W + kWStageBytes;
            mbar_arrive_expect_tx(&full[s], kWStageBytes + nbox * kRouteBox * 128);
            const int k0 = ks * kBK;
            if (a.mode == 0) {
              // 64 gate rows then the matching 64 up rows of this tile
              tma_load_3d(W, &tmW, &full[s], k0, tile * 64, slot);
              tma_load_3d(W + kWStageBytes / 2, &tmW, &full[s], k0, a.I + tile * 64, slot);
            } else {
              tma_load_3d(W, &tmW, &full[s], k0, tile * kTileRows, slot);
            }
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(R + b * kRouteBox * 128, &tmR, &full[s], k0, pc + b * kRouteBox);
          }
        }
      }
      // drain: every stage this thread filled must have landed before the CTA exits
      if (!ok) {
        for (uint32_t j = (it >= kStages ? it - kStages : 0); j < it; ++j)
          mbar_wait(&full[j % kStages], (j / kStages) & 1, err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, c = 0;
      bool ok = true;
      const uint32_t idesc = idesc_bf16(kRoutesPerMma, kTileRows);
      for (int item = blockIdx.x; ok && item < sch.total; item += gridDim.x) {
        const int u = item / sch.tpe;
        const int p0 = a.seg_start[u], p1 = a.seg_start[u + 1];
        for (int pc = p0; ok && pc < p1; pc += kChunk, ++c) {
          const int n = min(kChunk, p1 - pc);
          const int acc = c & 1;
          if (!mbar_wait(&tempty[acc], ((c >> 1) & 1) ^ 1, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ks = 0; ks < kst; ++ks, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&full[s], (it / kStages) & 1, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t w_addr = smem_u32(smem + s * L::kStageBytes);
            const uint32_t r_addr = w_addr + kWStageBytes;
#pragma unroll
            for (int m = 0; m < kMTiles; ++m) {
              if (m * kRoutesPerMma >= n) break;
              const uint32_t d = tmem + (uint32_t)((acc * kMTiles + m) * kTileRows);
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                mma_bf16(d, umma_desc_sw128(r_addr + m * kRStageBytes + kk * 32),
                         umma_desc_sw128(w_addr + kk * 32), idesc, (ks | kk) != 0);
              }
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&tfull[acc]);
        }
      }
      // every MMA this thread issued has finished before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t c = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < sch.total; item += gridDim.x) {
      const int u = item / sch.tpe, tile = item % sch.tpe;
      const int p0 = a.seg_start[u], p1 = a.seg_start[u + 1];
      for (int pc = p0; ok && pc < p1; pc += kChunk, ++c) {
        const int n = min(kChunk, p1 - pc);
        const int acc = c & 1;
        if (!mbar_wait(&tfull[acc], (c >> 1) & 1, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int m = 0; m < kMTiles; ++m) {
          const int r0 = m * kRoutesPerMma + q * 32;  // first route row of this warp
          if (r0 >= n) continue;                       // warp-uniform
          const int r = r0 + lane;
          const bool valid = r < n;
          const int p = pc + r;
          const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) +
                              (uint32_t)((acc * kMTiles + m) * kTileRows);
          if (a.mode == 0) {
            __nv_bfloat16* dst = a.out + (int64_t)p * a.I + tile * 64;
#pragma unroll 1
            for (int cb = 0; cb < 64; cb += 16) {
              float g[16], up[16];
              tmem_ld16(tb + cb, g);
              tmem_ld16(tb + 64 + cb, up);
              uint32_t pk[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float g0 = bf16_round(g[2 * i]), g1 = bf16_round(g[2 * i + 1]);
                const float u0 = bf16_round(up[2 * i]), u1 = bf16_round(up[2 * i + 1]);
                const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(silu_f(g0) * u0));
                const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(silu_f(g1) * u1));
                pk[i] = lo | (hi << 16);
              }
              if (valid) {
                uint4* d4 = reinterpret_cast<uint4*>(dst + cb);
                d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
              }
            }
          } else {
            const float w = valid ? a.topk_w[a.perm[p]] : 0.f;
            __nv_bfloat16* dst = a.out + (int64_t)p * a.H + tile * kTileRows;
#pragma unroll 1
            for (int cb = 0; cb < kTileRows; cb += 16) {
              float v[16];
              tmem_ld16(tb + cb, v);
              uint32_t pk[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i] * w));
                const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1] * w));
                pk[i] = lo | (hi << 16);
              }
              if (valid) {
                uint4* d4 = reinterpret_cast<uint4*>(dst + cb);
                d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Gather the input row of every grouped route: xg[p] = x[perm[p] / K].
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint4* __restrict__ x, int K, int H8, const int32_t* __restrict__ perm,
                   const int32_t* __restrict__ seg_start, const int32_t* __restrict__ num_unique,
                   uint4* __restrict__ xg) {
  const int used = seg_start[num_unique[0]];
  const int64_t total = (int64_t)used * H8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / H8, c = i % H8;
    xg[i] = x[(int64_t)(perm[p] / K) * H8 + c];
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      set_error("cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
      return TW_ERR_CUDA;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *out = g_encode;
  return TW_OK;
}

template <int kMTiles, int kStages>
int launch_gemm(const CUtensorMap& tw_, const CUtensorMap& tr, const TcArgs& args, int grid,
                cudaStream_t st) {
  using L = Smem<kMTiles, kStages>;
  auto kern = expert_gemm_tc_kernel<kMTiles, kStages>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    attr_set = true;
  }
  kern<<<grid, kTcThreads, L::kBytes, st>>>(tw_, tr, args);
  TW_CHECK_LAUNCH("expert_gemm_tc_kernel");
  return TW_OK;
}

}  // namespace

int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (int rc = encoder(&enc)) return rc;
  cuuint64_t gd[3];
  cuuint64_t gs[2];
  cuuint32_t bx[3], es[3];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gd, gs,
                   bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

int launch_expert_ffn_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                         const __nv_bfloat16* w1, const __nv_bfloat16* w2, int64_t S,
                         const float* topk_w, const Workspace& ws, int64_t n, cudaStream_t st) {
  TW_CHECK_ARG(H % 128 == 0 && I % 64 == 0, "tensor-core FFN: need H %% 128 == 0, I %% 64 == 0");
  TW_CHECK_ARG(n <= (int64_t)1 << 30 && S < (1 << 30), "tensor-core FFN: sizes out of range");
  // tensor maps: weight banks (3-D, slot outermost) and the position-ordered route rows
  CUtensorMap m_w1, m_w2, m_xg, m_act;
  {
    const uint64_t d[3] = {(uint64_t)H, (uint64_t)(2 * I), (uint64_t)S};
    const uint64_t s[2] = {(uint64_t)H * 2, (uint64_t)(2 * I) * H * 2};
    const uint32_t b[3] = {kBK, 64, 1};
    if (int rc = make_tmap_bf16(&m_w1, w1, 3, d, s, b)) return rc;
  }
  {
    const uint64_t d[3] = {(uint64_t)I, (uint64_t)H, (uint64_t)S};
    const uint64_t s[2] = {(uint64_t)I * 2, (uint64_t)H * I * 2};
    const uint32_t b[3] = {kBK, kTileRows, 1};
    if (int rc = make_tmap_bf16(&m_w2, w2, 3, d, s, b)) return rc;
  }
  {
    const uint64_t d[2] = {(uint64_t)H, (uint64_t)n};
    const uint64_t s[1] = {(uint64_t)H * 2};
    const uint32_t b[2] = {kBK, kRouteBox};
    if (int rc = make_tmap_bf16(&m_xg, ws.xg, 2, d, s, b)) return rc;
  }
  {
    const uint64_t d[2] = {(uint64_t)I, (uint64_t)n};
    const uint64_t s[1] = {(uint64_t)I * 2};
    const uint32_t b[2] = {kBK, kRouteBox};
    if (int rc = make_tmap_bf16(&m_act, ws.act, 2, d, s, b)) return rc;
  }
  const int sms = num_sms();
  {
    const int H8 = H / 8;
    const int64_t work = n * H8;
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, (int64_t)sms * 8);
    gather_rows_kernel<<<blocks > 0 ? blocks : 1, 256, 0, st>>>(
        reinterpret_cast<const uint4*>(x), K, H8, ws.perm, ws.seg_start, ws.num_unique,
        reinterpret_cast<uint4*>(ws.xg));
    TW_CHECK_LAUNCH("gather_rows_kernel");
  }
  // the number of distinct slots is only known on the device: size the persistent grid
  // for the worst case it can reach with n routes
  const int64_t max_u = std::min<int64_t>(n, S);
  TcArgs up{0, H, I, H, I / 64, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm, topk_w,
            ws.act, ws.err};
  TcArgs dn{1, I, I, H, H / kTileRows, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm,
            topk_w, ws.c3, ws.err};
  const int g_up = (int)std::min<int64_t>(max_u * up.tiles_per_expert, sms);
  const int g_dn = (int)std::min<int64_t>(max_u * dn.tiles_per_expert, sms);
  if (T <= kRoutesPerMma) {  // every slot has <= T <= 128 routes: one M tile, deeper ring
    if (int rc = launch_gemm<1, 6>(m_w1, m_xg, up, g_up, st)) return rc;
    if (int rc = launch_gemm<1, 6>(m_w2, m_act, dn, g_dn, st)) return rc;
  } else {
    if (int rc = launch_gemm<2, 4>(m_w1, m_xg, up, g_up, st)) return rc;
    if (int rc = launch_gemm<2, 4>(m_w2, m_act, dn, g_dn, st)) return rc;
  }
  return TW_OK;
}

}  // namespace tw
