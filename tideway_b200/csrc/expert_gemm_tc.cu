// Slot-indirect SwiGLU expert FFN on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA, as one persistent kernel per call.
//
// Work items are (slot, weight tile) pairs: first every up tile (64 gate rows + the
// matching 64 up rows of w1), then every down tile (128 rows of w2); CTAs claim them from a
// device counter in that order.  Each item computes
//   D[weight rows, routes] = W[weight rows, K] . R[routes, K]^T
// with the weight tile as the M = 128 operand, streamed by a 3-D TMA whose outer
// coordinate is the slot id read from the device-side route grouping (so the kernel reads
// straight out of the fixed-address slot bank and stays valid inside a captured graph), and
// the slot's routes as the N operand (gathered input rows, or the SwiGLU activations).
// A down item's producer waits until every up item of its slot has published its
// activations (per-slot counter, release/acquire + async-proxy fence).
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0      producer: claims items, TMA weight tile + route rows per 64-element K
//               stage into a ring of 128-byte-swizzled shared-memory stages.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=16..256, K=16) into a
//               double-buffered TMEM accumulator and frees stages with tcgen05.commit.
//   warps 2-9   epilogue (two warps per TMEM lane quarter, alternate 16-column chunks):
//               tcgen05.ld; up tiles hold gate and up rows interleaved, so a lane
//               pair swaps values with one shuffle and writes bf16(silu(bf16 gate) * bf16 up);
//               down items write bf16(acc * route weight) with the weights staged in smem.
//
// Every wait is bounded; on a timeout the kernel records an error word, drains its
// outstanding copies and MMAs, frees TMEM and exits.
#include <algorithm>

#include "ffn_sched.cuh"

namespace tw {
namespace {

using namespace tc;

constexpr int kTcThreads = 320;   // warp 0 TMA, 1 MMA, 2-9 epilogue (two per TMEM lane quarter)
constexpr int kEpiThreads = 256;
constexpr int kBK = 64;            // K elements per TMA box (128-byte rows)
#ifndef TW_FFN_KB
#define TW_FFN_KB 4                // K boxes per pipeline stage
#endif
constexpr int kKBMax = TW_FFN_KB;
#ifndef TW_FFN_KROT
#define TW_FFN_KROT 1              // rotate each item's K order to decorrelate DRAM streams
#endif
constexpr int kSmemBudget = 216 * 1024;
constexpr int kWRows = 128;        // weight rows per tile = MMA M
constexpr int kRouteBox = 16;      // smallest route-row box

// Route rows are loaded as one box of R rows x kKB K boxes per stage, R the smallest of
// these heights that covers the chunk's routes (rows past the chunk are never multiplied).
constexpr int kRouteRowsN = 4;
__host__ __device__ constexpr int route_rows_nominal(int i) {
  return i == 0 ? 16 : i == 1 ? 64 : i == 2 ? 128 : 256;
}
// the tallest box is the route tile itself (16, 64, 160 or 256 rows)
template <int kNCap>
__host__ __device__ constexpr int route_rows(int i) {
  return route_rows_nominal(i) < kNCap ? route_rows_nominal(i) : kNCap;
}
__device__ __forceinline__ int route_box_index(int n) {
  return n <= 16 ? 0 : n <= 64 ? 1 : n <= 128 ? 2 : 3;
}

struct RouteMaps {
  CUtensorMap xg[kRouteRowsN];   // [K box][n][64] views of the gathered input rows
  CUtensorMap act[kRouteRowsN];  // [K box][n][64] views of the activations
};
constexpr int kWStageBytes = kWRows * 128;



template <int kNCap>
struct FfnSmem {
  static constexpr int kThreads = kTcThreads;
  static constexpr int kRBoxBytes = kNCap * 128;                 // route rows of one K box
  static constexpr int kBoxPair = kWStageBytes + kRBoxBytes;      // one K box of both operands
  // K boxes per stage: up to kKBMax while at least kMinStages stages fit (latency hiding needs
  // several loads in flight more than it needs large ones)
  // decode tiles: 4 stages; prefill tiles (MMA N >= 128): 3 stages of 2+ K boxes, which halves
  // the MMA thread's per-stage overhead next to 64-cycle MMAs
  static constexpr int kMinStages = kNCap <= 64 ? 4 : 3;
  static constexpr int kFit = kSmemBudget / (kMinStages * kBoxPair);
  static constexpr int kKB = kFit < 1 ? 1 : (kFit < kKBMax ? kFit : kKBMax);
  static constexpr int kStageBytes = kKB * kBoxPair;
  static constexpr int kStages = kSmemBudget / kStageBytes;
  static constexpr int kXchgOffset = kStages * kStageBytes;
  static constexpr int kXchgBytes = 1024;  // route weights of a down chunk (<= 256 floats)
  static constexpr int kBarOffset = kXchgOffset + kXchgBytes;
  static constexpr int kBytes = kBarOffset + 512 + 1024;
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kStages >= 2 && kBytes <= 227 * 1024, "shared memory budget");
  static_assert((2 * kStages + 4 + 2 * kRing + 2) * 8 + 16 + 12 * kRing <= 512, "barriers");
  static_assert(kRBoxBytes % 1024 == 0, "route box alignment");
};

// One launch per FFN: every (slot, up tile) item, then every (slot, down tile) item,
// claimed dynamically.  A down item's activations come from up items of the same slot
// (possibly on other CTAs): its producer waits on up_done before loading them.
template <int kNCap>
__global__ void __launch_bounds__(FfnSmem<kNCap>::kThreads, 1)
expert_ffn_tc_kernel(const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_w2,
                     const __grid_constant__ RouteMaps rm, FfnArgs a) {
  using L = FfnSmem<kNCap>;
  constexpr int kStages = L::kStages;
  constexpr int kKB = L::kKB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* wbuf = reinterpret_cast<float*>(smem + L::kXchgOffset);   // [kNCap] route weights
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;      // [2] accumulator ready
  uint64_t* tempty = tfull + 2;           // [2] accumulator drained
  uint64_t* ifull = tempty + 2;           // [kRing] item published
  uint64_t* iempty = ifull + kRing;       // [kRing] item consumed
  uint64_t* drain = iempty + kRing;
  uint64_t* esync = drain + 1;            // the four epilogue warps meet here (bounded waits)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(esync + 1);
  Item* ring = reinterpret_cast<Item*>(tmem_slot + 4);  // [kRing] claimed items

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiThreads);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&ifull[i], 1);
      mbar_init(&iempty[i], 1 + kEpiThreads);  // the MMA thread and every epilogue thread
    }
    mbar_init(drain, 1);
    mbar_init(esync, kEpiThreads);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_w2);
    for (int i = 0; i < kRouteRowsN; ++i) {
      prefetch_tmap(&rm.xg[i]);
      prefetch_tmap(&rm.act[i]);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the prologue above overlaps the predecessor; inputs are read from here on
  pdl_trigger();
  const int U = a.num_unique[0];
  int* err = a.err;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      Claimer claimer;
      for (uint32_t r = 0; ok; ++r) {
        const int e = r % kRing;
        if (!mbar_wait(&iempty[e], ((r / kRing) & 1) ^ 1, err)) break;
        Item item;
        if (!claim_item(a, U, claimer, item, err)) {
          ok = false;
          item.kind = -1;
        }
        ring[e] = item;
        mbar_arrive(&ifull[e]);
        if (item.kind < 0) break;
        const int slot = a.seg_slot[item.u];
        const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
        const int kbox = (item.kind == 0 ? a.H : a.I) / kBK;
        const int kst = (kbox + kKB - 1) / kKB;
        if (item.kind == 1) fence_proxy_async_global();  // activations came from other CTAs
        for (int pc = p0; ok && pc < p1; pc += kNCap) {
          const int n = min(kNCap, p1 - pc);
          const int ri = route_box_index(n);
          const CUtensorMap* tr = item.kind == 0 ? &rm.xg[ri] : &rm.act[ri];
          const int rot = k_rotation(item, kst);
          for (int kq = 0; kq < kst; ++kq, ++it) {
            const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err)) {
              ok = false;
              break;
            }
            uint8_t* W = smem + s * L::kStageBytes;
            uint8_t* R = W + kKB * kWStageBytes;
            // one TMA instruction each for the stage's weight tile (kKB K boxes x 128 rows)
            // and route rows (kKB K boxes x route_rows(ri) rows); K boxes past the end of a
            // row read as zeros and are not multiplied
            mbar_arrive_expect_tx(&full[s], kKB * (kWStageBytes + route_rows<kNCap>(ri) * 128));
            if (item.kind == 0)
              tma_load_5d(W, &tm_w1, &full[s], 0, 0, item.tile * 64, ks * kKB, slot);
            else
              tma_load_4d(W, &tm_w2, &full[s], 0, item.tile * kWRows, ks * kKB, slot);
            tma_load_3d(R, tr, &full[s], 0, pc, ks * kKB);
          }
        }
      }
      if (!ok) {  // let every load already issued land before the CTA can exit
        for (uint32_t j = (it >= kStages ? it - kStages : 0); j < it; ++j)
          mbar_wait(&full[j % kStages], (j / kStages) & 1, err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, c = 0;
      bool ok = true;
      for (uint32_t r = 0; ok; ++r) {
        const int e = r % kRing;
        if (!mbar_wait(&ifull[e], (r / kRing) & 1, err)) break;
        const Item item = ring[e];
        mbar_arrive(&iempty[e]);
        if (item.kind < 0) break;
        const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
        const int kbox = (item.kind == 0 ? a.H : a.I) / kBK;
        const int kst = (kbox + kKB - 1) / kKB;
        for (int pc = p0; ok && pc < p1; pc += kNCap, ++c) {
          const int n = min(kNCap, p1 - pc);
          const uint32_t idesc = idesc_bf16(kWRows, (n + 15) & ~15);
          const uint32_t rbox16 = (uint32_t)(route_rows<kNCap>(route_box_index(n)) * 128) >> 4;
          const int acc = c & 1;
          if (!mbar_wait(&tempty[acc], ((c >> 1) & 1) ^ 1, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(acc * 256);
          const int rot = k_rotation(item, kst);
          for (int kq = 0; kq < kst; ++kq, ++it) {
            const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
            const int s = it % kStages;
            if (!mbar_wait(&full[s], (it / kStages) & 1, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // descriptors built once per stage, constant offsets per MMA (keeps the issuing
            // thread ahead of the tensor pipe at small N)
            const uint64_t w_desc = umma_desc_sw128(smem_u32(smem + s * L::kStageBytes));
            const uint64_t r_desc = w_desc + (uint64_t)((kKB * kWStageBytes) >> 4);
            const int nkb = min(kKB, kbox - ks * kKB);
            if (nkb == kKB) {
#pragma unroll
              for (int j = 0; j < kKB * (kBK / 16); ++j) {
                const int kb = j / (kBK / 16), kk = j % (kBK / 16);
                mma_bf16(d, w_desc + (uint64_t)((kb * kWStageBytes + kk * 32) >> 4),
                         r_desc + (uint64_t)(kb * rbox16 + ((kk * 32) >> 4)), idesc,
                         (kq | j) != 0);
              }
            } else {
              for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                  mma_bf16(d, w_desc + (uint64_t)((kb * kWStageBytes + kk * 32) >> 4),
                           r_desc + (uint64_t)(kb * rbox16 + ((kk * 32) >> 4)), idesc,
                           (kq | kb | kk) != 0);
              }
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&tfull[acc]);
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-9)
    const int q = warp & 3;  // TMEM lane quarter: rows 32q .. 32q+31 of the weight tile
    const int colhalf = (warp - 2) >> 2;  // which 16-column chunks of a tile this warp takes
    const int etid = (warp - 2) * 32 + lane;
    const int row = q * 32 + lane;
    uint32_t c = 0, ephase = 0;
    bool ok = true;
    auto epilogue_sync = [&]() -> bool {  // all kEpiThreads epilogue threads, bounded
      mbar_arrive(esync);
      const bool r = mbar_wait(esync, ephase, err);
      ephase ^= 1;
      return r;
    };
    for (uint32_t r = 0; ok; ++r) {
      const int e = r % kRing;
      if (!mbar_wait(&ifull[e], (r / kRing) & 1, err)) break;
      const Item item = ring[e];
      mbar_arrive(&iempty[e]);
      if (item.kind < 0) break;
      const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
      for (int pc = p0; ok && pc < p1; pc += kNCap, ++c) {
        const int n = min(kNCap, p1 - pc);
        const int acc = c & 1;
        if (!mbar_wait(&tfull[acc], (c >> 1) & 1, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256);
        if (item.kind == 0) {
          // tile rows alternate gate and up of one intermediate index: row 2i is gate
          // j = tile*64 + i, row 2i+1 its up row, in neighbouring lanes.  The pair swaps values
          // with one shuffle; the gate lane writes even columns, the up lane odd ones.
          const int j = item.tile * 64 + (row >> 1);
          const int odd = row & 1;
          for (int cb = 16 * colhalf; cb < n; cb += 32) {
            float v[16];
            tmem_ld16(tb + cb, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
              const int col = cb + i;
              if ((i & 1) == odd && col < n) {
                const float g = bf16_round(odd ? other : v[i]);
                const float u = bf16_round(odd ? v[i] : other);
                a.act[(int64_t)(pc + col) * a.I + j] = __float2bfloat16_rn(silu_fast(g) * u);
              }
            }
          }
          // publish this warp's activation writes to the down tiles of this slot: every lane
          // orders its writes for the async proxy, the warp synchronises, lane 0 releases
          fence_proxy_async_global();
          __syncwarp();
          if (lane == 0) {
            const int target = up_target(a, item.u, kNCap, 8);
            if (atom_add_acq_rel(a.up_done + item.u * kDoneStride, 1) + 1 == target) {
              const int pos = atomicAdd(a.ready_tail, 1);
              st_release(a.ready_slots + pos, item.u);
            }
          }
        } else {
          // the chunk's route weights, staged once in shared memory for all epilogue warps
          if (!epilogue_sync()) {
            ok = false;
            break;
          }
          for (int t = etid; t < n; t += kEpiThreads) wbuf[t] = a.topk_w[a.perm[pc + t]];
          if (!epilogue_sync()) {
            ok = false;
            break;
          }
          const int h = item.tile * kWRows + row;
          for (int cb = 16 * colhalf; cb < n; cb += 32) {
            float v[16];
            tmem_ld16(tb + cb, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = cb + i;
              if (col < n)
                a.c3[(int64_t)(pc + col) * a.H + h] = __float2bfloat16_rn(v[i] * wbuf[col]);
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
  pdl_wait();
  pdl_trigger();
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

// Weight and route tensor maps whose boxes cover one pipeline stage (kKB K boxes), then the
// launch.  w1 is viewed 5-D as [S][K box][I rows][gate|up][64] so that one box holds the
// stage's 64 gate rows and their 64 up rows, interleaved, for kKB K boxes in the
// shared-memory order the MMA reads ([K box][g0 u0 g1 u1 ...][64]); w2 4-D as
// [S][K box][H rows][64]; the route rows
// 3-D as [K box][n][64], one map per route-box height.
template <int kNCap>
int launch_ffn(const __nv_bfloat16* w1, const __nv_bfloat16* w2, const Workspace& ws, int64_t n,
               const FfnArgs& args, int grid, cudaStream_t st) {
  using L = FfnSmem<kNCap>;
  const uint64_t H = args.H, I = args.I, S = args.num_slots;
  CUtensorMap m1, m2;
  {
    const uint64_t d[5] = {kBK, 2, I, H / kBK, S};
    const uint64_t sb[4] = {I * H * 2, H * 2, kBK * 2, 2 * I * H * 2};
    const uint32_t b[5] = {kBK, 2, 64, (uint32_t)L::kKB, 1};
    if (int rc = make_tmap_bf16(&m1, w1, 5, d, sb, b)) return rc;
  }
  {
    const uint64_t d[4] = {kBK, H, I / kBK, S};
    const uint64_t sb[3] = {I * 2, kBK * 2, H * I * 2};
    const uint32_t b[4] = {kBK, kWRows, (uint32_t)L::kKB, 1};
    if (int rc = make_tmap_bf16(&m2, w2, 4, d, sb, b)) return rc;
  }
  RouteMaps rm;
  for (int i = 0; i < kRouteRowsN; ++i) {
    const int rows = route_rows<kNCap>(i);
    {
      const uint64_t d[3] = {kBK, (uint64_t)n, H / kBK};
      const uint64_t sb[2] = {H * 2, kBK * 2};
      const uint32_t b[3] = {kBK, (uint32_t)rows, (uint32_t)L::kKB};
      if (int rc = make_tmap_bf16(&rm.xg[i], ws.xg, 3, d, sb, b)) return rc;
    }
    {
      const uint64_t d[3] = {kBK, (uint64_t)n, I / kBK};
      const uint64_t sb[2] = {I * 2, kBK * 2};
      const uint32_t b[3] = {kBK, (uint32_t)rows, (uint32_t)L::kKB};
      if (int rc = make_tmap_bf16(&rm.act[i], ws.act, 3, d, sb, b)) return rc;
    }
  }
  auto kern = expert_ffn_tc_kernel<kNCap>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    attr_set = true;
  }
  TW_LAUNCH(kern, dim3(grid), dim3(L::kThreads), L::kBytes, st, m1, m2, rm, args);
  TW_CHECK_LAUNCH("expert_ffn_tc_kernel");
  return TW_OK;
}

}  // namespace

int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (int rc = encoder(&enc)) return rc;
  if (rank < 2 || rank > 5) {
    set_error("make_tmap: rank %d unsupported", rank);
    return TW_ERR_INVALID;
  }
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = enc(map, dtype, rank, const_cast<void*>(base), gd, gs, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box) {
  return make_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_expert_ffn_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                         const __nv_bfloat16* w1, const __nv_bfloat16* w2, int64_t S,
                         const float* topk_w, const Workspace& ws, int64_t n, cudaStream_t st) {
  TW_CHECK_ARG(H % kWRows == 0 && I % 64 == 0, "tensor-core FFN: need H %% 128 == 0, I %% 64 == 0");
  TW_CHECK_ARG(n <= (int64_t)1 << 30 && S < (1 << 30), "tensor-core FFN: sizes out of range");
  const int sms = num_sms();
  {
    const int H8 = H / 8;
    const int64_t work = n * H8;
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, (int64_t)sms * 8);
    TW_LAUNCH(gather_rows_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st, 
        reinterpret_cast<const uint4*>(x), K, H8, ws.perm, ws.seg_start, ws.num_unique,
        reinterpret_cast<uint4*>(ws.xg));
    TW_CHECK_LAUNCH("gather_rows_kernel");
  }
  // the number of distinct slots is only known on the device: size the persistent grid
  // for the most work n routes can produce; idle CTAs find the item counter exhausted
  const int64_t max_u = std::min<int64_t>(n, S);
  FfnArgs fa{H, I, I / 64, H / kWRows, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm,
             topk_w, ws.act, ws.c3, ws.up_ctr, ws.down_ctr, ws.up_done, ws.ready_tail,
             ws.ready_slots, ws.err, nullptr, nullptr, S};
  const int grid = (int)std::min<int64_t>(max_u * (fa.tu + fa.td), sms);
  // route-tile capacity: a slot has at most T routes (one per token); for larger T the
  // expected routes per slot (T*K / S) decide between 160-route tiles (3 stages of 2 K boxes)
  // and 256-route tiles (fewer re-streamed weight tiles when slots get more than 160)
  if (T <= 16) {
    if (int rc = launch_ffn<16>(w1, w2, ws, n, fa, grid, st)) return rc;
  } else if (T <= 64) {
    if (int rc = launch_ffn<64>(w1, w2, ws, n, fa, grid, st)) return rc;
  } else if (T <= 160 || n <= 128 * S) {
    if (int rc = launch_ffn<160>(w1, w2, ws, n, fa, grid, st)) return rc;
  } else {
    if (int rc = launch_ffn<256>(w1, w2, ws, n, fa, grid, st)) return rc;
  }
  return TW_OK;
}

}  // namespace tw
