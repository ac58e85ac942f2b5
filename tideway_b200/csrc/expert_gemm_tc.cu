// Slot-indirect SwiGLU expert FFN on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA, as one persistent kernel per call.
//
// Work items are (route segment, weight tile) pairs: first every up tile (64 gate rows + the
// matching 64 up rows of w1), then every down tile (128 rows of w2); CTAs claim them from a
// device counter in that order.  With large route tiles (160 or 256 routes) an item takes
// two neighbouring weight tiles that share each route load.  Each item computes
//   D[weight rows, routes] = W[weight rows, K] . R[routes, K]^T
// with the weight tile as the M = 128 operand, streamed by a 3-D TMA whose outer
// coordinate is the slot id read from the device-side route grouping (so the kernel reads
// straight out of the fixed-address slot bank and stays valid inside a captured graph), and
// the slot's routes as the N operand (gathered input rows, or the SwiGLU activations).
// A down item's producer waits until every up item of its slot has published its
// activations (per-slot counter, release/acquire + async-proxy fence).
//
// Warp roles (320 or 576 threads, one CTA per SM):
//   warp 0      producer: claims items, TMA weight tile + route rows per 64-element K
//               stage into a ring of 128-byte-swizzled shared-memory stages.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=16..256, K=16) into a
//               double-buffered TMEM accumulator and frees stages with tcgen05.commit.
//   warps 2..    epilogue (8 warps, or 16 for paired tiles: one per TMEM lane quarter and
//               column group, the groups taking alternate 16-column chunks):
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

#ifndef TW_FFN_PAIR_EPI_WARPS
#define TW_FFN_PAIR_EPI_WARPS 16   // epilogue warps of the paired-tile variants
#endif
constexpr int kBK = 64;            // K elements per TMA box (128-byte rows)
#ifndef TW_FFN_KB
#define TW_FFN_KB 4                // K boxes per pipeline stage
#endif
constexpr int kKBMax = TW_FFN_KB;
#ifndef TW_FFN_KROT
#define TW_FFN_KROT 1              // rotate each item's K order to decorrelate DRAM streams
#endif
#ifndef TW_FFN_PAIR
#define TW_FFN_PAIR 1              // prefill tiles: two weight tiles per item share route loads
#endif
constexpr int kSmemBudget = 216 * 1024;
constexpr int kWRows = 128;        // weight rows per tile = MMA M

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
  // Weight tiles per item.  Large route tiles are TMA-throughput-bound (each K box moves
  // 16 KB of weights and kNCap * 128 B of routes for only 4 MMAs), so there an item takes
  // two weight tiles that share every route box: two MMAs per route load.
  static constexpr int kTiles = (TW_FFN_PAIR && kNCap >= 160) ? 2 : 1;
  // Epilogue warps: four per column group, one per TMEM lane quarter.  A paired item's
  // accumulator is single-buffered, so its epilogue is split over more column groups.
  static constexpr int kEpiWarps = kTiles == 2 ? TW_FFN_PAIR_EPI_WARPS : 8;
  static constexpr int kColGroups = kEpiWarps / 4;
  static constexpr int kEpiThreads = 32 * kEpiWarps;
  static constexpr int kThreads = 64 + kEpiThreads;  // warp 0 TMA, warp 1 MMA, then epilogue
  static constexpr int kWBoxBytes = kTiles * kWStageBytes;        // weight rows of one K box
  static constexpr int kRBoxBytes = kNCap * 128;                 // route rows of one K box
  static constexpr int kBoxPair = kWBoxBytes + kRBoxBytes;        // one K box of both operands
  // accumulator columns of one route chunk; double-buffered when two fit in TMEM
  static constexpr int kAccCols = kTiles * kNCap;
  static constexpr int kAccBufs = kAccCols <= 256 ? 2 : 1;
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
  // per epilogue warp: one 16-route chunk of its outputs, transposed for 16-byte stores
  static constexpr int kScratchOffset = kXchgOffset + kXchgBytes;
  static constexpr int kScratchBytes = kEpiWarps * 1024;
  static constexpr int kBarOffset = kScratchOffset + kScratchBytes;
  static constexpr int kBytes = kBarOffset + 512 + 1024;
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kStages >= 2 && kBytes <= 227 * 1024, "shared memory budget");
  static_assert((2 * kStages + 4 + 2 * kRing + 2) * 8 + 16 + (int)sizeof(Item) * kRing <= 512,
                "barriers");
  static_assert(kRBoxBytes % 1024 == 0, "route box alignment");
  static_assert(kTiles == 1 || kKB == 1, "paired tiles: one K box per stage");
  static_assert(kEpiWarps % 4 == 0 && kThreads <= 1024, "epilogue warps");
  static_assert(kAccCols * kAccBufs <= 512, "TMEM columns");
};

// One launch per FFN: every (slot, up tile) item, then every (slot, down tile) item,
// claimed dynamically.  A down item's activations come from up items of the same slot
// (possibly on other CTAs): its producer waits on up_done before loading them.
template <int kNCap>
__global__ void __launch_bounds__(FfnSmem<kNCap>::kThreads, 1)
expert_ffn_tc_kernel(const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_w2,
                     const __grid_constant__ CUtensorMap tm_w1p,
                     const __grid_constant__ CUtensorMap tm_w2p,
                     const __grid_constant__ RouteMaps rm, FfnArgs a) {
  using L = FfnSmem<kNCap>;
  constexpr int kStages = L::kStages;
  constexpr int kKB = L::kKB;
  constexpr int kTiles = L::kTiles;
  constexpr int kAccBufs = L::kAccBufs;
  // weight tiles of an item: tiles [item.tile * kTiles, + tiles_of(item)) of its kind
  auto tiles_of = [&](const Item& item) {
    const int all = item.kind == 0 ? a.I / 64 : a.H / kWRows;
    return min(kTiles, all - item.tile * kTiles);
  };
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
  uint64_t* esync = drain + 1;            // the epilogue warps meet here (bounded waits)
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
      mbar_init(&tempty[i], L::kEpiThreads);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&ifull[i], 1);
      mbar_init(&iempty[i], 1 + L::kEpiThreads);  // the MMA thread and every epilogue thread
    }
    mbar_init(drain, 1);
    mbar_init(esync, L::kEpiThreads);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_w2);
    if (kTiles > 1) {
      prefetch_tmap(&tm_w1p);
      prefetch_tmap(&tm_w2p);
    }
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
        if (!mbar_wait(&iempty[e], ((r / kRing) & 1) ^ 1, err, a.wait_limit)) break;
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
        const int nt = tiles_of(item), t0 = item.tile * kTiles;
        if (item.kind == 1) fence_proxy_async_global();  // activations came from other CTAs
        for (int pc = p0; ok && pc < p1; pc += kNCap) {
          const int n = min(kNCap, p1 - pc);
          const int ri = route_box_index(n);
          const CUtensorMap* tr = item.kind == 0 ? &rm.xg[ri] : &rm.act[ri];
          // token rows: the up tile multiplies all of x's (<= 16) token rows, the epilogue
          // picks each route's token column
          const int r0 = item.kind == 0 && a.token_rows ? 0 : pc;
          const int rot = k_rotation(item, kst);
          for (int kq = 0; kq < kst; ++kq, ++it) {
            const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err, a.wait_limit)) {
              ok = false;
              break;
            }
            uint8_t* W = smem + s * L::kStageBytes;
            uint8_t* R = W + kKB * L::kWBoxBytes;
            // one TMA instruction each for the stage's weight tiles (kKB K boxes x 128 rows
            // per tile; a paired item's two tiles are one 256-row box) and route rows (kKB K
            // boxes x route_rows(ri) rows); K boxes past the end of a row read as zeros and
            // are not multiplied
            mbar_arrive_expect_tx(&full[s],
                                  kKB * (nt * kWStageBytes + route_rows<kNCap>(ri) * 128));
            if (item.kind == 0)
              tma_load_5d(W, nt > 1 ? &tm_w1p : &tm_w1, &full[s], 0, 0, t0 * 64, ks * kKB, slot);
            else
              tma_load_4d(W, nt > 1 ? &tm_w2p : &tm_w2, &full[s], 0, t0 * kWRows, ks * kKB,
                          slot);
            tma_load_3d(R, tr, &full[s], 0, r0, ks * kKB);
          }
        }
      }
      if (!ok) {  // let every load already issued land before the CTA can exit
        for (uint32_t j = (it >= kStages ? it - kStages : 0); j < it; ++j)
          mbar_drain(&full[j % kStages], (j / kStages) & 1, err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, c = 0;
      bool ok = true;
      for (uint32_t r = 0; ok; ++r) {
        const int e = r % kRing;
        if (!mbar_wait(&ifull[e], (r / kRing) & 1, err, a.wait_limit)) break;
        const Item item = ring[e];
        mbar_arrive(&iempty[e]);
        if (item.kind < 0) break;
        const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
        const int kbox = (item.kind == 0 ? a.H : a.I) / kBK;
        const int kst = (kbox + kKB - 1) / kKB;
        const int nt = tiles_of(item);
        for (int pc = p0; ok && pc < p1; pc += kNCap, ++c) {
          const int n = min(kNCap, p1 - pc);
          const uint32_t idesc = idesc_bf16(kWRows, (n + 15) & ~15);
          const uint32_t rbox16 = (uint32_t)(route_rows<kNCap>(route_box_index(n)) * 128) >> 4;
          const int acc = c % kAccBufs;
          if (!mbar_wait(&tempty[acc], ((c / kAccBufs) & 1) ^ 1, err, a.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(acc * 256);  // tile t accumulates at d + t * kNCap
          const int rot = k_rotation(item, kst);
          for (int kq = 0; kq < kst; ++kq, ++it) {
            const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
            const int s = it % kStages;
            if (!mbar_wait(&full[s], (it / kStages) & 1, err, a.wait_limit)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // descriptors built once per stage, constant offsets per MMA (keeps the issuing
            // thread ahead of the tensor pipe at small N)
            const uint64_t w_desc = umma_desc_sw128(smem_u32(smem + s * L::kStageBytes));
            const uint64_t r_desc = w_desc + (uint64_t)((kKB * L::kWBoxBytes) >> 4);
            const int nkb = min(kKB, kbox - ks * kKB);
            if (nkb == kKB) {
#pragma unroll
              for (int j = 0; j < kKB * (kBK / 16); ++j) {
                const int kb = j / (kBK / 16), kk = j % (kBK / 16);
#pragma unroll
                for (int t = 0; t < kTiles; ++t)
                  if (t < nt)
                    mma_bf16(d + (uint32_t)(t * kNCap),
                             w_desc + (uint64_t)((kb * L::kWBoxBytes + t * kWStageBytes +
                                                  kk * 32) >> 4),
                             r_desc + (uint64_t)(kb * rbox16 + ((kk * 32) >> 4)), idesc,
                             (kq | j) != 0);
              }
            } else {
              for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
#pragma unroll
                  for (int t = 0; t < kTiles; ++t)
                    if (t < nt)
                      mma_bf16(d + (uint32_t)(t * kNCap),
                               w_desc + (uint64_t)((kb * L::kWBoxBytes + t * kWStageBytes +
                                                    kk * 32) >> 4),
                               r_desc + (uint64_t)(kb * rbox16 + ((kk * 32) >> 4)), idesc,
                               (kq | kb | kk) != 0);
              }
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&tfull[acc]);
        }
      }
      mma_commit(drain);  // every MMA issued, error or not, completes before TMEM is freed
      mbar_drain(drain, 0, err);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..)
    const int q = warp & 3;  // TMEM lane quarter: rows 32q .. 32q+31 of the weight tile
    const int colgrp = (warp - 2) >> 2;  // which 16-column chunks of a tile this warp takes
    const int etid = (warp - 2) * 32 + lane;
    const int row = q * 32 + lane;
    // this warp's transpose scratch: up [16 routes][16 j], down [16 routes][32 h] (bf16)
    uint8_t* scr = smem + L::kScratchOffset + (warp - 2) * 1024;
    __nv_bfloat16* scr_h = reinterpret_cast<__nv_bfloat16*>(scr);
    uint32_t c = 0, ephase = 0;
    bool ok = true;
    auto epilogue_sync = [&]() -> bool {  // all epilogue threads, bounded
      mbar_arrive(esync);
      const bool r = warp_all(mbar_wait(esync, ephase, err, a.wait_limit));
      ephase ^= 1;
      return r;
    };
    for (uint32_t r = 0; ok; ++r) {
      const int e = r % kRing;
      if (!warp_all(mbar_wait(&ifull[e], (r / kRing) & 1, err, a.wait_limit))) break;
      const Item item = ring[e];
      mbar_arrive(&iempty[e]);
      if (item.kind < 0) break;
      const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
      const int nt = tiles_of(item), t0 = item.tile * kTiles;
      for (int pc = p0; ok && pc < p1; pc += kNCap, ++c) {
        const int n = min(kNCap, p1 - pc);
        const int acc = c % kAccBufs;
        const int w_in = a.variant >> 2, gate_act = a.variant & 3;
        if (item.kind == 1 || w_in) {
          // the chunk's route weights, staged in shared memory for all epilogue warps while
          // the MMAs still run (two dependent global loads kept off the accumulator's path);
          // they multiply the down projection, or with w_in the up projection only
          if (!epilogue_sync()) {
            ok = false;
            break;
          }
          const bool weighted = a.topk_w != nullptr && (item.kind == 1) != (w_in != 0);
          for (int t = etid; t < n; t += L::kEpiThreads)
            wbuf[t] = weighted ? a.topk_w[a.perm[pc + t]] : 1.0f;
          if (!epilogue_sync()) {
            ok = false;
            break;
          }
        }
        if (!warp_all(mbar_wait(&tfull[acc], (c / kAccBufs) & 1, err, a.wait_limit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256);
        if (item.kind == 0) {
          // tile rows alternate gate and up of one intermediate index: row 2m is gate
          // j = tile*64 + m, row 2m+1 its up row, in neighbouring lanes.  Per pair of routes
          // the lanes swap values with shuffles: the gate lane finishes the even route, the up
          // lane the odd one.  The warp's 16 routes x 16 j go through the scratch so that
          // each lane stores 16 bytes (8 j of one route).
          const int odd = row & 1;
          for (int t = 0; t < nt; ++t) {
            const int jbase = (t0 + t) * 64 + q * 16;
            for (int cb = 16 * colgrp; cb < n; cb += 16 * L::kColGroups) {
              float v[16];
              tmem_ld16(tb + (uint32_t)(t * kNCap + cb), v);
              __syncwarp();
              if (gate_act == 0 && w_in == 0) {  // SwiGLU, weight on the down projection
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                  const float o0 = __shfl_xor_sync(0xffffffffu, v[i], 1);
                  const float o1 = __shfl_xor_sync(0xffffffffu, v[i + 1], 1);
                  const float g = bf16_round(odd ? o1 : v[i]);
                  const float u = bf16_round(odd ? v[i + 1] : o0);
                  scr_h[(i + odd) * 16 + (lane >> 1)] = __float2bfloat16_rn(silu_fast(g) * u);
                }
              } else {  // the other activations; with w_in this lane's route (column
                        // cb + i + odd) weighs both halves before their rounding
                for (int i = 0; i < 16; i += 2) {
                  const float o0 = __shfl_xor_sync(0xffffffffu, v[i], 1);
                  const float o1 = __shfl_xor_sync(0xffffffffu, v[i + 1], 1);
                  const float wc = w_in ? wbuf[cb + i + odd] : 1.0f;
                  const float g = bf16_round((odd ? o1 : v[i]) * wc);
                  const float u = bf16_round((odd ? v[i + 1] : o0) * wc);
                  const float ag = gate_act == 0 ? silu_fast(g) : gelu_act(gate_act, g);
                  scr_h[(i + odd) * 16 + (lane >> 1)] = __float2bfloat16_rn(ag * u);
                }
              }
              __syncwarp();
              const int col = cb + (lane >> 1);  // the route (position pc + col) this lane stores
              if (col < n) {
                // token rows: scratch row = the route's token; gathered rows: = the route
                const int srow = a.token_rows ? a.perm[pc + col] / a.route_k : (lane >> 1);
                const uint4 val = reinterpret_cast<const uint4*>(scr)[srow * 2 + (lane & 1)];
                *reinterpret_cast<uint4*>(a.act + (int64_t)(pc + col) * a.I + jbase +
                                          (lane & 1) * 8) = val;
              }
            }
          }
          // the accumulator is free once read: hand it back before the publish below waits
          // for the stores to land
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          // publish this warp's activation writes to the down tiles of this slot: every lane
          // orders its writes for the async proxy, the warp synchronises, lane 0 releases
          fence_proxy_async_global();
          __syncwarp();
          if (lane == 0) {
            // every epilogue warp publishes each (item, route chunk) once
            const int target = up_target(a, item.u, kNCap, L::kEpiWarps);
            if (atom_add_acq_rel(a.up_done + item.u * kDoneStride, 1) + 1 == target) {
              const int pos = atomicAdd(a.ready_tail, 1);
              st_release(a.ready_slots + pos, item.u);
            }
          }
        } else {
          // the warp's 16 routes x 32 h go through the scratch: each lane then stores
          // 2 x 16 bytes (8 h of one route each).  Lane i holds route cb + i's weight
          // (cb + 16 <= kNCap; entries past n are unused) and shuffles it out; neighbouring
          // lanes (h, h + 1) swap products so that each writes one packed word per route pair.
          const int odd = lane & 1;
          uint32_t* scr_w = reinterpret_cast<uint32_t*>(scr);
          for (int t = 0; t < nt; ++t) {
            const int hbase = (t0 + t) * kWRows + q * 32;
            for (int cb = 16 * colgrp; cb < n; cb += 16 * L::kColGroups) {
              const float wl = wbuf[cb + (lane & 15)];
              float v[16];
              tmem_ld16(tb + (uint32_t)(t * kNCap + cb), v);
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 16; i += 2) {
                const float p0 = v[i] * __shfl_sync(0xffffffffu, wl, i);
                const float p1 = v[i + 1] * __shfl_sync(0xffffffffu, wl, i + 1);
                const float o0 = __shfl_xor_sync(0xffffffffu, p0, 1);
                const float o1 = __shfl_xor_sync(0xffffffffu, p1, 1);
                // even lane: route i, h pair (own, partner); odd lane: route i + 1
                const __nv_bfloat162 pk = odd ? __floats2bfloat162_rn(o1, p1)
                                              : __floats2bfloat162_rn(p0, o0);
                scr_w[(i + odd) * 16 + (lane >> 1)] = *reinterpret_cast<const uint32_t*>(&pk);
              }
              __syncwarp();
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int rl = h2 * 8 + (lane >> 2);
                const uint4 val = reinterpret_cast<const uint4*>(scr + rl * 64)[lane & 3];
                if (cb + rl < n)
                  *reinterpret_cast<uint4*>(a.c3 + (int64_t)(pc + cb + rl) * a.H + hbase +
                                            (lane & 3) * 8) = val;
              }
            }
          }
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
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
  // a block copies whole rows (grid-stride over positions), four 16-byte loads in flight
  // per thread before the stores
  const int used = seg_start[num_unique[0]];
  for (int p = blockIdx.x; p < used; p += gridDim.x) {
    const uint4* src = x + (int64_t)(perm[p] / K) * H8;
    uint4* dst = xg + (int64_t)p * H8;
    for (int c = threadIdx.x; c < H8; c += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j * (int)blockDim.x < H8) v[j] = src[c + j * blockDim.x];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j * (int)blockDim.x < H8) dst[c + j * blockDim.x] = v[j];
    }
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
int launch_ffn(const __nv_bfloat16* w1, const __nv_bfloat16* w2, const void* routes,
               int64_t route_rows_n, const Workspace& ws, int64_t n, const FfnArgs& args,
               int grid, cudaStream_t st) {
  using L = FfnSmem<kNCap>;
  const uint64_t H = args.H, I = args.I, S = args.num_slots;
  // single-tile maps (m1, m2) and the paired-tile maps (m1p, m2p: twice the rows per box)
  CUtensorMap m1, m2, m1p, m2p;
  for (int t = 1; t <= 2; ++t) {
    const uint64_t d[5] = {kBK, 2, I, H / kBK, S};
    const uint64_t sb[4] = {I * H * 2, H * 2, kBK * 2, 2 * I * H * 2};
    const uint32_t b[5] = {kBK, 2, (uint32_t)(64 * t), (uint32_t)L::kKB, 1};
    if (int rc = make_tmap_bf16(t == 1 ? &m1 : &m1p, w1, 5, d, sb, b)) return rc;
  }
  for (int t = 1; t <= 2; ++t) {
    const uint64_t d[4] = {kBK, H, I / kBK, S};
    const uint64_t sb[3] = {I * 2, kBK * 2, H * I * 2};
    const uint32_t b[4] = {kBK, (uint32_t)(kWRows * t), (uint32_t)L::kKB, 1};
    if (int rc = make_tmap_bf16(t == 1 ? &m2 : &m2p, w2, 4, d, sb, b)) return rc;
  }
  // items per segment: weight tiles grouped kTiles at a time
  FfnArgs fa = args;
  fa.tu = (args.I / 64 + L::kTiles - 1) / L::kTiles;
  fa.td = (args.H / kWRows + L::kTiles - 1) / L::kTiles;
  RouteMaps rm;
  for (int i = 0; i < kRouteRowsN; ++i) {
    const int rows = route_rows<kNCap>(i);
    {
      const uint64_t d[3] = {kBK, (uint64_t)route_rows_n, H / kBK};
      const uint64_t sb[2] = {H * 2, kBK * 2};
      const uint32_t b[3] = {kBK, (uint32_t)rows, (uint32_t)L::kKB};
      if (int rc = make_tmap_bf16(&rm.xg[i], routes, 3, d, sb, b)) return rc;
    }
    {
      const uint64_t d[3] = {kBK, (uint64_t)n, I / kBK};
      const uint64_t sb[2] = {I * 2, kBK * 2};
      const uint32_t b[3] = {kBK, (uint32_t)rows, (uint32_t)L::kKB};
      if (int rc = make_tmap_bf16(&rm.act[i], ws.act, 3, d, sb, b)) return rc;
    }
  }
  auto kern = expert_ffn_tc_kernel<kNCap>;
  // the dynamic shared-memory limit is a per-device attribute: raise it once per device
  static bool attr_set[kMaxAttrDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxAttrDevices || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (dev >= 0 && dev < kMaxAttrDevices) attr_set[dev] = true;
  }
  TW_LAUNCH(kern, dim3(grid), dim3(L::kThreads), L::kBytes, st, m1, m2, m1p, m2p, rm, fa);
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

namespace {

int launch_ffn_cap(int cap, const __nv_bfloat16* w1, const __nv_bfloat16* w2, const void* routes,
                   int64_t route_rows_n,
                   const Workspace& ws, int64_t n, const FfnArgs& fa, int grid, cudaStream_t st) {
  switch (cap) {
    case 16: return launch_ffn<16>(w1, w2, routes, route_rows_n, ws, n, fa, grid, st);
    case 64: return launch_ffn<64>(w1, w2, routes, route_rows_n, ws, n, fa, grid, st);
    case 160: return launch_ffn<160>(w1, w2, routes, route_rows_n, ws, n, fa, grid, st);
    default: return launch_ffn<256>(w1, w2, routes, route_rows_n, ws, n, fa, grid, st);
  }
}

// Segments of a dense FFN over T rows: ceil(T / cap) segments of cap rows of slot 0, plus
// the hand-off state the FFN kernel expects zeroed (what the grouping kernel does for
// routed calls).
__global__ void __launch_bounds__(256) dense_segments_kernel(int T, int cap, Workspace ws) {
  pdl_wait();
  pdl_trigger();
  const int U = (T + cap - 1) / cap;
  if (threadIdx.x == 0) {
    ws.err[0] = 0;
    ws.up_ctr[0] = 0;
    ws.down_ctr[0] = 0;
    ws.ready_tail[0] = 0;
    ws.num_unique[0] = U;
  }
  for (int u = threadIdx.x; u <= U; u += blockDim.x) {
    ws.seg_start[u] = min(u * cap, T);
    if (u < U) {
      ws.seg_slot[u] = 0;
      ws.up_done[u * 32] = 0;
      ws.ready_slots[u] = -1;
    }
  }
}

}  // namespace

int launch_expert_ffn_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                         const __nv_bfloat16* w1, const __nv_bfloat16* w2, int64_t S,
                         const float* topk_w, const Workspace& ws, int64_t n, cudaStream_t st,
                         FfnAct fx) {
  TW_CHECK_ARG(H % kWRows == 0 && I % 64 == 0, "tensor-core FFN: need H %% 128 == 0, I %% 64 == 0");
  TW_CHECK_ARG(n <= (int64_t)1 << 30 && S < (1 << 30), "tensor-core FFN: sizes out of range");
  const int sms = num_sms();
  const int cap = expert_ffn_tc_route_cap(T, n, S);
  // decode (one 16-route tile covers every token): the up tiles multiply x's token rows
  // directly and the epilogue picks each route's column, so no gathered copy is made
  // (a route weight on the up projection differs between the routes of one token row: those
  // launches keep one gathered row per route)
  const bool token_rows = cap == 16 && T <= 16 && !fx.w_in;
  if (!token_rows) {
    const int H8 = H / 8;
    const int blocks = (int)std::min<int64_t>(n, (int64_t)sms * 8);
    TW_LAUNCH(gather_rows_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st, 
        reinterpret_cast<const uint4*>(x), K, H8, ws.perm, ws.seg_start, ws.num_unique,
        reinterpret_cast<uint4*>(ws.xg));
    TW_CHECK_LAUNCH("gather_rows_kernel");
  }
  // the number of segments is only known on the device: size the persistent grid for the
  // most work n routes can produce (every slot, plus one segment per full route tile);
  // idle CTAs find the item counter exhausted
  const int64_t max_u = std::min<int64_t>(n, S + n / cap);
  FfnArgs fa{H, I, I / 64, H / kWRows, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm,
             topk_w, ws.act, ws.c3, ws.up_ctr, ws.down_ctr, ws.up_done, ws.ready_tail,
             ws.ready_slots, ws.err, RowScale{}, RowScale{}, S, ffn_wait_limit(), K,
             token_rows ? 1 : 0};
  fa.variant = fx.act | (fx.w_in << 2);
  const int grid = (int)std::min<int64_t>(max_u * (fa.tu + fa.td), sms);
  if (token_rows) return launch_ffn_cap(cap, w1, w2, x, T, ws, n, fa, grid, st);
  return launch_ffn_cap(cap, w1, w2, ws.xg, n, ws, n, fa, grid, st);
}

// Dense gated FFN of one expert over all T rows (a shared expert): routes are the rows
// themselves, so the segments are arithmetic (T rows cut at the route-tile capacity),
// the FFN reads x and writes out directly and every route weight is 1 (so only the gate
// activation of fx applies).
int launch_expert_ffn_dense_tc(const __nv_bfloat16* x, int64_t T, int H, int I,
                               const __nv_bfloat16* w1, const __nv_bfloat16* w2,
                               const Workspace& ws, __nv_bfloat16* out, cudaStream_t st,
                               FfnAct fx) {
  TW_CHECK_ARG(H % kWRows == 0 && I % 64 == 0, "tensor-core FFN: need H %% 128 == 0, I %% 64 == 0");
  TW_CHECK_ARG(T > 0 && T <= (int64_t)1 << 30, "tensor-core FFN: sizes out of range");
  const int cap = expert_ffn_tc_route_cap(T, T, 1);
  TW_LAUNCH(dense_segments_kernel, dim3(1), dim3(256), 0, st, (int)T, cap, ws);
  TW_CHECK_LAUNCH("dense_segments_kernel");
  FfnArgs fa{H, I, I / 64, H / kWRows, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm,
             nullptr, ws.act, out, ws.up_ctr, ws.down_ctr, ws.up_done, ws.ready_tail,
             ws.ready_slots, ws.err, RowScale{}, RowScale{}, 1, ffn_wait_limit(), 1, 0};
  fa.variant = fx.act;
  const int64_t segs = (T + cap - 1) / cap;
  const int grid = (int)std::min<int64_t>(segs * (fa.tu + fa.td), num_sms());
  return launch_ffn_cap(cap, w1, w2, x, T, ws, T, fa, grid, st);
}

// Route-tile capacity: a slot has at most T routes (one per token); for larger T the
// expected routes per slot (T*K / S) decide between 160-route tiles (3 stages of 2 K boxes)
// and 256-route tiles (fewer re-streamed weight tiles when slots get more than 160).
int expert_ffn_tc_route_cap(int64_t T, int64_t n, int64_t S) {
  if (T <= 16) return 16;
  if (T <= 64) return 64;
  if (T <= 160 || n <= 128 * S) return 160;
  return 256;
}

}  // namespace tw
