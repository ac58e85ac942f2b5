// NVFP4 slot-indirect SwiGLU expert FFN on the 5th-generation tensor cores, with the weight
// operand dequantised straight into tensor memory.
//
// Bank format (per slot): packed e2m1 codes [rows, K/2] (element 2j in the low nibble),
// e4m3 block scales [rows, K/16], fp32 global scale per row.  The product of an e2m1 code
// and an e4m3 scale has at most five significant bits and lies in [2^-10, 2688], so it is
// exact in f16: the kernel multiplies f16(code) * f16(scale) on the CUDA cores, feeds the
// tensor cores f16 operands (kind::f16, fp32 accumulation) and applies the fp32 row global
// in the epilogue.  This is dequant-then-matmul up to the order of the fp32 sums.
//
// Data path per 256-element K stage of a 128-row weight tile:
//   TMA        packed codes (128 rows x 128 B, 128-byte swizzle, one box) + the routes'
//              f16 rows (one box of 4 x 64 elements for route tiles of 16) -> smem ring;
//              the item's e4m3 scales (128 rows x K/16 B) once per work item into a
//              double-buffered scale area.  An SM keeps only a few TMA instructions in
//              flight, so every stage is moved by as few, as large boxes as possible.
//   dequant    16 warps in four groups of four taking stages in turn (a decode warp is
//              latency-bound, so each group gets four stage times per stage); in a group
//              each thread owns one weight row (its TMEM lane) and the stage's K; codes ->
//              f16x2 (hardware e2m1x2 conversion) -> * scale -> tcgen05.st into a TMEM A stage
//   MMA        16 x tcgen05.mma M=128 N=16..128 K=16, A from TMEM, B from smem; for route
//              tiles up to 64 two issuing threads take alternate stages into two partial
//              accumulators (summed by the epilogue): the tensor pipe cannot run ahead of
//              its issuing thread at small N, so one thread's per-stage barrier wait and
//              commit would otherwise idle it
//   barriers   indexed by the stage modulo a count that their consumers' count divides, so
//              every barrier has one consumer taking its phases in order (see the kernel)
//   epilogue   4 warps, as the BF16 kernel, with the row global scale applied
// Dequantised weights never touch shared memory: at HBM speed the f16 operand is 4x the
// bytes of the packed one and shared memory could not carry both that and its re-read.
//
// Work items, claiming and the up -> down hand-off are those of the BF16 kernel
// (ffn_sched.cuh).  Every wait is bounded; on a timeout the kernel records an error word,
// drains its copies and MMAs, frees TMEM and exits.
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include <algorithm>

#include "ffn_sched.cuh"

namespace tw {
namespace {

#ifndef TW_FP4_DEQUANT_WARPS
#define TW_FP4_DEQUANT_WARPS 16
#endif
// warp 0 TMA, warps 1 and kF4MmaWarp2 MMA, 2-5 epilogue, 6 .. 6 + kF4DequantWarps - 1 dequant
constexpr int kF4DequantWarp0 = 6;
constexpr int kF4DequantWarps = TW_FP4_DEQUANT_WARPS;
constexpr int kF4MmaWarp2 = kF4DequantWarp0 + kF4DequantWarps;
constexpr int kF4Threads = 32 * (kF4MmaWarp2 + 1);
constexpr int kF4KS = 256;         // K elements per stage
#ifndef TW_FP4_GROUP_WARPS
#define TW_FP4_GROUP_WARPS 4
#endif
// Dequant warps per stage (one group); groups take stages in turn.  A group splits the
// stage's K into kF4Parts parts, one per four warps (one warp per TMEM lane quarter).
constexpr int kF4GroupWarps = TW_FP4_GROUP_WARPS;
constexpr int kF4Groups = kF4DequantWarps / kF4GroupWarps;
constexpr int kF4Parts = kF4GroupWarps / 4;
constexpr int kF4PartK = kF4KS / kF4Parts;  // K elements per thread per stage
static_assert(kF4Groups * kF4GroupWarps == kF4DequantWarps && kF4PartK % 32 == 0, "dequant split");
constexpr int kF4PackBytes = 128 * (kF4KS / 2);   // 128 rows x 128 B
constexpr int kF4ScaleSeg = 128 * 128;             // 128 rows x 128 scale bytes (2048 K)
constexpr int kF4MaxK = 4096;                      // K of one item (H or I) the scale area holds
constexpr int kF4ScaleBuf = kF4ScaleSeg * (kF4MaxK / 2048);
constexpr int kF4RouteBox = 16;
constexpr int kF4XRow = 17;
constexpr int kF4SmemTotal = 227 * 1024;

constexpr int gcd_c(int a, int b) { return b == 0 ? a : gcd_c(b, a % b); }
constexpr int lcm_c(int a, int b) { return a / gcd_c(a, b) * b; }

template <int kNCap>
struct Fp4Smem {
  static constexpr int kRBoxBytes = kNCap * 128;  // routes x 64 f16 of one K box
  static constexpr int kRouteOffset = kF4PackBytes;
  static constexpr int kStageBytes = kRouteOffset + 4 * kRBoxBytes;
  static constexpr int kScaleBufs = kNCap >= 128 ? 1 : 2;
  static constexpr int kScaleOffset = 0;
  static constexpr int kStageOffset = kScaleBufs * kF4ScaleBuf;
  static constexpr int kXchgBytes = 2 * 64 * kF4XRow * 4;
  static constexpr int kStages =
      (kF4SmemTotal - 1024 - 1024 - kXchgBytes - kStageOffset) / kStageBytes;
  static constexpr int kXchgOffset = kStageOffset + kStages * kStageBytes;
  static constexpr int kBarOffset = kXchgOffset + kXchgBytes;
  static constexpr int kBytes = kBarOffset + 1024 + 1024;
  // TMEM: two accumulator buffers (each kIssuers partials of kAccPart columns), then
  // 128-column A stages (256 f16 per row)
  static constexpr int kIssuers = kNCap <= 64 ? 2 : 1;
  static constexpr int kAccPart = kNCap < 32 ? 32 : kNCap;
  static constexpr int kAccBuf = kIssuers * kAccPart;
  static constexpr int kABase = 2 * kAccBuf;
  static constexpr int kAStages = (512 - kABase) / 128;
  static_assert(kRouteOffset % 1024 == 0 && kStageBytes % 1024 == 0, "1024-byte alignment");
  static_assert(kStages >= 2 && kBytes <= 227 * 1024, "shared memory budget");
  static_assert(kAStages >= 2, "tensor memory budget");
  static_assert(kAStages <= kStages, "a TMEM stage is released through its smem stage's barrier");
  // barrier sets indexed by stage modulo these counts: each barrier then has one consumer
  // (a dequant group, or an MMA issuer) that takes its phases in order
  static constexpr int kNF = lcm_c(kStages, kF4Groups);     // full: stage landed
  static constexpr int kNAE = lcm_c(kAStages, kF4Groups);   // aempty: A stage free again
  static constexpr int kNAF = lcm_c(kAStages, kIssuers);    // afull: A stage written
  static_assert((kNF + kStages + kNAF + kNAE + 4 + 4 + 2 * kRing + 4 + 2) * 8 + 16 +
                    (int)sizeof(Item) * kRing <= 1024,
                "barriers");
};

__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}

// Four packed bytes (8 codes) -> four f16x2 (element pairs in order) times one block scale.
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 s, uint32_t* o) {
  // the word's four bytes are register halves' bytes (no shifts or masks); one hardware
  // e2m1x2 -> f16x2 conversion per byte (low nibble -> low half), then the exact scale
  // multiply
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      ".reg .b32 h0, h1, h2, h3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 h0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 h1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 h2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 h3, b3;\n"
      "mul.rn.f16x2 %0, h0, %5;\n"
      "mul.rn.f16x2 %1, h1, %5;\n"
      "mul.rn.f16x2 %2, h2, %5;\n"
      "mul.rn.f16x2 %3, h3, %5;\n"
      "}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w), "r"(h2_bits(s)));
}

// Two e4m3 scale bytes -> f16 (exact).
__device__ __forceinline__ __half2 e4m3x2_to_h2(uint32_t two) {
  const __half2_raw r =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu), __NV_E4M3);
  return __half2(r);
}

template <int kNCap>
__global__ void __launch_bounds__(kF4Threads, 1)
expert_ffn_fp4_tc_kernel(const __grid_constant__ CUtensorMap tm_w1p,
                         const __grid_constant__ CUtensorMap tm_w1s,
                         const __grid_constant__ CUtensorMap tm_w2p,
                         const __grid_constant__ CUtensorMap tm_w2s,
                         const __grid_constant__ CUtensorMap tm_xg,
                         const __grid_constant__ CUtensorMap tm_act,
                         const __grid_constant__ CUtensorMap tm_xg3,
                         const __grid_constant__ CUtensorMap tm_act3, FfnArgs a) {
  using L = Fp4Smem<kNCap>;
  constexpr int kStages = L::kStages;
  constexpr int kAStages = L::kAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* xchg = reinterpret_cast<float*>(smem + L::kXchgOffset);  // [2][64][kF4XRow]
  // Stage `it` (a count over the launch's stages) uses smem stage it % kStages and TMEM A stage
  // it % kAStages; dequant group it % kF4Groups fills it, MMA issuer it % kIssuers consumes
  // it.  Groups and issuers run unevenly, so a barrier shared by several of them could be
  // polled two phases early, where a parity wait passes at once.  Every barrier below is
  // therefore indexed by the stage modulo a count that the consumers' count divides: each
  // barrier has one consumer, which takes its phases in order.
  //   full[it % kNF]    stage it landed (TMA; its group waits)
  //   done[s]           the MMAs of the stage that last used smem stage s completed (the
  //                     producer waits, in order)
  //   afull[it % kNAF]  A stage of stage it written (its issuer waits)
  //   aempty[it % kNAE] the A stage that stage it is about to fill is free: the MMAs of stage
  //                     it - kAStages completed (its group waits)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* done = full + L::kNF;
  uint64_t* afull = done + kStages;
  uint64_t* aempty = afull + L::kNAF;
  uint64_t* sfull = aempty + L::kNAE;   // [2] scale buffer landed
  uint64_t* sempty = sfull + 2;         // [2] scale buffer released by the dequant warps
  uint64_t* tfull = sempty + 2;
  uint64_t* tempty = tfull + 2;
  uint64_t* ifull = tempty + 2;
  uint64_t* iempty = ifull + kRing;
  uint64_t* xfull = iempty + kRing;
  uint64_t* xempty = xfull + 2;
  uint64_t* drain = xempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  Item* ring = reinterpret_cast<Item*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kDequantWarps = kF4DequantWarps;
  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNF; ++i) mbar_init(&full[i], 1);
    for (int s = 0; s < kStages; ++s) mbar_init(&done[s], 1);
    for (int i = 0; i < L::kNAF; ++i) mbar_init(&afull[i], kF4GroupWarps);
    for (int i = 0; i < L::kNAE; ++i) mbar_init(&aempty[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], kDequantWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], L::kIssuers);
      mbar_init(&tempty[i], 128);
      mbar_init(&xfull[i], 64);
      mbar_init(&xempty[i], 64);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&ifull[i], 1);
      mbar_init(&iempty[i], L::kIssuers + 128 + 32 * kDequantWarps);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w1p);
    prefetch_tmap(&tm_w1s);
    prefetch_tmap(&tm_w2p);
    prefetch_tmap(&tm_w2s);
    prefetch_tmap(&tm_xg);
    prefetch_tmap(&tm_act);
    prefetch_tmap(&tm_xg3);
    prefetch_tmap(&tm_act3);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();
  const int U = a.num_unique[0];
  int* err = a.err;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0, ic = 0;  // stages, items
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
        const int kdim = item.kind == 0 ? a.H : a.I;
        const int kst = kdim / kF4KS;
        if (item.kind == 1) fence_proxy_async_global();  // activations came from other CTAs
        // the item's block scales: 128-byte segments (2048 K) of all 128 rows, one box
        {
          const int b = ic % L::kScaleBufs;
          if (!mbar_wait(&sempty[b], ((ic / L::kScaleBufs) & 1) ^ 1, err, a.wait_limit)) break;
          const int nseg = (kdim / 16 + 127) / 128;
          uint8_t* Sb = smem + L::kScaleOffset + b * kF4ScaleBuf;
          mbar_arrive_expect_tx(&sfull[b], nseg * kF4ScaleSeg);
          if (item.kind == 0)
            tma_load_5d(Sb, &tm_w1s, &sfull[b], 0, item.tile * 64, 0, 0, slot);
          else
            tma_load_4d(Sb, &tm_w2s, &sfull[b], 0, item.tile * 128, 0, slot);
          ++ic;
        }
        const CUtensorMap* tr = item.kind == 0 ? &tm_xg : &tm_act;
        const CUtensorMap* tr3 = item.kind == 0 ? &tm_xg3 : &tm_act3;
        for (int pc = p0; ok && pc < p1; pc += kNCap) {
          const int n = min(kNCap, p1 - pc);
          const int nbox = (n + kF4RouteBox - 1) / kF4RouteBox;
          const int rot = k_rotation(item, kst);
          for (int kq = 0; kq < kst; ++kq, ++it) {
            const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
            const int s = it % kStages;
            if (!mbar_wait(&done[s], ((it / kStages) & 1) ^ 1, err, a.wait_limit)) {
              ok = false;
              break;
            }
            uint8_t* P = smem + L::kStageOffset + s * L::kStageBytes;
            uint8_t* R = P + L::kRouteOffset;
            const int k0 = ks * kF4KS;
            const uint32_t rbytes = kNCap == kF4RouteBox ? 4 * kF4RouteBox * 128
                                                         : 4 * nbox * kF4RouteBox * 128;
            uint64_t* fb = &full[it % L::kNF];
            mbar_arrive_expect_tx(fb, kF4PackBytes + rbytes);
            if (item.kind == 0)
              tma_load_4d(P, &tm_w1p, fb, k0 / 2, item.tile * 64, 0, slot);
            else
              tma_load_3d(P, &tm_w2p, fb, k0 / 2, item.tile * 128, slot);
            if (kNCap == kF4RouteBox) {
              tma_load_3d(R, tr3, fb, 0, pc, k0 / 64);
            } else {
              for (int kb = 0; kb < 4; ++kb)
                for (int b = 0; b < nbox; ++b)
                  tma_load_2d(R + kb * L::kRBoxBytes + b * kF4RouteBox * 128, tr, fb,
                              k0 + kb * 64, pc + b * kF4RouteBox);
            }
          }
        }
      }
      if (!ok) {  // let every load already issued land before the CTA can exit
        for (uint32_t j = (it >= kStages ? it - kStages : 0); j < it; ++j)
          mbar_drain(&full[j % L::kNF], (j / L::kNF) & 1, err);
        for (uint32_t j = (ic >= (uint32_t)L::kScaleBufs ? ic - L::kScaleBufs : 0); j < ic; ++j)
          mbar_drain(&sfull[j % L::kScaleBufs], (j / L::kScaleBufs) & 1, err);
      }
    }
  } else if (warp == 1 || warp == kF4MmaWarp2) {
    // ------------------------------------------------------------ MMA issuers
    const int ix = warp == 1 ? 0 : 1;  // with two issuers: the stages it with it % 2 == ix
    if (lane == 0 && ix < L::kIssuers) {
      uint32_t it = 0, c = 0;
      bool ok = true;
      for (uint32_t r = 0; ok; ++r) {
        const int e = r % kRing;
        if (!mbar_wait(&ifull[e], (r / kRing) & 1, err, a.wait_limit)) break;
        const Item item = ring[e];
        mbar_arrive(&iempty[e]);
        if (item.kind < 0) break;
        const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
        const int kst = (item.kind == 0 ? a.H : a.I) / kF4KS;
        for (int pc = p0; ok && pc < p1; pc += kNCap, ++c) {
          const int n = min(kNCap, p1 - pc);
          const uint32_t idesc = idesc_f16(128, (n + 15) & ~15);
          const int acc = c & 1;
          if (!mbar_wait(&tempty[acc], ((c >> 1) & 1) ^ 1, err, a.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(acc * L::kAccBuf + ix * L::kAccPart);
          bool first = true;
          for (int kq = 0; kq < kst; ++kq, ++it) {
            if (L::kIssuers == 2 && (int)(it & 1) != ix) continue;
            const int s = it % kStages;
            const int t = it % kAStages;
            // the dequant warps acquired this stage's full barrier before releasing its afull
            // barrier, so the route rows of stage s are visible here as well
            if (!mbar_wait(&afull[it % L::kNAF], (it / L::kNAF) & 1, err, a.wait_limit)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // descriptors built once per stage; the 16 MMAs add constant offsets (the
            // issuing thread's own instruction latency, not the tensor pipe, bounds small-N
            // MMA rates, so the loop body is kept to the MMA and an add)
            const uint64_t b_desc =
                umma_desc_sw128(smem_u32(smem + L::kStageOffset + s * L::kStageBytes +
                                         L::kRouteOffset));
            const uint32_t a_tm = tmem + (uint32_t)(L::kABase + t * 128);
            mma_f16_tmem_a(d, a_tm, b_desc, idesc, first ? 0u : 1u);
            first = false;
#pragma unroll
            for (int j = 1; j < 16; ++j)
              mma_f16_tmem_a(d, a_tm + (uint32_t)(j * 8),
                             b_desc + (uint64_t)(((j >> 2) * L::kRBoxBytes + (j & 3) * 32) >> 4),
                             idesc, 1);
            mma_commit(&done[s]);
            mma_commit(&aempty[(it + kAStages) % L::kNAE]);  // the stage that refills t
          }
          if (ok) mma_commit(&tfull[acc]);
        }
      }
      mma_commit(&drain[ix]);  // every MMA issued, error or not, completes before TMEM is freed
      mbar_drain(&drain[ix], 0, err);
    }
  } else if (warp < kF4DequantWarp0) {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t c = 0, xb = 0;
    uint32_t eit = 0;  // the launch's stage count at the chunk's first stage
    bool ok = true;
    for (uint32_t r = 0; ok; ++r) {
      const int e = r % kRing;
      if (!warp_all(mbar_wait(&ifull[e], (r / kRing) & 1, err, a.wait_limit))) break;
      const Item item = ring[e];
      mbar_arrive(&iempty[e]);
      if (item.kind < 0) break;
      const int slot = a.seg_slot[item.u];
      const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
      const int kst = (item.kind == 0 ? a.H : a.I) / kF4KS;
      for (int pc = p0; ok && pc < p1; pc += kNCap, ++c, eit += kst) {
        const int n = min(kNCap, p1 - pc);
        const int acc = c & 1;
        if (!warp_all(mbar_wait(&tfull[acc], (c >> 1) & 1, err, a.wait_limit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * L::kAccBuf);
        // partial accumulators of the two issuers; a chunk of one stage has only that
        // stage's issuer's (issuers take the stages it with it % 2 == ix)
        const bool two = L::kIssuers == 2 && kst >= 2;
        const uint32_t only = L::kIssuers == 2 ? (eit & 1u) * (uint32_t)L::kAccPart : 0u;
        auto load_acc = [&](int cb, float* v) {
          tmem_ld16(tb + (two ? 0u : only) + cb, v);
          if (two) {
            float v2[16];
            tmem_ld16(tb + L::kAccPart + cb, v2);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += v2[i];
          }
        };
        if (item.kind == 0) {
          const bool up_rows = q >= 2;
          const int j = item.tile * 64 + (row & 63);
          const float g = a.g1.at((int64_t)slot * 2 * a.I + (up_rows ? a.I + j : j));
          __half* act = reinterpret_cast<__half*>(a.act);
          for (int cb = 0; ok && cb < n; cb += 16, ++xb) {
            const int x = xb & 1;
            float* xs = xchg + x * 64 * kF4XRow;
            float v[16];
            load_acc(cb, v);
            if (up_rows) {
              if (!warp_all(mbar_wait(&xempty[x], ((xb >> 1) & 1) ^ 1, err, a.wait_limit))) {
                ok = false;
                break;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) xs[(row - 64) * kF4XRow + i] = v[i] * g;
              mbar_arrive(&xfull[x]);
            } else {
              if (!warp_all(mbar_wait(&xfull[x], (xb >> 1) & 1, err, a.wait_limit))) {
                ok = false;
                break;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int col = cb + i;
                if (col < n) {
                  // with w_in the route's weight multiplies both halves before rounding
                  const float wr = (a.variant >> 2) ? a.topk_w[a.perm[pc + col]] : 1.0f;
                  const float gv = bf16_round(v[i] * g * wr);
                  const float uv = bf16_round(xs[row * kF4XRow + i] * wr);
                  // c2 = bf16(act(c1_gate) * c1_up), handed to the down GEMM as f16
                  const float ag = (a.variant & 3) == 0 ? silu_f(gv) : gelu_act(a.variant & 3, gv);
                  const float c2 = bf16_round(ag * uv);
                  act[(int64_t)(pc + col) * a.I + j] =
                      __float2half_rn(fminf(fmaxf(c2, -65504.f), 65504.f));
                }
              }
              mbar_arrive(&xempty[x]);
            }
          }
          if (ok && !up_rows) {
            fence_proxy_async_global();
            __syncwarp();
            if (lane == 0) {
              const int target = up_target(a, item.u, kNCap, 2);
              if (atom_add_acq_rel(a.up_done + item.u * kDoneStride, 1) + 1 == target) {
                const int pos = atomicAdd(a.ready_tail, 1);
                st_release(a.ready_slots + pos, item.u);
              }
            }
          }
        } else {
          const int h = item.tile * 128 + row;
          const float g = a.g2.at((int64_t)slot * a.H + h);
          for (int cb = 0; cb < n; cb += 16) {
            float v[16];
            load_acc(cb, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = cb + i;
              if (col < n) {
                const int p = pc + col;
                const float w = (a.variant >> 2) ? 1.0f : a.topk_w[a.perm[p]];
                a.c3[(int64_t)p * a.H + h] = __float2bfloat16_rn(v[i] * g * w);
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ dequant (warps 6-21)
    const int dw = warp - kF4DequantWarp0;
    const int grp = dw / kF4GroupWarps;     // stages it with it % kF4Groups == grp
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int part = (dw % kF4GroupWarps) >> 2;  // which kF4PartK of the stage's K
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t it = 0, ic = 0;
    bool ok = true;
    for (uint32_t r = 0; ok; ++r) {
      const int e = r % kRing;
      if (!warp_all(mbar_wait(&ifull[e], (r / kRing) & 1, err, a.wait_limit))) break;
      const Item item = ring[e];
      mbar_arrive(&iempty[e]);
      if (item.kind < 0) break;
      const int p0 = a.seg_start[item.u], p1 = a.seg_start[item.u + 1];
      const int kst = (item.kind == 0 ? a.H : a.I) / kF4KS;
      const int nchunk = (p1 - p0 + kNCap - 1) / kNCap;
      const int sb = ic % L::kScaleBufs;
      if (!warp_all(mbar_wait(&sfull[sb], (ic / L::kScaleBufs) & 1, err, a.wait_limit))) break;
      const uint8_t* Sb = smem + L::kScaleOffset + sb * kF4ScaleBuf;
      const int rot = k_rotation(item, kst);
      for (int ch = 0; ok && ch < nchunk; ++ch) {
        for (int kq = 0; kq < kst; ++kq, ++it) {
          if (kF4Groups > 1 && (int)(it % kF4Groups) != grp) continue;
          const int ks = kq + rot < kst ? kq + rot : kq + rot - kst;
          const int s = it % kStages;
          const int t = it % kAStages;
          // this stage's load, then (from the second use of A stage t on) the MMAs of stage
          // it - kAStages, which read A stage t before this fill; phase counts of the
          // group's own barriers: full[b] once per stage it with it % kNF == b, aempty[b]
          // once per stage it >= kAStages with it % kNAE == b
          if (!warp_all(mbar_wait(&full[it % L::kNF], (it / L::kNF) & 1, err, a.wait_limit) &&
                        (it < (uint32_t)kAStages ||
                         mbar_wait(&aempty[it % L::kNAE], ((it - kAStages) / L::kNAE) & 1, err,
                                   a.wait_limit)))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* P = smem + L::kStageOffset + s * L::kStageBytes;
          // this row's scale bytes for K chunk ks, this part: row byte ks * 16 + part *
          // kF4PartK / 16, in 128-byte segments of 128 rows with the 128-byte swizzle
          constexpr int kSB = kF4PartK / 16;  // scale bytes (= 16-element blocks) per part
          const int off = ks * 16 + part * kSB;
          const uint8_t* sp = Sb + (off >> 7) * kF4ScaleSeg + row * 128 +
                              ((((off >> 4) & 7) ^ (row & 7)) << 4) + (off & 15);
          uint32_t scw[kSB / 4];
#pragma unroll
          for (int i = 0; i < kSB / 4; ++i) scw[i] = reinterpret_cast<const uint32_t*>(sp)[i];
          const uint32_t a_col = lane_base + (uint32_t)(L::kABase + t * 128 + part * (kF4PartK / 2));
#pragma unroll
          for (int c4 = 0; c4 < kF4PartK / 32; ++c4) {
            // 16 bytes = 32 codes = blocks 2*c4 and 2*c4+1 of this part; the 128-byte swizzle
            // puts logical 16-byte chunk k of row r at chunk k ^ (r & 7)
            const int chunk = (part * (kF4PartK / 32) + c4) ^ (row & 7);
            const uint4 pk = *reinterpret_cast<const uint4*>(P + row * 128 + chunk * 16);
            const __half2 s2 = e4m3x2_to_h2(scw[c4 >> 1] >> (16 * (c4 & 1)));
            const __half2 slo = __low2half2(s2), shi = __high2half2(s2);
            uint32_t o[16];
            dequant_word(pk.x, slo, o);
            dequant_word(pk.y, slo, o + 4);
            dequant_word(pk.z, shi, o + 8);
            dequant_word(pk.w, shi, o + 12);
            tmem_st16(a_col + c4 * 16, o);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[it % L::kNAF]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[sb]);  // this warp's reads of the item's scales are done
      ++ic;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Gather the input row of every grouped route as f16: xg[p] = f16(x[perm[p] / K]),
// saturated to the f16 range.
__global__ void __launch_bounds__(256)
gather_rows_f16_kernel(const uint4* __restrict__ x, int K, int H8,
                       const int32_t* __restrict__ perm, const int32_t* __restrict__ seg_start,
                       const int32_t* __restrict__ num_unique, uint4* __restrict__ xg) {
  pdl_wait();
  pdl_trigger();
  // a block converts whole rows (grid-stride over positions), four 16-byte loads in flight
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
      for (int j = 0; j < 4; ++j) {
        if (c + j * (int)blockDim.x >= H8) continue;
        float f[8];
        bf16x8_to_f32(v[j], f);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float lo = fminf(fmaxf(f[2 * k], -65504.f), 65504.f);
          const float hi = fminf(fmaxf(f[2 * k + 1], -65504.f), 65504.f);
          ow[k] = h2_bits(__floats2half2_rn(lo, hi));
        }
        dst[c + j * blockDim.x] = o;
      }
    }
  }
}

// Dequantise NVFP4 rows to fp32 with the FFN kernel's own decoding (f16 code * scale, then
// the row global): one thread per 32 elements.
__global__ void __launch_bounds__(256)
nvfp4_dequant_kernel(const uint4* __restrict__ packed, const uint32_t* __restrict__ scale,
                     RowScale global_, int64_t rows, int K, float* __restrict__ out) {
  const int per_row = K / 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * per_row) return;
  const int64_t r = i / per_row;
  const int c = (int)(i % per_row);
  const uint4 pk = packed[i];
  const uint32_t sc = reinterpret_cast<const uint16_t*>(scale)[i];
  const __half2 s2 = e4m3x2_to_h2(sc);
  uint32_t o[16];
  dequant_word(pk.x, __low2half2(s2), o);
  dequant_word(pk.y, __low2half2(s2), o + 4);
  dequant_word(pk.z, __high2half2(s2), o + 8);
  dequant_word(pk.w, __high2half2(s2), o + 12);
  const float g = global_.at(r);
  float* dst = out + r * K + c * 32;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&o[k]));
    dst[2 * k] = f.x * g;
    dst[2 * k + 1] = f.y * g;
  }
}

template <int kNCap>
int launch_fp4(const CUtensorMap* maps, const FfnArgs& args, int grid, cudaStream_t st) {
  using L = Fp4Smem<kNCap>;
  auto kern = expert_ffn_fp4_tc_kernel<kNCap>;
  // the dynamic shared-memory limit is a per-device attribute: raise it once per device
  static bool attr_set[kMaxAttrDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxAttrDevices || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (dev >= 0 && dev < kMaxAttrDevices) attr_set[dev] = true;
  }
  TW_LAUNCH(kern, dim3(grid), dim3(kF4Threads), L::kBytes, st, maps[0], maps[1], maps[2],
            maps[3], maps[4], maps[5], maps[6], maps[7], args);
  TW_CHECK_LAUNCH("expert_ffn_fp4_tc_kernel");
  return TW_OK;
}

}  // namespace

int launch_expert_ffn_fp4_tc(const __nv_bfloat16* x, int64_t T, int K, int H, int I,
                             const uint8_t* w1p, const uint8_t* w1s, RowScale w1g,
                             const uint8_t* w2p, const uint8_t* w2s, RowScale w2g,
                             int64_t S, const float* topk_w, const Workspace& ws, int64_t n,
                             cudaStream_t st, FfnAct fx) {
  TW_CHECK_ARG(H % kF4KS == 0 && I % kF4KS == 0,
               "NVFP4 tensor-core FFN: need H %% 256 == 0 and I %% 256 == 0");
  TW_CHECK_ARG(n <= (int64_t)1 << 30 && S < (1 << 30), "NVFP4 tensor-core FFN: sizes out of range");
  TW_CHECK_ARG(aligned16(w1s) && aligned16(w2s), "NVFP4 tensor-core FFN: scale banks must be 16-byte aligned");
  TW_CHECK_ARG(H <= kF4MaxK && I <= kF4MaxK, "NVFP4 tensor-core FFN: need H, I <= %d", kF4MaxK);
  // w1 packed, w1 scales, w2 packed, w2 scales, route rows and activations (2-D, 16-row
  // boxes), route rows and activations (3-D: four K boxes of a stage in one box)
  CUtensorMap maps[8];
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint64_t uH = H, uI = I, uS = S;
  {  // [S][half][I rows][H/2]: one box = the stage's 64 gate rows and 64 up rows
    const uint64_t d[4] = {uH / 2, uI, 2, uS};
    const uint64_t sb[3] = {uH / 2, uI * uH / 2, 2 * uI * uH / 2};
    const uint32_t b[4] = {kF4KS / 2, 64, 2, 1};
    if (int rc = make_tmap(&maps[0], u8, w1p, 4, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {  // [S][128-byte segment][half][I rows][128]: all of an up item's scales in one box
    const uint64_t row = uH / 16, nseg = (row + 127) / 128;
    const uint64_t d[5] = {row < 128 ? row : 128, uI, 2, nseg, uS};
    const uint64_t sb[4] = {row, uI * row, 128, 2 * uI * row};
    const uint32_t b[5] = {128, 64, 2, (uint32_t)nseg, 1};
    if (int rc = make_tmap(&maps[1], u8, w1s, 5, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {
    const uint64_t d[3] = {uI / 2, uH, uS};
    const uint64_t sb[2] = {uI / 2, uH * uI / 2};
    const uint32_t b[3] = {kF4KS / 2, 128, 1};
    if (int rc = make_tmap(&maps[2], u8, w2p, 3, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {
    const uint64_t row = uI / 16, nseg = (row + 127) / 128;
    const uint64_t d[4] = {row < 128 ? row : 128, uH, nseg, uS};
    const uint64_t sb[3] = {row, 128, uH * row};
    const uint32_t b[4] = {128, 128, (uint32_t)nseg, 1};
    if (int rc = make_tmap(&maps[3], u8, w2s, 4, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  const CUtensorMapDataType f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    const uint64_t d[2] = {uH, (uint64_t)n};
    const uint64_t sb[1] = {uH * 2};
    const uint32_t b[2] = {64, kF4RouteBox};
    if (int rc = make_tmap(&maps[4], f16, ws.xg, 2, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {
    const uint64_t d[2] = {uI, (uint64_t)n};
    const uint64_t sb[1] = {uI * 2};
    const uint32_t b[2] = {64, kF4RouteBox};
    if (int rc = make_tmap(&maps[5], f16, ws.act, 2, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {
    const uint64_t d[3] = {64, (uint64_t)n, uH / 64};
    const uint64_t sb[2] = {uH * 2, 128};
    const uint32_t b[3] = {64, kF4RouteBox, 4};
    if (int rc = make_tmap(&maps[6], f16, ws.xg, 3, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  {
    const uint64_t d[3] = {64, (uint64_t)n, uI / 64};
    const uint64_t sb[2] = {uI * 2, 128};
    const uint32_t b[3] = {64, kF4RouteBox, 4};
    if (int rc = make_tmap(&maps[7], f16, ws.act, 3, d, sb, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  const int sms = num_sms();
  {
    const int H8 = H / 8;
    const int blocks = (int)std::min<int64_t>(n, (int64_t)sms * 8);
    TW_LAUNCH(gather_rows_f16_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st,
              reinterpret_cast<const uint4*>(x), K, H8, ws.perm, ws.seg_start, ws.num_unique,
              reinterpret_cast<uint4*>(ws.xg));
    TW_CHECK_LAUNCH("gather_rows_f16_kernel");
  }
  const int cap = expert_ffn_fp4_tc_route_cap(T);
  const int64_t max_u = std::min<int64_t>(n, S + n / cap);
  FfnArgs fa{H, I, I / 64, H / 128, ws.num_unique, ws.seg_start, ws.seg_slot, ws.perm,
             topk_w, ws.act, ws.c3, ws.up_ctr, ws.down_ctr, ws.up_done, ws.ready_tail,
             ws.ready_slots, ws.err, w1g, w2g, S, ffn_wait_limit(), K, 0};
  fa.variant = fx.act | (fx.w_in << 2);
  const int grid = (int)std::min<int64_t>(max_u * (fa.tu + fa.td), sms);
  if (cap == 16) return launch_fp4<16>(maps, fa, grid, st);
  if (cap == 64) return launch_fp4<64>(maps, fa, grid, st);
  return launch_fp4<128>(maps, fa, grid, st);
}

// Route-tile capacity (routes per MMA chunk): a slot has at most T routes.
int expert_ffn_fp4_tc_route_cap(int64_t T) { return T <= 16 ? 16 : T <= 64 ? 64 : 128; }

}  // namespace tw

using namespace tw;

extern "C" int tw_nvfp4_dequantize(const void* packed, const void* scale, const void* global_,
                                   int global_dtype, int64_t rows, int K, float* out,
                                   void* stream) {
  TW_CHECK_ARG(rows >= 0 && K > 0 && K % 32 == 0, "nvfp4_dequantize: need K %% 32 == 0");
  TW_CHECK_ARG(global_dtype == TW_F32 || global_dtype == TW_F16,
               "nvfp4_dequantize: row globals must be fp32 or fp16");
  TW_CHECK_ARG(aligned16(packed) && (reinterpret_cast<uintptr_t>(scale) & 1) == 0,
               "nvfp4_dequantize: packed must be 16-byte and scale 2-byte aligned");
  if (rows == 0) return TW_OK;
  const int64_t threads = rows * (K / 32);
  nvfp4_dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(packed), reinterpret_cast<const uint32_t*>(scale),
      RowScale{global_, global_dtype == TW_F16}, rows, K, out);
  TW_CHECK_LAUNCH("nvfp4_dequant_kernel");
  return TW_OK;
}
