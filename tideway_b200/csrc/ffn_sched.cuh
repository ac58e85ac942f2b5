// Work scheduling shared by the persistent tensor-core expert-FFN kernels (BF16 and NVFP4
// weights): the argument block, dependency-aware item claiming and the memory-order
// helpers the up -> down hand-off uses.
#pragma once

#include "moe_common.cuh"
#include "tc_common.cuh"

namespace tw {
namespace {

using namespace tc;

constexpr int kRing = 4;  // claimed work items in flight inside a CTA

struct FfnArgs {
  int H, I;
  int tu, td;               // weight tiles per slot: up (64 gate + 64 up rows), down (128 rows)
  const int32_t* num_unique;
  const int32_t* seg_start;
  const int32_t* seg_slot;
  const int32_t* perm;
  const float* topk_w;
  __nv_bfloat16* act;       // [n, I]  position order
  __nv_bfloat16* c3;        // [n, H]  position order
  int* up_ctr;              // next unclaimed up tile   (zeroed by the grouping kernel)
  int* down_ctr;            // next unclaimed down tile (zeroed by the grouping kernel)
  int* up_done;             // [n * 32] per-segment up-tile arrivals (128-byte stride)
  int* ready_tail;          // number of slots appended to ready_slots
  int* ready_slots;         // [n] slots in the order their activations became complete
  int* err;
  RowScale g1;              // NVFP4 only: [S, 2I] per-row global scale of w1
  RowScale g2;              // NVFP4 only: [S, H] per-row global scale of w2
  int64_t num_slots;        // S (host side: tensor-map extents)
  uint32_t wait_limit;      // polls before a bounded wait gives up (tw_set_wait_limit)
  int route_k;              // routes per token (position p holds token perm[p] / route_k)
  int token_rows;           // 1: up tiles read x's token rows (decode), not gathered rows
  // epilogue variant (fills the struct's tail padding): bits 0-1 the gate activation (0 SiLU,
  // 1 GELU, 2 GELU tanh form), bit 2 the route weight on the up projection (gathered rows)
  int variant;
};

struct Item {
  int kind;  // 0 up, 1 down, -1 end
  int u, tile;
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Slot u's completion counter lives on its own 128-byte line.
constexpr int kDoneStride = 32;

// Number of arrivals that make a slot's activations complete: every up item and route chunk
// is published by `per_tile` epilogue warps (all of the kernel's epilogue warps, or the ones
// that write activations), a.tu items per segment.
__device__ __forceinline__ int up_target(const FfnArgs& a, int u, int n_cap, int per_tile) {
  const int n = a.seg_start[u + 1] - a.seg_start[u];
  return a.tu * per_tile * ((n + n_cap - 1) / n_cap);
}

__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Producer-side work claiming.  Up tiles come from one counter in slot order.  When the
// last up tile of a slot publishes its activations, the slot is appended to a ready list;
// down tiles are tickets over that list (ticket x = tile x % td of the (x / td)-th slot to
// become ready).  A producer prefers a ready down tile; a ticket whose slot is not yet
// listed is kept pending while the producer goes on claiming up tiles, so no producer
// idles while up work remains and claims never serialise on a compare-and-swap.
struct Claimer {
  bool up_left = true;
  int pending = -1;  // a down ticket not yet resolvable
};

__device__ bool claim_item(const FfnArgs& a, int U, Claimer& c, Item& it, int* err) {
  const int n_up = U * a.tu, n_dn = U * a.td;
  for (uint32_t spins = 0; spins < a.wait_limit; ++spins) {
    if (c.pending < 0) {
      const int dn = ld_relaxed(a.down_ctr);
      if (dn >= n_dn) {
        it.kind = -1;
        return true;
      }
      if (!c.up_left || dn < ld_relaxed(a.ready_tail) * a.td) {
        const int x = atomicAdd(a.down_ctr, 1);
        if (x >= n_dn) {
          it.kind = -1;
          return true;
        }
        c.pending = x;
      }
    }
    if (c.pending >= 0) {
      const int u = ld_acquire(a.ready_slots + c.pending / a.td);
      if (u >= 0) {
        it.kind = 1;
        it.u = u;
        it.tile = c.pending % a.td;
        c.pending = -1;
        return true;
      }
    }
    if (c.up_left) {
      const int x = atomicAdd(a.up_ctr, 1);
      if (x < n_up) {
        it.kind = 0;
        it.u = x / a.tu;
        it.tile = x % a.tu;
        return true;
      }
      c.up_left = false;
      continue;
    }
    if ((spins & 255) == 255 && ld_relaxed(err) != 0) return false;
    __nanosleep(256);  // only unresolved down work is left: back off
  }
  atomicCAS(err, 0, kErrWaitTimeout);
  return false;
}

// First K stage of an item: consecutive items start at different K offsets so the CTAs
// streaming at the same moment do not walk the same column of neighbouring rows.
__device__ __forceinline__ int k_rotation(const Item& item, int kst) {
#if TW_FFN_KROT
  const unsigned key = (unsigned)item.u * 64u + (unsigned)item.tile * 2u + (unsigned)item.kind;
  return (int)((key * 2654435761u) >> 16) % kst;
#else
  return 0;
#endif
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

}  // namespace
}  // namespace tw
