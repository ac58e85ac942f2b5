// Route grouping by slot for the expert-FFN kernels: a stable counting sort of the T*K
// routes by slot id into positions, with slots of more routes than one MMA route tile cut
// into segments.  Shared by the FFN's own grouping launch (moe_ffn.cu) and the LRU ensure
// that groups the routes it has just rewritten into slots (slot_cache.cu).
#pragma once

#include "moe_common.cuh"

namespace tw {
namespace {

constexpr int kGroupThreads = 1024;
constexpr int kIdsPerLane = 16;  // grouping: ids a lane keeps in registers (n <= 16384 fully)

// Lanes of this warp whose key equals this lane's, for keys in [0, 2^nbits): one ballot per
// key bit (the peer set is the intersection of the lanes agreeing on every bit).  The same
// set as __match_any_sync, at a fraction of its cost when most keys differ.
__device__ __forceinline__ unsigned match_by_ballots(int key, int nbits) {
  unsigned peers = 0xffffffffu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1;
    const unsigned bb = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? bb : ~bb;
  }
  return peers;
}

// Stable grouping of the n routes by slot.  Small problems: shared-memory atomics count,
// one warp places the routes 32 at a time.  Many routes over few slots (prefill: per_warp):
// each of the 32 warps counts and later places its own contiguous slice of routes through a
// per-warp histogram, so placement runs 32-wide and counting needs no atomics.
// Exclusive scan over slots of packed (count | segments << 16): low half = route offset,
// high half = segment index.  A slot with more than `split` routes (split > 0) becomes
// ceil(count / split) consecutive segments of at most `split` routes each, so the FFN
// kernels take its route chunks as independent work items.  n <= 65535 and at most one
// segment per route keep the halves apart (unsigned: the high half may reach 65535).
// Writes num_unique, seg_start and seg_slot, clears the FFN kernels' hand-off state of the
// segments in use and leaves cnt[s] = the slot's first position.  Every thread of a
// kGroupThreads block calls it, with cnt[s] = the slot's route count (visible to all).
__device__ void scan_slots(int* cnt, int S, int split, const Workspace& ws, unsigned* warp_tot,
                           unsigned* s_total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (S + kGroupThreads - 1) / kGroupThreads;
  const int s0 = tid * per;
  auto packed = [&](int c) -> unsigned {
    const unsigned segs = c <= 0 ? 0u : split > 0 ? (unsigned)((c + split - 1) / split) : 1u;
    return (unsigned)c + (segs << 16);
  };
  unsigned local = 0;
  for (int i = 0; i < per; ++i) {
    const int s = s0 + i;
    if (s < S) local += packed(cnt[s]);
  }
  unsigned inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const unsigned w = warp_tot[lane];
    unsigned wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    warp_tot[lane] = wi - w;
    if (lane == 31) *s_total = wi;
  }
  __syncthreads();
  const unsigned tot = *s_total;
  unsigned run = warp_tot[warp] + inc - local;
  for (int i = 0; i < per; ++i) {
    const int s = s0 + i;
    if (s < S) {
      const int c = cnt[s];
      const int p = (int)(run & 0xffffu);
      if (c > 0) {
        const int u = (int)(run >> 16);
        const int step = split > 0 ? split : c;
        for (int j = 0; j * step < c; ++j) {
          ws.seg_start[u + j] = p + j * step;
          ws.seg_slot[u + j] = s;
        }
      }
      cnt[s] = p;  // cursor = the slot's first position
      run += packed(c);
    }
  }
  if (tid == 0) {
    ws.num_unique[0] = (int)(tot >> 16);
    ws.seg_start[tot >> 16] = (int)(tot & 0xffffu);
  }
  __syncthreads();
  // the FFN kernels' per-segment hand-off state: only the segments in use
  for (int u = tid; u < (int)(tot >> 16); u += kGroupThreads) {
    ws.up_done[u * 32] = 0;
    ws.ready_slots[u] = -1;
  }
}

// Decode batches (n <= kSmallRoutes routes): the same grouping without a pass over the S
// slots.  Route r's position is the number of valid routes before it in (slot, route) order
// -- the counting sort's stable order -- found by one thread per route over the n keys;
// each slot's first route computes its segment index from the slots before it and writes
// its segments.  The outputs are those of the counting sort, bit for bit.
constexpr int kSmallRoutes = 256;

__device__ void group_routes_small(const int32_t* __restrict__ ids, int n, int S, int split,
                                   const Workspace& ws) {
  __shared__ int key[kSmallRoutes];    // slot of route r, or S for a skipped route
  __shared__ int count[kSmallRoutes];  // first route of a slot: the slot's routes; else -1
  __shared__ int s_routes, s_segs;
  const int tid = threadIdx.x;
  auto segs_of = [&](int c) { return split > 0 ? (c + split - 1) / split : 1; };
  if (tid == 0) s_routes = s_segs = 0;
  int s = S;
  if (tid < n) {
    const int v = ids[tid];
    s = v >= 0 && v < S ? v : S;
    key[tid] = s;
  }
  __syncthreads();
  int pos = -1, before = 0, same = 0;
  if (tid < n && s < S) {
    int rank = 0;
    for (int r = 0; r < n; ++r) {
      const int k = key[r];
      rank += k < s;
      before += k == s && r < tid;
      same += k == s;
    }
    pos = rank + before;
  }
  if (tid < n) count[tid] = (s < S && before == 0) ? same : -1;
  __syncthreads();
  if (tid < n && s < S && before == 0) {  // the slot's first route: its segments
    int u = 0;
    for (int r = 0; r < n; ++r)
      if (count[r] > 0 && key[r] < s) u += segs_of(count[r]);
    const int step = split > 0 ? split : same;
    for (int j = 0; j * step < same; ++j) {
      ws.seg_start[u + j] = pos + j * step;
      ws.seg_slot[u + j] = s;
    }
    atomicAdd(&s_routes, same);
    atomicAdd(&s_segs, segs_of(same));
  }
  if (tid < n) {
    ws.pos[tid] = pos;
    if (pos >= 0) ws.perm[pos] = tid;
  }
  __syncthreads();
  const int total = s_segs;
  if (tid == 0) {
    ws.num_unique[0] = total;
    ws.seg_start[total] = s_routes;
  }
  // the FFN kernels' per-segment hand-off state: only the segments in use
  for (int u = tid; u < total; u += kGroupThreads) {
    ws.up_done[u * 32] = 0;
    ws.ready_slots[u] = -1;
  }
}

// One block of kGroupThreads threads: the stable grouping of the n routes by slot into the
// workspace (positions, segments, the FFN kernels' hand-off state).  cnt: dynamic shared
// memory of S ints (+ 32 * S uint16 with per_warp).  kSmall: decode batches take
// group_routes_small (the FFN's own grouping launch; inside the LRU ensure's launch, which
// is register-bound at 1024 threads, the extra path spilled and the step measured 3% slower).
template <bool kSmall>
__device__ void group_routes(const int32_t* __restrict__ ids, int n, int S, int per_warp,
                             int split, const Workspace& ws, int* cnt) {
  // per_warp: uint16 hist[32][S] after cnt: a warp's count per slot, then its offset within
  // the slot's segment (routes of lower warps first), then its running cursor
  unsigned short* hist = reinterpret_cast<unsigned short*>(cnt + S);
  __shared__ unsigned warp_tot[32];
  __shared__ unsigned s_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    ws.err[0] = 0;
    ws.up_ctr[0] = 0;
    ws.down_ctr[0] = 0;
    ws.ready_tail[0] = 0;
  }
  if (kSmall && !per_warp && n <= kSmallRoutes) {
    group_routes_small(ids, n, S, split, ws);
    return;
  }
  const int seg = (n + 31) / 32;  // per_warp: routes [warp * seg, warp * seg + seg)
  const int kbits = 32 - __clz(S);  // bits of the keys 0..S (S marks a skipped route)
  const int wr0 = min(n, warp * seg), wr1 = min(n, wr0 + seg);
  // per_warp: the warp's first kIdsPerLane * 32 ids, loaded once (all loads in flight
  // together) and kept in registers for both the count and the placement pass
  int vid[kIdsPerLane];
  if (per_warp) {
#pragma unroll
    for (int j = 0; j < kIdsPerLane; ++j) {
      const int r = wr0 + 32 * j + lane;
      vid[j] = r < wr1 ? ids[r] : -1;
    }
    for (int i = tid; i < 32 * S; i += kGroupThreads) hist[i] = 0;
    __syncthreads();
    for (int base = wr0; base < wr1; base += 32) {
      const int r = base + lane;
      const int jj = (base - wr0) >> 5;
      int s = -1;
#pragma unroll
      for (int j = 0; j < kIdsPerLane; ++j)
        if (j == jj) s = vid[j];
      if (jj >= kIdsPerLane) s = r < wr1 ? ids[r] : -1;
      const bool ok = r < wr1 && s >= 0 && s < S;
      const unsigned peers = match_by_ballots(ok ? s : S, kbits);  // key S: skipped routes
      if (ok && lane == __ffs(peers) - 1) hist[warp * S + s] += (unsigned short)__popc(peers);
      __syncwarp();
    }
    __syncthreads();
    for (int s = tid; s < S; s += kGroupThreads) {
      int run = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = hist[w * S + s];
        hist[w * S + s] = (unsigned short)run;
        run += c;
      }
      cnt[s] = run;
    }
    __syncthreads();
  } else {
    for (int s = tid; s < S; s += kGroupThreads) cnt[s] = 0;
    __syncthreads();
    for (int r = tid; r < n; r += kGroupThreads) {
      const int s = ids[r];
      if (s >= 0 && s < S) atomicAdd(&cnt[s], 1);
    }
    __syncthreads();
  }
  scan_slots(cnt, S, split, ws, warp_tot, &s_total);
  if (per_warp) {
    // stable placement, every warp over its own slice: segment start + the warp's offset
    for (int base = wr0; base < wr1; base += 32) {
      const int r = base + lane;
      const int jj = (base - wr0) >> 5;
      int s = -1;
#pragma unroll
      for (int j = 0; j < kIdsPerLane; ++j)
        if (j == jj) s = vid[j];
      if (jj >= kIdsPerLane) s = r < wr1 ? ids[r] : -1;
      const bool ok = r < wr1 && s >= 0 && s < S;
      const unsigned peers = match_by_ballots(ok ? s : S, kbits);
      const int leader = __ffs(peers) - 1;
      int start = 0;
      if (ok && lane == leader) {
        start = cnt[s] + hist[warp * S + s];
        hist[warp * S + s] += (unsigned short)__popc(peers);
      }
      start = __shfl_sync(0xffffffffu, start, leader);
      if (ok) {
        const int p = start + __popc(peers & ((1u << lane) - 1));
        ws.perm[p] = r;
        ws.pos[r] = p;
      } else if (r < wr1) {
        ws.pos[r] = -1;
      }
      __syncwarp();
    }
  } else if (warp == 0) {
    // stable placement: warp 0 walks the routes in order, 32 at a time
    for (int base = 0; base < n; base += 32) {
      const int r = base + lane;
      const int s = r < n ? ids[r] : -1;
      const bool ok = r < n && s >= 0 && s < S;
      const unsigned peers = match_by_ballots(ok ? s : S, kbits);  // key S: skipped routes
      const int leader = __ffs(peers) - 1;
      int start = 0;
      if (ok && lane == leader) {
        start = cnt[s];
        cnt[s] = start + __popc(peers);
      }
      start = __shfl_sync(0xffffffffu, start, leader);
      if (ok) {
        const int p = start + __popc(peers & ((1u << lane) - 1));
        ws.perm[p] = r;
        ws.pos[r] = p;
      } else if (r < n) {
        ws.pos[r] = -1;
      }
      __syncwarp();
    }
  }
}

}  // namespace
}  // namespace tw
