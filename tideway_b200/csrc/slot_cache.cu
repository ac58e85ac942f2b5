// Expert-slot table kernels: LRU ensure, whole-layer materialise, reset, prefill hit
// compaction, and the graph-safe multi-bank row copy.
//
// The LRU ensure is one CTA of 1024 threads.  The reference picks victims by a sequential
// argmin over slot usage (backends/freetoken_tideway/freetoken/moe/shift.py:761-773); since
// each pick only retires the chosen slot, the picks are exactly the M smallest
// (usage, slot) keys among eligible slots, in ascending order.  This kernel finds them with
// a block-wide radix select over 64-bit keys and ranks the M winners, so the cost does not
// grow with the number of misses.
#include <algorithm>

#include "common.cuh"
#include "moe_group.cuh"

namespace tw {
namespace {

constexpr int kEnsureThreads = 1024;
constexpr int kMaxIds = 8192;
constexpr int kMaxExperts = 1024;
constexpr int kMaxSlots = 16384;
constexpr int kSlotBits = 14;  // kMaxSlots == 1 << kSlotBits
constexpr int kSlotsPerThread = kMaxSlots / kEnsureThreads;
constexpr unsigned long long kIneligibleHigh = (~0ull) << kSlotBits;

__device__ __forceinline__ int block_excl_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const int r = warp_tot[warp] + inc - v;
  __syncthreads();
  return r;
}

// The M smallest (usage << 14 | slot) keys among the slots not touched this step (usage !=
// step) and not pinned, ranked ascending into vslot[0..M): the victims of M sequential
// argmin picks.  A block-wide radix select over 64-bit keys finds the M-th smallest key;
// the winners are then ranked among themselves.  Every thread of the block calls it.
struct VictimScratch {
  int* vslot;                 // [kMaxExperts] victim of rank i
  unsigned long long* vkey;   // [kMaxExperts]
  int* hist;                  // [256]
  int* warp_tot;              // [32]
  int* s_total;
  int* s_nvict;
  int* s_digit;
  int* s_rem;
  unsigned long long* s_maxkey;
};

__device__ void select_victims(int M, int S, long long step, const int64_t* __restrict__ usage,
                               const int32_t* __restrict__ pinned, const VictimScratch& v) {
  const int tid = threadIdx.x;
  int* const vslot = v.vslot;
  unsigned long long* const vkey = v.vkey;
  int* const hist = v.hist;
  int* const warp_tot = v.warp_tot;
  int& s_total = *v.s_total;
  int& s_nvict = *v.s_nvict;
  int& s_digit = *v.s_digit;
  int& s_rem = *v.s_rem;
  unsigned long long& s_maxkey = *v.s_maxkey;
  if (tid == 0) s_maxkey = 0ull;
  __syncthreads();
  // keys: (usage << 14) | slot for eligible slots; ineligible slots keep the slot order
  // above every eligible key (the reference's argmin then picks the lowest such index).
  unsigned long long key[kSlotsPerThread];
  int nelig = 0;
#pragma unroll
  for (int j = 0; j < kSlotsPerThread; ++j) {
    const int s = tid + j * kEnsureThreads;
    key[j] = ~0ull;
    if (s < S) {
      const long long u = usage[s];
      const bool elig = u != step && !(pinned && pinned[s] != 0);
      key[j] = elig ? (((unsigned long long)u << kSlotBits) | (unsigned)s)
                    : (kIneligibleHigh | (unsigned)s);
      if (elig) {
        ++nelig;
        atomicMax(&s_maxkey, key[j]);
      }
    }
  }
  // count eligible slots
  int tot_elig;
  {
    const int dummy = block_excl_scan(nelig, warp_tot, &s_total);
    (void)dummy;
    tot_elig = s_total;
  }
  // radix select of the M-th smallest key
  unsigned long long prefix = 0ull, mask = 0ull;
  int first_shift = 56;
  if (tot_elig >= M) {
    const unsigned long long mk = s_maxkey;
    const int topbit = 63 - __clzll(mk | 1ull);
    first_shift = (topbit / 8) * 8;
    mask = first_shift >= 56 ? 0ull : (~0ull << (first_shift + 8));
  }
  if (tid == 0) s_rem = M;
  __syncthreads();
  for (int shift = first_shift; shift >= 0; shift -= 8) {
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSlotsPerThread; ++j) {
      if (tid + j * kEnsureThreads < S && (key[j] & mask) == prefix)
        atomicAdd(&hist[(key[j] >> shift) & 255], 1);
    }
    __syncthreads();
    if (tid < 32) {
      // warp 0: lane l owns bins 8l..8l+7
      int c[8], lsum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c[q] = hist[tid * 8 + q];
        lsum += c[q];
      }
      int inc = lsum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (tid >= o) inc += v;
      }
      const int rem = s_rem;
      const int before = inc - lsum;
      const unsigned ball = __ballot_sync(0xffffffffu, inc >= rem);
      const int owner = __ffs(ball) - 1;
      if (tid == owner) {
        int cum = before, d = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (cum + c[q] >= rem) {
            d = q;
            break;
          }
          cum += c[q];
        }
        s_digit = tid * 8 + d;
        s_rem = rem - cum;
      }
    }
    __syncthreads();
    prefix |= (unsigned long long)s_digit << shift;
    mask |= 255ull << shift;
    __syncthreads();
  }
  // prefix is now the M-th smallest key; gather the winners and rank them
  if (tid == 0) s_nvict = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kSlotsPerThread; ++j) {
    if (tid + j * kEnsureThreads < S && key[j] <= prefix) {
      const int p = atomicAdd(&s_nvict, 1);
      if (p < kMaxExperts) vkey[p] = key[j];
    }
  }
  __syncthreads();
  if (tid < M) {
    const unsigned long long mine = vkey[tid];
    int r = 0;
    for (int j = 0; j < M; ++j) r += vkey[j] < mine;
    vslot[r] = (int)(mine & ((1ull << kSlotBits) - 1));
  }
  __syncthreads();
}

// The LRU ensure of one call, by one block of kEnsureThreads threads; ends with every id
// rewritten to its slot (written by several threads: a __syncthreads() makes them visible to
// the whole block).
__device__ void lru_ensure_block(int32_t* __restrict__ ids, int n,
                                 int32_t* __restrict__ slot_for_id,
                                 int32_t* __restrict__ id_of_slot, int64_t* __restrict__ usage,
                                 int64_t* __restrict__ step_ptr, int S, int E, int base,
                                 int32_t* __restrict__ evict, int32_t* __restrict__ src,
                                 int64_t* __restrict__ num_out, int64_t* __restrict__ stats,
                                 const int32_t* __restrict__ pinned) {
  __shared__ int eflag[kMaxExperts];   // bit0 queried, bit1 miss
  __shared__ int eslot[kMaxExperts];   // slot per expert (victim for misses)
  __shared__ int mexp[kMaxExperts];    // expert of miss rank i
  __shared__ int vslot[kMaxExperts];   // victim slot of rank i
  __shared__ unsigned long long vkey[kMaxExperts];
  __shared__ int hist[256];
  __shared__ int warp_tot[32];
  __shared__ int s_total, s_nvict, s_digit, s_rem;
  __shared__ long long s_step;
  __shared__ unsigned long long s_maxkey;

  const int tid = threadIdx.x;
  if (tid == 0) {
    s_step = step_ptr[0] + 1;
    s_maxkey = 0ull;
  }
  for (int e = tid; e < E; e += kEnsureThreads) eflag[e] = 0;
  __syncthreads();
  const long long step = s_step;
  if (tid == 0) step_ptr[0] = step;

  for (int k = tid; k < n; k += kEnsureThreads) {
    const int e = ids[k];
    if (e >= 0 && e < E) atomicOr(&eflag[e], 1);
  }
  __syncthreads();

  // lookup, hits, miss flags (one expert per thread; E <= 1024)
  int is_miss = 0, is_q = 0;
  if (tid < E && (eflag[tid] & 1)) {
    is_q = 1;
    const int s = slot_for_id[base + tid];
    eslot[tid] = s;
    if (s >= 0) {
      usage[s] = step;
    } else {
      is_miss = 1;
    }
  }
  const int rank = block_excl_scan(is_miss, warp_tot, &s_total);
  const int M = s_total;
  if (is_miss) mexp[rank] = tid;
  const int nq_rank = block_excl_scan(is_q, warp_tot, &s_total);
  (void)nq_rank;
  const int nuniq = s_total;
  if (tid == 0) {
    num_out[0] = M;
    if (stats) {
      atomicAdd(reinterpret_cast<unsigned long long*>(stats + 0), (unsigned long long)nuniq);
      atomicAdd(reinterpret_cast<unsigned long long*>(stats + 1), (unsigned long long)M);
      atomicAdd(reinterpret_cast<unsigned long long*>(stats + 2), 1ull);
    }
  }
  __syncthreads();  // hit usage writes visible to the block

  if (M > 0) {
    const VictimScratch vs{vslot, vkey, hist, warp_tot, &s_total, &s_nvict, &s_digit, &s_rem,
                           &s_maxkey};
    select_victims(M, S, step, usage, pinned, vs);
    // unmap evicted ids first, then map the misses
    if (tid < M) {
      const int v = vslot[tid];
      const int old = id_of_slot[v];
      if (old >= 0) slot_for_id[old] = -1;
    }
    __syncthreads();
    if (tid < M) {
      const int v = vslot[tid];
      const int e = mexp[tid];
      id_of_slot[v] = base + e;
      slot_for_id[base + e] = v;
      usage[v] = step;
      evict[tid] = v;
      src[tid] = e;
      eslot[e] = v;
    }
    __syncthreads();
  }

  for (int k = tid; k < n; k += kEnsureThreads) {
    const int e = ids[k];
    ids[k] = (e >= 0 && e < E) ? eslot[e] : -1;
  }
}

__global__ void __launch_bounds__(kEnsureThreads)
lru_ensure_kernel(int32_t* __restrict__ ids, int n, int32_t* __restrict__ slot_for_id,
                  int32_t* __restrict__ id_of_slot, int64_t* __restrict__ usage,
                  int64_t* __restrict__ step_ptr, int S, int E, int base,
                  int32_t* __restrict__ evict, int32_t* __restrict__ src,
                  int64_t* __restrict__ num_out, int64_t* __restrict__ stats,
                  const int32_t* __restrict__ pinned) {
  pdl_wait();
  pdl_trigger();
  lru_ensure_block(ids, n, slot_for_id, id_of_slot, usage, step_ptr, S, E, base, evict, src,
                   num_out, stats, pinned);
}

// The LRU ensure followed, in the same block, by the expert FFN's route grouping over the
// slot ids it has just written (decode sizes: one launch fewer per layer than the ensure and
// the FFN's own grouping).  cnt: dynamic shared memory of S ints.
__global__ void __launch_bounds__(kEnsureThreads)
lru_ensure_group_kernel(int32_t* __restrict__ ids, int n, int32_t* __restrict__ slot_for_id,
                        int32_t* __restrict__ id_of_slot, int64_t* __restrict__ usage,
                        int64_t* __restrict__ step_ptr, int S, int E, int base,
                        int32_t* __restrict__ evict, int32_t* __restrict__ src,
                        int64_t* __restrict__ num_out, int64_t* __restrict__ stats,
                        const int32_t* __restrict__ pinned, int split, Workspace ws) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int cnt[];
  lru_ensure_block(ids, n, slot_for_id, id_of_slot, usage, step_ptr, S, E, base, evict, src,
                   num_out, stats, pinned);
  __syncthreads();  // every rewritten id is visible to the block
  group_routes<false>(ids, n, S, 0, split, ws, cnt);
}

// Capped-fetch LRU of the hybrid backend: as lru_ensure_kernel, but only the first
// fetch-cap misses -- ordered by (recency descending, id ascending), or by id without a
// recency row -- get a victim slot and a pending copy; the rest keep no slot and their ids
// become -1.  active_mask[e] = expert e routed this step; recency[e] = step for those.
__global__ void __launch_bounds__(kEnsureThreads)
hybrid_ensure_kernel(int32_t* __restrict__ ids, int n, int32_t* __restrict__ slot_for_id,
                     int32_t* __restrict__ id_of_slot, int64_t* __restrict__ usage,
                     int64_t* __restrict__ step_ptr, int S, int E, int base,
                     int32_t* __restrict__ active_mask, int32_t* __restrict__ evict,
                     int32_t* __restrict__ src, int64_t* __restrict__ num_out,
                     int64_t* __restrict__ num_full_out, int64_t* __restrict__ recency,
                     int max_fetch, int frac_q16) {
  pdl_wait();
  pdl_trigger();
  __shared__ int eflag[kMaxExperts];   // bit0 routed this step
  __shared__ int eslot[kMaxExperts];   // slot per routed expert (-1: miss not fetched)
  __shared__ int mexp[kMaxExperts];    // misses in id order
  __shared__ long long mrec[kMaxExperts];  // their recency
  __shared__ int fexp[kMaxExperts];    // misses in fetch-priority order
  __shared__ int vslot[kMaxExperts];
  __shared__ unsigned long long vkey[kMaxExperts];
  __shared__ int hist[256];
  __shared__ int warp_tot[32];
  __shared__ int s_total, s_nvict, s_digit, s_rem, s_fetch;
  __shared__ long long s_step;
  __shared__ unsigned long long s_maxkey;

  const int tid = threadIdx.x;
  if (tid == 0) s_step = step_ptr[0] + 1;
  for (int e = tid; e < E; e += kEnsureThreads) eflag[e] = 0;
  __syncthreads();
  const long long step = s_step;
  if (tid == 0) step_ptr[0] = step;
  for (int k = tid; k < n; k += kEnsureThreads) {
    const int e = ids[k];
    if (e >= 0 && e < E) atomicOr(&eflag[e], 1);
  }
  __syncthreads();

  // active mask, lookup, hits, misses (one expert per thread; E <= 1024)
  int is_miss = 0;
  if (tid < E) {
    const int act = eflag[tid] & 1;
    active_mask[tid] = act;
    if (act) {
      const int s = slot_for_id[base + tid];
      eslot[tid] = s;
      if (s >= 0) {
        usage[s] = step;
      } else {
        is_miss = 1;
      }
    }
  }
  const int rank = block_excl_scan(is_miss, warp_tot, &s_total);
  const int M = s_total;
  if (is_miss) {
    mexp[rank] = tid;
    mrec[rank] = recency ? recency[tid] : 0;
  }
  __syncthreads();
  // fetch priority: (recency desc, id asc) with a recency row, else id asc (mexp's order)
  if (tid < M) {
    int r = tid;
    if (recency) {
      const long long mine = mrec[tid];
      r = 0;
      for (int j = 0; j < M; ++j) r += mrec[j] > mine || (mrec[j] == mine && j < tid);
    }
    fexp[r] = mexp[tid];
  }
  if (tid == 0) {
    long long cap = max_fetch;
    if (frac_q16 > 0) {  // the integer F near frac * M balancing F*(1-frac) and (M-F)*frac
      const long long m = M, q = 1ll << 16, f = frac_q16;
      const long long lo = (m * f) >> 16;
      const long long c_lo = max(lo * (q - f), (m - lo) * f);
      const long long c_hi = max((lo + 1) * (q - f), (m - lo - 1) * f);
      cap = c_lo <= c_hi ? lo : lo + 1;
    }
    s_fetch = (int)min((long long)M, max(cap, 0ll));
    num_out[0] = s_fetch;
    num_full_out[0] = M;
  }
  __syncthreads();  // hit usage writes and the fetch order visible to the block
  const int F = s_fetch;

  if (F > 0) {
    const VictimScratch vs{vslot, vkey, hist, warp_tot, &s_total, &s_nvict, &s_digit, &s_rem,
                           &s_maxkey};
    select_victims(F, S, step, usage, nullptr, vs);
    if (tid < F) {
      const int v = vslot[tid];
      const int old = id_of_slot[v];
      if (old >= 0) slot_for_id[old] = -1;
    }
    __syncthreads();
    if (tid < F) {
      const int v = vslot[tid];
      const int e = fexp[tid];
      id_of_slot[v] = base + e;
      slot_for_id[base + e] = v;
      usage[v] = step;
      evict[tid] = v;
      src[tid] = e;
      eslot[e] = v;
    }
    __syncthreads();
  }
  if (recency && tid < E && (eflag[tid] & 1)) recency[tid] = step;

  for (int k = tid; k < n; k += kEnsureThreads) {
    const int e = ids[k];
    ids[k] = (e >= 0 && e < E) ? eslot[e] : -1;
  }
}

__global__ void __launch_bounds__(kEnsureThreads)
materialize_kernel(int32_t* __restrict__ slot_for_id, int32_t* __restrict__ id_of_slot,
                   int64_t* __restrict__ usage, int64_t* __restrict__ step_ptr, int S, int E,
                   int base, int32_t* __restrict__ evict, int32_t* __restrict__ src,
                   int64_t* __restrict__ num_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ long long s_step;
  const int tid = threadIdx.x;
  // read every slot's owner before any store, as the reference's single vector load does
  int old[kSlotsPerThread];
#pragma unroll
  for (int j = 0; j < kSlotsPerThread; ++j) {
    const int s = tid + j * kEnsureThreads;
    old[j] = s < S ? id_of_slot[s] : -1;
  }
  if (tid == 0) s_step = step_ptr[0] + 1;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kSlotsPerThread; ++j) {
    const int s = tid + j * kEnsureThreads;
    if (s >= S) continue;
    const bool same = old[j] >= base && old[j] < base + E;
    if (same) {
      id_of_slot[s] = -1;
      usage[s] = 0;
    } else if (s < E && old[j] >= 0) {
      slot_for_id[old[j]] = -1;
    }
  }
  __syncthreads();
  const long long step = s_step;
  if (tid == 0) {
    step_ptr[0] = step;
    num_out[0] = E;
  }
  for (int e = tid; e < E; e += kEnsureThreads) {
    id_of_slot[e] = base + e;
    slot_for_id[base + e] = e;
    usage[e] = step;
    evict[e] = e;
    src[e] = e;
  }
}

__global__ void reset_kernel(int32_t* __restrict__ slot_for_id, int64_t n_ids,
                             int32_t* __restrict__ id_of_slot, int64_t* __restrict__ usage,
                             int64_t S, int64_t* __restrict__ step, int64_t* __restrict__ num) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_ids) slot_for_id[i] = -1;
  if (i < S) {
    id_of_slot[i] = -1;
    usage[i] = 0;
  }
  if (i == 0) {
    step[0] = 0;
    if (num) num[0] = 0;
  }
}

__global__ void __launch_bounds__(kEnsureThreads)
hit_compact_kernel(const int32_t* __restrict__ row, int E, int buffer_base,
                   int32_t* __restrict__ dst, int32_t* __restrict__ srcs,
                   int64_t* __restrict__ num) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_total;
  const int tid = threadIdx.x;
  const int s = tid < E ? row[tid] : -1;
  const int hit = s >= 2 * E;
  const int pos = block_excl_scan(hit, warp_tot, &s_total);
  if (hit) {
    dst[pos] = buffer_base + tid;
    srcs[pos] = s;
  }
  if (tid == 0) num[0] = s_total;
}

// ---------------------------------------------------------------- multi-bank row copy

constexpr int kCopyBanks = 8;
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 8;
constexpr int64_t kCopyChunk = (int64_t)kCopyThreads * kCopyUnroll * 16;  // 32 KiB

struct CopyPlan {
  char* dst[kCopyBanks];
  const char* src[kCopyBanks];
  int64_t bytes[kCopyBanks];
};

// Persistent CTAs walk the (bank, row, 32 KiB chunk) items of the *num_rows staged rows;
// with nothing staged every CTA exits after one load, so the launch stays cheap inside a
// captured decode step.
__global__ void __launch_bounds__(kCopyThreads)
copy_rows_kernel(CopyPlan plan, int n_banks, const int32_t* __restrict__ dst_rows,
                 const int32_t* __restrict__ src_rows, const int64_t* __restrict__ num_rows,
                 int64_t max_rows) {
  pdl_wait();
  pdl_trigger();
  const int64_t nr = min(num_rows[0], max_rows);
  for (int b = 0; b < n_banks; ++b) {
    const int64_t rb = plan.bytes[b];
    const int64_t cpr = (rb + kCopyChunk - 1) / kCopyChunk;
    for (int64_t item = blockIdx.x; item < nr * cpr; item += gridDim.x) {
      const int64_t r = item / cpr;
      const int64_t off0 = (item % cpr) * kCopyChunk;
      const char* s = plan.src[b] + (int64_t)src_rows[r] * rb;
      char* d = plan.dst[b] + (int64_t)dst_rows[r] * rb;
      uint4 v[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t o = off0 + ((int64_t)u * kCopyThreads + threadIdx.x) * 16;
        if (o < rb) v[u] = ld_stream16(s + o);
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t o = off0 + ((int64_t)u * kCopyThreads + threadIdx.x) * 16;
        if (o < rb) *reinterpret_cast<uint4*>(d + o) = v[u];
      }
    }
  }
}

}  // namespace
}  // namespace tw

using namespace tw;

extern "C" int tw_lru_ensure(int32_t* ids, int64_t n, int32_t* slot_for_id,
                             int32_t* id_of_slot, int64_t* usage, int64_t* step,
                             int64_t num_slots, int num_experts, int layer_id,
                             int32_t* evict_slots, int32_t* src_indices, int64_t* num_indices,
                             int64_t* stats, const int32_t* pinned, void* stream) {
  TW_CHECK_ARG(n >= 0 && n <= kMaxIds, "lru_ensure: need 0 <= n <= %d (got %lld)", kMaxIds,
               (long long)n);
  TW_CHECK_ARG(num_experts > 0 && num_experts <= kMaxExperts,
               "lru_ensure: need 0 < E <= %d", kMaxExperts);
  TW_CHECK_ARG(num_slots > 0 && num_slots <= kMaxSlots,
               "lru_ensure: need 0 < S <= %d (got S=%lld)", kMaxSlots, (long long)num_slots);
  TW_CHECK_ARG(layer_id >= 0, "lru_ensure: layer_id must be >= 0");
  TW_LAUNCH(lru_ensure_kernel, dim3(1), dim3(kEnsureThreads), 0, as_stream(stream), 
      ids, (int)n, slot_for_id, id_of_slot, usage, step, (int)num_slots, num_experts,
      layer_id * num_experts, evict_slots, src_indices, num_indices, stats, pinned);
  TW_CHECK_LAUNCH("lru_ensure_kernel");
  return TW_OK;
}

extern "C" int tw_lru_ensure_group(int32_t* ids, int64_t T, int K, int32_t* slot_for_id,
                                   int32_t* id_of_slot, int64_t* usage, int64_t* step,
                                   int64_t num_slots, int num_experts, int layer_id,
                                   int32_t* evict_slots, int32_t* src_indices,
                                   int64_t* num_indices, int64_t* stats, const int32_t* pinned,
                                   int H, int I, int nvfp4, void* workspace, size_t ws_bytes,
                                   void* stream) {
  const int64_t n = T * K;
  TW_CHECK_ARG(T >= 0 && K > 0 && n < 1024,
               "lru_ensure_group: decode batches only (T*K < 1024, got %lld)", (long long)n);
  TW_CHECK_ARG(num_experts > 0 && num_experts <= kMaxExperts,
               "lru_ensure_group: need 0 < E <= %d", kMaxExperts);
  TW_CHECK_ARG(num_slots > 0 && num_slots <= kMaxSlots,
               "lru_ensure_group: need 0 < S <= %d (got S=%lld)", kMaxSlots, (long long)num_slots);
  TW_CHECK_ARG(layer_id >= 0 && H > 0 && I > 0, "lru_ensure_group: bad layer or shape");
  Workspace ws;
  const size_t need = workspace_layout(n, H, I, static_cast<char*>(workspace), &ws);
  TW_CHECK_ARG(workspace != nullptr && ws_bytes >= need && aligned16(workspace),
               "lru_ensure_group: workspace too small or misaligned (%zu < %zu bytes)", ws_bytes,
               need);
  // the segment split the FFN kernel of this shape expects (its route-tile capacity)
  const int cap = nvfp4 ? expert_ffn_fp4_tc_route_cap(T) : expert_ffn_tc_route_cap(T, n, num_slots);
  const int split = cap > 0 && T > cap ? cap : 0;
  const size_t smem = sizeof(int) * (size_t)num_slots;
  static bool attr_set[kMaxAttrDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 16 * 1024 && (dev < 0 || dev >= kMaxAttrDevices || !attr_set[dev])) {
    cudaFuncSetAttribute(lru_ensure_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)std::max<size_t>(smem, 64 * 1024));
    if (dev >= 0 && dev < kMaxAttrDevices) attr_set[dev] = true;
  }
  TW_LAUNCH(lru_ensure_group_kernel, dim3(1), dim3(kEnsureThreads), smem, as_stream(stream),
            ids, (int)n, slot_for_id, id_of_slot, usage, step, (int)num_slots, num_experts,
            layer_id * num_experts, evict_slots, src_indices, num_indices, stats, pinned, split,
            ws);
  TW_CHECK_LAUNCH("lru_ensure_group_kernel");
  return TW_OK;
}

extern "C" int tw_hybrid_ensure(int32_t* ids, int64_t n, int32_t* slot_for_id,
                                int32_t* id_of_slot, int64_t* usage, int64_t* step,
                                int64_t num_slots, int num_experts, int layer_id,
                                int32_t* active_mask, int32_t* evict_slots,
                                int32_t* src_indices, int64_t* num_indices,
                                int64_t* num_missing_full, int64_t* recency, int max_fetch,
                                int fetch_frac_q16, void* stream) {
  TW_CHECK_ARG(n >= 0 && n <= kMaxIds, "hybrid_ensure: need 0 <= n <= %d (got %lld)", kMaxIds,
               (long long)n);
  TW_CHECK_ARG(num_experts > 0 && num_experts <= kMaxExperts,
               "hybrid_ensure: need 0 < E <= %d", kMaxExperts);
  TW_CHECK_ARG(num_slots > 0 && num_slots <= kMaxSlots,
               "hybrid_ensure: need 0 < S <= %d (got S=%lld)", kMaxSlots, (long long)num_slots);
  TW_CHECK_ARG(layer_id >= 0 && max_fetch >= 0 && fetch_frac_q16 >= 0 &&
                   fetch_frac_q16 <= (1 << 16),
               "hybrid_ensure: need layer_id >= 0, max_fetch >= 0, 0 <= frac_q16 <= 65536");
  TW_LAUNCH(hybrid_ensure_kernel, dim3(1), dim3(kEnsureThreads), 0, as_stream(stream), ids,
            (int)n, slot_for_id, id_of_slot, usage, step, (int)num_slots, num_experts,
            layer_id * num_experts, active_mask, evict_slots, src_indices, num_indices,
            num_missing_full, recency ? recency + (int64_t)layer_id * num_experts : nullptr,
            max_fetch, fetch_frac_q16);
  TW_CHECK_LAUNCH("hybrid_ensure_kernel");
  return TW_OK;
}

extern "C" int tw_materialize_layer(int32_t* slot_for_id, int32_t* id_of_slot, int64_t* usage,
                                    int64_t* step, int64_t num_slots, int num_experts,
                                    int layer_id, int32_t* evict_slots, int32_t* src_indices,
                                    int64_t* num_indices, void* stream) {
  TW_CHECK_ARG(num_experts > 0 && num_slots >= num_experts && num_slots <= kMaxSlots,
               "materialize_layer: need 0 < E <= S <= %d", kMaxSlots);
  TW_LAUNCH(materialize_kernel, dim3(1), dim3(kEnsureThreads), 0, as_stream(stream), 
      slot_for_id, id_of_slot, usage, step, (int)num_slots, num_experts,
      layer_id * num_experts, evict_slots, src_indices, num_indices);
  TW_CHECK_LAUNCH("materialize_kernel");
  return TW_OK;
}

extern "C" int tw_reset_slots(int32_t* slot_for_id, int64_t num_ids, int32_t* id_of_slot,
                              int64_t* usage, int64_t num_slots, int64_t* step,
                              int64_t* num_indices, void* stream) {
  const int64_t n = num_ids > num_slots ? num_ids : num_slots;
  const int64_t blocks = (n + 255) / 256;
  TW_LAUNCH(reset_kernel, dim3((unsigned)(blocks > 0 ? blocks : 1)), dim3(256), 0, as_stream(stream), 
      slot_for_id, num_ids, id_of_slot, usage, num_slots, step, num_indices);
  TW_CHECK_LAUNCH("reset_kernel");
  return TW_OK;
}

extern "C" int tw_prefill_hit_compact(const int32_t* row, int num_experts, int buffer_id,
                                      int32_t* dst_rows, int32_t* src_slots, int64_t* num_hits,
                                      void* stream) {
  TW_CHECK_ARG(num_experts > 0 && num_experts <= kEnsureThreads,
               "prefill_hit_compact: need 0 < E <= %d", kEnsureThreads);
  TW_LAUNCH(hit_compact_kernel, dim3(1), dim3(kEnsureThreads), 0, as_stream(stream), 
      row, num_experts, buffer_id * num_experts, dst_rows, src_slots, num_hits);
  TW_CHECK_LAUNCH("hit_compact_kernel");
  return TW_OK;
}

extern "C" int tw_host_register(void* ptr, size_t bytes) {
  TW_CHECK_ARG(ptr != nullptr && bytes > 0, "host_register: empty range");
  const cudaError_t e =
      cudaHostRegister(ptr, bytes, cudaHostRegisterPortable | cudaHostRegisterMapped);
  if (e != cudaSuccess) {
    cudaGetLastError();  // a failed registration leaves no error behind for later launches
    set_error("cudaHostRegister of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

extern "C" int tw_host_unregister(void* ptr) {
  const cudaError_t e = cudaHostUnregister(ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaHostUnregister failed: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

extern "C" int tw_copy_rows(int n_banks, void* const* dst_base, const void* const* src_base,
                            const int64_t* row_bytes, const int32_t* dst_rows,
                            const int32_t* src_rows, const int64_t* num_rows, int64_t max_rows,
                            void* stream) {
  TW_CHECK_ARG(n_banks > 0 && n_banks <= kCopyBanks, "copy_rows: need 0 < n_banks <= %d",
               kCopyBanks);
  TW_CHECK_ARG(max_rows >= 0, "copy_rows: need max_rows >= 0");
  if (max_rows == 0) return TW_OK;
  CopyPlan plan{};
  int64_t maxb = 0;
  for (int b = 0; b < n_banks; ++b) {
    TW_CHECK_ARG(aligned16(dst_base[b]) && aligned16(src_base[b]) && row_bytes[b] % 16 == 0 &&
                     row_bytes[b] > 0,
                 "copy_rows: bank %d base or row size not 16-byte aligned", b);
    plan.dst[b] = static_cast<char*>(dst_base[b]);
    plan.src[b] = static_cast<const char*>(src_base[b]);
    plan.bytes[b] = row_bytes[b];
    if (row_bytes[b] > maxb) maxb = row_bytes[b];
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_row = (maxb + kCopyChunk - 1) / kCopyChunk;
  const int64_t most = per_row * max_rows;
  const int grid = (int)std::min<int64_t>(most, (int64_t)sms * 4);
  TW_LAUNCH(copy_rows_kernel, dim3(grid), dim3(kCopyThreads), 0, as_stream(stream), plan, n_banks, dst_rows,
                                                                  src_rows, num_rows, max_rows);
  TW_CHECK_LAUNCH("copy_rows_kernel");
  return TW_OK;
}
