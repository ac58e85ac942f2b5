// Expert-parallel exchange over NVLink peer memory: dispatch and combine written by our own
// kernels straight into the other GPUs' memory (CUDA IPC mappings of one buffer per GPU),
// with device-side flags instead of NCCL all-to-alls.
//
// Every GPU of the expert-parallel group owns one exchange buffer of the same layout:
//   header  : per-source dispatch and combine flags (written by the peers), this GPU's
//             exchange count, the arrival counters of its two kernels, an error word
//   recv_x  : [world * T, H] bf16   row src * T + t = token t of GPU src (if it routes here)
//   recv_ids: [world * T, K] int32  local expert ids of those routes (-1: routed elsewhere)
//   recv_w  : [world * T, K] fp32   router weights
//   back    : [world * T, H] bf16   row src * T + t = GPU src's partial output for token t
//
// Dispatch (one launch): for every token and destination GPU d, the K local ids and
// weights go into d's recv_ids/recv_w row, and the token's input row into d's recv_x only
// when it has a route on d (routed rows only: the other rows cost K ids and weights).  The
// CTA that completes the launch's arrival count raises this GPU's flag on every peer
// (release, system scope) and waits -- bounded -- until every peer's flag for this step is
// up in its own header; the launch ends once every row addressed to this GPU has landed.
// The received rows then run through the slot cache and the expert FFN like any batch.
// Combine (one launch): for every received row, the sum of its local routes' outputs
// (k order) goes back into the source GPU's `back` row; the completing CTA raises the
// combine flags; then each local token waits for every peer's flag, adds the partials of
// the GPUs its routes went to in GPU order and (optionally) applies the next residual add
// and RMSNorm -- the same arithmetic as the all-to-all path's tw_ep_combine followed by
// tw_rmsnorm.
//
// Flags carry the exchange count (monotonic, never reset), so nothing has to be cleared
// between steps and a captured graph replays as is.  A buffer row is rewritten only after
// its previous contents were consumed: a GPU dispatches step s + 1 only after it received
// every partial of step s, which each peer sends only after its FFN read the rows of step s.
// Every wait is bounded (tw_set_wait_limit); a wait that gives up sets the header's error
// word and the launch returns.  Kernels that wait on other GPUs run one per GPU (one process
// per GPU), never as several launches on one GPU.  No TMA or bulk copy touches peer memory:
// plain 16-byte stores only.
#include <algorithm>
#include <cstring>

#include <cuda.h>

#include "common.cuh"
#include "moe_common.cuh"

namespace tw {
namespace {

constexpr int kMaxEpWorld = 8;
constexpr int kEpThreads = 128;
constexpr int kEpMaxK = 64;
constexpr int kEpNormVec = 4;  // H <= 128 * 8 * 4 = 4096

struct EpHeader {
  uint32_t flag_dispatch[kMaxEpWorld];  // [src]: src's last dispatch step into this buffer
  uint32_t flag_combine[kMaxEpWorld];   // [src]: src's last partials step into this buffer
  uint32_t step;                        // this GPU's exchange count
  uint32_t arrive_dispatch;             // CTAs of the running dispatch that are done
  uint32_t arrive_combine;              // CTAs of the running combine's first phase
  int32_t err;                          // 1: a bounded wait gave up
};

struct EpLayout {
  size_t x, ids, w, back, bytes;
};

inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

EpLayout ep_layout(int world, int64_t T, int H, int K) {
  EpLayout l;
  size_t off = al256(sizeof(EpHeader));
  const size_t rows = (size_t)world * (size_t)T;
  l.x = off;
  off += al256(rows * H * 2);
  l.ids = off;
  off += al256(rows * K * 4);
  l.w = off;
  off += al256(rows * K * 4);
  l.back = off;
  off += al256(rows * H * 2);
  l.bytes = off;
  return l;
}

struct Peers {
  char* base[kMaxEpWorld];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 of the CTA that completes `counter`'s count of gridDim.x arrivals gets true (and
// resets the counter for the next launch); every thread of the CTA learns it.  Each CTA's
// earlier stores, peer stores included, are ordered before its arrival.
__device__ __forceinline__ bool completes_launch(uint32_t* counter, int* s_last) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t done = atomicAdd(counter, 1u) + 1u;
    *s_last = done == gridDim.x;
    if (*s_last) {
      *counter = 0;
      __threadfence_system();
    }
  }
  __syncthreads();
  return *s_last != 0;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (threads 0..world-1, one source each) until flags[src] == target; a wait that
// gives up sets the error word.  The flags live in this GPU's memory; each peer fenced its
// data stores (system scope) before its release store of the flag, and the poll is an
// acquire load at system scope, so it pairs with that release across GPUs; the barrier
// after the wait orders the whole CTA's later loads of the data after it.
__device__ __forceinline__ void wait_flags(const uint32_t* flags, int world, uint32_t target,
                                           int32_t* err, uint32_t limit) {
  if (threadIdx.x < world) {
    const uint32_t* f = flags + threadIdx.x;
    uint32_t it = 0;
    while (ld_acquire_sys(f) != target) {
      if (++it >= limit) {
        atomicExch(err, 1);
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kEpThreads)
ep_p2p_dispatch_kernel(const uint4* __restrict__ x, const float* __restrict__ topk_w,
                       const int32_t* __restrict__ topk_ids, int T, int K, int H, int Eg,
                       int world, int rank, Peers peers, EpLayout lay, uint32_t limit) {
  pdl_wait();
  pdl_trigger();
  __shared__ int any;
  __shared__ int last;
  EpHeader* h = reinterpret_cast<EpHeader*>(peers.base[rank]);
  const uint32_t target = *reinterpret_cast<volatile uint32_t*>(&h->step) + 1u;
  const int H8 = H / 8;
  for (int item = blockIdx.x; item < T * world; item += gridDim.x) {
    const int t = item / world, d = item % world;
    char* dst = peers.base[d];
    const int64_t row = (int64_t)rank * T + t;
    int32_t* ids = reinterpret_cast<int32_t*>(dst + lay.ids) + row * K;
    float* w = reinterpret_cast<float*>(dst + lay.w) + row * K;
    if (threadIdx.x == 0) any = 0;
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += kEpThreads) {
      const int e = topk_ids[(int64_t)t * K + k];
      const bool mine = e >= 0 && e / Eg == d;
      ids[k] = mine ? e % Eg : -1;
      w[k] = topk_w[(int64_t)t * K + k];
      if (mine) atomicOr(&any, 1);
    }
    __syncthreads();
    if (any) {  // routed rows only: a row without a route on d is never read there
      uint4* xr = reinterpret_cast<uint4*>(dst + lay.x) + row * H8;
      for (int c = threadIdx.x; c < H8; c += kEpThreads) xr[c] = x[(int64_t)t * H8 + c];
    }
    __syncthreads();  // `any` is reused by the next item
  }
  if (!completes_launch(&h->arrive_dispatch, &last)) return;
  if (threadIdx.x < world) {
    EpHeader* peer = reinterpret_cast<EpHeader*>(peers.base[threadIdx.x]);
    st_release_sys(&peer->flag_dispatch[rank], target);
  }
  wait_flags(h->flag_dispatch, world, target, &h->err, limit);
  if (threadIdx.x == 0) h->step = target;
}

template <int kThreads>
__device__ __forceinline__ float ep_block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < (kThreads / 32) ? red[lane] : 0.f;
  r = warp_sum(r);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint4 ep_pack_bf16x8(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i])) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1])) << 16);
  return r;
}

struct EpTail {          // the token-side epilogue of the combine
  const uint4* resid;    // residual [T, H] (null: write the routed sum to y only)
  uint4* resid_out;      // bf16(sum + resid) (may alias resid)
  const uint4* norm_w;
  float eps;
  uint4* h_out;          // RMSNorm(resid_out) * norm_w
  uint4* y;              // the routed sum itself (may be null when resid is given)
};

__global__ void __launch_bounds__(kEpThreads)
ep_p2p_combine_kernel(const int32_t* __restrict__ pos, const __nv_bfloat16* __restrict__ c3,
                      const int32_t* __restrict__ topk_ids, int T, int K, int H, int Eg,
                      int world, int rank, Peers peers, EpLayout lay, EpTail tail,
                      uint32_t limit) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sp[kEpMaxK];
  __shared__ int any;
  __shared__ int last;
  __shared__ float red[32];
  __shared__ int routed[kMaxEpWorld];
  EpHeader* h = reinterpret_cast<EpHeader*>(peers.base[rank]);
  const uint32_t target = *reinterpret_cast<volatile uint32_t*>(&h->step);  // set by dispatch
  const int H8 = H / 8;
  // phase 1: the partial output of every received row, back to its source GPU
  for (int r = blockIdx.x; r < world * T; r += gridDim.x) {
    const int src = r / T, t = r % T;
    if (threadIdx.x == 0) any = 0;
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += kEpThreads) {
      sp[k] = pos[(int64_t)r * K + k];
      if (sp[k] >= 0) atomicOr(&any, 1);
    }
    __syncthreads();
    if (any) {
      uint4* dst = reinterpret_cast<uint4*>(peers.base[src] + lay.back) +
                   ((int64_t)rank * T + t) * H8;
      for (int c = threadIdx.x; c < H8; c += kEpThreads) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < K; ++k) {
          const int p = sp[k];
          if (p < 0) continue;
          float f[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(c3 + (int64_t)p * H + c * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += f[e];
        }
        dst[c] = ep_pack_bf16x8(acc);
      }
    }
    __syncthreads();
  }
  if (completes_launch(&h->arrive_combine, &last) && threadIdx.x < world) {
    EpHeader* peer = reinterpret_cast<EpHeader*>(peers.base[threadIdx.x]);
    st_release_sys(&peer->flag_combine[rank], target);
  }
  // phase 2: every local token, once every GPU's partials are in
  bool waited = false;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (!waited) {
      wait_flags(h->flag_combine, world, target, &h->err, limit);
      waited = true;
    }
    if (threadIdx.x < world) routed[threadIdx.x] = 0;
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += kEpThreads) {
      const int e = topk_ids[(int64_t)t * K + k];
      if (e >= 0 && e / Eg < world) routed[e / Eg] = 1;
    }
    __syncthreads();
    const uint4* back = reinterpret_cast<const uint4*>(peers.base[rank] + lay.back);
    float v[kEpNormVec][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kEpNormVec; ++j) {
      const int c = threadIdx.x + j * kEpThreads;
      if (c < H8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int d = 0; d < world; ++d) {  // GPU order; a GPU without routes adds zero
          if (!routed[d]) continue;
          float f[8];
          bf16x8_to_f32(back[((int64_t)d * T + t) * H8 + c], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += f[e];
        }
        const uint4 y = ep_pack_bf16x8(acc);
        if (tail.y != nullptr) tail.y[(int64_t)t * H8 + c] = y;
        if (tail.resid != nullptr) {
          float yf[8], rr[8];
          bf16x8_to_f32(y, yf);
          bf16x8_to_f32(tail.resid[(int64_t)t * H8 + c], rr);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[j][q] = bf16_round(yf[q] + rr[q]);
            ss += v[j][q] * v[j][q];
          }
        }
      }
    }
    if (tail.resid != nullptr) {
      const float tot = ep_block_sum<kEpThreads>(ss, red);
      const float rstd = rsqrtf(tot / (float)H + tail.eps);
#pragma unroll
      for (int j = 0; j < kEpNormVec; ++j) {
        const int c = threadIdx.x + j * kEpThreads;
        if (c < H8) {
          tail.resid_out[(int64_t)t * H8 + c] = ep_pack_bf16x8(v[j]);
          float wf[8], o[8];
          bf16x8_to_f32(tail.norm_w[c], wf);
#pragma unroll
          for (int q = 0; q < 8; ++q) o[q] = v[j][q] * rstd * wf[q];
          tail.h_out[(int64_t)t * H8 + c] = ep_pack_bf16x8(o);
        }
      }
    }
    __syncthreads();
  }
}

int check_peers(void* const* peers, int world, int rank) {
  TW_CHECK_ARG(world > 0 && world <= kMaxEpWorld, "ep_p2p: need 0 < world <= %d", kMaxEpWorld);
  TW_CHECK_ARG(rank >= 0 && rank < world, "ep_p2p: rank %d outside world %d", rank, world);
  TW_CHECK_ARG(peers != nullptr, "ep_p2p: peer buffer table required");
  for (int d = 0; d < world; ++d)
    TW_CHECK_ARG(peers[d] != nullptr && aligned16(peers[d]), "ep_p2p: peer %d buffer missing", d);
  return TW_OK;
}

// CTAs of an exchange launch: every CTA of a combine must be resident at once (its second
// phase waits on flags that the first phase of all CTAs, here and on the peers, raises).
int ep_grid(int64_t items) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(items, (int64_t)num_sms() * 4));
}

}  // namespace
}  // namespace tw

using namespace tw;

extern "C" size_t tw_ep_p2p_bytes(int world, int64_t T, int H, int K) {
  return ep_layout(world, T, H, K).bytes;
}

extern "C" int tw_ep_p2p_offsets(int world, int64_t T, int H, int K, size_t* out4) {
  TW_CHECK_ARG(out4 != nullptr, "ep_p2p_offsets: output required");
  const EpLayout l = ep_layout(world, T, H, K);
  out4[0] = l.x;
  out4[1] = l.ids;
  out4[2] = l.w;
  out4[3] = l.back;
  return TW_OK;
}

namespace {
using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
GetRangeFn g_get_range = nullptr;

int address_range(const void* ptr, CUdeviceptr* base) {
  if (g_get_range == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    const cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000,
                                                           cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      set_error("cuMemGetAddressRange unavailable (%s)", cudaGetErrorString(e));
      return TW_ERR_CUDA;
    }
    g_get_range = reinterpret_cast<GetRangeFn>(fn);
  }
  size_t size = 0;
  const CUresult r = g_get_range(base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) {
    set_error("cuMemGetAddressRange failed (%d)", (int)r);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}
}  // namespace

extern "C" int tw_ep_p2p_export(const void* buffer, void* ipc_handle, uint64_t* offset) {
  TW_CHECK_ARG(buffer != nullptr && ipc_handle != nullptr && offset != nullptr,
               "ep_p2p_export: bad arguments");
  CUdeviceptr base = 0;
  if (int rc = address_range(buffer, &base)) return rc;
  cudaIpcMemHandle_t hdl;
  const cudaError_t e = cudaIpcGetMemHandle(&hdl, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("ep_p2p_export: %s (the buffer must come from cudaMalloc, not a VMM pool)",
              cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &hdl, sizeof(hdl));
  *offset = reinterpret_cast<uint64_t>(buffer) - static_cast<uint64_t>(base);
  return TW_OK;
}

extern "C" size_t tw_ep_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int tw_ep_p2p_open(const void* ipc_handle, uint64_t offset, void** peer_buffer,
                              void** mapping) {
  TW_CHECK_ARG(ipc_handle != nullptr && peer_buffer != nullptr && mapping != nullptr,
               "ep_p2p_open: bad arguments");
  cudaIpcMemHandle_t hdl;
  std::memcpy(&hdl, ipc_handle, sizeof(hdl));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, hdl, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("ep_p2p_open: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  *mapping = base;
  *peer_buffer = static_cast<char*>(base) + offset;
  return TW_OK;
}

extern "C" int tw_ep_p2p_close(void* mapping) {
  const cudaError_t e = cudaIpcCloseMemHandle(mapping);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("ep_p2p_close: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

extern "C" int tw_ep_p2p_dispatch(const void* x, const float* topk_w, const int32_t* topk_ids,
                                  int64_t T, int K, int H, int experts_per_rank, int world,
                                  int rank, void* const* peers, void* stream) {
  if (int rc = check_peers(peers, world, rank)) return rc;
  TW_CHECK_ARG(T >= 0 && T <= 4096 && K > 0 && K <= kEpMaxK, "ep_p2p_dispatch: need T <= 4096, 0 < K <= %d", kEpMaxK);
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && experts_per_rank > 0, "ep_p2p_dispatch: bad H/experts");
  TW_CHECK_ARG(aligned16(x), "ep_p2p_dispatch: x must be 16-byte aligned");
  Peers p{};
  for (int d = 0; d < world; ++d) p.base[d] = static_cast<char*>(peers[d]);
  const EpLayout lay = ep_layout(world, T, H, K);
  TW_LAUNCH(ep_p2p_dispatch_kernel, dim3((unsigned)ep_grid(T * world)), dim3(kEpThreads), 0,
            as_stream(stream), reinterpret_cast<const uint4*>(x), topk_w, topk_ids, (int)T, K,
            H, experts_per_rank, world, rank, p, lay, ffn_wait_limit());
  TW_CHECK_LAUNCH("ep_p2p_dispatch_kernel");
  return TW_OK;
}

extern "C" int tw_ep_p2p_combine(const void* workspace, int64_t T, int K, int H, int I,
                                 int experts_per_rank, const int32_t* topk_ids, int world,
                                 int rank, void* const* peers, const void* residual,
                                 void* residual_out, const void* norm_w, float eps,
                                 void* h_out, void* y, void* stream) {
  if (int rc = check_peers(peers, world, rank)) return rc;
  TW_CHECK_ARG(T >= 0 && T <= 4096 && K > 0 && K <= kEpMaxK, "ep_p2p_combine: need T <= 4096, 0 < K <= %d", kEpMaxK);
  TW_CHECK_ARG(H > 0 && H % 8 == 0 && H <= kEpThreads * 8 * kEpNormVec,
               "ep_p2p_combine: need H %% 8 == 0 and H <= %d", kEpThreads * 8 * kEpNormVec);
  TW_CHECK_ARG(world * T <= (int64_t)num_sms() * 4 || T == 0,
               "ep_p2p_combine: world * T rows must fit one resident wave (%d)", num_sms() * 4);
  TW_CHECK_ARG((residual != nullptr) == (norm_w != nullptr) &&
                   (residual == nullptr || (residual_out != nullptr && h_out != nullptr)),
               "ep_p2p_combine: residual, residual_out, norm_w and h_out go together");
  TW_CHECK_ARG(y != nullptr || residual != nullptr, "ep_p2p_combine: nothing to write");
  if (T == 0) return TW_OK;
  Workspace ws;
  workspace_layout(world * T * K, H, I, static_cast<char*>(const_cast<void*>(workspace)), &ws);
  Peers p{};
  for (int d = 0; d < world; ++d) p.base[d] = static_cast<char*>(peers[d]);
  const EpLayout lay = ep_layout(world, T, H, K);
  const EpTail tail{static_cast<const uint4*>(residual), static_cast<uint4*>(residual_out),
                    static_cast<const uint4*>(norm_w), eps, static_cast<uint4*>(h_out),
                    static_cast<uint4*>(y)};
  TW_LAUNCH(ep_p2p_combine_kernel, dim3((unsigned)ep_grid(world * T)), dim3(kEpThreads), 0,
            as_stream(stream), ws.pos, ws.c3, topk_ids, (int)T, K, H, experts_per_rank, world,
            rank, p, lay, tail, ffn_wait_limit());
  TW_CHECK_LAUNCH("ep_p2p_combine_kernel");
  return TW_OK;
}

extern "C" int tw_ep_p2p_error(const void* buffer, int32_t* err_out, void* stream) {
  TW_CHECK_ARG(buffer != nullptr && err_out != nullptr, "ep_p2p_error: bad arguments");
  const EpHeader* h = static_cast<const EpHeader*>(buffer);
  const cudaError_t e = cudaMemcpyAsync(err_out, &h->err, sizeof(int32_t), cudaMemcpyDefault,
                                        as_stream(stream));
  if (e != cudaSuccess) {
    set_error("ep_p2p_error: %s", cudaGetErrorString(e));
    return TW_ERR_CUDA;
  }
  return TW_OK;
}
