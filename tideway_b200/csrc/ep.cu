// Expert-parallel dispatch/combine around the slot-indirect expert FFN.
//
// Experts of a layer are sharded evenly over G GPUs (GPU d owns experts [d*Eg, (d+1)*Eg)).
// Dispatch packs, for every destination GPU d and local token t, one fixed-size row
// [input row (H bf16) | K local expert ids (int32, -1 where route k lives elsewhere) |
//  K router weights (fp32)] at row d*T + t — fixed shapes, no host sync, so the step stays
// capturable and one all-to-all moves everything.  The receiver unpacks the rows into the
// FFN's [G*T, H] / [G*T, K] operands, runs the expert FFN (one partial sum per row) and
// sends the rows back; the combine adds the G partials of each token in GPU order.
#include "common.cuh"

namespace tw {
namespace {

inline int64_t row_bytes(int H, int K) { return ((int64_t)H * 2 + (int64_t)K * 8 + 15) / 16 * 16; }

__global__ void __launch_bounds__(256)
ep_pack_kernel(const uint4* __restrict__ x, const float* __restrict__ topk_w,
               const int32_t* __restrict__ topk_ids, int T, int K, int H, int Eg,
               int64_t rb, char* __restrict__ send) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, d = blockIdx.y;
  char* row = send + ((int64_t)d * T + t) * rb;
  int32_t* ids = reinterpret_cast<int32_t*>(row + (int64_t)H * 2);
  float* w = reinterpret_cast<float*>(ids + K);
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int e = topk_ids[t * K + k];
    const bool mine = e >= 0 && e / Eg == d;
    ids[k] = mine ? e % Eg : -1;
    w[k] = topk_w[t * K + k];
    if (mine) atomicOr(&any, 1);
  }
  __syncthreads();
  if (!any) return;  // no route of this token on GPU d: its input row is never read
  uint4* dst = reinterpret_cast<uint4*>(row);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = x[(int64_t)t * (H / 8) + c];
}

__global__ void __launch_bounds__(256)
ep_unpack_kernel(const char* __restrict__ recv, int K, int H, int64_t rb,
                 uint4* __restrict__ x, int32_t* __restrict__ ids, float* __restrict__ w) {
  pdl_wait();
  pdl_trigger();
  const int64_t r = blockIdx.x;
  const char* row = recv + r * rb;
  const int32_t* ri = reinterpret_cast<const int32_t*>(row + (int64_t)H * 2);
  const float* rw = reinterpret_cast<const float*>(ri + K);
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int e = ri[k];
    ids[r * K + k] = e;
    w[r * K + k] = rw[k];
    if (e >= 0) atomicOr(&any, 1);
  }
  __syncthreads();
  if (!any) return;
  const uint4* src = reinterpret_cast<const uint4*>(row);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) x[r * (H / 8) + c] = src[c];
}

__global__ void __launch_bounds__(256)
ep_sum_kernel(const uint4* __restrict__ parts, int T, int H8, int G, uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < H8; c += gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < G; ++d) {
      float v[8];
      bf16x8_to_f32(parts[((int64_t)d * T + t) * H8 + c], v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += v[i];
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      ow[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i])) |
              ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i + 1])) << 16);
    out[(int64_t)t * H8 + c] = o;
  }
}

}  // namespace
}  // namespace tw

using namespace tw;

extern "C" size_t tw_ep_row_bytes(int H, int K) { return (size_t)row_bytes(H, K); }

extern "C" int tw_ep_dispatch(const void* x, const float* topk_w, const int32_t* topk_ids,
                              int64_t T, int K, int H, int experts_per_rank, int world,
                              void* send_rows, void* stream) {
  TW_CHECK_ARG(T >= 0 && T < 65536 && K > 0 && K <= 256, "ep_dispatch: need T < 65536, 0 < K <= 256");
  TW_CHECK_ARG(H > 0 && H % 8 == 0, "ep_dispatch: H must be a multiple of 8");
  TW_CHECK_ARG(world > 0 && world <= 65535 && experts_per_rank > 0, "ep_dispatch: bad world/experts");
  TW_CHECK_ARG(aligned16(x) && aligned16(send_rows), "ep_dispatch: rows must be 16-byte aligned");
  if (T == 0) return TW_OK;
  TW_LAUNCH(ep_pack_kernel, dim3((unsigned)T, (unsigned)world), dim3(256), 0, as_stream(stream),
            reinterpret_cast<const uint4*>(x), topk_w, topk_ids, (int)T, K, H, experts_per_rank,
            row_bytes(H, K), static_cast<char*>(send_rows));
  return TW_OK;
}

extern "C" int tw_ep_receive(const void* recv_rows, int64_t rows, int K, int H, void* x,
                             int32_t* ids, float* w, void* stream) {
  TW_CHECK_ARG(rows >= 0 && rows < (1 << 30) && K > 0 && K <= 256 && H > 0 && H % 8 == 0,
               "ep_receive: bad shape");
  TW_CHECK_ARG(aligned16(recv_rows) && aligned16(x), "ep_receive: rows must be 16-byte aligned");
  if (rows == 0) return TW_OK;
  TW_LAUNCH(ep_unpack_kernel, dim3((unsigned)rows), dim3(256), 0, as_stream(stream),
            static_cast<const char*>(recv_rows), K, H, row_bytes(H, K),
            reinterpret_cast<uint4*>(x), ids, w);
  return TW_OK;
}

extern "C" int tw_ep_combine(const void* parts, int64_t T, int H, int world, void* out,
                             void* stream) {
  TW_CHECK_ARG(T >= 0 && T < 65536 && H > 0 && H % 8 == 0 && world > 0,
               "ep_combine: need T < 65536, H %% 8 == 0");
  TW_CHECK_ARG(aligned16(parts) && aligned16(out), "ep_combine: rows must be 16-byte aligned");
  if (T == 0) return TW_OK;
  const int H8 = H / 8;
  TW_LAUNCH(ep_sum_kernel, dim3((unsigned)((H8 + 255) / 256), (unsigned)T), dim3(256), 0,
            as_stream(stream), reinterpret_cast<const uint4*>(parts), (int)T, H8, world,
            reinterpret_cast<uint4*>(out));
  return TW_OK;
}
