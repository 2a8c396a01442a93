// Expert-parallel dispatch and combine kernels.
//
// Rank r of G owns experts [r*E/G, (r+1)*E/G), or, with a replica table
// (EpPlace, EPLB), the physical expert slots [r*S, (r+1)*S) that the table
// gives replicas of the logical experts. A token is sent once to every
// rank that holds the chosen replica of at least one of its top-k experts, as
// one fixed-size packed row (layout in include/b200moe.h, b200moe_ep_row_bytes):
//   [ fp8 row (H B) | 1x128 scales (H/128 f32) | k local ids (int32, -1 = not
//     on that rank) | k router weights (f32) ]
// Rows for destination d occupy block d of the send buffer, rows_per_rank rows
// per block, in ascending token order; unused rows carry ids -1. With equal
// blocks the exchange is one equal-split all-to-all and needs no host-side
// count exchange. The receiving rank runs the layer on the packed rows and
// returns one bf16 row per received row (its experts' weighted sum); the
// source adds the rows from each rank in rank order.
#include "common.cuh"
#include "ep_place.cuh"
#include "launch.h"
#include "ptx.cuh"

namespace b200moe {

namespace {

constexpr int kPlanThreads = 1024;

// One CTA per destination rank: stable positions of the tokens it needs (the
// tokens with at least one routed slot whose replica, ep_target, is on it).
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* __restrict__ ids, int64_t M, int topk,
                                                                const EpPlace pl, int64_t rows_per_rank,
                                                                int32_t* __restrict__ pos,
                                                                int32_t* __restrict__ tok_of,
                                                                int32_t* __restrict__ counts, int32_t* err) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  griddep_launch_dependents();  // the pack may start launching (it waits for this grid)
  const int d = blockIdx.x;
  const int G = pl.G, num_experts = pl.num_experts;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  for (int64_t t0 = 0; t0 < M; t0 += kPlanThreads) {
    const int64_t t = t0 + threadIdx.x;
    int need = 0;
    if (t < M) {
      for (int j = 0; j < topk; ++j) {
        const int id = __ldg(&ids[t * topk + j]);
        const int p = ep_target(pl, id, t, j, topk);
        if (p >= 0 && p / pl.slots == d) need = 1;
        // ids outside the expert range (other than -1), or a replica table that
        // names no physical slot for a valid id, are dropped and reported
        if (d == 0 && id != -1 && p < 0) atomicOr(err, ERR_DEV_BAD_EXPERT);
      }
    }
    int x = need;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int v = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      warp_tot[lane] = v;
    }
    __syncthreads();
    const int excl = x - need + (warp > 0 ? warp_tot[warp - 1] : 0);
    const int base = base_s;
    if (t < M) {
      const int r = base + excl;
      const bool fits = need && r < rows_per_rank;
      pos[t * G + d] = fits ? r : -1;
      if (fits) tok_of[(int64_t)d * rows_per_rank + r] = (int32_t)t;
      if (need && !fits) atomicOr(err, ERR_DEV_CAPACITY);
    }
    __syncthreads();
    if (threadIdx.x == 0) base_s = base + warp_tot[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[d] = base_s < rows_per_rank ? base_s : (int32_t)rows_per_rank;
}

// One warp per destination row: copy the token's fp8 row and scales and write
// its local ids and weights; rows past the count get ids -1.
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint8_t* __restrict__ q, const float* __restrict__ s,
                                                      const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                      int64_t H, int topk, const EpPlace pl,
                                                      int64_t rows_per_rank, const int32_t* __restrict__ tok_of,
                                                      const int32_t* __restrict__ counts, uint8_t* __restrict__ send,
                                                      int64_t row_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= (int64_t)pl.G * rows_per_rank) return;
  const int d = (int)(row / rows_per_rank);
  const int64_t r = row - (int64_t)d * rows_per_rank;
  uint8_t* dst = send + row * row_bytes;
  int32_t* dst_ids = reinterpret_cast<int32_t*>(dst + H + (H / 128) * 4);
  float* dst_w = reinterpret_cast<float*>(dst_ids + topk);
  if (r >= __ldg(&counts[d])) {
    for (int j = lane; j < topk; j += 32) {
      dst_ids[j] = -1;
      dst_w[j] = 0.f;
    }
    return;
  }
  const int64_t t = __ldg(&tok_of[row]);
  const uint4* src = reinterpret_cast<const uint4*>(q + t * H);
  uint4* out = reinterpret_cast<uint4*>(dst);
  for (int64_t i = lane; i < H / 16; i += 32) out[i] = __ldg(&src[i]);
  float* dst_s = reinterpret_cast<float*>(dst + H);
  for (int64_t g = lane; g < H / 128; g += 32) dst_s[g] = __ldg(&s[t * (H / 128) + g]);
  for (int j = lane; j < topk; j += 32) {
    const int p = ep_target(pl, __ldg(&ids[t * topk + j]), t, j, topk);
    const bool mine = p >= 0 && p / pl.slots == d;
    dst_ids[j] = mine ? p - d * pl.slots : -1;
    dst_w[j] = mine ? __ldg(&w[t * topk + j]) : 0.f;
  }
}

// Packed rows -> contiguous (R, topk) ids and weights.
__global__ void ep_unpack_meta_kernel(const uint8_t* __restrict__ rows, int64_t R, int64_t row_bytes, int64_t H,
                                      int topk, int32_t* __restrict__ ids, float* __restrict__ w) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * topk) return;
  const int64_t r = i / topk;
  const int j = (int)(i - r * topk);
  const int32_t* src = reinterpret_cast<const int32_t*>(rows + r * row_bytes + H + (H / 128) * 4);
  ids[i] = __ldg(&src[j]);
  w[i] = __ldg(reinterpret_cast<const float*>(src + topk) + j);
}

// out[t] = bf16( sum over ranks d (ascending) of comb[d][pos[t][d]] ).
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ comb,
                                                         const int32_t* __restrict__ pos, int64_t M, int64_t H,
                                                         int G, int64_t rows_per_rank,
                                                         __nv_bfloat16* __restrict__ out) {
  const int64_t per_row = H / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = idx / per_row;
  if (t >= M) return;
  const int64_t c = (idx - t * per_row) * 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int d = 0; d < G; ++d) {
    const int r = __ldg(&pos[t * G + d]);
    if (r < 0) continue;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(comb + ((int64_t)d * rows_per_rank + r) * H + c));
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  __nv_bfloat162 o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  *reinterpret_cast<uint4*>(out + t * H + c) = *reinterpret_cast<const uint4*>(o);
}

}  // namespace

cudaError_t launch_ep_plan(const int32_t* ids, int64_t M, int topk, const EpPlace& pl, int64_t rows_per_rank,
                           int32_t* pos, int32_t* tok_of, int32_t* counts, int32_t* err, cudaStream_t stream) {
  ep_plan_kernel<<<pl.G, kPlanThreads, 0, stream>>>(ids, M, topk, pl, rows_per_rank, pos, tok_of, counts, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const uint8_t* q, const float* s, const int32_t* ids, const float* w, int64_t M,
                               int64_t H, int topk, const EpPlace& pl, int64_t rows_per_rank, uint8_t* send,
                               int64_t row_bytes, int32_t* pos, int32_t* tok_of, int32_t* counts, int32_t* err,
                               cudaStream_t stream) {
  cudaError_t e = launch_ep_plan(ids, M, topk, pl, rows_per_rank, pos, tok_of, counts, err, stream);
  if (e != cudaSuccess) return e;
  const int64_t rows = (int64_t)pl.G * rows_per_rank;
  if (rows == 0) return cudaSuccess;
  ep_pack_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(q, s, ids, w, H, topk, pl, rows_per_rank, tok_of,
                                                                  counts, send, row_bytes);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack_meta(const uint8_t* rows, int64_t R, int64_t row_bytes, int64_t H, int topk,
                                  int32_t* ids, float* w, cudaStream_t stream) {
  const int64_t n = R * topk;
  if (n <= 0) return cudaSuccess;
  ep_unpack_meta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(rows, R, row_bytes, H, topk, ids, w);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const void* comb, const int32_t* pos, int64_t M, int64_t H, int G,
                              int64_t rows_per_rank, void* out, cudaStream_t stream) {
  const int64_t n = M * (H / 8);
  if (n <= 0) return cudaSuccess;
  ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(comb), pos, M, H, G, rows_per_rank,
      reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace b200moe
