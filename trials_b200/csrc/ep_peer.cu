// Expert-parallel exchange through NVLink peer memory: the two all-to-alls of
// the NCCL form (ep.cu) are folded into the kernels on either side of them.
//
// Every rank owns one exchange buffer (layout: EpPeerLayout in launch.h) that
// the other ranks map through CUDA IPC:
//   - the dispatch pack kernel stores each destination's rows straight into
//     that rank's receive area (block = source rank) and, when the last of its
//     CTAs is done, raises flag dflag[src] = epoch in every rank's header;
//   - on the receiving side a one-CTA kernel waits for the G dispatch flags
//     before the layer kernels read the rows;
//   - the layer's top-k reduce stores each result row straight into the
//     return area of the rank the token came from (block = expert-side rank)
//     and raises cflag[src] = epoch the same way;
//   - the combine kernel waits for the G combine flags, then sums.
// Flags only grow (epoch = call count, from 1), so nothing is reset between
// calls. Areas are double-buffered by epoch parity. Rank a stores into b's
// receive area (e & 1) in call e after a's layer of call e-1, which waited for
// b's dispatch of call e-1, which b issued after its layer of call e-2 had
// read that area. Likewise b stores into a's return area (e & 1) in call e+2
// after waiting for a's dispatch of call e+2, which a issued after its combine
// of call e had read the area. Waits are bounded by %globaltimer and set
// B200MOE_DEVERR_TIMEOUT on expiry.
#include "common.cuh"
#include "ep_place.cuh"
#include "ep_wait.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "rowops.cuh"

namespace b200moe {

namespace {

// Called by every thread of every CTA after its stores: the last CTA to finish
// raises this rank's flag (at byte offset flag_off of each rank's buffer) to
// epoch on all G ranks and resets the CTA counter for the next launch. The G
// flags are raised by G threads at once: each release store waits for the
// writes before it to reach the system (about 1 us apiece), so one thread
// raising them in turn cost G of those waits.
__device__ __forceinline__ void signal_done(const EpPeerArgs& a, int64_t flag_off, int32_t* counter) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(counter, 1) == (int)(gridDim.x * gridDim.y) - 1;
    if (last) {
      atomicExch(counter, 0);
      __threadfence_system();
    }
  }
  __syncthreads();
  if (last) {
    for (int g = threadIdx.x; g < a.G; g += blockDim.x)
      st_release_sys(reinterpret_cast<int32_t*>(a.bases[g] + flag_off) + a.rank, a.epoch);
  }
}

// One warp per (destination row, 1024-column segment), the rows as
// ep_pack_kernel builds them, stored into the destination's receive area (row
// rank*rows_per_rank + r). With bf16 input the warp quantises its segment 1x128
// on the way (the arithmetic of b200moe_quant_1x128, once per destination);
// otherwise it copies the fp8 bytes and scales. Segment 0 writes the ids and
// weights.
__global__ void __launch_bounds__(256) ep_pack_peer_kernel(const __nv_bfloat16* __restrict__ hidden,
                                                           const uint8_t* __restrict__ q, const float* __restrict__ s,
                                                           const int32_t* __restrict__ ids,
                                                           const float* __restrict__ w, int64_t H, int topk,
                                                           const EpPlace pl, const int32_t* __restrict__ tok_of,
                                                           const int32_t* __restrict__ counts, int64_t row_bytes,
                                                           const EpPeerArgs a, int32_t* counter) {
  griddep_wait();  // the plan ahead of it (programmatic launch)
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t seg0 = (int64_t)blockIdx.y * kQuantSegCols;
  if (row < (int64_t)a.G * a.rows_per_rank) {
    const int d = (int)(row / a.rows_per_rank);
    const int64_t r = row - (int64_t)d * a.rows_per_rank;
    uint8_t* dst = a.bases[d] + a.area_off + ((int64_t)a.rank * a.rows_per_rank + r) * row_bytes;
    int32_t* dst_ids = reinterpret_cast<int32_t*>(dst + H + (H / 128) * 4);
    float* dst_w = reinterpret_cast<float*>(dst_ids + topk);
    const bool used = r < __ldg(&counts[d]);
    const int64_t t = used ? __ldg(&tok_of[row]) : 0;
    if (used) {
      // a one-row view: input row t, output row 0 of a zero-stride destination
      QuantArgs qa{};
      qa.K = H;
      qa.q = dst;
      qa.s = reinterpret_cast<float*>(dst + H);
      qa.s_grp = 1;
      if (hidden) {
        qa.x = hidden + t * H;
      } else {
        qa.xq = q + t * H;
        qa.xs = s + t * (H / 128);
      }
      quant_row_segment(qa, 0, seg0, lane);
    }
    if (blockIdx.y == 0) {
      for (int j = lane; j < topk; j += 32) {
        const int p = used ? ep_target(pl, __ldg(&ids[t * topk + j]), t, j, topk) : -1;
        const bool mine = p >= 0 && p / pl.slots == d;
        dst_ids[j] = mine ? p - d * pl.slots : -1;
        dst_w[j] = mine ? __ldg(&w[t * topk + j]) : 0.f;
      }
    }
  }
  signal_done(a, EpPeerLayout::kDispatchFlags, counter);
}

// Packed rows -> contiguous (R, topk) ids and weights (as ep_unpack_meta_kernel),
// once the G dispatch flags of this epoch are up.
__global__ void ep_unpack_meta_peer_kernel(const uint8_t* own, const uint8_t* rows, int64_t R, int64_t row_bytes,
                                           int64_t H, int topk, int G, int32_t epoch, int32_t* __restrict__ ids,
                                           float* __restrict__ w, int32_t* err, uint64_t limit_ns) {
  wait_flags(reinterpret_cast<const int32_t*>(own + EpPeerLayout::kDispatchFlags), G, epoch, err, limit_ns);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * topk) return;
  const int64_t r = i / topk;
  const int j = (int)(i - r * topk);
  const int32_t* src = reinterpret_cast<const int32_t*>(rows + r * row_bytes + H + (H / 128) * 4);
  ids[i] = __ldcg(&src[j]);  // stored by other GPUs during this kernel's wait: read through L2
  w[i] = __ldcg(reinterpret_cast<const float*>(src + topk) + j);
}

// Top-k reduce of the received rows (R = G*rows_per_rank, row i = row
// i % rows_per_rank of source rank i / rows_per_rank), each bf16 result row
// stored into the source rank's return area at row rank*rows_per_rank + r.
template <int B>
__global__ void __launch_bounds__(256) ep_reduce_peer_kernel(const __nv_bfloat16* __restrict__ pair,
                                                             const int32_t* __restrict__ slot_pos, int sorted_rows,
                                                             int topk, int64_t H, const EpPeerArgs a,
                                                             int32_t* counter) {
  griddep_wait();  // the experts launch ahead of it (programmatic launch)
  const int64_t per_row = H / 8;
  const int64_t R = (int64_t)a.G * a.rows_per_rank;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = idx / per_row;
  if (t < R) {
    const int src = (int)(t / a.rows_per_rank);
    const int64_t r = t - (int64_t)src * a.rows_per_rank;
    __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(a.bases[src] + a.area_off) +
                         ((int64_t)a.rank * a.rows_per_rank + r) * H;
    // rows past a source's count carry no slot and are never read: not sent
    reduce_token_cols<B, true>(pair, slot_pos, sorted_rows, topk, H, t, (idx - t * per_row) * 8, row);
  }
  signal_done(a, EpPeerLayout::kCombineFlags, counter);
}

// out[t] = bf16(sum over ranks d, ascending, of the return-area row d*rpr + pos[t][d]),
// after the G combine flags of this epoch are up.
__global__ void __launch_bounds__(256) ep_combine_peer_kernel(const uint8_t* own, int64_t area_off,
                                                              const int32_t* __restrict__ pos, int64_t M, int64_t H,
                                                              int G, int64_t rows_per_rank, int32_t epoch,
                                                              __nv_bfloat16* __restrict__ out, int32_t* err,
                                                              uint64_t limit_ns) {
  griddep_wait();  // the reduce ahead of it (programmatic launch)
  wait_flags(reinterpret_cast<const int32_t*>(own + EpPeerLayout::kCombineFlags), G, epoch, err, limit_ns);
  const __nv_bfloat16* comb = reinterpret_cast<const __nv_bfloat16*>(own + area_off);
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
    // Written by another GPU in this kernel's lifetime: read through L2.
    const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(comb + ((int64_t)d * rows_per_rank + r) * H + c));
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

cudaError_t launch_ep_pack_peer(const void* hidden, const uint8_t* q, const float* s, const int32_t* ids,
                                const float* w, int64_t H, int topk, const EpPlace& pl, const int32_t* tok_of,
                                const int32_t* counts, int64_t row_bytes, const EpPeerArgs& a, int32_t* counter,
                                cudaStream_t stream) {
  const int64_t rows = (int64_t)a.G * a.rows_per_rank;
  const dim3 grid((unsigned)(rows > 0 ? (rows + 7) / 8 : 1),  // one CTA at least, to raise the flags
                  (unsigned)((H + kQuantSegCols - 1) / kQuantSegCols));
  return launch_pdl(ep_pack_peer_kernel, grid, dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(hidden), q, s,
                    ids, w, H, topk, pl, tok_of, counts, row_bytes, a, counter);
}

cudaError_t launch_ep_unpack_meta_peer(const uint8_t* own, const uint8_t* rows, int64_t R, int64_t row_bytes,
                                       int64_t H, int topk, int G, int32_t epoch, int32_t* ids, float* w,
                                       int32_t* err, uint64_t limit_ns, cudaStream_t stream) {
  const int64_t n = R * topk;
  const int64_t blocks = n > 0 ? (n + 255) / 256 : 1;
  ep_unpack_meta_peer_kernel<<<(unsigned)blocks, 256, 0, stream>>>(own, rows, R, row_bytes, H, topk, G, epoch, ids,
                                                                    w, err, limit_ns);
  return cudaGetLastError();
}

cudaError_t launch_ep_reduce_peer(const __nv_bfloat16* pair, const int32_t* slot_pos, int sorted_rows, int topk, int64_t H,
                                  const EpPeerArgs& a, int32_t* counter, cudaStream_t stream) {
  const int64_t R = (int64_t)a.G * a.rows_per_rank;
  const int64_t n = R * (H / 8);
  const int64_t blocks = n > 0 ? (n + 255) / 256 : 1;
  if (R * topk <= 1024)
    return launch_pdl(ep_reduce_peer_kernel<8>, dim3((unsigned)blocks), dim3(256), 0, stream, pair, slot_pos,
                      sorted_rows, topk, H, a, counter);
  return launch_pdl(ep_reduce_peer_kernel<4>, dim3((unsigned)blocks), dim3(256), 0, stream, pair, slot_pos,
                    sorted_rows, topk, H, a, counter);
}

cudaError_t launch_ep_combine_peer(const uint8_t* own, int64_t area_off, const int32_t* pos, int64_t M, int64_t H,
                                   int G, int64_t rows_per_rank, int32_t epoch, void* out, int32_t* err,
                                   uint64_t limit_ns, cudaStream_t stream) {
  const int64_t n = M * (H / 8);
  if (n <= 0) return cudaSuccess;
  return launch_pdl(ep_combine_peer_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, own, area_off,
                    pos, M, H, G, rows_per_rank, epoch, reinterpret_cast<__nv_bfloat16*>(out), err, limit_ns);
}

}  // namespace b200moe
