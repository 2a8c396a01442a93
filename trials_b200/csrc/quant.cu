// FP8 quantisation kernels (HBM-bound) and the top-k combine reduction.
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "rowops.cuh"

namespace b200moe {

// ---------------------------------------------------------------------------
// 1 x 128 per-token-group quantisation (per_token_group_quant_fp8,
// phase5_orchestrator.py:26-32). One warp per (output row, 1024-column
// segment): each lane converts 8 consecutive bf16 per 16-byte load, a
// half-warp covers one 128-column group, and the warp issues the loads of its
// four 256-column steps before it reduces any of them, so a row's latency is
// one load round trip rather than K/256 of them.
// ---------------------------------------------------------------------------
constexpr int kQuantWarps = 8;

__global__ void __launch_bounds__(kQuantWarps * 32) quant_1x128_kernel(const QuantArgs a) {
  griddep_wait();  // the routing ahead of it (programmatic launch)
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  const int64_t n_rows = a.num_rows ? (int64_t)(*a.num_rows) : a.rows;
  if (row >= n_rows || row >= a.rows) return;
  quant_row_segment(a, row, (int64_t)blockIdx.y * kQuantSegCols, lane);
}

cudaError_t launch_quant_1x128(const QuantArgs& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.K <= 0) return cudaSuccess;
  const int64_t blocks = (a.rows + kQuantWarps - 1) / kQuantWarps;
  const dim3 grid((unsigned)blocks, (unsigned)((a.K + kQuantSegCols - 1) / kQuantSegCols));
  return launch_pdl(quant_1x128_kernel, grid, dim3(kQuantWarps * 32), 0, stream, a);
}

// ---------------------------------------------------------------------------
// 128 x 128 block quantisation of weights (per_block_quant_fp8,
// phase5_orchestrator.py:35-41). One CTA of 256 threads per block; thread t
// owns row t/2, columns (t%2)*64 .. +64.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quant_block128_kernel(const __nv_bfloat16* __restrict__ w, int64_t N,
                                                             int64_t K, uint8_t* __restrict__ q,
                                                             float* __restrict__ s) {
  __shared__ float wmax[8];
  const int kb = blockIdx.x, nb = blockIdx.y;
  const int64_t e = blockIdx.z;
  const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int64_t off = (e * N + (int64_t)nb * 128 + r) * K + (int64_t)kb * 128 + half * 64;
  float v[64];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(w + off) + i);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f2 = __bfloat1622float2(h2[k]);
      v[i * 8 + 2 * k] = f2.x;
      v[i * 8 + 2 * k + 1] = f2.y;
    }
  }
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = wmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, wmax[i]);
  const float scale = group_scale(amax);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t word[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t b = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) b |= (uint32_t)quant_e4m3(v[i * 16 + k * 4 + t], scale) << (8 * t);
      word[k] = b;
    }
    *reinterpret_cast<uint4*>(q + off + i * 16) = make_uint4(word[0], word[1], word[2], word[3]);
  }
  if (threadIdx.x == 0) s[(e * (N / 128) + nb) * (K / 128) + kb] = scale;
}

cudaError_t launch_quant_block128(const void* w, int64_t E, int64_t N, int64_t K, uint8_t* q, float* s,
                                  cudaStream_t stream) {
  if (E <= 0) return cudaSuccess;
  dim3 grid((unsigned)(K / 128), (unsigned)(N / 128), (unsigned)E);
  quant_block128_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(w), N, K, q, s);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Top-k combine: out[t, n] = bf16(sum_j pair[pos(t, j), n]) over the routed
// slots, summed in slot order j (the view(M, k, K).sum(1) of
// sglang_integration/aiter.py:176-177, on bf16 rows that already carry the
// router weight). pos = slot_pos[t*topk+j] (-1: slot dropped); the slot's row
// of pair is pos (sorted_rows) or t*topk+j. One thread per 8 output columns.
// ---------------------------------------------------------------------------
// Slots whose row loads a thread issues together: 8 for small batches (the
// loads are the latency), 4 for large ones (measured: 0.167 vs 0.185 ms with 1
// and 0.28 with 8 at 8192 tokens).
#ifndef B200MOE_REDUCE_B_LARGE
#define B200MOE_REDUCE_B_LARGE 4
#endif

template <int B>
__global__ void __launch_bounds__(256) combine_reduce_kernel(const __nv_bfloat16* __restrict__ pair,
                                                             const int32_t* __restrict__ slot_pos, int sorted_rows,
                                                             int64_t M, int topk, int64_t H,
                                                             __nv_bfloat16* __restrict__ out) {
  griddep_wait();  // the experts launch ahead of it (programmatic launch)
  const int64_t per_row = H / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = idx / per_row;
  if (t >= M) return;
  reduce_token_cols<B>(pair, slot_pos, sorted_rows, topk, H, t, (idx - t * per_row) * 8, out + t * H);
}

cudaError_t launch_combine_reduce(const void* pair_rows, const int32_t* slot_pos, int sorted_rows, int64_t M, int topk,
                                  int64_t H, void* out, cudaStream_t stream) {
  const int64_t n = M * (H / 8);
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  const __nv_bfloat16* pair = static_cast<const __nv_bfloat16*>(pair_rows);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  if (M * topk <= 1024)
    return launch_pdl(combine_reduce_kernel<8>, dim3((unsigned)blocks), dim3(256), 0, stream, pair, slot_pos,
                      sorted_rows, M, topk, H, o);
  return launch_pdl(combine_reduce_kernel<B200MOE_REDUCE_B_LARGE>, dim3((unsigned)blocks), dim3(256), 0, stream,
                    pair, slot_pos, sorted_rows, M, topk, H, o);
}

// ---------------------------------------------------------------------------
// Bounded-wait self test: waits on an mbarrier that nothing completes.
// ---------------------------------------------------------------------------
__global__ void wait_timeout_selftest_kernel(int32_t* err, uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait_bounded(&bar, 0, timeout_ns)) atomicOr(err, ERR_DEV_TIMEOUT);
  }
}

cudaError_t launch_wait_timeout_selftest(int32_t* err, uint64_t timeout_ns, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(err, timeout_ns);
  return cudaGetLastError();
}

}  // namespace b200moe
