// Router: scores -> top-k expert ids and weights, one warp per token.
//
// Replaces the router stage in front of the MoE layer (aiter's
// topksoftmax kernel in the reference's runs, MBR/micro/glm52_fp8_moe.log;
// GLM's sigmoid "noaux_tc" routing, measure_xcd_imbalance.py:50-55 and
// phase1_xcd_imbalance_and_proof.md:37-39):
//   softmax: p = softmax(logits); select the k largest p (= largest logits);
//   sigmoid: s = 1 / (1 + exp(-logits)); select the k largest s + bias
//            (bias = per-expert correction, optional);
//   weights = unbiased p or s of the selected experts, optionally divided by
//   their sum, times scaling (routed_scaling_factor).
// Output order: descending selection value; equal values -> lower id first.
#include "common.cuh"
#include "launch.h"

namespace b200moe {

namespace {

constexpr int kRouterWarps = 4;
constexpr int kMaxPerLane = 32;  // E <= 1024

template <typename T>
__device__ __forceinline__ float load_logit(const T* p);
template <>
__device__ __forceinline__ float load_logit<float>(const float* p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32) router_topk_kernel(const T* __restrict__ logits, int64_t M, int E,
                                                                        int topk, int scoring,
                                                                        const float* __restrict__ bias,
                                                                        int renormalize, float scaling,
                                                                        float* __restrict__ out_w,
                                                                        int32_t* __restrict__ out_ids) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (t >= M) return;
  const T* row = logits + t * E;
  const int per = (E + 31) / 32;  // values per lane: expert e = lane + 32 * i
  float x[kMaxPerLane], sel[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    x[i] = (i < per && e < E) ? load_logit<T>(row + e) : -INFINITY;
  }
  float denom = 1.f, xmax = 0.f;
  if (scoring == 0) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (i < per && lane + 32 * i < E) sum += expf(x[i] - m);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    denom = sum;
    xmax = m;
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    if (i < per && e < E) {
      if (scoring == 0) {
        sel[i] = x[i];  // softmax is monotone in the logit
      } else {
        const float s = 1.0f / (1.0f + expf(-x[i]));
        x[i] = s;
        sel[i] = bias ? s + __ldg(&bias[e]) : s;
      }
    } else {
      sel[i] = -INFINITY;
    }
  }
  float wsum = 0.f;
  float wk[16];
  int idk[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (k >= topk) break;
    // lane-local best, then warp argmax (larger value, then lower id)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (sel[i] > bv || (sel[i] == bv && e < bi && sel[i] != -INFINITY)) {
        bv = sel[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // owner lane marks it and publishes the weight
    float w = 0.f;
    if ((bi & 31) == lane) {
      const int i = bi >> 5;
#pragma unroll
      for (int ii = 0; ii < kMaxPerLane; ++ii)
        if (ii == i) {
          w = scoring == 0 ? expf(x[ii] - xmax) / denom : x[ii];
          sel[ii] = -INFINITY;
        }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    wk[k] = w;
    idk[k] = bi;
    wsum += w;
  }
  if (lane < topk) {
    float w = 0.f;
    int id = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k == lane) {
        w = wk[k];
        id = idk[k];
      }
    if (renormalize) w = w / wsum;
    out_w[t * topk + lane] = w * scaling;
    out_ids[t * topk + lane] = id;
  }
}

}  // namespace

cudaError_t launch_router_topk(const void* logits, int bf16, int64_t M, int E, int topk, int scoring,
                               const float* bias, int renormalize, float scaling, float* out_w, int32_t* out_ids,
                               cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((M + kRouterWarps - 1) / kRouterWarps);
  if (bf16)
    router_topk_kernel<__nv_bfloat16><<<blocks, kRouterWarps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits), M, E, topk, scoring, bias, renormalize, scaling, out_w,
        out_ids);
  else
    router_topk_kernel<float><<<blocks, kRouterWarps * 32, 0, stream>>>(reinterpret_cast<const float*>(logits), M,
                                                                         E, topk, scoring, bias, renormalize,
                                                                         scaling, out_w, out_ids);
  return cudaGetLastError();
}

}  // namespace b200moe
