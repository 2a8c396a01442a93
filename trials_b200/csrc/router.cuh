// Router top-k of one token by one warp: scores -> k expert ids and weights.
//
// The router in front of the reference's MoE call (aiter's topksoftmax kernel
// in its runs, MBR/micro/glm52_fp8_moe.log; GLM's sigmoid "noaux_tc" routing,
// measure_xcd_imbalance.py:50-55 and phase1_xcd_imbalance_and_proof.md:37-39):
//   softmax: p = softmax(logits); select the k largest p (= largest logits);
//   sigmoid: s = 1 / (1 + exp(-logits)); select the k largest s + bias
//            (bias = per-expert correction, optional);
//   weights = unbiased p or s of the selected experts, optionally divided by
//   their sum, times scaling (routed_scaling_factor).
// Output order: descending selection value; equal values -> lower id first.
// Used by the standalone router kernel (router.cu) and by routing's first
// launch when routing starts from logits (route.cu): the same arithmetic, so
// the two give the same bits.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace b200moe {

constexpr int kRouterMaxPerLane = 32;  // E <= 1024
constexpr int kRouterMaxTopk = 16;

struct RouterArgs {
  const void* logits;  // (M, E) f32, or bf16 when bf16 != 0
  int bf16;
  int E, topk, scoring, renormalize;
  const float* bias;   // nullable (sigmoid only)
  float scaling;
  float* out_w;        // (M, topk)
  int32_t* out_ids;    // (M, topk)
};

__device__ __forceinline__ float router_logit(const RouterArgs& r, int64_t t, int e) {
  if (r.bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(r.logits)[t * r.E + e]);
  return __ldg(reinterpret_cast<const float*>(r.logits) + t * r.E + e);
}

// Warp-wide: routes token t; lane j < topk returns the j-th id and weight and
// also stores them to r.out_ids / r.out_w. All 32 lanes must call it.
__device__ __forceinline__ void route_token_warp(const RouterArgs& r, int64_t t, int lane, int& id_out,
                                                 float& w_out) {
  const int E = r.E, topk = r.topk;
  const int per = (E + 31) / 32;  // values per lane: expert e = lane + 32 * i
  float x[kRouterMaxPerLane], sel[kRouterMaxPerLane];
#pragma unroll
  for (int i = 0; i < kRouterMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    x[i] = (i < per && e < E) ? router_logit(r, t, e) : -INFINITY;
  }
  float denom = 1.f, xmax = 0.f;
  if (r.scoring == 0) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kRouterMaxPerLane; ++i) m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kRouterMaxPerLane; ++i)
      if (i < per && lane + 32 * i < E) sum += expf(x[i] - m);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    denom = sum;
    xmax = m;
  }
#pragma unroll
  for (int i = 0; i < kRouterMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    if (i < per && e < E) {
      if (r.scoring == 0) {
        sel[i] = x[i];  // softmax is monotone in the logit
      } else {
        const float s = 1.0f / (1.0f + expf(-x[i]));
        x[i] = s;
        sel[i] = r.bias ? s + __ldg(&r.bias[e]) : s;
      }
    } else {
      sel[i] = -INFINITY;
    }
  }
  float wsum = 0.f;
  float wk[kRouterMaxTopk];
  int idk[kRouterMaxTopk];
#pragma unroll
  for (int k = 0; k < kRouterMaxTopk; ++k) {
    if (k >= topk) break;
    // lane-local best, then warp argmax (larger value, then lower id)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kRouterMaxPerLane; ++i) {
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
      for (int ii = 0; ii < kRouterMaxPerLane; ++ii)
        if (ii == i) {
          w = r.scoring == 0 ? expf(x[ii] - xmax) / denom : x[ii];
          sel[ii] = -INFINITY;
        }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    wk[k] = w;
    idk[k] = bi;
    wsum += w;
  }
  id_out = 0;
  w_out = 0.f;
  if (lane < topk) {
#pragma unroll
    for (int k = 0; k < kRouterMaxTopk; ++k)
      if (k == lane) {
        w_out = wk[k];
        id_out = idk[k];
      }
    if (r.renormalize) w_out = w_out / wsum;
    w_out *= r.scaling;
    r.out_w[t * topk + lane] = w_out;
    r.out_ids[t * topk + lane] = id_out;
  }
}

}  // namespace b200moe
