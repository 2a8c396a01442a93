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

constexpr int kRouterMaxTopk = 16;  // E <= 1024 (32 values per lane)

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
// also stores them to r.out_ids / r.out_w. All 32 lanes must call it. PER =
// values per lane (expert e = lane + 32 i, i < PER): 8 for E <= 256, 16 for
// E <= 512, 32 for E <= 1024 (router_per_lane), so the logits stay in
// registers; the selected id and weight of round k stay in lane k.
template <int PER>
__device__ __forceinline__ void route_token_warp(const RouterArgs& r, int64_t t, int lane, int& id_out,
                                                 float& w_out) {
  const int E = r.E, topk = r.topk;
  float x[PER], sel[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    x[i] = e < E ? router_logit(r, t, e) : -INFINITY;
  }
  float denom = 1.f, xmax = 0.f;
  if (r.scoring == 0) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i < E) sum += expf(x[i] - m);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    denom = sum;
    xmax = m;
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
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
  float wsum = 0.f, my_w = 0.f;
  int my_id = 0;
  for (int k = 0; k < topk; ++k) {
    // lane-local best, then warp argmax (larger value, then lower id)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
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
      for (int ii = 0; ii < PER; ++ii)
        if (ii == i) {
          w = r.scoring == 0 ? expf(x[ii] - xmax) / denom : x[ii];
          sel[ii] = -INFINITY;
        }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    if (lane == k) {
      my_w = w;
      my_id = bi;
    }
    wsum += w;
  }
  id_out = 0;
  w_out = 0.f;
  if (lane < topk) {
    w_out = my_w;
    id_out = my_id;
    if (r.renormalize) w_out = w_out / wsum;
    w_out *= r.scaling;
    r.out_w[t * topk + lane] = w_out;
    r.out_ids[t * topk + lane] = id_out;
  }
}

// Values per lane for E experts (see route_token_warp).
__host__ __device__ __forceinline__ int router_per_lane(int E) { return E <= 256 ? 8 : (E <= 512 ? 16 : 32); }

}  // namespace b200moe
