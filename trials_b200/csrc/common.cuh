// Shared definitions for the b200moe kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200moe.h"

namespace b200moe {

// Device error word bits (the word lives in caller memory).
constexpr int32_t ERR_DEV_BAD_EXPERT = B200MOE_DEVERR_BAD_EXPERT_ID;
constexpr int32_t ERR_DEV_TIMEOUT = B200MOE_DEVERR_TIMEOUT;
constexpr int32_t ERR_DEV_CAPACITY = B200MOE_DEVERR_CAPACITY;

// FP8 E4M3 quantisation of one value with a per-group fp32 scale, following
// the torch expression (x / s).clamp(-448, 448).to(float8_e4m3fn)
// (phase5_orchestrator.py:26-32): IEEE division, clamp, round-to-nearest-even.
__device__ __forceinline__ uint8_t quant_e4m3(float x, float scale) {
  float v = __fdiv_rn(x, scale);
  v = fminf(fmaxf(v, -448.0f), 448.0f);
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// Group scale: max(amax / 448, 1e-12) in fp32 (phase5_orchestrator.py:29-30).
__device__ __forceinline__ float group_scale(float amax) { return fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f); }

// Work-unit order of the grouped GEMMs. A unit is (chunk, weight tile nt).
// Chunks are taken in groups of `group` consecutive chunks, and inside a group
// weight-tile-major: (c0, 0), (c1, 0), ..., (c0, 1), (c1, 1), ... CTAs running
// at the same time then share the weight tile of an expert that has several
// chunks (one HBM read, the rest from L2) and reuse the group's activation rows
// from L2. group = 1 is plain chunk-major order. A bijection of
// [0, n_chunks * NT) for every group >= 1.
__device__ __forceinline__ void unit_coords(int u, int n_chunks, int NT, int group, int& chunk, int& nt) {
  const int span = group * NT;
  const int g = u / span;
  const int r = u - g * span;
  const int first = g * group;
  const int gc = n_chunks - first < group ? n_chunks - first : group;
  nt = r / gc;
  chunk = first + (r - nt * gc);
}

}  // namespace b200moe
