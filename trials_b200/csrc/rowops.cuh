// Per-row device routines shared by the stand-alone kernels (quant.cu) and
// the fused experts launch (moe_gemm.cuh): 1x128 quantisation / row copy of
// one (row, 1024-column segment) by one warp, and the top-k reduce of eight
// output columns of one token by one thread.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace b200moe {

constexpr int kQuantSegSteps = 4;
constexpr int kQuantSegCols = 256 * kQuantSegSteps;

__device__ __forceinline__ int32_t ld_index(const QuantArgs& a, const int32_t* p) {
  return a.meta_l2 ? __ldcg(p) : __ldg(p);
}

// One warp: launch row `row` of `a` (see QuantArgs), columns seg0 .. seg0+1023.
// Each lane converts 8 consecutive bf16 per 16-byte load, a half-warp covers
// one 128-column group, and the warp issues the loads of its four 256-column
// steps before it reduces any of them (one load round trip per row). In fan-out
// mode the segment is quantised (or loaded) once and stored to each of the
// token's slot rows.
__device__ __forceinline__ void quant_row_segment(const QuantArgs& a, int64_t row, int64_t seg0, int lane) {
  const int64_t seg_end = seg0 + kQuantSegCols < a.K ? seg0 + kQuantSegCols : a.K;
  int64_t src = row, dst = row;
  int32_t pos = 0;
  const bool fan = a.slot_pos && a.fanout;
  if (fan) {
    src = row;  // lane j holds the row of slot j; consumed after the loads are issued
    pos = lane < a.topk ? ld_index(a, &a.slot_pos[row * a.topk + lane]) : -1;
  } else if (a.slot_pos) {
    src = row / a.topk;
    pos = ld_index(a, &a.slot_pos[row]);  // consumed after the row's loads are issued
  } else if (a.sorted_ids) {
    const int f = ld_index(a, &a.sorted_ids[row]);
    src = (f >= 0 && f < a.sentinel) ? (int64_t)(f / a.topk) : -1;
    // Padding rows are not written: a padding row only feeds its own MMA
    // column (or row), whose results no epilogue keeps.
    if (src < 0) return;
  }
  if (a.xq != nullptr) {
    // Copy mode: the input is already quantised.
    const uint8_t* sq = a.xq + src * a.ldxq;
    uint4 v[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t b = seg0 + lane * 16 + i * 512;
      if (b < seg_end) v[i] = __ldg(reinterpret_cast<const uint4*>(sq + b));
    }
    const int64_t g = (seg0 >> 7) + lane;
    const bool gs = lane < kQuantSegCols / 128 && g * 128 < seg_end;
    const float sv = gs ? __ldg(&a.xs[src * a.ldxs + g]) : 0.f;
    auto put = [&](int64_t d) {
      uint8_t* qr = a.q + d * a.ldq;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int64_t b = seg0 + lane * 16 + i * 512;
        if (b < seg_end) *reinterpret_cast<uint4*>(qr + b) = v[i];
      }
      if (gs) a.s[d * a.s_row + g * a.s_grp] = sv;
    };
    if (fan) {
      for (int j = 0; j < a.topk; ++j) {
        const int d = __shfl_sync(0xffffffffu, pos, j);
        if (d >= 0) put(d);
      }
      return;
    }
    if (a.slot_pos) {
      if (pos < 0) return;
      dst = pos;
    }
    put(dst);
    return;
  }
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(a.x) + src * a.ldx;
  float v[kQuantSegSteps][8];
#pragma unroll
  for (int i = 0; i < kQuantSegSteps; ++i) {
    const int64_t c = seg0 + i * 256 + lane * 8;
    if (c < seg_end) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr + c));
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f2 = __bfloat1622float2(h2[j]);
        v[i][2 * j] = f2.x;
        v[i][2 * j + 1] = f2.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }
  uint2 packed[kQuantSegSteps];
  float scl[kQuantSegSteps];
#pragma unroll
  for (int i = 0; i < kQuantSegSteps; ++i) {
    packed[i] = make_uint2(0, 0);
    scl[i] = 0.f;
    if (seg0 + i * 256 >= seg_end) continue;  // warp-uniform
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    uint32_t lo = 0, hi = 0;
    const float scale = group_scale(m);
#pragma unroll
    for (int j = 0; j < 4; ++j) lo |= (uint32_t)quant_e4m3(v[i][j], scale) << (8 * j);
#pragma unroll
    for (int j = 0; j < 4; ++j) hi |= (uint32_t)quant_e4m3(v[i][4 + j], scale) << (8 * j);
    packed[i] = make_uint2(lo, hi);
    scl[i] = scale;
  }
  auto put = [&](int64_t d) {
    uint8_t* qr = a.q + d * a.ldq;
#pragma unroll
    for (int i = 0; i < kQuantSegSteps; ++i) {
      const int64_t c = seg0 + i * 256 + lane * 8;
      if (c >= seg_end) continue;
      *reinterpret_cast<uint2*>(qr + c) = packed[i];
      if ((lane & 15) == 0) a.s[d * a.s_row + (c >> 7) * a.s_grp] = scl[i];
    }
  };
  if (fan) {
    for (int j = 0; j < a.topk; ++j) {
      const int d = __shfl_sync(0xffffffffu, pos, j);
      if (d >= 0) put(d);
    }
    return;
  }
  if (a.slot_pos) {
    if (pos < 0) return;
    dst = pos;
  }
  put(dst);
}

// One thread: out_row[c .. c+7] = bf16(sum over the routed slots j of token t's
// stage-2 rows), slots summed in order j. pos = slot_pos[t*topk + j]
// (-1: dropped); the row is pos (sorted_rows) or t*topk + j. Slots in groups of
// B: all positions, then all row loads of the group are issued before the
// sums consume them. Loads go through L2 (the rows may have been written by
// other CTAs of the same launch). SKIP_EMPTY: a row with no routed slot is not
// stored (rows nobody reads: unused rows of an expert-parallel exchange block).
template <int B, bool SKIP_EMPTY = false>
__device__ __forceinline__ void reduce_token_cols(const __nv_bfloat16* pair, const int32_t* slot_pos, int sorted_rows,
                                                  int topk, int64_t H, int64_t t, int64_t c,
                                                  __nv_bfloat16* out_row) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  bool any = false;
  for (int j0 = 0; j0 < topk; j0 += B) {
    int pos[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      pos[j] = j0 + j < topk ? __ldcg(&slot_pos[t * topk + j0 + j]) : -1;
      any |= pos[j] >= 0;
    }
    uint4 x[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      if (pos[j] >= 0) {
        const int64_t row = sorted_rows ? (int64_t)pos[j] : t * topk + j0 + j;
        x[j] = __ldcg(reinterpret_cast<const uint4*>(pair + row * H + c));
      }
    }
#pragma unroll
    for (int j = 0; j < B; ++j) {
      if (pos[j] < 0) continue;
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&x[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
  }
  if (SKIP_EMPTY && !any) return;
  __nv_bfloat162 o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  *reinterpret_cast<uint4*>(out_row + c) = *reinterpret_cast<const uint4*>(o);
}

}  // namespace b200moe
