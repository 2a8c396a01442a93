// One-CTA routing body (moe_align_block_size with a stable order inside each
// expert, plus the grouped-GEMM work list), for a CTA of NTHR threads.
//
// Semantics follow the reference's routing contract:
//   * flat index i = t*topk + j, grouped by expert, ascending i inside an
//     expert (the stable argsort of build_routing_from_topk,
//     phase5_orchestrator.py:51-57);
//   * each expert padded to a multiple of block_m with the sentinel M*topk and
//     experts laid out in ascending id order (moe_align_block_size as used at
//     sglang_integration/aiter.py:113-123);
//   * everything past the routed rows is defined: sentinel ids, expert id -1
//     (the reference leaves that tail uninitialised; MBR/phase13_findings.md:27-47).
//
// The flat ids are cut into NTHR/32 contiguous segments, one per warp. Pass 1
// counts per (warp, expert) with __match_any_sync; a column scan over warps
// gives each warp its starting offset inside every expert; pass 2 walks the
// same segments in order and places each id at offset + (rank among equal
// experts in lower lanes). That makes the order stable without sorting. The
// layout is a function of the ids alone, so every CTA width gives the same
// bits. Used by the routing kernels (1,024 threads) and by the whole-layer
// launch of the grouped GEMM (its own CTA width).
#pragma once

#include "common.cuh"
#include "launch.h"

namespace b200moe {

constexpr int kRouteBatch = 8;  // 32-id steps whose loads a warp issues together

// Loads flat id i. COH: the ids were stored earlier in the same launch (by a
// router), so they are read through L2, not the read-only path.
template <bool COH>
__device__ __forceinline__ int load_id(const AlignArgs& a, int64_t i) {
  return COH ? __ldcg(&a.topk_ids[i]) : __ldg(&a.topk_ids[i]);
}

// Maps a raw id to the weight index, -1 = drop. Reports bad ids when `report`.
__device__ __forceinline__ int map_expert(const AlignArgs& a, int raw, bool report) {
  if (raw == -1) return -1;
  if (raw < 0 || raw >= a.num_experts) {
    if (report) atomicOr(a.err, ERR_DEV_BAD_EXPERT);
    return -1;
  }
  if (a.expert_map == nullptr) return raw < a.E ? raw : -1;
  const int m = __ldg(&a.expert_map[raw]);
  if (m >= a.E) {
    if (report) atomicOr(a.err, ERR_DEV_BAD_EXPERT);
    return -1;
  }
  return m < 0 ? -1 : m;
}

// Exclusive scan over the NTHR threads of the block (every thread calls it);
// *total receives the sum. warp_tot: 32 ints of shared memory.
template <int NTHR>
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  constexpr int NW = NTHR / 32;
  static_assert(NTHR % 32 == 0 && NW <= 32, "block of whole warps, at most 32");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < NW ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < NW) warp_tot[lane] = t;
  }
  __syncthreads();
  const int excl = x - v + (warp > 0 ? warp_tot[warp - 1] : 0);
  *total = warp_tot[NW - 1];
  __syncthreads();
  return excl;
}

// Shared memory of align_body for E experts and NW warps, in ints.
__host__ __device__ constexpr int64_t align_smem_ints(int E, int NW) { return (int64_t)NW * E + 4 * E + 3 + 32; }

// All NTHR threads of the CTA call it (E <= 1024). sm: align_smem_ints(E,
// NTHR/32) ints of shared memory.
template <bool COH, int NTHR>
__device__ void align_body(const AlignArgs& a, int32_t* sm) {
  constexpr int NW = NTHR / 32;
  constexpr int PEM = (1024 + NTHR - 1) / NTHR;  // experts per thread, at most
  const int E = a.E;
  int32_t* cnt = sm;                   // [NW][E]
  int32_t* base = cnt + NW * E;        // [E + 1] padded row offsets
  int32_t* padded = base + E + 1;      // [E]
  int32_t* chbase = padded + E;        // [E + 1] chunk offsets
  int32_t* chbase2 = chbase + E + 1;   // [E + 1] heavy-list chunk offsets (mixed lists)
  int32_t* warp_tot = chbase2 + E + 1; // [32] scan scratch
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool mixed = a.heavy_rows > 0;
  if (a.chunk_ready)  // per-chunk counters and the two phase counters after them
    for (int64_t i = tid; i < a.chunks_cap + 2; i += NTHR) a.chunk_ready[i] = 0;
  if (mixed && tid < 2) a.counters2[tid] = 0;

  for (int i = tid; i < NW * E; i += NTHR) cnt[i] = 0;
  __syncthreads();

  const int64_t n = a.n;
  const int64_t seg = (n + NW - 1) / NW;
  const int64_t beg = warp * seg;
  const int64_t end = beg + seg < n ? beg + seg : n;

  // Pass 1: per-(warp, expert) counts. Each warp loads kRouteBatch steps of
  // ids before it counts any (one load round trip per batch, not per step).
  for (int64_t i0 = beg; i0 < end; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < end) ? map_expert(a, load_id<COH>(a, i), true) : -2;
    }
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const unsigned peers = __match_any_sync(0xffffffffu, ev[u]);
      if (ev[u] >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + ev[u]] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  // Thread tid owns experts [e0, e0 + pe): column scan over warps
  // (cnt[w][e] <- rows of expert e in warps < w) and the padded size.
  const int pe = (E + NTHR - 1) / NTHR;
  const int e0 = tid * pe;
  const int bm = a.block_m;
  int pad[PEM];
  int light = 0, heavy = 0, nch = 0, nch2 = 0;
#pragma unroll
  for (int k = 0; k < PEM; ++k) {
    const int e = e0 + k;
    pad[k] = 0;
    if (k < pe && e < E) {
      int tot = 0;
      for (int w = 0; w < NW; ++w) {
        const int c = cnt[w * E + e];
        cnt[w * E + e] = tot;
        tot += c;
      }
      pad[k] = (tot + bm - 1) / bm * bm;
      // Mixed lists: heavy experts (more than heavy_rows padded rows) after
      // all the light ones, each group in expert order.
      if (mixed && pad[k] > a.heavy_rows) {
        heavy += pad[k];
        nch2 += (pad[k] + kHeavyTile - 1) / kHeavyTile;
      } else {
        light += pad[k];
        if (a.tile_tokens > 0) nch += (pad[k] + a.tile_tokens - 1) / a.tile_tokens;
      }
    }
  }
  int total_light = 0, total_heavy = 0, total_chunks = 0, total_chunks2 = 0;
  int ro = block_exclusive_scan<NTHR>(light, warp_tot, &total_light);
  int rh = mixed ? block_exclusive_scan<NTHR>(heavy, warp_tot, &total_heavy) : 0;
  int co = block_exclusive_scan<NTHR>(nch, warp_tot, &total_chunks);
  int ch = mixed ? block_exclusive_scan<NTHR>(nch2, warp_tot, &total_chunks2) : 0;
  const int total_rows = total_light + total_heavy;
#pragma unroll
  for (int k = 0; k < PEM; ++k) {
    const int e = e0 + k;
    if (k < pe && e < E) {
      const bool hv = mixed && pad[k] > a.heavy_rows;
      base[e] = hv ? total_light + rh : ro;
      padded[e] = pad[k];
      chbase[e] = co;
      chbase2[e] = ch;
      if (hv) {
        rh += pad[k];
        ch += (pad[k] + kHeavyTile - 1) / kHeavyTile;
      } else {
        ro += pad[k];
        if (a.tile_tokens > 0) co += (pad[k] + a.tile_tokens - 1) / a.tile_tokens;
      }
    }
  }
  if (tid == 0) {
    base[E] = total_rows;
    chbase[E] = total_chunks;
    chbase2[E] = total_chunks2;
  }
  const bool overflow = total_rows > a.sorted_cap || (a.tile_tokens > 0 && total_chunks > a.chunks_cap) ||
                        (mixed && total_chunks2 > a.chunks_cap2);
  if (tid == 0) {
    if (overflow) atomicOr(a.err, ERR_DEV_CAPACITY);
    *a.ntp = overflow ? 0 : total_rows;
    if (a.n_chunks) *a.n_chunks = overflow ? 0 : total_chunks;
    if (mixed) {
      *a.n_chunks2 = overflow ? 0 : total_chunks2;
      *a.heavy_row0 = overflow ? 0 : total_light;
    }
  }
  // Defined contents everywhere: sentinel ids (and no position for any slot)
  // first, then the scatter below.
  for (int64_t i = tid; i < a.sorted_cap; i += NTHR) a.sorted_ids[i] = a.sentinel;
  if (a.slot_pos)
    for (int64_t i = tid; i < a.n; i += NTHR) a.slot_pos[i] = -1;
  __syncthreads();
  if (overflow) return;

  // Pass 2: stable scatter.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t i0 = beg; i0 < end; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < end) ? map_expert(a, load_id<COH>(a, i), false) : -2;
    }
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      const int e = ev[u];
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      int step = 0;
      if (e >= 0) {
        const int rank = __popc(peers & lt_mask);
        const int32_t pos = base[e] + cnt[warp * E + e] + rank;
        a.sorted_ids[pos] = (int32_t)i;
        if (a.slot_pos) a.slot_pos[i] = pos;
        step = __popc(peers);
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += step;
      __syncwarp();
    }
  }

  // Expert id of every block_m block; -1 past the routed rows.
  if (a.expert_ids != nullptr) {
    for (int64_t b = tid; b < a.blocks_cap; b += NTHR) {
      const int64_t row = b * bm;
      int eid = -1;
      if (row < total_rows) {
        int lo = 0, hi = E - 1;  // largest e with base[e] <= row
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (base[mid] <= row) lo = mid;
          else hi = mid - 1;
        }
        eid = lo;
      }
      a.expert_ids[b] = eid;
    }
  }

  // GEMM work list: each expert's rows cut into nearly equal chunks of at
  // most tile_tokens rows (multiples of block_m); heavy experts of mixed
  // lists into chunks of at most kHeavyTile rows in the second list.
  if (a.tile_tokens > 0) {
#pragma unroll
    for (int k = 0; k < PEM; ++k) {
      const int e = e0 + k;
      if (k >= pe || e >= E) continue;
      const int P = pad[k];
      const bool hv = mixed && P > a.heavy_rows;
      if (P > 0) {
        const int* cb = hv ? chbase2 : chbase;
        int32_t* ce = hv ? a.chunk_expert2 : a.chunk_expert;
        int32_t* cr0 = hv ? a.chunk_row0_2 : a.chunk_row0;
        int32_t* crw = hv ? a.chunk_rows2 : a.chunk_rows;
        const int blocks = P / bm;
        const int nc = cb[e + 1] - cb[e];
        const int per = blocks / nc, extra = blocks % nc;
        int row0 = base[e];
        for (int c = 0; c < nc; ++c) {
          const int rows = (per + (c < extra ? 1 : 0)) * bm;
          ce[cb[e] + c] = e;
          cr0[cb[e] + c] = row0;
          crw[cb[e] + c] = rows;
          row0 += rows;
        }
      }
    }
  }
}

}  // namespace b200moe
