// Routing: moe_align_block_size with a stable within-expert order, plus the
// grouped-GEMM work list (chunks).
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
// One CTA of 1024 threads (32 warps). The flat ids are cut into 32 contiguous
// segments, one per warp. Pass 1 counts per (warp, expert) with
// __match_any_sync; a column scan over warps gives each warp its starting
// offset inside every expert; pass 2 walks the same segments in order and
// places each id at offset + (rank among equal experts in lower lanes).
// That makes the order stable without sorting.
#include "common.cuh"
#include "launch.h"

namespace b200moe {

constexpr int kRouteWarps = 32;
constexpr int kRouteThreads = kRouteWarps * 32;
constexpr int kRouteBatch = 8;  // 32-id steps whose loads a warp issues together

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

// Exclusive scan over the 1024 threads of the block; *total receives the sum.
__device__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
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
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;
  }
  __syncthreads();
  const int excl = x - v + (warp > 0 ? warp_tot[warp - 1] : 0);
  *total = warp_tot[31];
  __syncthreads();
  return excl;
}

__global__ void __launch_bounds__(kRouteThreads, 1) align_kernel(const AlignArgs a) {
  extern __shared__ int32_t sm[];
  __shared__ int warp_tot[32];
  const int E = a.E;
  int32_t* cnt = sm;                        // [kRouteWarps][E]
  int32_t* base = cnt + kRouteWarps * E;    // [E + 1] padded row offsets
  int32_t* padded = base + E + 1;           // [E]
  int32_t* chbase = padded + E;             // [E + 1] chunk offsets
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (a.chunk_ready)  // per-chunk counters and the two phase counters after them
    for (int64_t i = tid; i < a.chunks_cap + 2; i += kRouteThreads) a.chunk_ready[i] = 0;

  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) cnt[i] = 0;
  __syncthreads();

  const int64_t n = a.n;
  const int64_t seg = (n + kRouteWarps - 1) / kRouteWarps;
  const int64_t beg = warp * seg;
  const int64_t end = beg + seg < n ? beg + seg : n;

  // Pass 1: per-(warp, expert) counts. Each warp loads kRouteBatch steps of
  // ids before it counts any (one load round trip per batch, not per step).
  for (int64_t i0 = beg; i0 < end; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < end) ? map_expert(a, __ldg(&a.topk_ids[i]), true) : -2;
    }
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const unsigned peers = __match_any_sync(0xffffffffu, ev[u]);
      if (ev[u] >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + ev[u]] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  // Column scan over warps: cnt[w][e] <- rows of expert e in warps < w.
  int tot = 0;
  if (tid < E) {
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = cnt[w * E + tid];
      cnt[w * E + tid] = tot;
      tot += c;
    }
  }
  const int bm = a.block_m;
  const int pad = tid < E ? (tot + bm - 1) / bm * bm : 0;
  int total_rows = 0;
  const int off = block_exclusive_scan(pad, warp_tot, &total_rows);
  int nch = 0;
  if (tid < E) {
    base[tid] = off;
    padded[tid] = pad;
    if (a.tile_tokens > 0) nch = (pad + a.tile_tokens - 1) / a.tile_tokens;
  }
  int total_chunks = 0;
  const int choff = block_exclusive_scan(nch, warp_tot, &total_chunks);
  if (tid < E) chbase[tid] = choff;
  if (tid == 0) {
    base[E] = total_rows;
    chbase[E] = total_chunks;
  }
  const bool overflow = total_rows > a.sorted_cap || (a.tile_tokens > 0 && total_chunks > a.chunks_cap);
  if (tid == 0) {
    if (overflow) atomicOr(a.err, ERR_DEV_CAPACITY);
    *a.ntp = overflow ? 0 : total_rows;
    if (a.n_chunks) *a.n_chunks = overflow ? 0 : total_chunks;
  }
  // Defined contents everywhere: sentinel ids (and no position for any slot)
  // first, then the scatter below.
  for (int64_t i = tid; i < a.sorted_cap; i += kRouteThreads) a.sorted_ids[i] = a.sentinel;
  if (a.slot_pos)
    for (int64_t i = tid; i < a.n; i += kRouteThreads) a.slot_pos[i] = -1;
  __syncthreads();
  if (overflow) return;

  // Pass 2: stable scatter.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t i0 = beg; i0 < end; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < end) ? map_expert(a, __ldg(&a.topk_ids[i]), false) : -2;
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
    for (int64_t b = tid; b < a.blocks_cap; b += kRouteThreads) {
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
  // most tile_tokens rows (multiples of block_m).
  if (a.tile_tokens > 0 && tid < E) {
    const int P = padded[tid];
    if (P > 0) {
      const int blocks = P / bm;
      const int nc = chbase[tid + 1] - chbase[tid];
      const int per = blocks / nc, extra = blocks % nc;
      int row0 = base[tid];
      for (int c = 0; c < nc; ++c) {
        const int rows = (per + (c < extra ? 1 : 0)) * bm;
        a.chunk_expert[chbase[tid] + c] = tid;
        a.chunk_row0[chbase[tid] + c] = row0;
        a.chunk_rows[chbase[tid] + c] = rows;
        row0 += rows;
      }
    }
  }
}

size_t align_smem_bytes(int E) { return (size_t)(kRouteWarps * E + 3 * E + 2) * sizeof(int32_t); }

cudaError_t launch_align(const AlignArgs& a, cudaStream_t stream) {
  const size_t smem = align_smem_bytes(a.E);
  cudaError_t err = cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  align_kernel<<<1, kRouteThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace b200moe
