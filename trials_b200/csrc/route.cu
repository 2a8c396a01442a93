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
#include "router.cuh"

namespace b200moe {

constexpr int kRouteWarps = 32;
constexpr int kRouteThreads = kRouteWarps * 32;
constexpr int kRouteBatch = 8;  // 32-id steps whose loads a warp issues together
constexpr int64_t kRouteMultiMinSlots = 16384;  // flat slots from which routing uses several CTAs
constexpr int64_t kRouteSlotsPerCta = 2048;
constexpr int kRouteMaxCtas = 128;

// Loads flat id i. COH: the ids were stored earlier in the same launch (the
// router part of routing from logits), so they are read through L2, not the
// read-only path.
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

// The one-CTA routing of align_kernel (all 1024 threads of the CTA call it).
template <bool COH>
__device__ void align_body(const AlignArgs& a, int32_t* sm) {
  __shared__ int warp_tot[32];
  const int E = a.E;
  int32_t* cnt = sm;                        // [kRouteWarps][E]
  int32_t* base = cnt + kRouteWarps * E;    // [E + 1] padded row offsets
  int32_t* padded = base + E + 1;           // [E]
  int32_t* chbase = padded + E;             // [E + 1] chunk offsets
  int32_t* chbase2 = chbase + E + 1;        // [E + 1] heavy-list chunk offsets (mixed lists)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool mixed = a.heavy_rows > 0;
  if (a.chunk_ready)  // per-chunk counters and the two phase counters after them
    for (int64_t i = tid; i < a.chunks_cap + 2; i += kRouteThreads) a.chunk_ready[i] = 0;
  if (mixed && tid < 2) a.counters2[tid] = 0;

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
  // Mixed lists: heavy experts (more than heavy_rows padded rows) after all
  // the light ones, each group in expert order.
  const bool heavy = mixed && pad > a.heavy_rows;
  int total_rows = 0, total_heavy = 0;
  const int off = block_exclusive_scan(heavy ? 0 : pad, warp_tot, &total_rows);
  const int off_h = mixed ? block_exclusive_scan(heavy ? pad : 0, warp_tot, &total_heavy) : 0;
  const int total_light = total_rows;
  total_rows += total_heavy;
  int nch = 0, nch2 = 0;
  if (tid < E) {
    base[tid] = heavy ? total_light + off_h : off;
    padded[tid] = pad;
    if (heavy) nch2 = (pad + kHeavyTile - 1) / kHeavyTile;
    else if (a.tile_tokens > 0) nch = (pad + a.tile_tokens - 1) / a.tile_tokens;
  }
  int total_chunks = 0, total_chunks2 = 0;
  const int choff = block_exclusive_scan(nch, warp_tot, &total_chunks);
  const int choff2 = mixed ? block_exclusive_scan(nch2, warp_tot, &total_chunks2) : 0;
  if (tid < E) {
    chbase[tid] = choff;
    chbase2[tid] = choff2;
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
  // most tile_tokens rows (multiples of block_m); heavy experts of mixed
  // lists into chunks of at most kHeavyTile rows in the second list.
  if (a.tile_tokens > 0 && tid < E) {
    const int P = padded[tid];
    const bool hv = mixed && P > a.heavy_rows;
    if (P > 0) {
      const int* cb = hv ? chbase2 : chbase;
      int32_t* ce = hv ? a.chunk_expert2 : a.chunk_expert;
      int32_t* cr0 = hv ? a.chunk_row0_2 : a.chunk_row0;
      int32_t* crw = hv ? a.chunk_rows2 : a.chunk_rows;
      const int blocks = P / bm;
      const int nc = cb[tid + 1] - cb[tid];
      const int per = blocks / nc, extra = blocks % nc;
      int row0 = base[tid];
      for (int c = 0; c < nc; ++c) {
        const int rows = (per + (c < extra ? 1 : 0)) * bm;
        ce[cb[tid] + c] = tid;
        cr0[cb[tid] + c] = row0;
        crw[cb[tid] + c] = rows;
        row0 += rows;
      }
    }
  }
}

__global__ void __launch_bounds__(kRouteThreads, 1) align_kernel(const AlignArgs a) {
  extern __shared__ int32_t sm[];
  align_body<false>(a, sm);
}

// Router + routing of small batches in one launch: warp w < tpc of CTA c
// routes token tpc*c + w and stores its ids and weights (a.topk_ids =
// r.out_ids); the last CTA to finish (a counter, left at zero again) routes
// every id as align_kernel does, reading the ids the other CTAs stored
// through L2. Few tokens per CTA (one up to 128 tokens) spread the router's
// per-token work over many SMs.
template <int PER>
__global__ void __launch_bounds__(kRouteThreads, 1) router_align_kernel(const AlignArgs a, const RouterArgs r,
                                                                       int64_t M, int tpc, int32_t* counter) {
  extern __shared__ int32_t sm[];
  __shared__ int last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = (int64_t)blockIdx.x * tpc + warp;
  if (warp < tpc && t < M) {
    int id;
    float w;
    route_token_warp<PER>(r, t, lane, id, w);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
    if (last) {
      atomicExch(counter, 0);
      __threadfence();
    }
  }
  __syncthreads();
  if (!last) return;
  align_body<true>(a, sm);
}

size_t align_smem_bytes(int E) { return (size_t)(kRouteWarps * E + 4 * E + 3) * sizeof(int32_t); }

cudaError_t launch_align(const AlignArgs& a, cudaStream_t stream) {
  const size_t smem = align_smem_bytes(a.E);
  cudaError_t err = cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  align_kernel<<<1, kRouteThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Routing on several CTAs (large batches): the same result as align_kernel.
// CTA c of C owns the flat ids [c*S, (c+1)*S). Launch 1 counts each CTA's ids
// per expert into scratch[c][e]. Launch 2: every CTA derives the per-expert
// totals, its own prefix over lower CTAs and the padded layout from scratch
// (the same scans as align_kernel), counts its segment again per warp and
// scatters it; padding and tail rows get the sentinel, dropped slots
// slot_pos -1. CTA segments, warp segments and lanes are in flat-index order,
// so the order inside an expert is the stable one of the single-CTA kernel.
// ---------------------------------------------------------------------------
int route_ctas(int64_t n) {
  if (n < kRouteMultiMinSlots) return 1;
  const int64_t c = (n + kRouteSlotsPerCta - 1) / kRouteSlotsPerCta;
  return c > kRouteMaxCtas ? kRouteMaxCtas : (int)c;
}

namespace {

// Per-(warp, expert) counts of ids [beg, end) cut into 32 warp segments.
template <bool COH>
__device__ void count_segment(const AlignArgs& a, int64_t beg, int64_t end, int32_t* cnt, bool report) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t seg = (end - beg + kRouteWarps - 1) / kRouteWarps;
  const int64_t wb = beg + warp * seg;
  const int64_t we = wb + seg < end ? wb + seg : end;
  for (int64_t i0 = wb; i0 < we; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < we) ? map_expert(a, load_id<COH>(a, i), report) : -2;
    }
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const unsigned peers = __match_any_sync(0xffffffffu, ev[u]);
      if (ev[u] >= 0 && lane == __ffs(peers) - 1) cnt[warp * a.E + ev[u]] += __popc(peers);
      __syncwarp();
    }
  }
}

// CTA segments of the flat ids, whole tokens each when a.seg_align = topk
// (routing from logits: a CTA routes the tokens whose ids it then counts).
__device__ __forceinline__ void cta_segment(const AlignArgs& a, int64_t& beg, int64_t& end) {
  const int64_t n = a.n;
  const int64_t al = a.seg_align > 1 ? a.seg_align : 1;
  const int64_t S = ((n + gridDim.x - 1) / gridDim.x + al - 1) / al * al;
  beg = (int64_t)blockIdx.x * S < n ? (int64_t)blockIdx.x * S : n;
  end = beg + S < n ? beg + S : n;
}

// ROUTER: the CTA first routes the tokens of its segment (a.seg_align = topk,
// a.topk_ids = r.out_ids) and counts the ids it just stored.
template <bool ROUTER, int PER>
__global__ void __launch_bounds__(kRouteThreads, 1) route_count_kernel(const AlignArgs a, int32_t* scratch,
                                                                      const RouterArgs r) {
  extern __shared__ int32_t sm[];
  const int E = a.E;
  int32_t* cnt = sm;  // [kRouteWarps][E]
  const int tid = threadIdx.x;
  if (a.chunk_ready)
    for (int64_t i = (int64_t)blockIdx.x * kRouteThreads + tid; i < a.chunks_cap + 2;
         i += (int64_t)gridDim.x * kRouteThreads)
      a.chunk_ready[i] = 0;
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) cnt[i] = 0;
  int64_t beg, end;
  cta_segment(a, beg, end);
  if (ROUTER) {
    const int lane = tid & 31;
    for (int64_t t = beg / r.topk + (tid >> 5); t < end / r.topk; t += kRouteWarps) {
      int id;
      float w;
      route_token_warp<PER>(r, t, lane, id, w);
    }
  }
  __syncthreads();
  count_segment<ROUTER>(a, beg, end, cnt, true);
  __syncthreads();
  for (int e = tid; e < E; e += kRouteThreads) {
    int t = 0;
    for (int w = 0; w < kRouteWarps; ++w) t += cnt[w * E + e];
    scratch[(int64_t)blockIdx.x * E + e] = t;
  }
}

__global__ void __launch_bounds__(kRouteThreads, 1) route_scatter_kernel(const AlignArgs a,
                                                                        const int32_t* __restrict__ scratch) {
  extern __shared__ int32_t sm[];
  __shared__ int warp_tot[32];
  const int E = a.E;
  int32_t* cnt = sm;                      // [kRouteWarps][E]
  int32_t* base = cnt + kRouteWarps * E;  // [E + 1]
  int32_t* padded = base + E + 1;         // [E]
  int32_t* chbase = padded + E;           // [E + 1]
  int32_t* pre = chbase + E + 1;          // [E] rows of expert e in lower CTAs
  int32_t* tots = pre + E;                // [E] rows of expert e
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, c = blockIdx.x;
  const int64_t gtid = (int64_t)c * kRouteThreads + tid, gstride = (int64_t)C * kRouteThreads;
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) cnt[i] = 0;
  int tot = 0;
  if (tid < E) {
    int p = 0;
    for (int k = 0; k < C; ++k) {
      const int v = __ldg(&scratch[(int64_t)k * E + tid]);
      if (k < c) p += v;
      tot += v;
    }
    pre[tid] = p;
    tots[tid] = tot;
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
  if (c == 0 && tid == 0) {
    if (overflow) atomicOr(a.err, ERR_DEV_CAPACITY);
    *a.ntp = overflow ? 0 : total_rows;
    if (a.n_chunks) *a.n_chunks = overflow ? 0 : total_chunks;
  }
  if (overflow) {
    for (int64_t i = gtid; i < a.sorted_cap; i += gstride) a.sorted_ids[i] = a.sentinel;
    if (a.slot_pos)
      for (int64_t i = gtid; i < a.n; i += gstride) a.slot_pos[i] = -1;
    if (a.expert_ids)
      for (int64_t b = gtid; b < a.blocks_cap; b += gstride) a.expert_ids[b] = -1;
    return;
  }
  __syncthreads();
  // Sentinels: each expert's padding rows, then the tail past the routed rows
  // (neither overlaps a scattered row).
  for (int64_t g = gtid; g < (int64_t)E * bm; g += gstride) {
    const int e = (int)(g / bm), k = (int)(g - (int64_t)e * bm);
    if (tots[e] + k < padded[e]) a.sorted_ids[base[e] + tots[e] + k] = a.sentinel;
  }
  for (int64_t i = total_rows + gtid; i < a.sorted_cap; i += gstride) a.sorted_ids[i] = a.sentinel;

  int64_t beg, end;
  cta_segment(a, beg, end);
  count_segment<false>(a, beg, end, cnt, false);
  __syncthreads();
  if (tid < E) {
    int t = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int v = cnt[w * E + tid];
      cnt[w * E + tid] = t;
      t += v;
    }
  }
  __syncthreads();

  const unsigned lt_mask = (1u << lane) - 1u;
  const int64_t seg = (end - beg + kRouteWarps - 1) / kRouteWarps;
  const int64_t wb = beg + warp * seg;
  const int64_t we = wb + seg < end ? wb + seg : end;
  for (int64_t i0 = wb; i0 < we; i0 += 32 * kRouteBatch) {
    int ev[kRouteBatch];
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = (i < we) ? map_expert(a, __ldg(&a.topk_ids[i]), false) : -2;
    }
#pragma unroll
    for (int u = 0; u < kRouteBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      const int e = ev[u];
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      int step = 0;
      if (e >= 0) {
        const int rank = __popc(peers & lt_mask);
        const int32_t pos = base[e] + pre[e] + cnt[warp * E + e] + rank;
        a.sorted_ids[pos] = (int32_t)i;
        if (a.slot_pos) a.slot_pos[i] = pos;
        step = __popc(peers);
      } else if (e == -1 && a.slot_pos) {
        a.slot_pos[i] = -1;
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += step;
      __syncwarp();
    }
  }

  if (a.expert_ids != nullptr) {
    for (int64_t b = gtid; b < a.blocks_cap; b += gstride) {
      const int64_t row = b * bm;
      int eid = -1;
      if (row < total_rows) {
        int lo = 0, hi = E - 1;
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

  // Work list: expert e's chunks by CTA e % C.
  if (a.tile_tokens > 0)
    for (int e = tid; e < E; e += kRouteThreads) {
      if (e % C != c) continue;
      const int P = padded[e];
      if (P == 0) continue;
      const int blocks = P / bm;
      const int nc = chbase[e + 1] - chbase[e];
      const int per = blocks / nc, extra = blocks % nc;
      int row0 = base[e];
      for (int k = 0; k < nc; ++k) {
        const int rows = (per + (k < extra ? 1 : 0)) * bm;
        a.chunk_expert[chbase[e] + k] = e;
        a.chunk_row0[chbase[e] + k] = row0;
        a.chunk_rows[chbase[e] + k] = rows;
        row0 += rows;
      }
    }
}

}  // namespace

int64_t route_scratch_ints(int64_t n, int E) {
  const int C = route_ctas(n);
  return C > 1 ? (int64_t)C * E : 0;
}

namespace {

template <bool ROUTER, int PER>
cudaError_t launch_route_multi(const AlignArgs& a, const RouterArgs& r, int C, int32_t* scratch,
                               cudaStream_t stream) {
  const size_t smem1 = (size_t)kRouteWarps * a.E * sizeof(int32_t);
  const size_t smem2 = (size_t)(kRouteWarps * a.E + 5 * a.E + 2) * sizeof(int32_t);
  cudaError_t err = cudaFuncSetAttribute(route_count_kernel<ROUTER, PER>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
  if (err != cudaSuccess) return err;
  route_count_kernel<ROUTER, PER><<<C, kRouteThreads, smem1, stream>>>(a, scratch, r);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  route_scatter_kernel<<<C, kRouteThreads, smem2, stream>>>(a, scratch);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_route(const AlignArgs& a, int32_t* scratch, int64_t scratch_ints, cudaStream_t stream) {
  const int C = route_ctas(a.n);
  // mixed work lists are built by the one-CTA kernel only
  if (C == 1 || a.heavy_rows > 0 || !scratch || scratch_ints < (int64_t)C * a.E) return launch_align(a, stream);
  return launch_route_multi<false, 8>(a, RouterArgs{}, C, scratch, stream);
}

int64_t route_logits_scratch_ints(int64_t n, int E) { return kRouteLogitsCounterInts + route_scratch_ints(n, E); }

cudaError_t launch_route_logits(const AlignArgs& a_in, const RouterArgs& r, int64_t M, int32_t* counter,
                                int32_t* counts, cudaStream_t stream) {
  AlignArgs a = a_in;
  a.topk_ids = r.out_ids;
  a.seg_align = r.topk;
  const int C = route_ctas(a.n);
  const int per = router_per_lane(r.E);
  if (C > 1 && a.heavy_rows == 0) {
    if (per == 8) return launch_route_multi<true, 8>(a, r, C, counts, stream);
    if (per == 16) return launch_route_multi<true, 16>(a, r, C, counts, stream);
    return launch_route_multi<true, 32>(a, r, C, counts, stream);
  }
  const size_t smem = align_smem_bytes(a.E);
  // tokens per CTA: one up to 128 tokens, then as many as keep 128 CTAs (at most 32)
  int tpc = M <= 128 ? 1 : (int)((M + 127) / 128);
  if (tpc > kRouteWarps) tpc = kRouteWarps;
  const int64_t ctas = M > 0 ? (M + tpc - 1) / tpc : 1;
  auto kernel = per == 8 ? router_align_kernel<8> : (per == 16 ? router_align_kernel<16> : router_align_kernel<32>);
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  kernel<<<(unsigned)ctas, kRouteThreads, smem, stream>>>(a, r, M, tpc, counter);
  return cudaGetLastError();
}

}  // namespace b200moe
