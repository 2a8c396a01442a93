// Routing: moe_align_block_size with a stable within-expert order, plus the
// grouped-GEMM work list (chunks). The one-CTA body (align.cuh) runs on one
// CTA of 1024 threads below 16,384 routed slots; larger batches use the
// count / scatter kernels below on several CTAs (same result, bit for bit).
#include "align.cuh"
#include "common.cuh"
#include "ep_wait.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "router.cuh"

namespace b200moe {

constexpr int kRouteWarps = 32;
constexpr int kRouteThreads = kRouteWarps * 32;
constexpr int64_t kRouteMultiMinSlots = 16384;  // flat slots from which routing uses several CTAs
constexpr int64_t kRouteSlotsPerCta = 2048;
constexpr int kRouteMaxCtas = 128;

__global__ void __launch_bounds__(kRouteThreads, 1) align_kernel(const AlignArgs a) {
  extern __shared__ int32_t sm[];
  griddep_launch_dependents();  // the gather may start launching (it waits for this grid)
  align_body<false, kRouteThreads>(a, sm);
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
  griddep_launch_dependents();  // the gather may start launching (it waits for this grid)
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
  align_body<true, kRouteThreads>(a, sm);
}

// Expert-parallel layer: waits for the G dispatch flags, unpacks the received
// rows' ids and weights (as ep_unpack_meta_peer_kernel), then routes them as
// align_kernel does (reading the ids just stored through L2).
__global__ void __launch_bounds__(kRouteThreads, 1) unpack_align_kernel(const AlignArgs a, const PackedMeta pm) {
  extern __shared__ int32_t sm[];
  griddep_launch_dependents();  // the gather may start launching (it waits for this grid)
  wait_flags(reinterpret_cast<const int32_t*>(pm.own + EpPeerLayout::kDispatchFlags), pm.G, pm.epoch, a.err,
             pm.limit_ns);
  const int64_t n = pm.R * pm.topk;
  for (int64_t i = threadIdx.x; i < n; i += kRouteThreads) {
    const int64_t r = i / pm.topk;
    const int j = (int)(i - r * pm.topk);
    const int32_t* src = reinterpret_cast<const int32_t*>(pm.rows + r * pm.row_bytes + pm.H + (pm.H / 128) * 4);
    pm.ids[i] = __ldcg(&src[j]);  // stored by other GPUs during the wait: read through L2
    pm.w[i] = __ldcg(reinterpret_cast<const float*>(src + pm.topk) + j);
  }
  __syncthreads();
  align_body<true, kRouteThreads>(a, sm);
}

size_t align_smem_bytes(int E) { return (size_t)align_smem_ints(E, kRouteWarps) * sizeof(int32_t); }

cudaError_t launch_align_packed(const AlignArgs& a, const PackedMeta& pm, cudaStream_t stream) {
  const size_t smem = align_smem_bytes(a.E);
  cudaError_t err = cudaFuncSetAttribute(unpack_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  unpack_align_kernel<<<1, kRouteThreads, smem, stream>>>(a, pm);
  return cudaGetLastError();
}

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
  griddep_launch_dependents();  // the gather may start launching (it waits for this grid)
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
  const int off = block_exclusive_scan<kRouteThreads>(pad, warp_tot, &total_rows);
  int nch = 0;
  if (tid < E) {
    base[tid] = off;
    padded[tid] = pad;
    if (a.tile_tokens > 0) nch = (pad + a.tile_tokens - 1) / a.tile_tokens;
  }
  int total_chunks = 0;
  const int choff = block_exclusive_scan<kRouteThreads>(nch, warp_tot, &total_chunks);
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
