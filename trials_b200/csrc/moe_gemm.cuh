// Persistent FP8 block-scaled grouped GEMM for the two MoE stages (sm_100a).
//
// Math (both stages), for one expert e and the rows p of the expert-sorted
// activation matrix A that were routed to e:
//   C[p, n] = sum_kb  w_s[e, n/128, kb] * a_s[p, kb] * sum_{k in kb} W[e, n, k] * A[p, k]
// which is the block-scaled dequant order of the reference Triton kernel
// (aiter_module/moe_decode_megakernel.py:71-81: acc += dot(a, b) * a_s * b_s per
// 128-wide K block).
//
// Orientation ("swap-AB"): the tensor-core MMA M side is 128 weight rows (N of
// the layer), the MMA N side is the expert's routed tokens (16..T columns).
// At decode an expert sees a handful of tokens, so the weight tile fills the
// 128-row MMA and the token count only sets the (cheap) N width.
//
// One work unit = (token chunk of one expert, 256 consecutive weight rows).
// Per 128-wide K block the MMA warp issues 4 (K=32) x 2 (two 128-row halves)
// tcgen05.mma into a fresh TMEM buffer; the epilogue warps read that partial
// sum back with tcgen05.ld, multiply by the two block scales and accumulate in
// fp32 registers ("promotion" - the fp32 128x128 scales are not MX scales, so
// the tensor core cannot apply them). TMEM holds NBUF partial buffers so the
// MMA of block kb+1.. overlaps the promotion of block kb.
//
// Warp roles: warp 0 = TMA producer, warp 1 = MMA issuer (+ TMEM owner),
// warps 2.. = epilogue: 8 * CS warps, one per (TMEM lane quarter w%4, 128-row
// half, token-column slice of T/CS columns); warp w reads TMEM lanes
// 32*(w%4)..+31.
//
// Epilogues:
//   EPI_SILU    (stage 1, gate/up interleaved rows): inter = silu(gate) * up in
//               fp32, then 1x128 FP8 re-quantisation of inter (amax/448 scale)
//               straight into the stage-2 activation buffer (sorted row order).
//   EPI_COMBINE (stage 2): out_pair[f, n] = topk_w[f] * C[p, n] for the flat
//               (token, slot) id f = sorted_ids[p]; padding rows are skipped.
#pragma once

#include <cuda_fp8.h>

#include "align.cuh"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "router.cuh"
#include "rowops.cuh"

// Weight tiles stream once per launch. An evict_first L2 hint on them measured
// slower than no hint on a pure TMA read stream (6.9 vs 7.0 TB/s) and no faster
// in this kernel, so it is off unless this is set to 1 - except in the
// whole-layer launch (EPI_WHOLE), whose routing and gather phases run on code
// and rows that the previous call's weight stream would otherwise have evicted
// from L2 (measured: one token, 114 -> 91 us per layer).
#ifndef B200MOE_W_EVICT_FIRST
#define B200MOE_W_EVICT_FIRST 0
#endif
// K blocks the epilogue promotes per round when a thread holds 32 token
// columns: the TMEM loads of a round share one wait, and the barrier waits and
// releases of a round follow each other, so the epilogue's fixed latency per
// K block shrinks by this factor.
#ifndef B200MOE_EPI_KR
#define B200MOE_EPI_KR 2
#endif

// SiLU with the fast (2 ulp) division; 0 selects IEEE division.
#ifndef B200MOE_FAST_SILU
#define B200MOE_FAST_SILU 1
#endif

namespace b200moe {

// EPI_LAYER: EPI_FUSED plus the in-launch phases (gather + quantise first,
// top-k reduce last) set up in GemmParams.q0 / red_*. EPI_WHOLE: EPI_LAYER
// with the routing (and optionally the router) at the start of the launch.
enum { EPI_SILU = 0, EPI_COMBINE = 1, EPI_FUSED = 2, EPI_LAYER = 3, EPI_WHOLE = 4 };

struct GemmParams {
  // routing: chunk list produced by the route kernel (device memory)
  const int32_t* chunk_expert;
  const int32_t* chunk_row0;
  const int32_t* chunk_rows;
  const int32_t* n_chunks;
  // weight block scales (E, Nw/128, K/128) contiguous
  const float* w_scale;
  // activation scales, transposed: a_sT[kb * as_ld + p]
  const float* a_sT;
  int64_t as_ld;
  int K;        // reduction width (bytes of fp8)
  int Nw;       // weight rows per expert
  // EPI_SILU outputs: q rows p (width Nw/2), scales transposed (Nw/256 x as_ld)
  uint8_t* out_q;
  int64_t out_q_ld;
  float* out_sT;
  int64_t out_s_ld;
  // EPI_COMBINE
  const int32_t* sorted_ids;
  const float* topk_w;
  int32_t sentinel;   // M * topk
  // bf16 rows of Nw (router weight applied): row f = slot (tiles <= 64) or
  // sorted row p (tiles >= 128, unless rows_by_slot)
  __nv_bfloat16* out_pair;
  int rows_by_slot;   // token-major stage 2: write row f (slot) instead of sorted row p
  // EPI_FUSED: per-chunk count of finished stage-1 units (zeroed by routing),
  // followed by two phase counters (CTAs done with phase 0 / with all units)
  int32_t* chunk_ready;
  int32_t* phase_count;
  // EPI_FUSED, small batches: activation gather + quantisation as phase 0 of
  // the launch (q0.rows > 0, slot mode) and the top-k reduce as its last phase
  // (red_out != nullptr; stage-2 rows by slot, red_slot_pos from routing).
  QuantArgs q0;
  const int32_t* red_slot_pos;
  __nv_bfloat16* red_out;
  int64_t red_M;
  int red_topk;
  // unit order: chunks per group (see unit_coords); 1 = chunk-major
  int chunk_group;
  // token-major kernels: a zeroed counter from which CTAs take their next unit
  // (dynamic queue); nullptr = static round-robin over the grid
  int32_t* unit_counter;
  // EPI_WHOLE: the one-CTA routing run inside the launch (ra), after the
  // router top-k of every token (rr, when router != 0; ra.topk_ids =
  // rr.out_ids); route_sync: 3 ints that are zero between launches (router
  // CTA counter, routing done, CTAs past the routing wait).
  AlignArgs ra;
  RouterArgs rr;
  int router;
  int32_t* route_sync;
  // diagnostics
  int32_t* err;
  uint64_t timeout_ns;
};

template <int T_, int CS_>
struct GemmCfg {
  static constexpr int T = T_;                 // max tokens (MMA N) per unit
  static constexpr int CS = CS_;               // token-column slices of the epilogue
  static constexpr int NSUB = 2;               // 128-row halves per unit
  static constexpr int EW = 4 * NSUB * CS;     // epilogue warps
  static constexpr int UNIT_ROWS = 128 * NSUB; // weight rows per unit
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr int TC = T / CS;            // token columns per epilogue thread
  static constexpr int KR = (TC <= 32 && CS == 1) ? B200MOE_EPI_KR : 1;  // K blocks per epilogue round
  static constexpr int W_BYTES = UNIT_ROWS * 128;
  static constexpr int A_BYTES = T * 128;
  static constexpr int TILE_BYTES = W_BYTES + A_BYTES;  // multiple of 1024
  static constexpr int S_BYTES = T * 4;                 // activation scales of one K block
  static constexpr int NBUF = 512 / (NSUB * T);         // TMEM partial buffers
  static constexpr int TMEM_COLS = 512;
  static constexpr int STAGING = T * 128;               // EPI_SILU output tile
  static constexpr int RED = 4 * NSUB * T * 4;          // EPI_SILU amax exchange (per warp, per column)
  static constexpr int SMEM_LIMIT = 232448;
  static constexpr int MAX_STAGE = 8;
  // Scale ring: the producer can run at most NSTAGE K blocks ahead of the MMA,
  // which runs at most NBUF ahead of the epilogue, so NSTAGE + NBUF slots never
  // make the producer wait on the epilogue.
  static constexpr int FIXED = 1024 /*align slack*/ + STAGING + RED + (MAX_STAGE + NBUF) * S_BYTES +
                               1024 /*barriers etc*/;
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - FIXED) / TILE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > MAX_STAGE ? MAX_STAGE : NSTAGE_RAW;
  static constexpr int NSLOT = NSTAGE + NBUF;
  static constexpr int SMEM_BYTES = FIXED + NSTAGE * TILE_BYTES;
  static_assert(T % 16 == 0 && T >= 16 && T <= 256, "MMA N must be a multiple of 16 in [16, 256]");
  static_assert(TC % 32 == 0, "columns per epilogue thread must be a multiple of 32");
  static_assert(NBUF >= 2, "need at least two TMEM buffers");
  static_assert(KR >= 1 && 2 * KR <= NBUF, "epilogue round must leave the MMA TMEM buffers to fill");
  static_assert(NSTAGE >= 2, "shared memory too small");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
};

__device__ __forceinline__ float silu_f32(float g) {
#if B200MOE_FAST_SILU
  // __fdividef is accurate to 2 ulp for divisors below 2^126; above that
  // (g < -87) silu(g) rounds to -0 anyway.
  const float d = 1.0f + __expf(-g);
  return d < 1e30f ? __fdividef(g, d) : -0.0f;
#else
  return g / (1.0f + __expf(-g));
#endif
}

// Column maxima for values spread over lane pairs: lane l holds, for m < 16,
// |value| of column 2m + (l & 1). Returns, in lane l, the max over the 16
// lanes of l's parity for column l. Butterfly over lane bits 4..1 that halves
// the values each lane keeps per step (15 shuffles).
__device__ __forceinline__ float warp_pair_transpose_max(const float* vals, int lane) {
  float m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = fabsf(vals[i]);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool hi = (lane & (2 * o)) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = hi ? m[i] : m[i + o];
      const float recv = __shfl_xor_sync(0xffffffffu, send, 2 * o);
      m[i] = fmaxf(hi ? m[i + o] : m[i], recv);
    }
  }
  return m[0];
}

// Acquire load of a counter another CTA releases.
__device__ __forceinline__ int ld_acquire_gpu(const int32_t* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

// Routing metadata (chunk lists, sorted ids, router weights): read-only for
// the launch unless the launch wrote it itself (EPI_WHOLE), then through L2.
template <bool COH>
__device__ __forceinline__ int32_t ld_meta(const int32_t* ptr) {
  return COH ? __ldcg(ptr) : __ldg(ptr);
}
template <bool COH>
__device__ __forceinline__ float ld_meta(const float* ptr) {
  return COH ? __ldcg(ptr) : __ldg(ptr);
}

// Waits until *counter >= target (bounded like every wait in this library);
// then orders the following async-proxy (TMA) reads after the acquire.
__device__ __forceinline__ bool wait_count_bounded(const int32_t* counter, int target, uint64_t limit_ns,
                                                   volatile int* abort_flag) {
  bool ok = ld_acquire_gpu(counter) >= target;
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    while (!ok) {
      __nanosleep(128);
      ok = ld_acquire_gpu(counter) >= target;
      if (!ok && (*abort_flag || globaltimer_ns() - t0 > limit_ns)) return false;
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// mbarrier wait that gives up after limit_ns or once the CTA's abort flag is set.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                                   volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (*abort_flag || globaltimer_ns() - t0 > limit_ns) return false;
  return true;
}

// EPI_WHOLE, first phase (every thread of every CTA). With a router, token t
// is routed by warp t / G of CTA t % G (G CTAs) and the last CTA to finish its
// tokens (counter sync[0]) runs the routing; without, CTA 0 does. The routing
// CTA releases sync[1] = 1 and the others wait for it (bounded). Every CTA then
// counts itself past (sync[2]); the last one clears sync[1..2] (every CTA is
// past the wait by then), so the words are zero again for the next launch.
// sm: shared memory for align_body. Returns false after a timeout.
template <int NTHR>
__device__ bool route_phase(const GemmParams& p, int32_t* sm, volatile int* abort_flag, volatile int* flag_sh) {
  constexpr int NW = NTHR / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* sync = p.route_sync;
  bool aligner = blockIdx.x == 0;
  if (p.router) {
    const int64_t M = p.ra.n / p.rr.topk;
    const int per = router_per_lane(p.rr.E);
    for (int64_t t = blockIdx.x + (int64_t)gridDim.x * warp; t < M; t += (int64_t)gridDim.x * NW) {
      int id;
      float w;
      if (per == 8) route_token_warp<8>(p.rr, t, lane, id, w);
      else if (per == 16) route_token_warp<16>(p.rr, t, lane, id, w);
      else route_token_warp<32>(p.rr, t, lane, id, w);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const bool last = atomicAdd(&sync[0], 1) == (int)gridDim.x - 1;
      if (last) {
        sync[0] = 0;
        __threadfence();
      }
      *flag_sh = last ? 1 : 0;
    }
    __syncthreads();
    aligner = *flag_sh != 0;
  }
  if (aligner) {
    if (p.router) align_body<true, NTHR>(p.ra, sm);
    else align_body<false, NTHR>(p.ra, sm);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(&sync[1]), "r"(1) : "memory");
    }
  } else if (threadIdx.x == 0) {
    if (!wait_count_bounded(&sync[1], 1, p.timeout_ns, abort_flag)) {
      atomicOr(p.err, ERR_DEV_TIMEOUT);
      *abort_flag = 1;
    }
  }
  if (threadIdx.x == 0 && atomicAdd(&sync[2], 1) == (int)gridDim.x - 1) {
    sync[1] = 0;
    sync[2] = 0;
  }
  // The routing's shared memory becomes the TMA ring: order its generic
  // writes before the async-proxy writes and reads that follow.
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  return *abort_flag == 0;
}

// The kernel runs one stage (EPI_SILU / EPI_COMBINE: parameters p, tensor
// maps tm_w / tm_a; the *2 copies are unused) or both (EPI_FUSED): units
// [0, n1) are stage-1 units with p, units [n1, n1 + n2) stage-2 units with
// p2, in one persistent grid. A stage-2 unit of chunk c reads the stage-1
// output rows of c, so its producer first waits until all NT1 stage-1 units
// of c have released p.chunk_ready[c]. Every CTA finishes issuing its stage-1
// units before it waits on any chunk, and the grid is co-resident (one CTA
// per SM, cooperative launch), so the waits always end. The count is released
// by an extra "publisher" warp: the epilogue warps hand it each finished
// stage-1 unit through an mbarrier, and its GPU-scope fence (which waits for
// the stores to land) stays off the epilogue's path.
template <int T, int CS, int EPI>
__global__ void __launch_bounds__(GemmCfg<T, CS>::THREADS + (EPI >= EPI_FUSED ? 32 : 0), 1)
    moe_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                            const __grid_constant__ GemmParams p, const __grid_constant__ CUtensorMap tm_w2,
                            const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ GemmParams p2) {
  using C = GemmCfg<T, CS>;
  constexpr int EW = C::EW;
  constexpr bool FUSED = EPI >= EPI_FUSED;
  constexpr bool PHASES = EPI >= EPI_LAYER;
  constexpr bool ROUTE = EPI == EPI_WHOLE;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled TMA tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;                                             // NSTAGE * TILE_BYTES
  float* sscale = reinterpret_cast<float*>(tiles + C::NSTAGE * C::TILE_BYTES);  // NSLOT * T
  uint8_t* staging = reinterpret_cast<uint8_t*>(sscale + C::NSLOT * T);       // T * 128
  float* red = reinterpret_cast<float*>(staging + C::STAGING);                // 4 * COL_SPLIT * T
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + C::RED);
  uint64_t* empty = full + C::NSTAGE;
  uint64_t* tfull = empty + C::NSTAGE;
  uint64_t* tempty = tfull + C::NBUF;
  uint64_t* sfull = tempty + C::NBUF;
  uint64_t* sempty = sfull + C::NSLOT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty + C::NSLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // The epilogue's stop decision for a unit, written by one thread before the
  // unit's first named barrier so that every epilogue warp reads the same value.
  volatile int* stop_sh = reinterpret_cast<volatile int*>(tmem_slot + 2);
  // EPI_FUSED hand-off of finished stage-1 units to the publisher warp:
  // pub[0..1] filled by the epilogue warps, pub[2..3] released by the publisher.
  uint64_t* pub = reinterpret_cast<uint64_t*>(tmem_slot + 4);
  // EPI_WHOLE: which CTA routes (broadcast from thread 0).
  volatile int* route_sh = reinterpret_cast<volatile int*>(tmem_slot + 3);
  // EPI_FUSED: units come from a counter (p.unit_counter, zeroed by routing)
  // in the order CTAs become free for them; the producer hands each one with
  // its chunk metadata {unit, expert, first row, rows} to the MMA thread and
  // the epilogue warps through a ring of kUnitRing slots (-1: no more units),
  // and the epilogue hands the chunk of each finished stage-1 unit to the
  // publisher in pub_chunk (-1: no more).
  constexpr bool DYN = EPI == EPI_FUSED;
  constexpr int kUnitRing = 4;
  uint64_t* ufull = pub + 4;
  uint64_t* uempty = ufull + kUnitRing;
  int4* uring = reinterpret_cast<int4*>(uempty + kUnitRing);
  volatile int* pub_chunk = reinterpret_cast<volatile int*>(uring + kUnitRing);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NT1 = p.Nw / C::UNIT_ROWS, NKB1 = p.K >> 7;
  const int NT2 = FUSED ? p2.Nw / C::UNIT_ROWS : 1, NKB2 = FUSED ? p2.K >> 7 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // released by the MMA commit
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EW);
    }
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], EW);  // released by every epilogue warp
    }
    *abort_flag = 0;
    if (FUSED) {
      mbar_init(&pub[0], EW);
      mbar_init(&pub[1], EW);
      mbar_init(&pub[2], 1);
      mbar_init(&pub[3], 1);
    }
    if (DYN)
      for (int s = 0; s < kUnitRing; ++s) {
        mbar_init(&ufull[s], 1);
        mbar_init(&uempty[s], 1 + EW);  // the MMA thread and every epilogue warp
      }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_a);
    if (FUSED) {
      prefetch_tmap(&tm_w2);
      prefetch_tmap(&tm_a2);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched programmatically after the gather: everything above overlapped
  // its end; nothing below may read its rows (or the routing) before this.
  griddep_wait();

  int n_chunks;
  if constexpr (ROUTE) {
    // The routing writes the work list the rest of the launch reads; the
    // tile ring is free until the producer starts.
    static_assert(align_smem_ints(1024, (C::THREADS + 32) / 32) * 4 <= C::NSTAGE * C::TILE_BYTES,
                  "routing shared memory");
    const bool routed = route_phase<C::THREADS + 32>(p, reinterpret_cast<int32_t*>(tiles), abort_flag, route_sh);
    n_chunks = routed ? __ldcg(p.n_chunks) : 0;
  } else {
    n_chunks = *p.n_chunks;
  }
  const int n1 = n_chunks * NT1;
  const int n_units = n1 + (FUSED ? n_chunks * NT2 : 0);
  // unit -> (stage 2?, chunk, weight-row tile)
  auto unit_of = [&](int u, bool& s2, int& chunk, int& nt) {
    s2 = FUSED && u >= n1;
    unit_coords(s2 ? u - n1 : u, n_chunks, s2 ? NT2 : NT1, p.chunk_group, chunk, nt);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      (void)pol_w;
      int stage = 0, slot = 0;
      uint32_t phase = 0, sphase = 0;
      long issued = 0;
      bool ok = true;
      // Chunk metadata is loaded one unit ahead, off the critical path.
      int e_n = 0, p0_n = 0;
      auto meta = [&](int u) {
        bool s2;
        int c, nt;
        unit_of(u, s2, c, nt);
        e_n = ld_meta<ROUTE>(&p.chunk_expert[c]);
        p0_n = ld_meta<ROUTE>(&p.chunk_row0[c]);
      };
      if (!DYN && blockIdx.x < n_units) meta(blockIdx.x);
      // With phase 0 in the launch (EPI_FUSED, q0.rows > 0) the stage-1
      // activation rows are written by the epilogue warps of every CTA first:
      // until all CTAs are done, stage-1 tiles get only their weight half, and
      // the activation halves and scales of up to NSTAGE stages wait here.
      bool a_ready = !PHASES;
      int np = 0;
      int pst[C::NSTAGE], psl[C::NSTAGE], pkb[C::NSTAGE], pp0[C::NSTAGE];
      auto flush = [&]() -> bool {
        const bool got = wait_count_bounded(p.phase_count, (int)gridDim.x, p.timeout_ns, abort_flag);
        // Issued even after a timeout, so that every barrier they feed completes
        // (the error word then marks the results).
        for (int i = 0; i < np; ++i) {
          tma_load_2d(tiles + pst[i] * C::TILE_BYTES + C::W_BYTES, &tm_a, &full[pst[i]], pkb[i] * 128, pp0[i],
                      pol_a);
          mbar_arrive_expect_tx(&sfull[psl[i]], C::S_BYTES);
          bulk_load(sscale + psl[i] * T, p.a_sT + (int64_t)pkb[i] * p.as_ld + pp0[i], C::S_BYTES, &sfull[psl[i]]);
        }
        np = 0;
        a_ready = true;
        return got;
      };
      int uslot = 0;
      uint32_t uphase = 0;
      for (int k = 0, u = blockIdx.x; ok; ++k) {
        bool s2 = false;
        int chunk = 0, nt = 0, e = 0, p0 = 0;
        if (DYN) {
          // take the next unit (round-robin without a counter) and hand it
          // on with its metadata
          u = p.unit_counter ? atomicAdd(p.unit_counter, 1) : (int)blockIdx.x + k * (int)gridDim.x;
          if (u >= n_units) u = -1;
          int rows = 0;
          if (u >= 0) {
            unit_of(u, s2, chunk, nt);
            e = __ldg(&p.chunk_expert[chunk]);
            p0 = __ldg(&p.chunk_row0[chunk]);
            rows = __ldg(&p.chunk_rows[chunk]);
          }
          if (*abort_flag || !mbar_wait_bounded(&uempty[uslot], uphase ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          uring[uslot] = make_int4(u, e, p0, rows);
          mbar_arrive(&ufull[uslot]);
          if (++uslot == kUnitRing) {
            uslot = 0;
            uphase ^= 1;
          }
          if (u < 0) break;
        } else {
          if (k > 0) u += gridDim.x;
          if (u >= n_units) break;
          unit_of(u, s2, chunk, nt);
          e = e_n;
          p0 = p0_n;
          if (u + (int)gridDim.x < n_units) meta(u + gridDim.x);
        }
        const GemmParams& q = s2 ? p2 : p;
        const CUtensorMap* tw = s2 ? &tm_w2 : &tm_w;
        const CUtensorMap* ta = s2 ? &tm_a2 : &tm_a;
        const int NKB = s2 ? NKB2 : NKB1;
        const int wrow = e * q.Nw + nt * C::UNIT_ROWS;
        if (FUSED && s2 && !a_ready && !flush()) {
          ok = false;
          break;
        }
        if (FUSED && s2 && !wait_count_bounded(p.chunk_ready + chunk, NT1, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        for (int kb = 0; kb < NKB; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns) ||
              !mbar_wait_bounded(&sempty[slot], sphase ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* tile = tiles + stage * C::TILE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::TILE_BYTES);
          if (B200MOE_W_EVICT_FIRST || ROUTE)
            tma_load_2d(tile, tw, &full[stage], kb * 128, wrow, pol_w);
          else
            tma_load_2d(tile, tw, &full[stage], kb * 128, wrow);
          if (a_ready) {
            tma_load_2d(tile + C::W_BYTES, ta, &full[stage], kb * 128, p0, pol_a);
            mbar_arrive_expect_tx(&sfull[slot], C::S_BYTES);
            bulk_load(sscale + slot * T, q.a_sT + (int64_t)kb * q.as_ld + p0, C::S_BYTES, &sfull[slot]);
          } else {
            pst[np] = stage;
            psl[np] = slot;
            pkb[np] = kb;
            pp0[np] = p0;
            ++np;
          }
          ++issued;
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1;
          }
          if (++slot == C::NSLOT) {
            slot = 0;
            sphase ^= 1;
          }
          if (np == C::NSTAGE && !flush()) {
            ok = false;
            break;
          }
        }
      }
      if (np > 0 && !flush()) ok = false;
      if (!ok) {
        atomicOr(p.err, ERR_DEV_TIMEOUT);
        *abort_flag = 1;
        // Let every copy already issued land before the CTA exits.
        long first = issued > C::NSTAGE ? issued - C::NSTAGE : 0;
        for (long g = first; g < issued; ++g)
          mbar_wait_bounded(&full[g % C::NSTAGE], (uint32_t)((g / C::NSTAGE) & 1), p.timeout_ns);
        first = issued > C::NSLOT ? issued - C::NSLOT : 0;
        for (long g = first; g < issued; ++g)
          mbar_wait_bounded(&sfull[g % C::NSLOT], (uint32_t)((g / C::NSLOT) & 1), p.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, buf = 0;
      uint32_t phase = 0, bphase = 0;
      long committed = 0;
      int last_buf = 0;
      uint32_t last_bphase = 0;
      bool ok = true;
      auto rows_of = [&](int u) {
        bool s2;
        int c, nt;
        unit_of(u, s2, c, nt);
        return ld_meta<ROUTE>(&p.chunk_rows[c]);
      };
      int rows_n = !DYN && blockIdx.x < n_units ? rows_of(blockIdx.x) : 0;
      int uslot = 0;
      uint32_t uphase = 0;
      for (int k = 0, u = blockIdx.x; ok; ++k) {
        int rows;
        if (DYN) {
          if (!mbar_wait_or_abort(&ufull[uslot], uphase, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          const int4 ent = uring[uslot];
          mbar_arrive(&uempty[uslot]);
          if (++uslot == kUnitRing) {
            uslot = 0;
            uphase ^= 1;
          }
          u = ent.x;
          rows = ent.w;
          if (u < 0) break;
        } else {
          if (k > 0) u += gridDim.x;
          if (u >= n_units) break;
          rows = rows_n;
          if (u + (int)gridDim.x < n_units) rows_n = rows_of(u + gridDim.x);
        }
        const int NKB = (FUSED && u >= n1) ? NKB2 : NKB1;
        const uint32_t idesc = idesc_e4m3_f32(128, rows);
        for (int kb = 0; kb < NKB; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&tempty[buf], bphase ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (*abort_flag || !mbar_wait_bounded(&full[stage], phase, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(tiles + stage * C::TILE_BYTES);
          const uint32_t a_addr = w_addr + C::W_BYTES;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int s = 0; s < C::NSUB; ++s) {
              const uint32_t d = tmem_base + (uint32_t)(buf * C::NSUB * T + s * T);
              umma_f8(d, sdesc_kmajor_sw128(w_addr + s * 16384 + ks * 32), sdesc_kmajor_sw128(a_addr + ks * 32),
                      idesc, ks > 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty[stage]);
          umma_commit(&tfull[buf]);
          ++committed;
          last_buf = buf;
          last_bphase = bphase;
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1;
          }
          if (++buf == C::NBUF) {
            buf = 0;
            bphase ^= 1;
          }
        }
      }
      if (!ok) {
        atomicOr(p.err, ERR_DEV_TIMEOUT);
        *abort_flag = 1;
      }
      // The tensor core must be done with TMEM before it is released.
      if (committed > 0) mbar_wait_bounded(&tfull[last_buf], last_bphase, p.timeout_ns);
    }
  } else if (warp < 2 + EW) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;                 // 0..EW-1
    const int q = warp & 3;                  // TMEM lane quarter
    const int hs = (ew >> 2) & 1;            // 128-row half of the unit
    const int col0 = (ew >> 3) * C::TC;      // first token column of this warp
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int slot = 0, buf = 0;
    uint32_t sphase = 0, bphase = 0;
    bool ok = true;
    // Chunk metadata is loaded one unit ahead, and the unit's weight block
    // scales (one per K block of this 128-row half) are spread over the lanes
    // (K blocks lane and lane + 32) and loaded before the previous unit's
    // final epilogue, so no global load sits on the per-K-block path.
    auto ws_row = [&](bool s2, int e, int nt) {
      const GemmParams& g = s2 ? p2 : p;
      return g.w_scale + ((int64_t)e * (g.Nw >> 7) + nt * 2 + hs) * (g.K >> 7);
    };
    int e_n = 0, p0_n = 0, rows_n = 0;
    float wl0 = 0.f, wl1 = 0.f;
    auto load_ws = [&](bool s2, int e, int nt) {
      const float* w = ws_row(s2, e, nt);
      const int nkb = s2 ? NKB2 : NKB1;
      wl0 = lane < nkb ? __ldg(w + lane) : 0.f;
      wl1 = lane + 32 < nkb ? __ldg(w + lane + 32) : 0.f;
    };
    int n_pub = 0;  // stage-1 units handed to the publisher (EPI_FUSED)
    const int tid = threadIdx.x - 64;  // 0 .. EW*32-1
    if (PHASES) {
      // Phase 0: gather + quantise the routed rows (one warp per routed slot
      // and 1024-column segment, strided over every epilogue warp of the
      // grid), then count this CTA done. The producer's first activation loads
      // wait for every CTA; its weight loads are already in flight.
      const int nseg = (int)((p.q0.K + kQuantSegCols - 1) / kQuantSegCols);
      const int64_t ntask = p.q0.rows * nseg;
      for (int64_t t = (int64_t)blockIdx.x * EW + ew; t < ntask; t += (int64_t)gridDim.x * EW)
        quant_row_segment(p.q0, t / nseg, (t % nseg) * kQuantSegCols, lane);
      named_bar_sync(1, EW * 32);
      if (tid == 0) {
        __threadfence();
        atomicAdd(p.phase_count, 1);
      }
    }
    // EPI_FUSED: the next ring entry ({-1}: none left, {-2}: the wait ended
    // without one). Every epilogue warp reads every entry.
    int uslot = 0;
    uint32_t uphase = 0;
    auto take = [&]() -> int4 {
      if (!mbar_wait_or_abort(&ufull[uslot], uphase, p.timeout_ns, abort_flag)) return make_int4(-2, 0, 0, 0);
      const int4 v = uring[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty[uslot]);
      if (++uslot == kUnitRing) {
        uslot = 0;
        uphase ^= 1;
      }
      return v;
    };
    int4 nxt = make_int4(-1, 0, 0, 0);
    if (DYN) {
      nxt = take();
      if (nxt.x >= 0) {
        bool s2;
        int c, nt;
        unit_of(nxt.x, s2, c, nt);
        load_ws(s2, nxt.y, nt);
      }
    } else if (blockIdx.x < n_units) {
      bool s2;
      int c, nt;
      unit_of(blockIdx.x, s2, c, nt);
      e_n = ld_meta<ROUTE>(&p.chunk_expert[c]);
      p0_n = ld_meta<ROUTE>(&p.chunk_row0[c]);
      rows_n = ld_meta<ROUTE>(&p.chunk_rows[c]);
      load_ws(s2, e_n, nt);
    }
    for (int k = 0, u = blockIdx.x;; ++k) {
      int e, p0, rows;
      if (DYN) {
        u = nxt.x;
        if (u < 0) {
          if (u == -2 && !*abort_flag) {
            atomicOr(p.err, ERR_DEV_TIMEOUT);
            *abort_flag = 1;
          }
          break;
        }
        e = nxt.y;
        p0 = nxt.z;
        rows = nxt.w;
      } else {
        if (k > 0) u += gridDim.x;
        if (u >= n_units) break;
        e = e_n;
        p0 = p0_n;
        rows = rows_n;
      }
      bool s2;
      int chunk, nt;
      unit_of(u, s2, chunk, nt);
      const int NKB = s2 ? NKB2 : NKB1;
      const float ws0 = wl0, ws1 = wl1;
      const float* wsp = ws_row(s2, e, nt);
      const int un = DYN ? -1 : u + (int)gridDim.x;
      bool s2n = false;
      int cn = 0, ntn = 0;
      if (!DYN && un < n_units) {
        unit_of(un, s2n, cn, ntn);
        e_n = ld_meta<ROUTE>(&p.chunk_expert[cn]);
        p0_n = ld_meta<ROUTE>(&p.chunk_row0[cn]);
        rows_n = ld_meta<ROUTE>(&p.chunk_rows[cn]);
      }

      float acc[C::TC];
#pragma unroll
      for (int j = 0; j < C::TC; ++j) acc[j] = 0.f;

      constexpr int KR = C::KR;
      for (int kb = 0; kb < NKB && ok; kb += KR) {
        const int nr = NKB - kb < KR ? NKB - kb : KR;
        float wsr[KR];
        int bufr[KR], slotr[KR];
        bool good = *abort_flag == 0;
#pragma unroll
        for (int r = 0; r < KR; ++r) {
          int b = buf + r, sl = slot + r;
          uint32_t bp = bphase, sp = sphase;
          if (b >= C::NBUF) {
            b -= C::NBUF;
            bp ^= 1;
          }
          if (sl >= C::NSLOT) {
            sl -= C::NSLOT;
            sp ^= 1;
          }
          bufr[r] = b;
          slotr[r] = sl;
          const int k = kb + r;
          const float wsh = __shfl_sync(0xffffffffu, k < 32 ? ws0 : ws1, k & 31);
          wsr[r] = k < 64 ? wsh : (k < NKB ? __ldg(wsp + k) : 0.f);
          if (r < nr && good)
            good = mbar_wait_bounded(&tfull[b], bp, p.timeout_ns) && mbar_wait_bounded(&sfull[sl], sp, p.timeout_ns);
        }
        if (!good) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < C::TC / 16; ++cc) {
          if (col0 + cc * 16 < rows) {  // warp-uniform
            uint32_t v[KR][16];
#pragma unroll
            for (int r = 0; r < KR; ++r)
              if (r < nr)
                tmem_ld16(tmem_base + lane_base + (uint32_t)(bufr[r] * 2 * T + hs * T + col0 + cc * 16), v[r]);
            tmem_wait_ld();
#pragma unroll
            for (int r = 0; r < KR; ++r)
              if (r < nr) {
                const float* ss = sscale + slotr[r] * T + col0 + cc * 16;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  tmem_reg_fence(v[r][i]);
                  acc[cc * 16 + i] = fmaf(__uint_as_float(v[r][i]), wsr[r] * ss[i], acc[cc * 16 + i]);
                }
              }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < KR; ++r)
            if (r < nr) {
              mbar_arrive(&tempty[bufr[r]]);
              mbar_arrive(&sempty[slotr[r]]);
            }
        }
        buf += nr;
        if (buf >= C::NBUF) {
          buf -= C::NBUF;
          bphase ^= 1;
        }
        slot += nr;
        if (slot >= C::NSLOT) {
          slot -= C::NSLOT;
          sphase ^= 1;
        }
      }
      if (!ok) {
        atomicOr(p.err, ERR_DEV_TIMEOUT);
        *abort_flag = 1;
      }
      if (DYN) {
        // The next unit only now: the producer hands it on after issuing this
        // unit's loads, which needed this unit's TMEM buffers drained first.
        nxt = ok ? take() : make_int4(-1, 0, 0, 0);
        if (nxt.x >= 0) {
          unit_of(nxt.x, s2n, cn, ntn);
          load_ws(s2n, nxt.y, ntn);
        }
      } else if (un < n_units) {
        load_ws(s2n, e_n, ntn);
      }

      if (EPI == EPI_SILU || (FUSED && !s2)) {
        // Lane pair (2k, 2k+1) holds weight rows 2k (gate) and 2k+1 (up) of
        // this half for every token column. The even lane produces inter for
        // the even token columns and the odd lane for the odd ones; inter
        // column i = hs*64 + q*16 + k of this unit's 128-wide group.
        const int par = lane & 1;
        const int icol = hs * 64 + q * 16 + (lane >> 1);
        constexpr int TH = C::TC / 2;
        constexpr int NG = C::TC / 32;
        // 32-column groups holding at least one of the chunk's rows (warp-uniform).
        const int live = rows > col0 ? ((rows - col0 + 31) >> 5) : 0;
        float v[TH];
#pragma unroll
        for (int m = 0; m < TH; ++m) {
          v[m] = 0.f;
          if (m / 16 < live) {
            const float send = par ? acc[2 * m] : acc[2 * m + 1];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const float gate = par ? recv : acc[2 * m];
            const float up = par ? acc[2 * m + 1] : recv;
            v[m] = silu_f32(gate) * up;  // token column col0 + 2m + par
          }
        }
        // Column amax: within the warp (transposed, lane l ends with column
        // l of each 32-column group), then over the 8 warps of this column slice.
#pragma unroll
        for (int g = 0; g < NG; ++g)
          if (g < live) red[(hs * 4 + q) * T + col0 + g * 32 + lane] = warp_pair_transpose_max(v + g * 16, lane);
        if (tid == 0) *stop_sh = *abort_flag;
        named_bar_sync(1, EW * 32);
        // The previous read of stop_sh happened before this unit's second
        // barrier, the write above after it: one slot suffices.
        if (*stop_sh) break;
        float colscale[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          colscale[g] = 1.f;
          if (g >= live) continue;
          const int c = col0 + g * 32 + lane;
          float amax = red[c];
#pragma unroll
          for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w * T + c]);
          colscale[g] = group_scale(amax);
          if (hs == 0 && q == 0 && c < rows) p.out_sT[(int64_t)nt * p.out_s_ld + p0 + c] = colscale[g];
        }
#pragma unroll
        for (int m = 0; m < TH; ++m) {
          if (m / 16 < live) {
            const float sc = __shfl_sync(0xffffffffu, colscale[m / 16], 2 * (m % 16) + par);
            staging[(col0 + 2 * m + par) * 128 + icol] = quant_e4m3(v[m], sc);
          }
        }
        named_bar_sync(1, EW * 32);
        // Coalesced copy of the quantised rows: 8 x 16 B per row.
        for (int idx = tid; idx < rows * 8; idx += EW * 32) {
          const int c = idx >> 3, part = idx & 7;
          const uint4 val = *reinterpret_cast<const uint4*>(staging + c * 128 + part * 16);
          *reinterpret_cast<uint4*>(p.out_q + (int64_t)(p0 + c) * p.out_q_ld + nt * 128 + part * 16) = val;
        }
        if (FUSED) {
          // The warp's stores are ordered before lane 0's arrive (release) by
          // __syncwarp; the publisher's acquire and GPU-scope fence follow.
          const int sl = n_pub & 1;
          bool free_slot = true;
          if (n_pub >= 2 && lane == 0)
            free_slot = mbar_wait_or_abort(&pub[2 + sl], ((n_pub >> 1) & 1) ^ 1, p.timeout_ns, abort_flag);
          __syncwarp();
          if (DYN && tid == 0 && free_slot) pub_chunk[sl] = chunk;
          if (lane == 0 && free_slot) mbar_arrive(&pub[sl]);
          ++n_pub;
        }
      } else {
        if (!ok) break;
        const GemmParams& pc = FUSED ? p2 : p;
        // Lane l fetches the slot id and router weight of column l of each
        // 32-column group once; the stores below broadcast them by shuffle.
        constexpr int NG = C::TC / 32;
        int fl[NG];
        float wl[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const int c = col0 + g * 32 + lane;
          fl[g] = c < rows ? ld_meta<ROUTE>(&pc.sorted_ids[p0 + c]) : pc.sentinel;
          wl[g] = fl[g] < pc.sentinel ? ld_meta<ROUTE>(&pc.topk_w[fl[g]]) : 0.f;
        }
        // Row f (the slot) of out_pair; one 64-byte store per column.
        __nv_bfloat16* dst = pc.out_pair + nt * C::UNIT_ROWS + hs * 128 + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < C::TC; ++j) {
          if (col0 + (j & ~31) < rows) {  // warp-uniform
            const int f = __shfl_sync(0xffffffffu, fl[j / 32], j % 32);
            const float w = __shfl_sync(0xffffffffu, wl[j / 32], j % 32);
            if (f < pc.sentinel) dst[(int64_t)f * pc.Nw] = __float2bfloat16_rn(w * acc[j]);
          }
        }
      }
    }
    if (DYN) {
      // No more stage-1 units from this CTA: the publisher may stop.
      const int sl = n_pub & 1;
      bool free_slot = true;
      if (n_pub >= 2 && lane == 0)
        free_slot = mbar_wait_or_abort(&pub[2 + sl], ((n_pub >> 1) & 1) ^ 1, p.timeout_ns, abort_flag);
      __syncwarp();
      if (tid == 0 && free_slot) pub_chunk[sl] = -1;
      if (lane == 0 && free_slot) mbar_arrive(&pub[sl]);
    }
    if (PHASES) {
      // Last phase: the top-k reduce, once every CTA has stored all its
      // stage-2 rows (each CTA counts itself after its epilogue warps' last
      // stores; the fence of that thread orders them all, as in phase 0).
      named_bar_sync(1, EW * 32);
      if (tid == 0) {
        bool go = *abort_flag == 0;
        __threadfence();
        atomicAdd(p.phase_count + 1, 1);
        if (go) go = wait_count_bounded(p.phase_count + 1, (int)gridDim.x, p.timeout_ns, abort_flag);
        if (!go && *abort_flag == 0) {
          atomicOr(p.err, ERR_DEV_TIMEOUT);
          *abort_flag = 1;
        }
        *stop_sh = go ? 0 : 1;
      }
      named_bar_sync(1, EW * 32);
      if (*stop_sh == 0) {
        const int64_t per_row = p2.Nw / 8;
        const int64_t n = p.red_M * per_row;
        for (int64_t i = (int64_t)blockIdx.x * (EW * 32) + tid; i < n; i += (int64_t)gridDim.x * (EW * 32)) {
          const int64_t t = i / per_row;
          reduce_token_cols<4>(p2.out_pair, p.red_slot_pos, 0, p.red_topk, p2.Nw, t, (i - t * per_row) * 8,
                               p.red_out + t * p2.Nw);
        }
      }
    }
  } else if (FUSED) {
    // ------------------------------------------------------------ publisher
    if (lane == 0) {
      int k = 0;
      for (int u = blockIdx.x; DYN || u < n1; u += gridDim.x, ++k) {
        const int sl = k & 1;
        if (!mbar_wait_or_abort(&pub[sl], (k >> 1) & 1, p.timeout_ns, abort_flag)) {
          if (!*abort_flag) {
            atomicOr(p.err, ERR_DEV_TIMEOUT);
            *abort_flag = 1;
          }
          break;
        }
        int chunk;
        if (DYN) {
          chunk = pub_chunk[sl];
          if (chunk < 0) break;
        } else {
          bool s2;
          int nt;
          unit_of(u, s2, chunk, nt);
        }
        __threadfence();
        atomicAdd(p.chunk_ready + chunk, 1);
        mbar_arrive(&pub[2 + sl]);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace b200moe
