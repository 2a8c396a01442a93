// Token-major persistent FP8 block-scaled grouped GEMM (sm_100a), used when
// experts receive many tokens (prefill). Same math and epilogues as
// moe_gemm.cuh; the MMA orientation is the other way round:
//   MMA M = 128 routed rows of one expert (A = activation tile),
//   MMA N = 256 weight rows (B = weight tile), one 128x256x32 MMA per K step.
// Each epilogue thread then owns one routed row and 128 consecutive weight
// rows (one 128-row scale block), so
//   * the block-scale promotion is a scalar per thread and K block
//     (a_s[row] * w_s[block]), applied with packed f32x2 FMAs;
//   * gate/up pairs (interleaved rows 2j, 2j+1) sit in the same thread, so
//     SiLU*up needs no shuffles and the 1x128 requant amax is the max of two
//     threads' values;
//   * each thread writes a contiguous run of its output row.
//
// Warp roles: warp 0 TMA producer, warp 1 MMA issuer and TMEM owner, warps
// 2..9 epilogue (TMEM lane quarter w%4 x column half).
#pragma once

#include "common.cuh"
#include "moe_gemm.cuh"
#include "ptx.cuh"

namespace b200moe {

// Epilogue warps of the stage-1 (SiLU) token-major kernel: 8 (two per SM
// sub-partition, 128 weight-row columns per thread) or 16 (four per
// sub-partition, 64 columns per thread, to hide more of the TMEM-load and FMA
// latencies of the per-K-block promotion). 16 measured 3% slower at 4,096
// and 8,192 tokens (96 registers a thread, some spilled), so 8 it is. Stage 2
// keeps 8 either way: its output staging would cost another pipeline stage.
#ifndef B200MOE_TOK_EW_SILU
#define B200MOE_TOK_EW_SILU 8
#endif

template <int EW_, bool OUT_>
struct TokCfgT {
  static constexpr int TM = 128;                 // routed rows per unit (MMA M)
  static constexpr int UNIT_ROWS = 256;          // weight rows per unit (MMA N)
  static constexpr int EW = EW_;                 // epilogue warps: 4 lane quarters x CQ column groups
  static constexpr int CQ = EW / 4;              // column groups
  static constexpr int COLS = UNIT_ROWS / CQ;    // weight-row columns per epilogue thread
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr int A_BYTES = TM * 128;
  static constexpr int W_BYTES = UNIT_ROWS * 128;
  static constexpr int TILE_BYTES = A_BYTES + W_BYTES;
  static constexpr int S_BYTES = TM * 4;
  static constexpr int NBUF = 2;                 // TMEM partial buffers of 256 columns
  static constexpr int TMEM_COLS = 512;
  static constexpr int RED = 2 * CQ * TM * 4;    // amax exchange, double-buffered by unit parity
  static constexpr int SMEM_LIMIT = 232448;
  static constexpr int MAX_STAGE = 6;
  // Stage 2: each epilogue warp's 32 rows x COLS bf16 output columns, staged
  // for TMA stores in 64-column boxes with the 128-byte swizzle (1024-byte
  // aligned, hence the extra 1024).
  static constexpr int OUT_STAGE = OUT_ ? EW * 32 * COLS * 2 : 0;
  static constexpr int NU = 4;                    // unit hand-off ring (producer -> MMA, epilogue)
  static constexpr int FIXED = 1024 + RED + (MAX_STAGE + NBUF) * S_BYTES + 1024 + (OUT_ ? OUT_STAGE + 1024 : 0);
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - FIXED) / TILE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > MAX_STAGE ? MAX_STAGE : NSTAGE_RAW;
  static constexpr int NSLOT = NSTAGE + NBUF;
  static constexpr int SMEM_BYTES = FIXED + NSTAGE * TILE_BYTES;
  static_assert(EW == 8 || EW == 16, "8 or 16 epilogue warps");
  static_assert(COLS % 32 == 0 && COLS <= 128, "a thread's columns lie in one 128-row scale block");
  static_assert(!OUT_ || COLS % 64 == 0, "stage-2 output boxes are 64 columns wide");
  static_assert(NSTAGE >= 2, "shared memory too small");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
};

// The configuration of each token-major stage kernel.
template <int EPI>
using TokCfgE = TokCfgT<EPI == EPI_SILU ? B200MOE_TOK_EW_SILU : 8, EPI != EPI_SILU>;
using TokCfg = TokCfgT<8, true>;


// Router-weighted fp32 rows of a token-major unit, in sorted row order. The
// calling warp holds rows row0 .. row0+31 of the unit (lane = row) x NC
// output columns in acc. They pass through tb (this warp's 32 x 20 floats of
// shared memory) 16 columns at a time, so that every store instruction writes
// 32 contiguous bytes (one whole sector) of each of 8 rows instead of 8 bytes
// of 32 rows. Only rows whose bit is set in `valid` (bit i = row row0 + i, a
// routed slot) are written; w_l is the lane's router weight.
template <int NC>
__device__ __forceinline__ void store_sorted_rows(const float (&acc)[NC], float w_l, unsigned valid, float* tb,
                                                  int lane, int row0, __nv_bfloat16* out, int64_t ld) {
#pragma unroll
  for (int cb = 0; cb < NC / 16; ++cb) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<float4*>(tb + lane * 20 + 4 * k) =
          make_float4(w_l * acc[cb * 16 + 4 * k], w_l * acc[cb * 16 + 4 * k + 1], w_l * acc[cb * 16 + 4 * k + 2],
                      w_l * acc[cb * 16 + 4 * k + 3]);
    __syncwarp();
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int row = rr * 8 + (lane >> 2);
      const float4 v = *reinterpret_cast<const float4*>(tb + row * 20 + 4 * (lane & 3));
      if ((valid >> row) & 1u) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(out + (int64_t)(row0 + row) * ld + cb * 16 + 4 * (lane & 3)) = pk;
      }
    }
    __syncwarp();
  }
}

// d = a * s + d on two fp32 lanes at once (IEEE fma on each).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float s) {
  uint64_t rd, ra, rs;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(rs) : "f"(s));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rd) : "f"(d0), "f"(d1));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(rd) : "l"(ra), "l"(rs));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(rd));
}

// Epilogue tuning: TMEM loads of 16 columns issued per wait (1, 2 or 4) and
// packed f32x2 FMA (1) or scalar FMA (0) for the promotion. Same results.
#ifndef B200MOE_TOK_LD_BATCH
#define B200MOE_TOK_LD_BATCH 2
#endif
// L2 hint on token-major weight tiles: 0 none, 1 evict_first, 2 evict_last.
#ifndef B200MOE_TOK_W_POLICY
#define B200MOE_TOK_W_POLICY 0
#endif
// L2 hint on token-major activation tiles: 1 evict_last, 0 none.
#ifndef B200MOE_TOK_A_POLICY
#define B200MOE_TOK_A_POLICY 1
#endif
#ifndef B200MOE_TOK_FFMA2
#define B200MOE_TOK_FFMA2 1
#endif

// tm_o: stage 2's out_pair (rows_capacity, Nw) bf16, boxes of 64 columns x 16
// rows with the 128-byte swizzle; read only when stage-2 rows go to their
// sorted position (not rows_by_slot).
template <int EPI>
__global__ void __launch_bounds__(TokCfgE<EPI>::THREADS, 1)
    moe_grouped_gemm_tok_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                                const __grid_constant__ CUtensorMap tm_o, const GemmParams p) {
  using C = TokCfgE<EPI>;
  constexpr int EW = C::EW;
  constexpr int COLS = C::COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;                                                       // NSTAGE * (A | W)
  float* sscale = reinterpret_cast<float*>(tiles + C::NSTAGE * C::TILE_BYTES);  // NSLOT * TM
  float* red = sscale + C::NSLOT * C::TM;                                       // 2 x 2 x TM
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + C::RED);
  uint64_t* empty = full + C::NSTAGE;
  uint64_t* tfull = empty + C::NSTAGE;
  uint64_t* tempty = tfull + C::NBUF;
  uint64_t* sfull = tempty + C::NBUF;
  uint64_t* sempty = sfull + C::NSLOT;
  uint64_t* ufull = sempty + C::NSLOT;
  uint64_t* uempty = ufull + C::NU;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(uempty + C::NU);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // The epilogue's stop decision for a unit, written by one thread before the
  // unit's first named barrier so that every epilogue warp reads the same value.
  volatile int* stop_sh = reinterpret_cast<volatile int*>(tmem_slot + 2);
  // Units in the order the producer takes them (-1 = no more), read by the MMA
  // thread and every epilogue warp before the slot is reused.
  volatile int* unit_sh = reinterpret_cast<volatile int*>(tmem_slot + 4);
  uint8_t* out_stage = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(full) + 1024 + 1023) & ~uintptr_t(1023));  // EW x 32 x COLS bf16

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NKB = p.K >> 7;
  const int NT = p.Nw / C::UNIT_ROWS;
  // Launched programmatically: the kernel ahead of it (the routing's work
  // list, the gather's rows, stage 1's rows) must be done before any read.
  griddep_wait();
  // An empty work list (the heavy list of a batch without heavy experts)
  // ends the launch before any set-up.
  if (*p.n_chunks == 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EW);
    }
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], EW);
    }
    for (int s = 0; s < C::NU; ++s) {
      mbar_init(&ufull[s], 1);
      mbar_init(&uempty[s], 1 + EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_a);
    if (EPI != EPI_SILU && !p.rows_by_slot) prefetch_tmap(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int n_chunks = *p.n_chunks;
  const int n_units = n_chunks * NT;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // Weight tiles of a group's chunks are shared through L2 by units that
      // run at the same time (unit_coords), activation tiles by the 2I/256 or
      // H/256 units of a chunk: neither may be evicted first.
      const uint64_t pol_w = B200MOE_TOK_W_POLICY == 2 ? policy_evict_last() : policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int stage = 0, slot = 0, uslot = 0;
      uint32_t phase = 0, sphase = 0, uphase = 0;
      long issued = 0;
      bool ok = true;
      // Units come from the shared counter when there is one (a CTA takes the
      // next unit when it is ready for it, so units that share weight tiles
      // through L2 keep running at the same time), else round-robin.
      for (int k = 0; ok; ++k) {
        int u = p.unit_counter ? atomicAdd(p.unit_counter, 1) : (int)blockIdx.x + k * (int)gridDim.x;
        if (u >= n_units) u = -1;
        if (*abort_flag || !mbar_wait_bounded(&uempty[uslot], uphase ^ 1, p.timeout_ns)) {
          ok = false;
          break;
        }
        unit_sh[uslot] = u;
        mbar_arrive(&ufull[uslot]);
        if (++uslot == C::NU) {
          uslot = 0;
          uphase ^= 1;
        }
        if (u < 0) break;
        int chunk, nt;
        unit_coords(u, n_chunks, NT, p.chunk_group, chunk, nt);
        const int e = __ldg(&p.chunk_expert[chunk]);
        const int p0 = __ldg(&p.chunk_row0[chunk]);
        const int wrow = e * p.Nw + nt * C::UNIT_ROWS;
        for (int kb = 0; kb < NKB; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns) ||
              !mbar_wait_bounded(&sempty[slot], sphase ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* tile = tiles + stage * C::TILE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::TILE_BYTES);
          if (B200MOE_TOK_A_POLICY)
            tma_load_2d(tile, &tm_a, &full[stage], kb * 128, p0, pol_a);
          else
            tma_load_2d(tile, &tm_a, &full[stage], kb * 128, p0);
          if (B200MOE_TOK_W_POLICY == 1 || B200MOE_TOK_W_POLICY == 2)
            tma_load_2d(tile + C::A_BYTES, &tm_w, &full[stage], kb * 128, wrow, pol_w);
          else
            tma_load_2d(tile + C::A_BYTES, &tm_w, &full[stage], kb * 128, wrow);
          mbar_arrive_expect_tx(&sfull[slot], C::S_BYTES);
          bulk_load(sscale + slot * C::TM, p.a_sT + (int64_t)kb * p.as_ld + p0, C::S_BYTES, &sfull[slot]);
          ++issued;
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1;
          }
          if (++slot == C::NSLOT) {
            slot = 0;
            sphase ^= 1;
          }
        }
      }
      if (!ok) {
        atomicOr(p.err, ERR_DEV_TIMEOUT);
        *abort_flag = 1;
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
      const uint32_t idesc = idesc_e4m3_f32(C::TM, C::UNIT_ROWS);
      int stage = 0, buf = 0;
      uint32_t phase = 0, bphase = 0;
      long committed = 0;
      int last_buf = 0, uslot = 0;
      uint32_t last_bphase = 0, uphase = 0;
      bool ok = true;
      while (ok) {
        if (*abort_flag || !mbar_wait_bounded(&ufull[uslot], uphase, p.timeout_ns)) {
          ok = false;
          break;
        }
        const int u = unit_sh[uslot];
        mbar_arrive(&uempty[uslot]);
        if (++uslot == C::NU) {
          uslot = 0;
          uphase ^= 1;
        }
        if (u < 0) break;
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
          const uint32_t a_addr = smem_u32(tiles + stage * C::TILE_BYTES);
          const uint32_t w_addr = a_addr + C::A_BYTES;
          const uint32_t d = tmem_base + (uint32_t)(buf * C::UNIT_ROWS);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_f8(d, sdesc_kmajor_sw128(a_addr + ks * 32), sdesc_kmajor_sw128(w_addr + ks * 32), idesc,
                    ks > 0 ? 1u : 0u);
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
      if (committed > 0) mbar_wait_bounded(&tfull[last_buf], last_bphase, p.timeout_ns);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;          // TMEM lane quarter = routed rows 32q..32q+31
    const int cq = ew >> 2;          // column group = weight rows COLS*cq .. COLS*cq+COLS-1 of the unit
    const int h = (cq * COLS) >> 7;  // its 128-row scale block
    const int r = q * 32 + lane;     // this thread's routed row within the chunk
    const uint32_t taddr0 = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(cq * COLS);
    int slot = 0, buf = 0;
    uint32_t sphase = 0, bphase = 0;
    bool ok = true;
    int parity = 0;
    // The unit's weight block scales (one per K block of this 128-row half)
    // are spread over the lanes (K blocks lane and lane + 32) and loaded
    // before the previous unit's final epilogue, so no global load sits on
    // the per-K-block path.
    auto ws_row = [&](int e, int nt) { return p.w_scale + ((int64_t)e * (p.Nw >> 7) + nt * 2 + h) * NKB; };
    float wl0 = 0.f, wl1 = 0.f;
    auto load_ws = [&](int u) {
      int c, t;
      unit_coords(u, n_chunks, NT, p.chunk_group, c, t);
      const float* w = ws_row(__ldg(&p.chunk_expert[c]), t);
      wl0 = lane < NKB ? __ldg(w + lane) : 0.f;
      wl1 = lane + 32 < NKB ? __ldg(w + lane + 32) : 0.f;
    };
    int uslot = 0;
    uint32_t uphase = 0;
    // The next unit of the producer's sequence (-1: none left, -2: timed out).
    auto next_unit = [&]() -> int {
      if (!mbar_wait_bounded(&ufull[uslot], uphase, p.timeout_ns)) return -2;
      const int v = unit_sh[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty[uslot]);
      if (++uslot == C::NU) {
        uslot = 0;
        uphase ^= 1;
      }
      return v;
    };
    int u = next_unit();
    if (u >= 0) load_ws(u);
    for (int nu = -1; u >= 0; u = nu, parity ^= 1) {
      int chunk, nt;
      unit_coords(u, n_chunks, NT, p.chunk_group, chunk, nt);
      const int e = __ldg(&p.chunk_expert[chunk]);
      const int p0 = __ldg(&p.chunk_row0[chunk]);
      const int rows = __ldg(&p.chunk_rows[chunk]);
      const float ws0 = wl0, ws1 = wl1;
      const bool live = q * 32 < rows;  // warp-uniform
      const float* wsp = ws_row(e, nt);
      // Stage 2: the row's slot id is loaded now and its router weight after
      // the first partial, so that neither load waits in the unit's tail.
      int f_row = p.sentinel;
      float w_row = 0.f;
      if constexpr (EPI != EPI_SILU)
        if (live && r < rows) f_row = __ldg(&p.sorted_ids[p0 + r]);

      float acc[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) acc[j] = 0.f;

      for (int kb = 0; kb < NKB && ok; ++kb) {
        const float wsh = __shfl_sync(0xffffffffu, kb < 32 ? ws0 : ws1, kb & 31);
        const float ws = kb < 64 ? wsh : __ldg(wsp + kb);
        if (*abort_flag || !mbar_wait_bounded(&tfull[buf], bphase, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if constexpr (EPI != EPI_SILU)
          if (kb == 0 && f_row < p.sentinel) w_row = __ldg(&p.topk_w[f_row]);
        if (!mbar_wait_bounded(&sfull[slot], sphase, p.timeout_ns)) {
          ok = false;
          break;
        }
        if (live) {
          const float sc = ws * sscale[slot * C::TM + r];
          const uint32_t taddr = taddr0 + (uint32_t)(buf * C::UNIT_ROWS);
          constexpr int LB = COLS == 128 ? B200MOE_TOK_LD_BATCH : 1;
#pragma unroll
          for (int c0 = 0; c0 < COLS / 16; c0 += LB) {
            uint32_t v[LB][16];
#pragma unroll
            for (int b = 0; b < LB; ++b) tmem_ld16(taddr + (c0 + b) * 16, v[b]);
            tmem_wait_ld();
#pragma unroll
            for (int b = 0; b < LB; ++b)
#pragma unroll
              for (int i = 0; i < 16; ++i) tmem_reg_fence(v[b][i]);
#pragma unroll
            for (int b = 0; b < LB; ++b)
#pragma unroll
              for (int i = 0; i < 16; i += 2) {
                float& d0 = acc[(c0 + b) * 16 + i];
                float& d1 = acc[(c0 + b) * 16 + i + 1];
#if B200MOE_TOK_FFMA2
                ffma2(d0, d1, __uint_as_float(v[b][i]), __uint_as_float(v[b][i + 1]), sc);
#else
                d0 = fmaf(__uint_as_float(v[b][i]), sc, d0);
                d1 = fmaf(__uint_as_float(v[b][i + 1]), sc, d1);
#endif
              }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[buf]);
          mbar_arrive(&sempty[slot]);
        }
        if (++slot == C::NSLOT) {
          slot = 0;
          sphase ^= 1;
        }
        if (++buf == C::NBUF) {
          buf = 0;
          bphase ^= 1;
        }
      }
      if (!ok) {
        atomicOr(p.err, ERR_DEV_TIMEOUT);
        *abort_flag = 1;
      }
      nu = ok ? next_unit() : -1;
      if (nu >= 0) load_ws(nu);

      if constexpr (EPI == EPI_SILU) {
        // inter column i of this column group = silu(acc[2i]) * acc[2i+1],
        // column NI*cq + i of the unit's 128 (the 1x128 requant group = all
        // CQ column groups of this row).
        constexpr int NI = COLS / 2;
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          acc[i] = silu_f32(acc[2 * i]) * acc[2 * i + 1];
          m = fmaxf(m, fabsf(acc[i]));
        }
        float* rb = red + parity * C::CQ * C::TM;
        rb[cq * C::TM + r] = m;
        if (threadIdx.x == 64) *stop_sh = *abort_flag;
        named_bar_sync(1, EW * 32);
        // All epilogue warps read the value one thread stored before the
        // barrier; the store for the next unit comes after the second barrier.
        const bool stop = *stop_sh != 0;
        float amax = rb[r];
#pragma unroll
        for (int g = 1; g < C::CQ; ++g) amax = fmaxf(amax, rb[g * C::TM + r]);
        const float scale = group_scale(amax);
        named_bar_sync(1, EW * 32);
        if (stop) break;
        if (r < rows) {
          uint32_t w[NI / 4];
#pragma unroll
          for (int k = 0; k < NI / 4; ++k) {
            uint32_t b = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) b |= (uint32_t)quant_e4m3(acc[4 * k + t], scale) << (8 * t);
            w[k] = b;
          }
          uint4* dst = reinterpret_cast<uint4*>(p.out_q + (int64_t)(p0 + r) * p.out_q_ld + nt * 128 + cq * NI);
#pragma unroll
          for (int k = 0; k < NI / 16; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          if (cq == 0) p.out_sT[(int64_t)nt * p.out_s_ld + p0 + r] = scale;
        }
      } else {
        if (!ok) break;
        // Row p of out_pair = sorted row p: a unit's rows are neighbours in
        // memory (rows by slot id scatter them over the whole buffer, and the
        // stores then cost more than the unit's MMAs at prefill sizes).
        if (live) {
          const int f = f_row;
          const float w = w_row;
          if (p.rows_by_slot) {
            // Row f (the slot), as the swap-AB tiles write it: COLS contiguous
            // bf16 per thread (few heavy experts of a decode batch take this path).
            if (f < p.sentinel) {
              uint4* dst = reinterpret_cast<uint4*>(p.out_pair + (int64_t)f * p.Nw + nt * C::UNIT_ROWS + cq * COLS);
#pragma unroll
              for (int k = 0; k < COLS / 8; ++k) {
                __nv_bfloat162 b[4];
#pragma unroll
                for (int t = 0; t < 4; ++t)
                  b[t] = __floats2bfloat162_rn(w * acc[8 * k + 2 * t], w * acc[8 * k + 2 * t + 1]);
                dst[k] = *reinterpret_cast<const uint4*>(b);
              }
            }
          } else {
            // The warp's 32 rows x COLS columns go to shared memory (bf16,
            // 64-column boxes of 32 rows x 128 bytes, 16-byte pieces swizzled
            // by row: piece c of row r at c ^ (r & 7), so the 8 rows of a
            // quarter-warp store hit different banks), then one lane stores
            // them with TMA, 16 rows per box. Chunks of an expert follow one
            // another in the sorted rows, so only the chunk's own rows are
            // written: 16-row blocks inside it by TMA (their rows without a
            // slot as zeros), the rows of a block that the chunk ends inside
            // by their own threads (chunks from routing are multiples of 16
            // rows and never end inside a block). The staging buffer is
            // reused once the warp's previous stores have read it.
            uint8_t* sb = out_stage + ew * (32 * COLS * 2);
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
            const bool valid = f < p.sentinel;
            const bool own_store = r < rows && (r & ~15) + 16 > rows;
            __nv_bfloat16* orow = p.out_pair + (int64_t)(p0 + r) * p.Nw + nt * C::UNIT_ROWS + cq * COLS;
#pragma unroll
            for (int b = 0; b < COLS / 64; ++b)
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                uint32_t pk[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const int j = b * 64 + c * 8 + 2 * t;
                  __nv_bfloat162 h = __floats2bfloat162_rn(valid ? w * acc[j] : 0.f, valid ? w * acc[j + 1] : 0.f);
                  pk[t] = *reinterpret_cast<uint32_t*>(&h);
                }
                const uint4 v = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4*>(sb + b * 4096 + lane * 128 + ((c ^ (lane & 7)) << 4)) = v;
                if (own_store) *reinterpret_cast<uint4*>(orow + b * 64 + c * 8) = v;
              }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
              for (int h = 0; h < 2; ++h)
                if (q * 32 + h * 16 + 16 <= rows)
#pragma unroll
                  for (int b = 0; b < COLS / 64; ++b)
                    tma_store_2d(&tm_o, sb + b * 4096 + h * 2048, nt * C::UNIT_ROWS + cq * COLS + b * 64,
                                 p0 + q * 32 + h * 16);
              bulk_commit_group();
            }
          }
        }
      }
    }
    if (u == -2) {  // the producer never handed over the next unit
      atomicOr(p.err, ERR_DEV_TIMEOUT);
      *abort_flag = 1;
    }
    // Stage-2 rows stored with TMA are complete (and the staging buffer
    // read) before the CTA exits.
    if (EPI != EPI_SILU && lane == 0) bulk_wait_all();
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
