// Token-major grouped GEMM on CTA pairs (tcgen05 cta_group::2), for experts
// with many routed rows (large prefill batches).
//
// A cluster of two CTAs computes one unit = (up to 256 routed rows of one
// expert, 256 weight rows): MMA M = 256 (each CTA holds 128 routed rows of A
// in its shared memory and gets those rows of D in its TMEM), N = 256 (each
// CTA loads 128 of the 256 weight rows; the pair MMA reads both halves). Per
// K block each SM therefore moves 16 KB of activations + 16 KB of weights
// instead of 16 KB + 32 KB for the one-CTA 128x256 tile: 1.5x less data per
// multiply. The epilogue is the one-CTA token-major epilogue
// (moe_gemm_tok.cuh): one routed row and 128 weight rows per thread.
//
// Synchronisation: each CTA's TMA loads complete on the leader CTA's `full`
// barrier (.cta_group::2 loads, no multicast); the leader's single MMA thread
// issues the pair MMA and its commits arrive on `empty` / `tfull` of both CTAs
// (commit multicast); both CTAs' epilogue warps release a TMEM buffer by
// arriving on the leader's `tempty`. Activation scales are loaded and consumed
// inside each CTA.
#pragma once

#include "common.cuh"
#include "moe_gemm.cuh"
#include "moe_gemm_tok.cuh"
#include "ptx.cuh"

namespace b200moe {

struct Tok2Cfg {
  static constexpr int TM = 128;                 // routed rows per CTA
  static constexpr int UNIT_ROWS = 256;          // weight rows per unit (pair MMA N)
  static constexpr int W_ROWS = 128;             // weight rows loaded by each CTA
  static constexpr int EW = 8;
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr int A_BYTES = TM * 128;
  static constexpr int W_BYTES = W_ROWS * 128;
  static constexpr int TILE_BYTES = A_BYTES + W_BYTES;  // per CTA
  static constexpr int S_BYTES = TM * 4;
  static constexpr int NBUF = 2;
  static constexpr int TMEM_COLS = 512;
  static constexpr int RED = 2 * 2 * TM * 4;
  static constexpr int SMEM_LIMIT = 232448;
  static constexpr int MAX_STAGE = 6;
  static constexpr int XPOSE = EW * 32 * 20 * 4;  // stage-2 store transpose blocks
  static constexpr int FIXED = 1024 + RED + (MAX_STAGE + NBUF) * S_BYTES + 1024 + XPOSE;
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - FIXED) / TILE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > MAX_STAGE ? MAX_STAGE : NSTAGE_RAW;
  static constexpr int NSLOT = NSTAGE + NBUF;
  static constexpr int SMEM_BYTES = FIXED + NSTAGE * TILE_BYTES;
  static_assert(NSTAGE >= 2, "shared memory too small");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Tok2Cfg::THREADS, 1)
    moe_grouped_gemm_tok2_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                                 const GemmParams p) {
  using C = Tok2Cfg;
  constexpr int EW = C::EW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  float* sscale = reinterpret_cast<float*>(tiles + C::NSTAGE * C::TILE_BYTES);
  float* red = sscale + C::NSLOT * C::TM;
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
  float* xpose = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 1024);  // EW x 32 x 20

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader of the pair
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int NKB = p.K >> 7;
  const int NT = p.Nw / C::UNIT_ROWS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);   // leader: its producer's expect_tx; bytes from both CTAs
      mbar_init(&empty[s], 1);  // the pair MMA's commit (multicast to both CTAs)
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EW);  // leader: epilogue warps of both CTAs
    }
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int n_chunks = *p.n_chunks;
  const int n_units = n_chunks * NT;

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_a);
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int stage = 0, slot = 0;
      uint32_t phase = 0, sphase = 0;
      long issued = 0;
      bool ok = true;
      for (int u = pair; u < n_units && ok; u += n_pairs) {
        int chunk, nt;
        unit_coords(u, n_chunks, NT, p.chunk_group, chunk, nt);
        const int e = __ldg(&p.chunk_expert[chunk]);
        const int p0 = __ldg(&p.chunk_row0[chunk]) + (int)rank * C::TM;
        const int wrow = e * p.Nw + nt * C::UNIT_ROWS + (int)rank * C::W_ROWS;
        for (int kb = 0; kb < NKB; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns) ||
              !mbar_wait_bounded(&sempty[slot], sphase ^ 1, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* tile = tiles + stage * C::TILE_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::TILE_BYTES);
          const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(tile, &tm_a, leader_full, kb * 128, p0, pol_a);
          tma_load_2d_pair(tile + C::A_BYTES, &tm_w, leader_full, kb * 128, wrow, pol_w);
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
        // Tile loads land on the leader's barriers; let this CTA's scale copies land.
        long first = issued > C::NSLOT ? issued - C::NSLOT : 0;
        for (long g = first; g < issued; ++g)
          mbar_wait_bounded(&sfull[g % C::NSLOT], (uint32_t)((g / C::NSLOT) & 1), p.timeout_ns);
        if (rank == 0) {
          first = issued > C::NSTAGE ? issued - C::NSTAGE : 0;
          for (long g = first; g < issued; ++g)
            mbar_wait_bounded(&full[g % C::NSTAGE], (uint32_t)((g / C::NSTAGE) & 1), p.timeout_ns);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ pair MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_e4m3_f32(2 * C::TM, C::UNIT_ROWS);
      int stage = 0, buf = 0;
      uint32_t phase = 0, bphase = 0;
      long committed = 0;
      int last_buf = 0;
      uint32_t last_bphase = 0;
      bool ok = true;
      for (int u = pair; u < n_units && ok; u += n_pairs) {
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
            umma_f8_pair(d, sdesc_kmajor_sw128(a_addr + ks * 32), sdesc_kmajor_sw128(w_addr + ks * 32), idesc,
                         ks > 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage], 0x3);
          umma_commit_pair(&tfull[buf], 0x3);
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
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int r = q * 32 + lane;  // routed row within this CTA's half of the chunk
    const uint32_t taddr0 = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 128);
    int slot = 0, buf = 0;
    uint32_t sphase = 0, bphase = 0;
    bool ok = true;
    int parity = 0;
    for (int u = pair; u < n_units; u += n_pairs, parity ^= 1) {
      int chunk, nt;
      unit_coords(u, n_chunks, NT, p.chunk_group, chunk, nt);
      const int e = __ldg(&p.chunk_expert[chunk]);
      const int p0 = __ldg(&p.chunk_row0[chunk]) + (int)rank * C::TM;
      const int chunk_rows = __ldg(&p.chunk_rows[chunk]);
      int rows = chunk_rows - (int)rank * C::TM;
      rows = rows < 0 ? 0 : (rows > C::TM ? C::TM : rows);
      const bool live = q * 32 < rows;
      const float* wsp = p.w_scale + ((int64_t)e * (p.Nw >> 7) + nt * 2 + h) * NKB;

      float acc[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;

      // The unit's weight block scales spread over the lanes (K blocks lane
      // and lane + 32), read by shuffle: no global load per K block.
      const float ws0 = lane < NKB ? __ldg(wsp + lane) : 0.f;
      const float ws1 = lane + 32 < NKB ? __ldg(wsp + lane + 32) : 0.f;
      for (int kb = 0; kb < NKB && ok; ++kb) {
        const float wsh = __shfl_sync(0xffffffffu, kb < 32 ? ws0 : ws1, kb & 31);
        const float ws = kb < 64 ? wsh : __ldg(wsp + kb);
        if (*abort_flag || !mbar_wait_bounded(&tfull[buf], bphase, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!mbar_wait_bounded(&sfull[slot], sphase, p.timeout_ns)) {
          ok = false;
          break;
        }
        if (live) {
          const float sc = ws * sscale[slot * C::TM + r];
          const uint32_t taddr = taddr0 + (uint32_t)(buf * C::UNIT_ROWS);
#pragma unroll
          for (int c0 = 0; c0 < 8; c0 += 2) {
            uint32_t v[2][16];
            tmem_ld16(taddr + c0 * 16, v[0]);
            tmem_ld16(taddr + (c0 + 1) * 16, v[1]);
            tmem_wait_ld();
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 16; ++i) tmem_reg_fence(v[b][i]);
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 16; i += 2)
                ffma2(acc[(c0 + b) * 16 + i], acc[(c0 + b) * 16 + i + 1], __uint_as_float(v[b][i]),
                      __uint_as_float(v[b][i + 1]), sc);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
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

      if constexpr (EPI == EPI_SILU) {
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          acc[i] = silu_f32(acc[2 * i]) * acc[2 * i + 1];
          m = fmaxf(m, fabsf(acc[i]));
        }
        float* rb = red + parity * 2 * C::TM;
        rb[h * C::TM + r] = m;
        if (threadIdx.x == 64) *stop_sh = *abort_flag;
        named_bar_sync(1, EW * 32);
        // All epilogue warps read the value one thread stored before the
        // barrier; the store for the next unit comes after the second barrier.
        const bool stop = *stop_sh != 0;
        const float scale = group_scale(fmaxf(rb[r], rb[C::TM + r]));
        named_bar_sync(1, EW * 32);
        if (stop) break;
        if (r < rows) {
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            uint32_t b = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) b |= (uint32_t)quant_e4m3(acc[4 * k + t], scale) << (8 * t);
            w[k] = b;
          }
          uint4* dst = reinterpret_cast<uint4*>(p.out_q + (int64_t)(p0 + r) * p.out_q_ld + nt * 128 + h * 64);
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          if (h == 0) p.out_sT[(int64_t)nt * p.out_s_ld + p0 + r] = scale;
        }
      } else {
        if (!ok) break;
        // Row p of out_pair = sorted row p (see the one-CTA kernel).
        if (live) {
          const int f = r < rows ? __ldg(&p.sorted_ids[p0 + r]) : p.sentinel;
          const float w = f < p.sentinel ? __ldg(&p.topk_w[f]) : 0.f;
          const unsigned valid = __ballot_sync(0xffffffffu, f < p.sentinel);
          store_sorted_rows(acc, w, valid, xpose + ew * (32 * 20), lane, q * 32,
                            p.out_pair + (int64_t)p0 * p.Nw + nt * C::UNIT_ROWS + h * 128, p.Nw);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // the pair MMA is done with both CTAs' shared memory and TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace b200moe
