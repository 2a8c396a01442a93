// Internal launcher interfaces between the C-ABI layer (capi.cu) and the
// kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200moe {

// Launch with the programmatic stream serialisation attribute: the kernel may
// begin while the kernel ahead of it in the stream finishes, so it must call
// griddep_wait() (ptx.cuh) before it touches memory that kernel writes.
#ifndef B200MOE_PDL
#define B200MOE_PDL 1
#endif
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = B200MOE_PDL ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

struct AlignArgs {
  const int32_t* topk_ids;
  int64_t n;               // M * topk
  int num_experts;         // id range of topk_ids
  const int32_t* expert_map;
  int E;                   // weight experts (map targets)
  int block_m;
  int32_t sentinel;
  int32_t* sorted_ids;
  int64_t sorted_cap;
  int32_t* expert_ids;     // nullable
  int64_t blocks_cap;
  int32_t* ntp;
  int tile_tokens;         // 0 = no chunk list
  int32_t* chunk_expert;
  int32_t* chunk_row0;
  int32_t* chunk_rows;
  int64_t chunks_cap;
  int32_t* n_chunks;
  int32_t* chunk_ready;    // nullable: zeroed over chunks_cap + 2 entries
  int32_t* slot_pos;       // nullable: sorted position of each flat slot (n entries), -1 if dropped
  int32_t* err;
  int seg_align;           // multi-CTA segments: multiple of this many ids (0/1 = any)
  // Mixed work lists (one-CTA routing only; 0 = off): experts with more than
  // heavy_rows padded rows are laid out after all the others and cut into
  // chunks of at most 128 rows in a second list (for the token-major stages);
  // the rest form the tile_tokens list as usual. *heavy_row0 receives the
  // first row of the heavy experts (= the light experts' rows), *n_chunks2
  // the heavy list's length; counters2 (2 ints) is zeroed.
  int heavy_rows;
  int32_t* chunk_expert2;
  int32_t* chunk_row0_2;
  int32_t* chunk_rows2;
  int64_t chunks_cap2;
  int32_t* n_chunks2;
  int32_t* heavy_row0;
  int32_t* counters2;
};
constexpr int kHeavyTile = 128;  // chunk rows of the heavy list

size_t align_smem_bytes(int E);
cudaError_t launch_align(const AlignArgs& a, cudaStream_t stream);
// Routing of large batches on several CTAs (two launches) when scratch holds
// route_scratch_ints() entries; otherwise launch_align.
int route_ctas(int64_t n);
int64_t route_scratch_ints(int64_t n, int E);
cudaError_t launch_route(const AlignArgs& a, int32_t* scratch, int64_t scratch_ints, cudaStream_t stream);
// Routing from router logits: the router (router.cuh) runs in routing's first
// launch and stores topk ids and weights to r.out_ids / r.out_w, which routing
// then uses as a.topk_ids. scratch: kRouteLogitsCounterInts ints (a CTA
// counter that must be zero before the first call; every call leaves it zero)
// followed by the route_scratch_ints(n, E) counts of the multi-CTA form.
struct RouterArgs;
constexpr int kRouteLogitsCounterInts = 4;
int64_t route_logits_scratch_ints(int64_t n, int E);
cudaError_t launch_route_logits(const AlignArgs& a, const RouterArgs& r, int64_t M, int32_t* counter,
                                int32_t* counts, cudaStream_t stream);

// Per-token-group (1 x 128) FP8 quantisation. With sorted_ids != nullptr the
// output row p takes its input from token sorted_ids[p] / topk (zeros for the
// sentinel) and the number of rows is read from *num_rows on the device.
struct QuantArgs {
  const void* x;
  int64_t ldx;
  // Pre-quantised input (copy mode, x unused): fp8 rows with row stride ldxq
  // bytes and 1x128 scales xs[t * ldxs + g].
  const uint8_t* xq;
  int64_t ldxq;
  const float* xs;
  int64_t ldxs;
  int64_t K;
  int64_t rows;            // rows (M) or the row capacity in gather mode
  const int32_t* num_rows; // gather mode: device row count
  const int32_t* sorted_ids;
  // Slot mode (takes precedence over sorted_ids): row r of the launch is the
  // flat slot r (rows = M*topk); it reads input row r / topk and writes output
  // row slot_pos[r] (skipped when -1).
  const int32_t* slot_pos;
  int topk;
  // With slot_pos: row r of the launch is token r instead (rows = M), written
  // to every one of its slots' rows slot_pos[r*topk + j] (topk <= 32).
  int fanout;
  // slot_pos / sorted_ids were written earlier in the same launch: read them
  // through L2 instead of the read-only path.
  int meta_l2;
  int32_t sentinel;
  uint8_t* q;
  int64_t ldq;
  float* s;
  int64_t s_row;
  int64_t s_grp;
};
cudaError_t launch_quant_1x128(const QuantArgs& a, cudaStream_t stream);

cudaError_t launch_quant_block128(const void* w, int64_t E, int64_t N, int64_t K, uint8_t* q, float* s,
                                  cudaStream_t stream);

cudaError_t launch_combine_reduce(const void* pair_rows, const int32_t* slot_pos, int sorted_rows, int64_t M, int topk,
                                  int64_t H, void* out, cudaStream_t stream);

// Where each expert's weights live for expert parallelism: physical expert
// slots p = rank * slots + local index. rep == nullptr: expert e only in slot
// e (slots = num_experts / G, rank r holds [r*slots, (r+1)*slots)). Otherwise
// rep[e * (1 + max_rep)] = n replicas of e, followed by their n slots; a
// routed slot (t, j) of expert e goes to the replica on src_rank if there is
// one, else to replica (t * topk + j) mod n (ep_place.cuh).
struct EpPlace {
  const int32_t* rep;
  int max_rep;
  int slots;
  int num_experts;
  int src_rank;
  int G;
};
cudaError_t launch_ep_plan(const int32_t* ids, int64_t M, int topk, const EpPlace& pl, int64_t rows_per_rank,
                           int32_t* pos, int32_t* tok_of, int32_t* counts, int32_t* err, cudaStream_t stream);
cudaError_t launch_ep_dispatch(const uint8_t* q, const float* s, const int32_t* ids, const float* w, int64_t M,
                               int64_t H, int topk, const EpPlace& pl, int64_t rows_per_rank, uint8_t* send,
                               int64_t row_bytes, int32_t* pos, int32_t* tok_of, int32_t* counts, int32_t* err,
                               cudaStream_t stream);
cudaError_t launch_ep_unpack_meta(const uint8_t* rows, int64_t R, int64_t row_bytes, int64_t H, int topk,
                                  int32_t* ids, float* w, cudaStream_t stream);
cudaError_t launch_ep_combine(const void* comb, const int32_t* pos, int64_t M, int64_t H, int G,
                              int64_t rows_per_rank, void* out, cudaStream_t stream);

// Exchange buffer of one rank for expert parallelism through peer memory:
// [header | receive area x 2 | return area x 2], areas double-buffered by the
// parity of the call count. Receive area: G blocks of rows_per_rank packed
// rows (block = source rank). Return area: G blocks of rows_per_rank bf16 rows
// of H (block = expert-side rank). Header: the flags the other ranks raise and
// this rank's CTA counters.
struct EpPeerLayout {
  static constexpr int64_t kDispatchFlags = 0;   // int32[kMaxRanks]: source rank -> epoch of its rows
  static constexpr int64_t kCombineFlags = 256;  // int32[kMaxRanks]: expert-side rank -> epoch of its results
  static constexpr int64_t kCounters = 512;      // int32[2]: CTAs done (pack, reduce), local
  static constexpr int64_t kHeader = 1024;
  static constexpr int kMaxRanks = 64;
  int64_t recv_bytes, ret_bytes;
  EpPeerLayout(int64_t rows_per_rank, int64_t H, int64_t row_bytes, int G)
      : recv_bytes(((int64_t)G * rows_per_rank * row_bytes + 255) / 256 * 256),
        ret_bytes(((int64_t)G * rows_per_rank * H * 2 + 255) / 256 * 256) {}
  int64_t recv_off(int32_t epoch) const { return kHeader + (epoch & 1) * recv_bytes; }
  int64_t ret_off(int32_t epoch) const { return kHeader + 2 * recv_bytes + (epoch & 1) * ret_bytes; }
  int64_t total() const { return kHeader + 2 * (recv_bytes + ret_bytes); }
};

struct EpPeerArgs {
  uint8_t* const* bases;  // device array: the G ranks' exchange buffers as mapped here
  int64_t area_off;       // the area written on the far side (receive or return, this call's parity)
  int64_t rows_per_rank;
  int G, rank;
  int32_t epoch;
};
cudaError_t launch_ep_pack_peer(const void* hidden, const uint8_t* q, const float* s, const int32_t* ids,
                                const float* w, int64_t H, int topk, const EpPlace& pl, const int32_t* tok_of,
                                const int32_t* counts, int64_t row_bytes, const EpPeerArgs& a, int32_t* counter,
                                cudaStream_t stream);
// Received packed rows whose ids and weights the routing launch unpacks
// itself, after waiting for the G dispatch flags (ep_unpack_meta_peer's work):
// ids / w (R * topk) receive them; a.topk_ids must be ids.
struct PackedMeta {
  const uint8_t* own;   // this rank's exchange buffer (its dispatch flags)
  const uint8_t* rows;  // receive area of this call
  int64_t R, row_bytes, H;
  int topk, G;
  int32_t epoch;
  uint64_t limit_ns;
  int32_t* ids;
  float* w;
};
// One-CTA routing that first waits for and unpacks the received rows' ids and
// weights (below 16,384 routed slots, or with mixed lists).
cudaError_t launch_align_packed(const AlignArgs& a, const PackedMeta& pm, cudaStream_t stream);
cudaError_t launch_ep_unpack_meta_peer(const uint8_t* own, const uint8_t* rows, int64_t R, int64_t row_bytes,
                                       int64_t H, int topk, int G, int32_t epoch, int32_t* ids, float* w,
                                       int32_t* err, uint64_t limit_ns, cudaStream_t stream);
cudaError_t launch_ep_reduce_peer(const __nv_bfloat16* pair, const int32_t* slot_pos, int sorted_rows, int topk, int64_t H,
                                  const EpPeerArgs& a, int32_t* counter, cudaStream_t stream);
cudaError_t launch_ep_combine_peer(const uint8_t* own, int64_t area_off, const int32_t* pos, int64_t M, int64_t H,
                                   int G, int64_t rows_per_rank, int32_t epoch, void* out, int32_t* err,
                                   uint64_t limit_ns, cudaStream_t stream);

cudaError_t launch_router_topk(const void* logits, int bf16, int64_t M, int E, int topk, int scoring,
                               const float* bias, int renormalize, float scaling, float* out_w, int32_t* out_ids,
                               cudaStream_t stream);

cudaError_t launch_wait_timeout_selftest(int32_t* err, uint64_t timeout_ns, cudaStream_t stream);

struct GemmParams;
// epi: 0 = SiLU + requant (stage 1), 1 = weighted combine (stage 2).
// Both stages in one cooperative persistent launch (tiles of 16..64 tokens):
// stage-2 units of a chunk start once its stage-1 units released
// p1.chunk_ready (zeroed by the route kernel).
cudaError_t launch_grouped_gemm_fused(int tile_tokens, const CUtensorMap& tm_w1, const CUtensorMap& tm_a1,
                                      const GemmParams& p1, const CUtensorMap& tm_w2, const CUtensorMap& tm_a2,
                                      const GemmParams& p2, int grid, cudaStream_t stream);
// tm_o: stage 2's out_pair for the token-major tiles of 128 that store sorted
// rows with TMA (make_tmap_rows_bf16); any map otherwise (not read).
cudaError_t launch_grouped_gemm(int epi, int tile_tokens, const CUtensorMap& tm_w, const CUtensorMap& tm_a,
                                const CUtensorMap& tm_o, const GemmParams& p, int grid, cudaStream_t stream);
// Activation tile rows the kernel for this tile_tokens loads per stage (per CTA).
int gemm_tile_rows(int tile_tokens);
// Weight rows per TMA box (per CTA).
inline int gemm_weight_box_rows(int tile_tokens) { return tile_tokens == 256 ? 128 : 256; }

// Records a message for b200moe_last_error_message() and returns status.
int record_error(int status, const char* message);

}  // namespace b200moe
