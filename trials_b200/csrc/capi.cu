// extern "C" entry points: argument checks, workspace carving, TMA tensor
// maps and kernel sequencing. No function here allocates device memory or
// synchronises the stream, except b200moe_read_error (which exists to do so)
// and the set-up calls of the peer exchange buffer (b200moe_ep_peer_alloc).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>

#include "../../include/b200moe.h"
#include "launch.h"
#include "moe_gemm.cuh"
#include "router.cuh"

using namespace b200moe;

namespace {

thread_local char g_last_error[256] = "";

int fail(int status, const char* fmt, const char* detail = "") {
  snprintf(g_last_error, sizeof(g_last_error), fmt, detail);
  return status;
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return B200MOE_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, cudaGetErrorString(e));
  return B200MOE_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// ---- TMA descriptor encoding through the driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D byte matrix [rows][cols] (row pitch = cols), box = 128 bytes x box_rows,
// 128-byte swizzle (the K-major canonical layout of the tcgen05 descriptors).
int make_tmap_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable%s");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed%s");
  return B200MOE_OK;
}

// 2D bf16 matrix [rows][cols] (row pitch = cols elements), boxes of 64
// columns (128 bytes) x box_rows, 128-byte swizzle: the token-major stage-2
// output, stored from swizzled shared-memory staging.
int make_tmap_rows_bf16(CUtensorMap* m, void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable%s");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed%s");
  return B200MOE_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 1;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

bool valid_tile(int t) { return t == 16 || t == 32 || t == 64 || t == 128 || t == 256; }

int pick_tile_tokens(int64_t numel, int E_local) {
  const double avg = (double)numel / (double)(E_local > 0 ? E_local : 1);
  // 32-token tiles up to 26 routed rows per expert (measured: 1.641 vs 1.687 ms
  // at 832 tokens of top-8 over 256 experts; 64-token tiles win from 28 rows).
  if (avg <= 26.0) return 32;
  if (avg <= 48.0) return 64;
  return 128;  // 256 (CTA pairs) is available to staged callers; measured slower so far
}

constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per pipeline wait

// Chunks per unit group (unit_coords): token-major tiles have several chunks
// per expert at prefill, whose CTAs then share weight tiles through L2.
#ifndef B200MOE_CHUNK_GROUP_TOK
#define B200MOE_CHUNK_GROUP_TOK 4
#endif
#ifndef B200MOE_CHUNK_GROUP_SWAP
#define B200MOE_CHUNK_GROUP_SWAP 1
#endif

// From this many routed (token, slot) pairs on, the gather runs one warp per
// (token, segment) that quantises (or loads) the token's segment once and
// stores it to each of its slot rows, instead of one warp per (slot, segment):
// topk-fold fewer loads and conversions, at the cost of fewer, longer warps,
// which only pays at prefill sizes.
constexpr int64_t kFanOutMinPairs = 2048;
bool fan_out_tokens(int64_t numel, int topk) { return numel >= kFanOutMinPairs && topk <= 32; }

// Stage-2 output row layout of a tile size: token-major tiles (128, 256)
// write rows in sorted order, the swap-AB tiles one row per slot.
int pair_sorted_rows(int tile_tokens) { return tile_tokens > 64 ? 1 : 0; }

// Mixed work lists: with tiles of 16..64 tokens, experts whose padded rows
// exceed this many (a skewed router's hot experts) are cut into 128-row
// chunks for the token-major stages instead, in the same layer call. An
// expert has at most M rows, so this needs M > kHeavyRows, and the one-CTA
// routing (below 16,384 routed slots), which builds the two lists.
constexpr int kHeavyRows = 128;
int heavy_rows_for(int64_t M, int64_t numel, int tile) {
  return (tile <= 64 && M > kHeavyRows && route_ctas(numel) == 1) ? kHeavyRows : 0;
}

// The whole layer in one launch (the routing, the gather, both GEMM stages and
// the top-k reduce: EPI_WHOLE) applies with tiles of 16..64 tokens, one-CTA
// routing, no mixed lists and local results. Policy (b200moe_set_layer_launch):
// 0 = the form measured faster, 1 = one launch wherever it applies, 2 = never.
// Measured on the GLM layer (CUDA graphs, alternating): one launch 91 vs 83 us
// at 1 token, 3-4% slower at 64 and 128 tokens. Its routing and gather phases
// take 20 and 15 us inside the launch (one 352-thread CTA routes, on code and
// rows fetched cold after the weight stream), against 9 and 7 us as launches
// of their own; so the default (0) keeps the separate launches everywhere.
std::atomic<int> g_layer_launch{0};
constexpr int64_t kWholeAutoTokens = 0;  // batches up to this many tokens take one launch under policy 0
bool whole_layer_for(int64_t M, int64_t numel, int tile, int heavy_rows, bool peer) {
  const int mode = g_layer_launch.load();
  if (mode == 2 || tile > 64 || heavy_rows > 0 || route_ctas(numel) != 1 || peer) return false;
  return mode == 1 || M <= kWholeAutoTokens;
}

struct LayerPlan {
  int tile_tokens;
  int heavy_rows;  // > 0: mixed work lists (second list in off_ce2.., counters in off_ready2)
  int64_t rows_cap, chunks_cap, chunks_cap2, as_ld;
  size_t off_sorted, off_pos, off_ce, off_cr0, off_crows, off_ready, off_counts, off_a1, off_a1s, off_a2, off_a2s,
      off_pair, off_rscratch, off_ce2, off_cr0_2, off_crows2, off_ready2, total;
  int64_t rscratch_ints;  // routing on several CTAs (large batches)
};

// tile = 0: the tile size picked for M*topk routed slots.
LayerPlan plan_layer(int64_t M, int64_t H, int64_t I, int E_local, int topk, int tile = 0) {
  LayerPlan p{};
  const int64_t numel = M * topk;
  p.tile_tokens = tile > 0 ? tile : pick_tile_tokens(numel, E_local);
  p.heavy_rows = heavy_rows_for(M, numel, p.tile_tokens);
  p.rows_cap = b200moe_route_capacity_rows(numel, E_local);
  p.chunks_cap = b200moe_route_capacity_chunks(numel, E_local, p.tile_tokens);
  p.chunks_cap2 = p.heavy_rows ? b200moe_route_capacity_chunks(numel, E_local, kHeavyTile) : 0;
  p.as_ld = round_up(p.rows_cap + 256, 64);
  size_t off = 256;  // device error word
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (size_t)round_up((int64_t)bytes, 256);
    return o;
  };
  p.off_sorted = take(sizeof(int32_t) * p.rows_cap);
  p.off_pos = take(sizeof(int32_t) * (numel > 0 ? numel : 1));
  p.off_ce = take(sizeof(int32_t) * p.chunks_cap);
  p.off_cr0 = take(sizeof(int32_t) * p.chunks_cap);
  p.off_crows = take(sizeof(int32_t) * p.chunks_cap);
  p.off_ready = take(sizeof(int32_t) * (p.chunks_cap + 2));
  p.off_counts = take(sizeof(int32_t) * 4);
  p.off_a1 = take((size_t)p.rows_cap * H);
  p.off_a1s = take(sizeof(float) * (size_t)(H / 128) * p.as_ld);
  p.off_a2 = take((size_t)p.rows_cap * I);
  p.off_a2s = take(sizeof(float) * (size_t)(I / 128) * p.as_ld);
  // Token-major tiles write sorted rows (rows_cap of them), the others slot rows.
  p.off_pair = take(sizeof(__nv_bfloat16) * (size_t)(pair_sorted_rows(p.tile_tokens) ? p.rows_cap : numel) * H);
  p.rscratch_ints = route_scratch_ints(numel, E_local);
  if (p.rscratch_ints > 0) p.off_rscratch = take(sizeof(int32_t) * (size_t)p.rscratch_ints);
  if (p.heavy_rows) {
    p.off_ce2 = take(sizeof(int32_t) * p.chunks_cap2);
    p.off_cr0_2 = take(sizeof(int32_t) * p.chunks_cap2);
    p.off_crows2 = take(sizeof(int32_t) * p.chunks_cap2);
    p.off_ready2 = take(sizeof(int32_t) * 2);
  }
  p.total = off;
  return p;
}

int check_gemm_shapes(int64_t H, int64_t I) {
  if (H <= 0 || I <= 0 || H % 256 != 0 || I % 128 != 0)
    return fail(B200MOE_ERR_UNSUPPORTED, "hidden must be a multiple of 256 and intermediate of 128%s");
  if (H > (1 << 20) || I > (1 << 20)) return fail(B200MOE_ERR_UNSUPPORTED, "dimension too large%s");
  return B200MOE_OK;
}

// Tensor maps and the operand / work-list fields of one grouped GEMM stage.
int prep_gemm(const uint8_t* a_q, const float* a_sT, int64_t as_ld, int64_t rows_cap, const uint8_t* w,
              const float* w_scale, int E_local, int64_t Nw, int64_t K, const int32_t* ce, const int32_t* cr0,
              const int32_t* crows, const int32_t* n_chunks, int tile_tokens, GemmParams& p, CUtensorMap& tm_w,
              CUtensorMap& tm_a) {
  int st = make_tmap_u8(&tm_w, w, (int64_t)E_local * Nw, K, gemm_weight_box_rows(tile_tokens));
  if (st) return st;
  st = make_tmap_u8(&tm_a, a_q, rows_cap, K, gemm_tile_rows(tile_tokens));
  if (st) return st;
  p.chunk_expert = ce;
  p.chunk_row0 = cr0;
  p.chunk_rows = crows;
  p.n_chunks = n_chunks;
  p.w_scale = w_scale;
  p.a_sT = a_sT;
  p.as_ld = as_ld;
  p.K = (int)K;
  p.Nw = (int)Nw;
  p.timeout_ns = kTimeoutNs;
  p.chunk_group = tile_tokens > 64 ? B200MOE_CHUNK_GROUP_TOK : B200MOE_CHUNK_GROUP_SWAP;
  return B200MOE_OK;
}

int run_gemm(int epi, const uint8_t* a_q, const float* a_sT, int64_t as_ld, int64_t rows_cap, const uint8_t* w,
             const float* w_scale, int E_local, int64_t Nw, int64_t K, const int32_t* ce, const int32_t* cr0,
             const int32_t* crows, const int32_t* n_chunks, int64_t chunks_cap, int tile_tokens, GemmParams p,
             int grid_ctas, cudaStream_t stream) {
  CUtensorMap tm_w, tm_a;
  int st = prep_gemm(a_q, a_sT, as_ld, rows_cap, w, w_scale, E_local, Nw, K, ce, cr0, crows, n_chunks, tile_tokens,
                     p, tm_w, tm_a);
  if (st) return st;
  // Token-major stage 2 (tiles of 128) stores its sorted rows with TMA.
  CUtensorMap tm_o = tm_w;
  if (epi == EPI_COMBINE && tile_tokens == 128 && !p.rows_by_slot) {
    if (!aligned16(p.out_pair)) return fail(B200MOE_ERR_UNSUPPORTED, "out_pair: 16-byte alignment required%s");
    st = make_tmap_rows_bf16(&tm_o, p.out_pair, rows_cap, Nw, 16);
    if (st) return st;
  }
  const int64_t units_cap = chunks_cap * (Nw / 256);
  int64_t grid = grid_ctas > 0 ? grid_ctas : sm_count();
  if (grid > units_cap) grid = units_cap;
  return cuda_status(launch_grouped_gemm(epi, tile_tokens, tm_w, tm_a, tm_o, p, (int)grid, stream), "grouped gemm");
}

}  // namespace

namespace b200moe {
int record_error(int status, const char* message) { return fail(status, "%s", message); }
}  // namespace b200moe

namespace {

// Host checks of the router arguments (b200moe_router_topk and routing from logits).
int check_router(const char* name, const void* logits, int64_t M, int num_experts, int topk, int scoring,
                 const float* correction_bias, const float* topk_weights, const int32_t* topk_ids) {
  if (M < 0 || num_experts <= 0 || topk <= 0 || topk > num_experts || (scoring != 0 && scoring != 1) ||
      (M > 0 && (!logits || !topk_weights || !topk_ids)) || (correction_bias && scoring != 1))
    return fail(B200MOE_ERR_INVALID_ARG, "%s: bad router argument", name);
  if (num_experts > 1024 || topk > kRouterMaxTopk)
    return fail(B200MOE_ERR_UNSUPPORTED, "%s: at most 1024 experts and top-16", name);
  return B200MOE_OK;
}

}  // namespace

extern "C" {

int b200moe_version(void) { return 100; }

const char* b200moe_status_string(int status) {
  switch (status) {
    case B200MOE_OK:
      return "ok";
    case B200MOE_ERR_INVALID_ARG:
      return "invalid argument";
    case B200MOE_ERR_UNSUPPORTED:
      return "unsupported shape or option";
    case B200MOE_ERR_WORKSPACE:
      return "workspace too small";
    case B200MOE_ERR_CUDA:
      return "CUDA error";
    default:
      return "unknown status";
  }
}

const char* b200moe_last_error_message(void) { return g_last_error; }

int64_t b200moe_align_capacity_rows(int64_t numel, int num_experts, int block_m) {
  return numel + (int64_t)(num_experts + 1) * (block_m - 1);
}

int64_t b200moe_align_capacity_blocks(int64_t numel, int num_experts, int block_m) {
  return ceil_div(b200moe_align_capacity_rows(numel, num_experts, block_m), block_m);
}

int b200moe_align(const int32_t* topk_ids, int64_t M, int topk, int num_experts, int block_m,
                  const int32_t* expert_map, int num_local_experts, int32_t* sorted_token_ids,
                  int64_t sorted_capacity, int32_t* expert_ids, int64_t blocks_capacity,
                  int32_t* num_tokens_post_pad, int32_t* err_word, void* stream) {
  if (M < 0 || topk <= 0 || num_experts <= 0 || block_m <= 0 || !sorted_token_ids || !num_tokens_post_pad ||
      !err_word || (M > 0 && !topk_ids))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_align: bad argument%s");
  const int E = expert_map ? num_local_experts : num_experts;
  if (E <= 0 || E > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_align: 1..1024 experts supported%s");
  const int64_t numel = M * topk;
  if (numel > INT32_MAX / 2) return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_align: too many tokens%s");
  if (sorted_capacity < b200moe_align_capacity_rows(numel, E, block_m) ||
      (expert_ids && blocks_capacity < b200moe_align_capacity_blocks(numel, E, block_m)))
    return fail(B200MOE_ERR_WORKSPACE, "b200moe_align: output capacity too small%s");
  AlignArgs a{};
  a.topk_ids = topk_ids;
  a.n = numel;
  a.num_experts = num_experts;
  a.expert_map = expert_map;
  a.E = E;
  a.block_m = block_m;
  a.sentinel = (int32_t)numel;
  a.sorted_ids = sorted_token_ids;
  a.sorted_cap = sorted_capacity;
  a.expert_ids = expert_ids;
  a.blocks_cap = blocks_capacity;
  a.ntp = num_tokens_post_pad;
  a.err = err_word;
  return cuda_status(launch_align(a, (cudaStream_t)stream), "align");
}

int b200moe_quant_1x128(const void* x, int64_t M, int64_t K, int64_t ldx, uint8_t* q, int64_t ldq, float* s,
                        int64_t s_stride_row, int64_t s_stride_group, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0 || ldx < K || ldq < K || (M > 0 && (!x || !q || !s)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_quant_1x128: bad argument%s");
  if (!aligned16(x) || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(q) & 7) || ldq % 8 != 0)
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_quant_1x128: x rows must be 16-byte aligned, q rows 8-byte%s");
  QuantArgs a{};
  a.x = x;
  a.ldx = ldx;
  a.K = K;
  a.rows = M;
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  a.s_row = s_stride_row;
  a.s_grp = s_stride_group;
  return cuda_status(launch_quant_1x128(a, (cudaStream_t)stream), "quant_1x128");
}

int b200moe_quant_block128(const void* w, int64_t E, int64_t N, int64_t K, uint8_t* q, float* s, void* stream) {
  if (E < 0 || N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0 || (E > 0 && (!w || !q || !s)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_quant_block128: bad argument%s");
  if (!aligned16(w) || !aligned16(q) || E > 65535 || N / 128 > 65535)
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_quant_block128: alignment or size%s");
  return cuda_status(launch_quant_block128(w, E, N, K, q, s, (cudaStream_t)stream), "quant_block128");
}

int64_t b200moe_route_capacity_rows(int64_t numel, int num_local_experts) {
  return numel + (int64_t)num_local_experts * 15;
}

int64_t b200moe_route_capacity_chunks(int64_t numel, int num_local_experts, int tile_tokens) {
  if (tile_tokens <= 0) return 0;
  return ceil_div(b200moe_route_capacity_rows(numel, num_local_experts), tile_tokens) + num_local_experts;
}

int64_t b200moe_route_scratch_ints(int64_t numel, int num_local_experts) {
  if (numel < 0 || num_local_experts <= 0) return 0;
  return route_scratch_ints(numel, num_local_experts);
}

}  // extern "C"

namespace {

// The second (heavy) work list of mixed routing.
struct MixedLists {
  int heavy_rows;
  int32_t* chunk_expert;
  int32_t* chunk_row0;
  int32_t* chunk_rows;
  int64_t chunks_cap;
  int32_t* n_chunks;
  int32_t* heavy_row0;
  int32_t* counters;  // 2 ints, zeroed: the unit counters of the two token-major stages
};

// The AlignArgs of one routing call, after the checks every routing entry
// point shares.
int make_align(const int32_t* topk_ids, int64_t M, int topk, int num_experts, const int32_t* expert_map,
               int num_local_experts, int tile_tokens, int32_t* sorted_ids, int64_t rows_capacity,
               int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows, int64_t chunks_capacity,
               int32_t* n_chunks, int32_t* num_rows, int32_t* slot_pos, int32_t* chunk_ready, int32_t* err_word,
               const MixedLists* mixed, AlignArgs& a) {
  if (M < 0 || topk <= 0 || num_experts <= 0 || !valid_tile(tile_tokens) || !sorted_ids || !chunk_expert ||
      !chunk_row0 || !chunk_rows || !n_chunks || !num_rows || !err_word || (M > 0 && !topk_ids))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_route: bad argument%s");
  const int E = expert_map ? num_local_experts : num_experts;
  if (E <= 0 || E > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_route: 1..1024 experts supported%s");
  const int64_t numel = M * topk;
  if (numel > INT32_MAX / 2) return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_route: too many tokens%s");
  if (rows_capacity < b200moe_route_capacity_rows(numel, E) ||
      chunks_capacity < b200moe_route_capacity_chunks(numel, E, tile_tokens))
    return fail(B200MOE_ERR_WORKSPACE, "b200moe_route: capacity too small%s");
  a = AlignArgs{};
  a.topk_ids = topk_ids;
  a.n = numel;
  a.num_experts = num_experts;
  a.expert_map = expert_map;
  a.E = E;
  a.block_m = 16;
  a.sentinel = (int32_t)numel;
  a.sorted_ids = sorted_ids;
  a.sorted_cap = rows_capacity;
  a.expert_ids = nullptr;
  a.ntp = num_rows;
  a.tile_tokens = tile_tokens;
  a.chunk_expert = chunk_expert;
  a.chunk_row0 = chunk_row0;
  a.chunk_rows = chunk_rows;
  a.chunks_cap = chunks_capacity;
  a.n_chunks = n_chunks;
  a.chunk_ready = chunk_ready;
  a.slot_pos = slot_pos;
  a.err = err_word;
  if (mixed && mixed->heavy_rows > 0) {
    if (route_ctas(numel) != 1 || tile_tokens > 64 || !mixed->chunk_expert || !mixed->chunk_row0 ||
        !mixed->chunk_rows || !mixed->n_chunks || !mixed->heavy_row0 || !mixed->counters ||
        mixed->chunks_cap < b200moe_route_capacity_chunks(numel, E, kHeavyTile))
      return fail(B200MOE_ERR_INVALID_ARG, "mixed work lists: bad argument (tiles of 16..64 tokens, below 16,384 "
                                           "routed slots, heavy list capacity)%s");
    a.heavy_rows = mixed->heavy_rows;
    a.chunk_expert2 = mixed->chunk_expert;
    a.chunk_row0_2 = mixed->chunk_row0;
    a.chunk_rows2 = mixed->chunk_rows;
    a.chunks_cap2 = mixed->chunks_cap;
    a.n_chunks2 = mixed->n_chunks;
    a.heavy_row0 = mixed->heavy_row0;
    a.counters2 = mixed->counters;
  }
  return B200MOE_OK;
}

// b200moe_route, and b200moe_route_logits when `router` is set (topk_ids then
// names the router's id output, which routing reads after the router stored it).
int route_impl(const int32_t* topk_ids, int64_t M, int topk, int num_experts, const int32_t* expert_map,
               int num_local_experts, int tile_tokens, int32_t* sorted_ids, int64_t rows_capacity,
               int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows, int64_t chunks_capacity,
               int32_t* n_chunks, int32_t* num_rows, int32_t* slot_pos, int32_t* chunk_ready,
               int32_t* route_scratch, int64_t route_scratch_ints, int32_t* err_word, void* stream,
               const RouterArgs* router, int32_t* router_counter, const MixedLists* mixed = nullptr,
               const PackedMeta* packed = nullptr) {
  AlignArgs a;
  const int st = make_align(topk_ids, M, topk, num_experts, expert_map, num_local_experts, tile_tokens, sorted_ids,
                            rows_capacity, chunk_expert, chunk_row0, chunk_rows, chunks_capacity, n_chunks, num_rows,
                            slot_pos, chunk_ready, err_word, mixed, a);
  if (st) return st;
  const int E = a.E;
  const int64_t numel = a.n;
  if (router) {
    // The CTA counter: router_counter, or the first ints of route_scratch.
    int32_t* counts = router_counter ? route_scratch : route_scratch + kRouteLogitsCounterInts;
    const int64_t counts_ints = router_counter ? route_scratch_ints : route_scratch_ints - kRouteLogitsCounterInts;
    int32_t* counter = router_counter ? router_counter : route_scratch;
    const int64_t need = b200moe::route_scratch_ints(numel, E);
    if (!counter || counts_ints < need || (need > 0 && !counts))
      return fail(B200MOE_ERR_WORKSPACE, "b200moe_route_logits: route_scratch too small%s");
    return cuda_status(launch_route_logits(a, *router, M, counter, counts, (cudaStream_t)stream), "route_logits");
  }
  if (packed) {
    // Received expert-parallel rows: the routing launch also waits for them and
    // unpacks their ids and weights; with several routing CTAs the unpack is a
    // launch of its own first.
    const int C = route_ctas(numel);
    if (C == 1 || a.heavy_rows > 0 || !route_scratch || route_scratch_ints < (int64_t)C * E)
      return cuda_status(launch_align_packed(a, *packed, (cudaStream_t)stream), "route_packed");
    const int st = cuda_status(launch_ep_unpack_meta_peer(packed->own, packed->rows, packed->R, packed->row_bytes,
                                                          packed->H, packed->topk, packed->G, packed->epoch,
                                                          packed->ids, packed->w, err_word, packed->limit_ns,
                                                          (cudaStream_t)stream),
                               "ep_unpack_meta_peer");
    if (st) return st;
  }
  return cuda_status(launch_route(a, route_scratch, route_scratch_ints, (cudaStream_t)stream), "route");
}

}  // namespace

extern "C" {

int b200moe_route(const int32_t* topk_ids, int64_t M, int topk, int num_experts, const int32_t* expert_map,
                  int num_local_experts, int tile_tokens, int32_t* sorted_ids, int64_t rows_capacity,
                  int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows, int64_t chunks_capacity,
                  int32_t* n_chunks, int32_t* num_rows, int32_t* slot_pos, int32_t* chunk_ready,
                  int32_t* route_scratch, int64_t route_scratch_ints, int32_t* err_word, void* stream) {
  return route_impl(topk_ids, M, topk, num_experts, expert_map, num_local_experts, tile_tokens, sorted_ids,
                    rows_capacity, chunk_expert, chunk_row0, chunk_rows, chunks_capacity, n_chunks, num_rows,
                    slot_pos, chunk_ready, route_scratch, route_scratch_ints, err_word, stream, nullptr, nullptr);
}

int b200moe_heavy_rows(int64_t M, int topk, int tile_tokens) {
  if (M < 0 || topk <= 0) return 0;
  return heavy_rows_for(M, M * topk, tile_tokens);
}

int b200moe_route_mixed(const int32_t* topk_ids, int64_t M, int topk, int num_experts, const int32_t* expert_map,
                        int num_local_experts, int tile_tokens, int heavy_rows, int32_t* sorted_ids,
                        int64_t rows_capacity, int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows,
                        int64_t chunks_capacity, int32_t* heavy_chunk_expert, int32_t* heavy_chunk_row0,
                        int32_t* heavy_chunk_rows, int64_t heavy_chunks_capacity, int32_t* counts,
                        int32_t* slot_pos, int32_t* chunk_ready, int32_t* heavy_counters, int32_t* err_word,
                        void* stream) {
  if (heavy_rows <= 0 || !counts)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_route_mixed: heavy_rows must be positive%s");
  const MixedLists mx{heavy_rows, heavy_chunk_expert, heavy_chunk_row0, heavy_chunk_rows, heavy_chunks_capacity,
                      counts + 2, counts + 3, heavy_counters};
  return route_impl(topk_ids, M, topk, num_experts, expert_map, num_local_experts, tile_tokens, sorted_ids,
                    rows_capacity, chunk_expert, chunk_row0, chunk_rows, chunks_capacity, counts, counts + 1,
                    slot_pos, chunk_ready, nullptr, 0, err_word, stream, nullptr, nullptr, &mx);
}

int64_t b200moe_route_logits_scratch_ints(int64_t numel, int num_local_experts) {
  if (numel < 0 || num_local_experts <= 0) return 0;
  return route_logits_scratch_ints(numel, num_local_experts);
}

int b200moe_route_logits(const void* logits, int logits_bf16, int64_t M, int num_experts, int topk, int scoring,
                         const float* correction_bias, int renormalize, float scaling, float* topk_weights,
                         int32_t* topk_ids, const int32_t* expert_map, int num_local_experts, int tile_tokens,
                         int32_t* sorted_ids, int64_t rows_capacity, int32_t* chunk_expert, int32_t* chunk_row0,
                         int32_t* chunk_rows, int64_t chunks_capacity, int32_t* n_chunks, int32_t* num_rows,
                         int32_t* slot_pos, int32_t* chunk_ready, int32_t* route_scratch,
                         int64_t route_scratch_ints, int32_t* err_word, void* stream) {
  int st = check_router("b200moe_route_logits", logits, M, num_experts, topk, scoring, correction_bias, topk_weights,
                        topk_ids);
  if (st) return st;
  const RouterArgs r{logits, logits_bf16 ? 1 : 0, num_experts, topk, scoring, renormalize ? 1 : 0,
                     correction_bias, scaling, topk_weights, topk_ids};
  return route_impl(topk_ids, M, topk, num_experts, expert_map, num_local_experts, tile_tokens, sorted_ids,
                    rows_capacity, chunk_expert, chunk_row0, chunk_rows, chunks_capacity, n_chunks, num_rows,
                    slot_pos, chunk_ready, route_scratch, route_scratch_ints, err_word, stream, &r, nullptr);
}

int b200moe_gather_quant(const void* hidden, int64_t M, int64_t H, int topk, const int32_t* slot_pos,
                         int64_t rows_capacity, uint8_t* a_q, float* a_sT, int64_t a_s_ld, void* stream) {
  if (M < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || rows_capacity < 0 || a_s_ld < rows_capacity ||
      (M > 0 && (!hidden || !slot_pos || !a_q || !a_sT)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_gather_quant: bad argument%s");
  if (!aligned16(hidden) || (reinterpret_cast<uintptr_t>(a_q) & 7))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_gather_quant: alignment%s");
  QuantArgs a{};
  a.x = hidden;
  a.ldx = H;
  a.K = H;
  // Large batches: one launch row per token, quantised once and stored to each
  // of its slot rows; small ones: one launch row per flat slot.
  const bool fan = fan_out_tokens(M * topk, topk);
  a.rows = fan ? M : M * topk;
  a.fanout = fan ? 1 : 0;
  a.slot_pos = slot_pos;
  a.topk = topk;
  a.sentinel = (int32_t)(M * topk);
  a.q = a_q;
  a.ldq = H;
  a.s = a_sT;
  a.s_row = 1;
  a.s_grp = a_s_ld;
  return cuda_status(launch_quant_1x128(a, (cudaStream_t)stream), "gather_quant");
}

int b200moe_gather_rows(const uint8_t* xq, const float* xs, int64_t ldxq, int64_t ldxs, int64_t M, int64_t H, int topk,
                        const int32_t* slot_pos, int64_t rows_capacity, uint8_t* a_q, float* a_sT, int64_t a_s_ld,
                        void* stream) {
  if (M < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || rows_capacity < 0 || a_s_ld < rows_capacity ||
      ldxq < H || ldxs < H / 128 || (M > 0 && (!xq || !xs || !slot_pos || !a_q || !a_sT)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_gather_rows: bad argument%s");
  if (!aligned16(xq) || ldxq % 16 != 0 || !aligned16(a_q) || H % 16 != 0)
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_gather_rows: fp8 rows must be 16-byte aligned%s");
  QuantArgs a{};
  a.xq = xq;
  a.ldxq = ldxq;
  a.xs = xs;
  a.ldxs = ldxs;
  a.K = H;
  const bool fan = fan_out_tokens(M * topk, topk);  // as b200moe_gather_quant
  a.rows = fan ? M : M * topk;
  a.fanout = fan ? 1 : 0;
  a.slot_pos = slot_pos;
  a.topk = topk;
  a.sentinel = (int32_t)(M * topk);
  a.q = a_q;
  a.ldq = H;
  a.s = a_sT;
  a.s_row = 1;
  a.s_grp = a_s_ld;
  return cuda_status(launch_quant_1x128(a, (cudaStream_t)stream), "gather_rows");
}

}  // extern "C"

namespace {

// The stage launches behind b200moe_gemm1_silu / b200moe_gemm2_combine;
// unit_counter (zeroed, or nullptr) gives token-major tiles a dynamic unit queue.
int gemm1_silu_core(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                    const uint8_t* w13, const float* w13_scale, int num_local_experts, int64_t H, int64_t I,
                    const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                    const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens, uint8_t* a2_q,
                    float* a2_sT, int32_t* err_word, int grid_ctas, void* stream, int32_t* unit_counter) {
  int st = check_gemm_shapes(H, I);
  if (st) return st;
  if (!valid_tile(tile_tokens) || num_local_experts <= 0 || rows_capacity <= 0 ||
      a_s_ld < rows_capacity + (tile_tokens < 32 ? 32 : tile_tokens) || a_s_ld % 4 != 0 || !a1_q || !a1_sT || !w13 ||
      !w13_scale || !chunk_expert || !chunk_row0 || !chunk_rows || !n_chunks || !a2_q || !a2_sT || !err_word)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_gemm1_silu: bad argument%s");
  if (!aligned16(a1_q) || !aligned16(w13) || !aligned16(a1_sT) || !aligned16(a2_q))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_gemm1_silu: 16-byte alignment required%s");
  GemmParams p{};
  p.out_q = a2_q;
  p.out_q_ld = I;
  p.out_sT = a2_sT;
  p.out_s_ld = a_s_ld;
  p.err = err_word;
  p.unit_counter = unit_counter;
  return run_gemm(EPI_SILU, a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, 2 * I, H,
                  chunk_expert, chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens, p, grid_ctas,
                  (cudaStream_t)stream);
}

int gemm2_combine_core(const uint8_t* a2_q, const float* a2_sT, int64_t a_s_ld, int64_t rows_capacity,
                       const uint8_t* w2, const float* w2_scale, int num_local_experts, int64_t H, int64_t I,
                       const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                       const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens,
                       const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk,
                       void* out_pair, int32_t* err_word, int grid_ctas, void* stream, int32_t* unit_counter,
                       int rows_by_slot = 0) {
  int st = check_gemm_shapes(H, I);
  if (st) return st;
  if (!valid_tile(tile_tokens) || num_local_experts <= 0 || rows_capacity <= 0 || M < 0 || topk <= 0 ||
      a_s_ld < rows_capacity + (tile_tokens < 32 ? 32 : tile_tokens) || a_s_ld % 4 != 0 || !a2_q || !a2_sT || !w2 ||
      !w2_scale || !chunk_expert || !chunk_row0 || !chunk_rows || !n_chunks || !sorted_ids || !topk_weights ||
      !out_pair || !err_word)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_gemm2_combine: bad argument%s");
  if (!aligned16(a2_q) || !aligned16(w2) || !aligned16(a2_sT))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_gemm2_combine: 16-byte alignment required%s");
  GemmParams p{};
  p.sorted_ids = sorted_ids;
  p.topk_w = topk_weights;
  p.sentinel = (int32_t)(M * topk);
  p.out_pair = static_cast<__nv_bfloat16*>(out_pair);
  p.rows_by_slot = rows_by_slot;
  p.err = err_word;
  p.unit_counter = unit_counter;
  return run_gemm(EPI_COMBINE, a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I,
                  chunk_expert, chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens, p, grid_ctas,
                  (cudaStream_t)stream);
}

// The token-major stages on the heavy list of mixed routing (128-row chunks,
// units from the two counters), stage-2 rows by slot like the swap-AB tiles.
int experts_heavy_core(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                       const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                       int num_local_experts, int64_t H, int64_t I, const int32_t* chunk_expert,
                       const int32_t* chunk_row0, const int32_t* chunk_rows, const int32_t* n_chunks,
                       int64_t chunks_capacity, int32_t* counters, uint8_t* a2_q, float* a2_sT,
                       const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk, void* out_pair,
                       int32_t* err_word, int grid_ctas, void* stream) {
  if (!counters) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_experts_heavy: null counters%s");
  int st = gemm1_silu_core(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, H, I,
                           chunk_expert, chunk_row0, chunk_rows, n_chunks, chunks_capacity, kHeavyTile, a2_q, a2_sT,
                           err_word, grid_ctas, stream, counters);
  if (st) return st;
  return gemm2_combine_core(a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I, chunk_expert,
                            chunk_row0, chunk_rows, n_chunks, chunks_capacity, kHeavyTile, sorted_ids, topk_weights,
                            M, topk, out_pair, err_word, grid_ctas, stream, counters + 1, /*rows_by_slot=*/1);
}

}  // namespace

extern "C" {

int b200moe_gemm1_silu(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                       const uint8_t* w13, const float* w13_scale, int num_local_experts, int64_t H, int64_t I,
                       const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                       const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens, uint8_t* a2_q,
                       float* a2_sT, int32_t* err_word, int grid_ctas, void* stream) {
  return gemm1_silu_core(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, H, I, chunk_expert,
                         chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens, a2_q, a2_sT, err_word,
                         grid_ctas, stream, nullptr);
}

int b200moe_gemm2_combine(const uint8_t* a2_q, const float* a2_sT, int64_t a_s_ld, int64_t rows_capacity,
                          const uint8_t* w2, const float* w2_scale, int num_local_experts, int64_t H, int64_t I,
                          const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                          const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens,
                          const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk,
                          void* out_pair, int32_t* err_word, int grid_ctas, void* stream) {
  return gemm2_combine_core(a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I, chunk_expert,
                            chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens, sorted_ids,
                            topk_weights, M, topk, out_pair, err_word, grid_ctas, stream, nullptr);
}

int b200moe_experts(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                    const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                    int num_local_experts, int64_t H, int64_t I, const int32_t* chunk_expert,
                    const int32_t* chunk_row0, const int32_t* chunk_rows, const int32_t* n_chunks,
                    int64_t chunks_capacity, int32_t* chunk_ready, int tile_tokens, uint8_t* a2_q, float* a2_sT,
                    const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk, void* out_pair,
                    int32_t* err_word, int grid_ctas, void* stream) {
  if (tile_tokens > 64) {
    // Token-major tiles: the two stages as two launches, each taking its units
    // from a counter after chunk_ready's per-chunk entries (zeroed by routing).
    int32_t* q1 = chunk_ready ? chunk_ready + chunks_capacity : nullptr;
    int st = gemm1_silu_core(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, H, I,
                             chunk_expert, chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens, a2_q,
                             a2_sT, err_word, grid_ctas, stream, q1);
    if (st) return st;
    return gemm2_combine_core(a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I,
                              chunk_expert, chunk_row0, chunk_rows, n_chunks, chunks_capacity, tile_tokens,
                              sorted_ids, topk_weights, M, topk, out_pair, err_word, grid_ctas, stream,
                              q1 ? q1 + 1 : nullptr);
  }
  int st = check_gemm_shapes(H, I);
  if (st) return st;
  if (!valid_tile(tile_tokens) || num_local_experts <= 0 || rows_capacity <= 0 || M < 0 || topk <= 0 ||
      a_s_ld < rows_capacity + (tile_tokens < 32 ? 32 : tile_tokens) || a_s_ld % 4 != 0 || !a1_q || !a1_sT ||
      !w13 || !w13_scale || !w2 || !w2_scale || !chunk_expert || !chunk_row0 || !chunk_rows || !n_chunks ||
      !chunk_ready || !a2_q || !a2_sT || !sorted_ids || !topk_weights || !out_pair || !err_word)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_experts: bad argument%s");
  if (!aligned16(a1_q) || !aligned16(w13) || !aligned16(a1_sT) || !aligned16(a2_q) || !aligned16(w2) ||
      !aligned16(a2_sT))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_experts: 16-byte alignment required%s");
  GemmParams p1{}, p2{};
  CUtensorMap tw1, ta1, tw2, ta2;
  st = prep_gemm(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, 2 * I, H, chunk_expert,
                 chunk_row0, chunk_rows, n_chunks, tile_tokens, p1, tw1, ta1);
  if (st) return st;
  st = prep_gemm(a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I, chunk_expert, chunk_row0,
                 chunk_rows, n_chunks, tile_tokens, p2, tw2, ta2);
  if (st) return st;
  p1.out_q = a2_q;
  p1.out_q_ld = I;
  p1.out_sT = a2_sT;
  p1.out_s_ld = a_s_ld;
  p1.chunk_ready = chunk_ready;
  p1.unit_counter = chunk_ready + chunks_capacity;  // zeroed by routing with the per-chunk entries
  p1.err = err_word;
  p2.sorted_ids = sorted_ids;
  p2.topk_w = topk_weights;
  p2.sentinel = (int32_t)(M * topk);
  p2.out_pair = static_cast<__nv_bfloat16*>(out_pair);
  p2.err = err_word;
  const int64_t units_cap = chunks_capacity * ((2 * I) / 256 + H / 256);
  int64_t grid = grid_ctas > 0 ? grid_ctas : sm_count();
  if (grid > units_cap) grid = units_cap;
  return cuda_status(launch_grouped_gemm_fused(tile_tokens, tw1, ta1, p1, tw2, ta2, p2, (int)grid,
                                               (cudaStream_t)stream),
                     "experts");
}

int b200moe_experts_heavy(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                          const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                          int num_local_experts, int64_t H, int64_t I, const int32_t* heavy_chunk_expert,
                          const int32_t* heavy_chunk_row0, const int32_t* heavy_chunk_rows,
                          const int32_t* n_heavy_chunks, int64_t heavy_chunks_capacity, int32_t* heavy_counters,
                          uint8_t* a2_q, float* a2_sT, const int32_t* sorted_ids, const float* topk_weights,
                          int64_t M, int topk, void* out_pair, int32_t* err_word, int grid_ctas, void* stream) {
  return experts_heavy_core(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, w2, w2_scale, num_local_experts, H,
                            I, heavy_chunk_expert, heavy_chunk_row0, heavy_chunk_rows, n_heavy_chunks,
                            heavy_chunks_capacity, heavy_counters, a2_q, a2_sT, sorted_ids, topk_weights, M, topk,
                            out_pair, err_word, grid_ctas, stream);
}

int b200moe_experts_fused(const void* hidden, int64_t M, int topk, const int32_t* slot_pos, uint8_t* a1_q,
                          float* a1_sT, int64_t a_s_ld, int64_t rows_capacity, const uint8_t* w13,
                          const float* w13_scale, const uint8_t* w2, const float* w2_scale, int num_local_experts,
                          int64_t H, int64_t I, const int32_t* chunk_expert, const int32_t* chunk_row0,
                          const int32_t* chunk_rows, const int32_t* n_chunks, int64_t chunks_capacity,
                          int32_t* chunk_ready, int tile_tokens, uint8_t* a2_q, float* a2_sT,
                          const int32_t* sorted_ids, const float* topk_weights, void* out_pair, void* out,
                          int32_t* err_word, int grid_ctas, void* stream) {
  int st = check_gemm_shapes(H, I);
  if (st) return st;
  if (tile_tokens > 64)
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_experts_fused: tiles of 16..64 tokens only%s");
  if (!valid_tile(tile_tokens) || num_local_experts <= 0 || rows_capacity <= 0 || M <= 0 || topk <= 0 ||
      a_s_ld < rows_capacity + (tile_tokens < 32 ? 32 : tile_tokens) || a_s_ld % 4 != 0 || !hidden || !slot_pos ||
      !a1_q || !a1_sT || !w13 || !w13_scale || !w2 || !w2_scale || !chunk_expert || !chunk_row0 || !chunk_rows ||
      !n_chunks || !chunk_ready || !a2_q || !a2_sT || !sorted_ids || !topk_weights || !out_pair || !out ||
      !err_word)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_experts_fused: bad argument%s");
  if (!aligned16(hidden) || !aligned16(a1_q) || !aligned16(w13) || !aligned16(a1_sT) || !aligned16(a2_q) ||
      !aligned16(w2) || !aligned16(a2_sT) || !aligned16(out_pair) || !aligned16(out))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_experts_fused: 16-byte alignment required%s");
  GemmParams p1{}, p2{};
  CUtensorMap tw1, ta1, tw2, ta2;
  st = prep_gemm(a1_q, a1_sT, a_s_ld, rows_capacity, w13, w13_scale, num_local_experts, 2 * I, H, chunk_expert,
                 chunk_row0, chunk_rows, n_chunks, tile_tokens, p1, tw1, ta1);
  if (st) return st;
  st = prep_gemm(a2_q, a2_sT, a_s_ld, rows_capacity, w2, w2_scale, num_local_experts, H, I, chunk_expert, chunk_row0,
                 chunk_rows, n_chunks, tile_tokens, p2, tw2, ta2);
  if (st) return st;
  p1.out_q = a2_q;
  p1.out_q_ld = I;
  p1.out_sT = a2_sT;
  p1.out_s_ld = a_s_ld;
  p1.chunk_ready = chunk_ready;
  p1.phase_count = chunk_ready + chunks_capacity;
  p1.err = err_word;
  // phase 0: quantise each routed slot's hidden row into its sorted row
  p1.q0.x = hidden;
  p1.q0.ldx = H;
  p1.q0.K = H;
  p1.q0.rows = M * topk;
  p1.q0.slot_pos = slot_pos;
  p1.q0.topk = topk;
  p1.q0.sentinel = (int32_t)(M * topk);
  p1.q0.q = a1_q;
  p1.q0.ldq = H;
  p1.q0.s = a1_sT;
  p1.q0.s_row = 1;
  p1.q0.s_grp = a_s_ld;
  // last phase: top-k reduce of the slot rows
  p1.red_slot_pos = slot_pos;
  p1.red_out = static_cast<__nv_bfloat16*>(out);
  p1.red_M = M;
  p1.red_topk = topk;
  p2.sorted_ids = sorted_ids;
  p2.topk_w = topk_weights;
  p2.sentinel = (int32_t)(M * topk);
  p2.out_pair = static_cast<__nv_bfloat16*>(out_pair);
  p2.err = err_word;
  const int64_t units_cap = chunks_capacity * ((2 * I) / 256 + H / 256);
  int64_t grid = grid_ctas > 0 ? grid_ctas : sm_count();
  if (grid > units_cap) grid = units_cap;
  return cuda_status(launch_grouped_gemm_fused(tile_tokens, tw1, ta1, p1, tw2, ta2, p2, (int)grid,
                                               (cudaStream_t)stream),
                     "experts_fused");
}

int b200moe_combine_reduce(const void* out_pair, const int32_t* slot_pos, int sorted_rows, int64_t M, int topk,
                           int64_t H, void* out, void* stream) {
  if (M < 0 || topk <= 0 || H <= 0 || H % 8 != 0 || (M > 0 && (!out_pair || !slot_pos || !out)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_combine_reduce: bad argument%s");
  if (!aligned16(out_pair) || !aligned16(out))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_combine_reduce: 16-byte alignment required%s");
  return cuda_status(launch_combine_reduce(out_pair, slot_pos, sorted_rows, M, topk, H, out, (cudaStream_t)stream),
                     "combine_reduce");
}

int b200moe_set_layer_launch(int mode) {
  if (mode < 0 || mode > 2) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_set_layer_launch: mode 0, 1 or 2%s");
  return g_layer_launch.exchange(mode);
}

int b200moe_layer_launches(int64_t M, int64_t H, int64_t I, int num_experts, int num_local_experts, int topk) {
  if (M <= 0 || H <= 0 || I <= 0 || topk <= 0 || num_experts <= 0) return 0;
  const int E = num_local_experts > 0 ? num_local_experts : num_experts;
  const LayerPlan pl = plan_layer(M, H, I, E, topk);
  const int64_t numel = M * topk;
  if (whole_layer_for(M, numel, pl.tile_tokens, pl.heavy_rows, false)) return 1;
  int n = (route_ctas(numel) > 1 && pl.heavy_rows == 0) ? 2 : 1;  // routing (with the router from logits)
  n += 1;                                                          // gather + quantise
  n += pl.tile_tokens > 64 ? 2 : 1;                                // both GEMM stages
  if (pl.heavy_rows) n += 2;                                       // the heavy list's token-major stages
  return n + 1;                                                    // top-k reduce
}

size_t b200moe_layer_workspace_size(int64_t M, int64_t H, int64_t I, int num_experts, int num_local_experts,
                                    int topk) {
  if (M < 0 || H <= 0 || I <= 0 || topk <= 0) return 0;
  const int E = num_local_experts > 0 ? num_local_experts : num_experts;
  return plan_layer(M, H, I, E, topk).total;
}

}  // extern "C"

namespace {

// Activation source of the layer: bf16 rows to quantise, or rows already
// quantised 1x128 (fp8 with row stride ldq bytes, scales s[t * lds + g]).
struct LayerInput {
  const void* hidden;
  const uint8_t* q;
  int64_t ldq;
  const float* s;
  int64_t lds;
};

// The layer as one cooperative launch (EPI_WHOLE) on the workspace regions of
// plan pl at wl: routing (after the router, when router is set) in one CTA
// while the others wait, then the gather of the routed rows, both GEMM stages
// and the top-k reduce (as b200moe_experts_fused). The launch's sync words are
// ints 1..3 of the workspace header (int 1 is also the router counter of the
// separate routing launch; every call leaves them zero).
int whole_layer(const char* name, const LayerInput& in, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
                const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                const float* topk_weights, const int32_t* topk_ids, const int32_t* expert_map, int E, void* out,
                const LayerPlan& pl, uint8_t* wl, int32_t* err, const RouterArgs* router, void* stream) {
  int32_t* sorted = reinterpret_cast<int32_t*>(wl + pl.off_sorted);
  int32_t* pos = reinterpret_cast<int32_t*>(wl + pl.off_pos);
  int32_t* ce = reinterpret_cast<int32_t*>(wl + pl.off_ce);
  int32_t* cr0 = reinterpret_cast<int32_t*>(wl + pl.off_cr0);
  int32_t* crows = reinterpret_cast<int32_t*>(wl + pl.off_crows);
  int32_t* ready = reinterpret_cast<int32_t*>(wl + pl.off_ready);
  int32_t* counts = reinterpret_cast<int32_t*>(wl + pl.off_counts);
  uint8_t* a1 = wl + pl.off_a1;
  float* a1s = reinterpret_cast<float*>(wl + pl.off_a1s);
  uint8_t* a2 = wl + pl.off_a2;
  float* a2s = reinterpret_cast<float*>(wl + pl.off_a2s);
  __nv_bfloat16* pair = reinterpret_cast<__nv_bfloat16*>(wl + pl.off_pair);
  if (!in.hidden && (!aligned16(in.q) || in.ldq % 16 != 0 || in.ldq < H || in.lds < H / 128 || !in.s))
    return fail(B200MOE_ERR_UNSUPPORTED, "%s: fp8 rows must be 16-byte aligned with scales per row", name);
  if (!aligned16(out) || (in.hidden && !aligned16(in.hidden)))
    return fail(B200MOE_ERR_UNSUPPORTED, "%s: 16-byte alignment required", name);
  GemmParams p1{}, p2{};
  int st = make_align(router ? router->out_ids : topk_ids, M, topk, num_experts, expert_map, E, pl.tile_tokens,
                      sorted, pl.rows_cap, ce, cr0, crows, pl.chunks_cap, counts, counts + 1, pos, ready, err, nullptr,
                      p1.ra);
  if (st) return st;
  CUtensorMap tw1, ta1, tw2, ta2;
  st = prep_gemm(a1, a1s, pl.as_ld, pl.rows_cap, w13, w13_scale, E, 2 * I, H, ce, cr0, crows, counts,
                 pl.tile_tokens, p1, tw1, ta1);
  if (st) return st;
  st = prep_gemm(a2, a2s, pl.as_ld, pl.rows_cap, w2, w2_scale, E, H, I, ce, cr0, crows, counts, pl.tile_tokens, p2,
                 tw2, ta2);
  if (st) return st;
  p1.out_q = a2;
  p1.out_q_ld = I;
  p1.out_sT = a2s;
  p1.out_s_ld = pl.as_ld;
  p1.chunk_ready = ready;
  p1.phase_count = ready + pl.chunks_cap;
  p1.err = err;
  p1.route_sync = err + 1;
  if (router) {
    p1.rr = *router;
    p1.router = 1;
  }
  // gather: as b200moe_gather_quant / b200moe_gather_rows, slot positions
  // read through L2 (the routing of this launch wrote them)
  QuantArgs& g = p1.q0;
  if (in.hidden) {
    g.x = in.hidden;
    g.ldx = H;
  } else {
    g.xq = in.q;
    g.ldxq = in.ldq;
    g.xs = in.s;
    g.ldxs = in.lds;
  }
  g.K = H;
  const bool fan = fan_out_tokens(M * topk, topk);
  g.rows = fan ? M : M * topk;
  g.fanout = fan ? 1 : 0;
  g.slot_pos = pos;
  g.topk = topk;
  g.sentinel = (int32_t)(M * topk);
  g.meta_l2 = 1;
  g.q = a1;
  g.ldq = H;
  g.s = a1s;
  g.s_row = 1;
  g.s_grp = pl.as_ld;
  p1.red_slot_pos = pos;
  p1.red_out = static_cast<__nv_bfloat16*>(out);
  p1.red_M = M;
  p1.red_topk = topk;
  p2.sorted_ids = sorted;
  p2.topk_w = router ? router->out_w : topk_weights;
  p2.sentinel = (int32_t)(M * topk);
  p2.out_pair = pair;
  p2.err = err;
  const int64_t units_cap = pl.chunks_cap * ((2 * I) / 256 + H / 256);
  int64_t grid = sm_count();
  if (grid > units_cap) grid = units_cap;
  return cuda_status(launch_grouped_gemm_fused(pl.tile_tokens, tw1, ta1, p1, tw2, ta2, p2, (int)grid,
                                               (cudaStream_t)stream),
                     name);
}

int layer_core(const char* name, const LayerInput& in, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
               const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
               const float* topk_weights, const int32_t* topk_ids, const int32_t* expert_map, int num_local_experts,
               void* out, void* workspace, size_t workspace_bytes, size_t workspace_offset, void* stream,
               const EpPeerArgs* peer_out = nullptr, int32_t* peer_counter = nullptr, int64_t tile_numel = -1,
               const RouterArgs* router = nullptr, const PackedMeta* packed = nullptr) {
  int st = check_gemm_shapes(H, I);
  if (st) return st;
  if (M < 0 || topk <= 0 || num_experts <= 0) return fail(B200MOE_ERR_INVALID_ARG, "%s: bad argument", name);
  if (M == 0) return B200MOE_OK;
  if ((!in.hidden && !in.q) || !w13 || !w13_scale || !w2 || !w2_scale || !topk_weights || !topk_ids ||
      (!out && !peer_out) || !workspace)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: null pointer", name);
  const int E = expert_map ? num_local_experts : num_experts;
  if (E <= 0 || E > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "%s: 1..1024 experts supported", name);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: workspace must be 256-byte aligned", name);
  // tile_numel: the routed slots expected when M*topk overstates them (received
  // expert-parallel rows carry ids for this rank's experts only).
  const LayerPlan pl = plan_layer(M, H, I, E, topk, tile_numel >= 0 ? pick_tile_tokens(tile_numel, E) : 0);
  if (workspace_bytes < workspace_offset + pl.total) return fail(B200MOE_ERR_WORKSPACE, "%s: workspace too small", name);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* err = reinterpret_cast<int32_t*>(ws);
  uint8_t* wl = ws + workspace_offset;  // layer regions (the error word stays at offset 0)
  int32_t* sorted = reinterpret_cast<int32_t*>(wl + pl.off_sorted);
  int32_t* pos = reinterpret_cast<int32_t*>(wl + pl.off_pos);
  int32_t* ce = reinterpret_cast<int32_t*>(wl + pl.off_ce);
  int32_t* cr0 = reinterpret_cast<int32_t*>(wl + pl.off_cr0);
  int32_t* crows = reinterpret_cast<int32_t*>(wl + pl.off_crows);
  int32_t* ready = reinterpret_cast<int32_t*>(wl + pl.off_ready);
  int32_t* counts = reinterpret_cast<int32_t*>(wl + pl.off_counts);  // [0] n_chunks, [1] num_rows
  uint8_t* a1 = wl + pl.off_a1;
  float* a1s = reinterpret_cast<float*>(wl + pl.off_a1s);
  uint8_t* a2 = wl + pl.off_a2;
  float* a2s = reinterpret_cast<float*>(wl + pl.off_a2s);
  __nv_bfloat16* pair = reinterpret_cast<__nv_bfloat16*>(wl + pl.off_pair);

  int32_t* rscratch = pl.rscratch_ints > 0 ? reinterpret_cast<int32_t*>(wl + pl.off_rscratch) : nullptr;
  // Routing from router logits: the router's CTA counter is int 1 of the
  // workspace header (zeroed with the error word; every call leaves it zero).
  // Mixed work lists (decode batches with heavy experts): counts[2] = heavy
  // chunks, counts[3] = first heavy row.
  if (whole_layer_for(M, M * topk, pl.tile_tokens, pl.heavy_rows, peer_out != nullptr))
    return whole_layer(name, in, M, H, I, num_experts, topk, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids,
                       expert_map, E, out, pl, wl, err, router, stream);
  MixedLists mx{};
  if (pl.heavy_rows) {
    mx = MixedLists{pl.heavy_rows, reinterpret_cast<int32_t*>(wl + pl.off_ce2),
                    reinterpret_cast<int32_t*>(wl + pl.off_cr0_2), reinterpret_cast<int32_t*>(wl + pl.off_crows2),
                    pl.chunks_cap2, counts + 2, counts + 3, reinterpret_cast<int32_t*>(wl + pl.off_ready2)};
  }
  st = route_impl(topk_ids, M, topk, num_experts, expert_map, E, pl.tile_tokens, sorted, pl.rows_cap, ce, cr0, crows,
                  pl.chunks_cap, counts, counts + 1, pos, ready, rscratch, pl.rscratch_ints, err, stream, router,
                  router ? err + 1 : nullptr, pl.heavy_rows ? &mx : nullptr, packed);
  if (st) return st;
  const LayerInput& src = in;
  if (src.hidden) {
    st = b200moe_gather_quant(in.hidden, M, H, topk, pos, pl.rows_cap, a1, a1s, pl.as_ld, stream);
  } else {
    if (!aligned16(src.q) || src.ldq % 16 != 0 || src.ldq < H || src.lds < H / 128 || !src.s)
      return fail(B200MOE_ERR_UNSUPPORTED, "%s: fp8 rows must be 16-byte aligned with scales per row", name);
    st = b200moe_gather_rows(src.q, src.s, src.ldq, src.lds, M, H, topk, pos, pl.rows_cap, a1, a1s, pl.as_ld,
                             stream);
  }
  if (st) return st;
  st = b200moe_experts(a1, a1s, pl.as_ld, pl.rows_cap, w13, w13_scale, w2, w2_scale, E, H, I, ce, cr0, crows, counts,
                       pl.chunks_cap, ready, pl.tile_tokens, a2, a2s, sorted, topk_weights, M, topk, pair, err, 0,
                       stream);
  if (st) return st;
  if (pl.heavy_rows) {
    st = experts_heavy_core(a1, a1s, pl.as_ld, pl.rows_cap, w13, w13_scale, w2, w2_scale, E, H, I, mx.chunk_expert,
                            mx.chunk_row0, mx.chunk_rows, mx.n_chunks, mx.chunks_cap, mx.counters, a2, a2s, sorted,
                            topk_weights, M, topk, pair, err, 0, stream);
    if (st) return st;
  }
  if (peer_out)  // results straight into the source ranks' return areas
    return cuda_status(launch_ep_reduce_peer(pair, pos, pair_sorted_rows(pl.tile_tokens), topk, H, *peer_out,
                                             peer_counter, (cudaStream_t)stream),
                       "ep_reduce_peer");
  return b200moe_combine_reduce(pair, pos, pair_sorted_rows(pl.tile_tokens), M, topk, H, out, stream);
}

}  // namespace

extern "C" {

int b200moe_layer(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
                  const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                  const float* topk_weights, const int32_t* topk_ids, const int32_t* expert_map,
                  int num_local_experts, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!hidden && M > 0) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer: null hidden%s");
  LayerInput in{hidden, nullptr, 0, nullptr, 0};
  return layer_core("b200moe_layer", in, M, H, I, num_experts, topk, w13, w13_scale, w2, w2_scale, topk_weights,
                    topk_ids, expert_map, num_local_experts, out, workspace, workspace_bytes, 0, stream);
}

int b200moe_layer_quantized(const uint8_t* hidden_q, const float* hidden_scale, int64_t M, int64_t H, int64_t I,
                            int num_experts, int topk, const uint8_t* w13, const float* w13_scale, const uint8_t* w2,
                            const float* w2_scale, const float* topk_weights, const int32_t* topk_ids,
                            const int32_t* expert_map, int num_local_experts, void* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if ((!hidden_q || !hidden_scale) && M > 0)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer_quantized: null input%s");
  LayerInput in{nullptr, hidden_q, H, hidden_scale, H / 128};
  return layer_core("b200moe_layer_quantized", in, M, H, I, num_experts, topk, w13, w13_scale, w2, w2_scale,
                    topk_weights, topk_ids, expert_map, num_local_experts, out, workspace, workspace_bytes, 0,
                    stream);
}

int b200moe_layer_logits(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
                         const void* router_logits, int logits_bf16, int scoring, const float* correction_bias,
                         int renormalize, float scaling, const uint8_t* w13, const float* w13_scale,
                         const uint8_t* w2, const float* w2_scale, const int32_t* expert_map, int num_local_experts,
                         float* topk_weights, int32_t* topk_ids, void* out, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!hidden && M > 0) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer_logits: null hidden%s");
  int st = check_router("b200moe_layer_logits", router_logits, M, num_experts, topk, scoring, correction_bias,
                        topk_weights, topk_ids);
  if (st) return st;
  const RouterArgs r{router_logits, logits_bf16 ? 1 : 0, num_experts, topk, scoring, renormalize ? 1 : 0,
                     correction_bias, scaling, topk_weights, topk_ids};
  LayerInput in{hidden, nullptr, 0, nullptr, 0};
  return layer_core("b200moe_layer_logits", in, M, H, I, num_experts, topk, w13, w13_scale, w2, w2_scale,
                    topk_weights, topk_ids, expert_map, num_local_experts, out, workspace, workspace_bytes, 0, stream,
                    nullptr, nullptr, -1, &r);
}

int64_t b200moe_ep_row_bytes(int64_t H, int topk) { return round_up(H + (H / 128) * 4 + 8 * (int64_t)topk, 16); }

}  // extern "C"

namespace {

// The expert placement of a dispatch: identity (replicas == nullptr: E/G
// experts per rank, slots_per_rank 0 or E/G) or a replica table.
int make_place(const char* name, int num_experts, int num_ranks, int rank, const int32_t* replicas,
               int max_replicas, int slots_per_rank, EpPlace& pl) {
  if (num_experts <= 0 || num_ranks <= 0 || num_ranks > EpPeerLayout::kMaxRanks || rank < 0 || rank >= num_ranks)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: bad expert or rank count", name);
  if (!replicas) {
    if (num_experts % num_ranks != 0 || (slots_per_rank != 0 && slots_per_rank != num_experts / num_ranks))
      return fail(B200MOE_ERR_INVALID_ARG, "%s: without a replica table num_experts must split evenly", name);
    pl = EpPlace{nullptr, 0, num_experts / num_ranks, num_experts, rank, num_ranks};
    return B200MOE_OK;
  }
  if (max_replicas < 1 || max_replicas > num_ranks || slots_per_rank < 1 ||
      (int64_t)slots_per_rank * num_ranks < num_experts || slots_per_rank > 1024)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: bad replica table shape", name);
  pl = EpPlace{replicas, max_replicas, slots_per_rank, num_experts, rank, num_ranks};
  return B200MOE_OK;
}

}  // namespace

extern "C" {

int b200moe_ep_dispatch(const uint8_t* hidden_q, const float* hidden_scale, const int32_t* topk_ids,
                        const float* topk_weights, int64_t M, int64_t H, int topk, int num_experts, int num_ranks,
                        int rank, const int32_t* replicas, int max_replicas, int slots_per_rank,
                        int64_t rows_per_rank, uint8_t* send_rows, int32_t* pos, int32_t* tok_of, int32_t* counts,
                        int32_t* err_word, void* stream) {
  if (M < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || rows_per_rank < 0 || !err_word || !counts ||
      (M > 0 && (!hidden_q || !hidden_scale || !topk_ids || !topk_weights || !pos)) ||
      (rows_per_rank > 0 && (!send_rows || !tok_of)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_dispatch: bad argument%s");
  EpPlace pl;
  int st = make_place("b200moe_ep_dispatch", num_experts, num_ranks, rank, replicas, max_replicas, slots_per_rank,
                      pl);
  if (st) return st;
  if (!aligned16(hidden_q) || !aligned16(send_rows))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_ep_dispatch: 16-byte alignment required%s");
  return cuda_status(launch_ep_dispatch(hidden_q, hidden_scale, topk_ids, topk_weights, M, H, topk, pl,
                                        rows_per_rank, send_rows, b200moe_ep_row_bytes(H, topk), pos, tok_of, counts,
                                        err_word, (cudaStream_t)stream),
                     "ep_dispatch");
}

size_t b200moe_layer_packed_workspace_size(int64_t R, int64_t H, int64_t I, int num_local_experts, int topk) {
  if (R < 0 || H <= 0 || I <= 0 || topk <= 0 || num_local_experts <= 0) return 0;
  const size_t meta = (size_t)round_up(R * topk * 8 + 256, 256);
  // Enough for every tile size the packed layers may pick (the peer form picks
  // from the expected slots per rank, not R*topk).
  size_t most = 0;
  for (int tile : {32, 64, 128}) {
    const size_t t = plan_layer(R, H, I, num_local_experts, topk, tile).total;
    most = t > most ? t : most;
  }
  return meta + most;
}

int b200moe_layer_packed(const uint8_t* rows, int64_t R, int num_ranks, int64_t row_bytes, int64_t H, int64_t I,
                         int num_local_experts, int topk, const uint8_t* w13, const float* w13_scale,
                         const uint8_t* w2, const float* w2_scale, void* out, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (R < 0 || num_ranks <= 0 || row_bytes != b200moe_ep_row_bytes(H, topk) || !workspace || (R > 0 && !rows))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer_packed: bad argument%s");
  if (R == 0) return B200MOE_OK;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer_packed: workspace must be 256-byte aligned%s");
  const size_t meta = (size_t)round_up(R * topk * 8 + 256, 256);
  if (workspace_bytes < b200moe_layer_packed_workspace_size(R, H, I, num_local_experts, topk))
    return fail(B200MOE_ERR_WORKSPACE, "b200moe_layer_packed: workspace too small%s");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* ids = reinterpret_cast<int32_t*>(ws + 256);
  float* w = reinterpret_cast<float*>(ids + R * topk);
  int st = cuda_status(launch_ep_unpack_meta(rows, R, row_bytes, H, topk, ids, w, (cudaStream_t)stream),
                       "ep_unpack_meta");
  if (st) return st;
  LayerInput in{nullptr, rows, row_bytes, reinterpret_cast<const float*>(rows + H), row_bytes / 4};
  // About R*topk/num_ranks of the id fields name this rank's experts: the tile size follows them.
  return layer_core("b200moe_layer_packed", in, R, H, I, num_local_experts, topk, w13, w13_scale, w2, w2_scale, w,
                    ids, nullptr, num_local_experts, out, workspace, workspace_bytes, meta, stream, nullptr, nullptr,
                    R * topk / num_ranks);
}

int b200moe_ep_combine(const void* returned_rows, const int32_t* pos, int64_t M, int64_t H, int num_ranks,
                       int64_t rows_per_rank, void* out, void* stream) {
  if (M < 0 || H <= 0 || H % 8 != 0 || num_ranks <= 0 || (M > 0 && (!returned_rows || !pos || !out)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_combine: bad argument%s");
  if (!aligned16(returned_rows) || !aligned16(out))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_ep_combine: 16-byte alignment required%s");
  return cuda_status(launch_ep_combine(returned_rows, pos, M, H, num_ranks, rows_per_rank, out, (cudaStream_t)stream),
                     "ep_combine");
}

size_t b200moe_ep_peer_bytes(int64_t rows_per_rank, int64_t H, int topk, int num_ranks) {
  if (rows_per_rank < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || num_ranks <= 0 ||
      num_ranks > EpPeerLayout::kMaxRanks)
    return 0;
  return (size_t)EpPeerLayout(rows_per_rank, H, b200moe_ep_row_bytes(H, topk), num_ranks).total();
}

int b200moe_ep_peer_alloc(size_t bytes, void** base, void* ipc_handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == B200MOE_IPC_HANDLE_BYTES, "IPC handle size");
  if (bytes < (size_t)EpPeerLayout::kHeader || !base || !ipc_handle)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_peer_alloc: bad argument%s");
  void* p = nullptr;
  int st = cuda_status(cudaMalloc(&p, bytes), "ep_peer_alloc");
  if (st) return st;
  // Flags start at 0 (epochs count from 1); done before the handle leaves.
  st = cuda_status(cudaMemset(p, 0, EpPeerLayout::kHeader), "ep_peer_alloc memset");
  if (!st) st = cuda_status(cudaDeviceSynchronize(), "ep_peer_alloc sync");
  cudaIpcMemHandle_t h;
  if (!st) st = cuda_status(cudaIpcGetMemHandle(&h, p), "ep_peer_alloc handle");
  if (st) {
    cudaFree(p);
    return st;
  }
  memcpy(ipc_handle, &h, sizeof h);
  *base = p;
  return B200MOE_OK;
}

int b200moe_ep_peer_open(const void* ipc_handle, void** base) {
  if (!ipc_handle || !base) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_peer_open: null pointer%s");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof h);
  return cuda_status(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "ep_peer_open");
}

int b200moe_ep_peer_close(void* base) {
  if (!base) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_peer_close: null pointer%s");
  return cuda_status(cudaIpcCloseMemHandle(base), "ep_peer_close");
}

int b200moe_ep_peer_free(void* base) {
  if (!base) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_peer_free: null pointer%s");
  return cuda_status(cudaFree(base), "ep_peer_free");
}

namespace {
// Limit of every peer flag wait (dispatch and combine). Ranks may start a
// call seconds apart, so the default is long; b200moe_ep_peer_wait_limit_us
// changes it for the whole process (tests use a short one).
constexpr uint64_t kPeerWaitDefaultNs = 10ull * 1000 * 1000 * 1000;
constexpr int64_t kPeerWaitMaxUs = 60ll * 1000 * 1000;
std::atomic<uint64_t> g_peer_wait_ns{kPeerWaitDefaultNs};

bool peer_args_ok(int num_ranks, int rank, int64_t rows_per_rank, int32_t epoch, void* const* peer_bases,
                  const void* own_base) {
  return num_ranks > 0 && num_ranks <= EpPeerLayout::kMaxRanks && rank >= 0 && rank < num_ranks &&
         rows_per_rank >= 0 && epoch >= 1 && peer_bases && own_base &&
         (reinterpret_cast<uintptr_t>(own_base) & 255) == 0;
}
}  // namespace

int b200moe_ep_dispatch_peer(const void* hidden, const uint8_t* hidden_q, const float* hidden_scale,
                             const int32_t* topk_ids, const float* topk_weights, int64_t M, int64_t H, int topk,
                             int num_experts, int num_ranks, int rank, const int32_t* replicas, int max_replicas,
                             int slots_per_rank, int64_t rows_per_rank, void* const* peer_bases, void* own_base,
                             int32_t epoch, int32_t* pos, int32_t* tok_of, int32_t* counts, int32_t* err_word,
                             void* stream) {
  if (M < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || !err_word || !counts ||
      !peer_args_ok(num_ranks, rank, rows_per_rank, epoch, peer_bases, own_base) ||
      (M > 0 && (!(hidden || (hidden_q && hidden_scale)) || !topk_ids || !topk_weights || !pos)) ||
      (rows_per_rank > 0 && !tok_of))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_dispatch_peer: bad argument%s");
  EpPlace pl;
  int st0 = make_place("b200moe_ep_dispatch_peer", num_experts, num_ranks, rank, replicas, max_replicas,
                       slots_per_rank, pl);
  if (st0) return st0;
  if (!aligned16(hidden) || !aligned16(hidden_q))
    return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_ep_dispatch_peer: 16-byte alignment%s");
  const int64_t rb = b200moe_ep_row_bytes(H, topk);
  const EpPeerLayout lay(rows_per_rank, H, rb, num_ranks);
  cudaStream_t s = (cudaStream_t)stream;
  int st = cuda_status(launch_ep_plan(topk_ids, M, topk, pl, rows_per_rank, pos, tok_of, counts, err_word, s),
                       "ep_plan");
  if (st) return st;
  const EpPeerArgs a{reinterpret_cast<uint8_t* const*>(peer_bases), lay.recv_off(epoch), rows_per_rank, num_ranks,
                     rank, epoch};
  int32_t* counter = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(own_base) + EpPeerLayout::kCounters);
  return cuda_status(launch_ep_pack_peer(hidden, hidden_q, hidden_scale, topk_ids, topk_weights, H, topk, pl, tok_of,
                                         counts, rb, a, counter, s),
                     "ep_pack_peer");
}

int b200moe_layer_packed_peer(void* own_base, void* const* peer_bases, int num_ranks, int rank,
                              int64_t rows_per_rank, int32_t epoch, int64_t H, int64_t I, int num_local_experts,
                              int topk, const uint8_t* w13, const float* w13_scale, const uint8_t* w2,
                              const float* w2_scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (!peer_args_ok(num_ranks, rank, rows_per_rank, epoch, peer_bases, own_base) || H <= 0 || H % 128 != 0 ||
      topk <= 0 || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_layer_packed_peer: bad argument%s");
  const int64_t R = (int64_t)num_ranks * rows_per_rank;
  const int64_t rb = b200moe_ep_row_bytes(H, topk);
  const EpPeerLayout lay(rows_per_rank, H, rb, num_ranks);
  uint8_t* own = static_cast<uint8_t*>(own_base);
  cudaStream_t s = (cudaStream_t)stream;
  if (R > 0 && workspace_bytes < b200moe_layer_packed_workspace_size(R, H, I, num_local_experts, topk))
    return fail(B200MOE_ERR_WORKSPACE, "b200moe_layer_packed_peer: workspace too small%s");
  int32_t* err = static_cast<int32_t*>(workspace);
  const EpPeerArgs a{reinterpret_cast<uint8_t* const*>(peer_bases), lay.ret_off(epoch), rows_per_rank, num_ranks,
                     rank, epoch};
  int32_t* counter = reinterpret_cast<int32_t*>(own + EpPeerLayout::kCounters) + 1;
  if (R == 0) return cuda_status(launch_ep_reduce_peer(nullptr, nullptr, 0, topk, H, a, counter, s), "ep_reduce_peer");
  const uint8_t* rows = own + lay.recv_off(epoch);
  const size_t meta = (size_t)round_up(R * topk * 8 + 256, 256);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* ids = reinterpret_cast<int32_t*>(ws + 256);
  float* w = reinterpret_cast<float*>(ids + R * topk);
  // The routing launch waits for the G dispatch flags and unpacks the ids
  // and weights before it routes them.
  const PackedMeta pm{own, rows, R, rb, H, topk, num_ranks, epoch, g_peer_wait_ns.load(), ids, w};
  LayerInput in{nullptr, rows, rb, reinterpret_cast<const float*>(rows + H), rb / 4};
  // R*topk counts every id field of the G blocks; about rows_per_rank*topk of
  // them name this rank's experts, which sets the tile size.
  return layer_core("b200moe_layer_packed_peer", in, R, H, I, num_local_experts, topk, w13, w13_scale, w2, w2_scale, w,
                    ids, nullptr, num_local_experts, nullptr, workspace, workspace_bytes, meta, stream, &a, counter,
                    rows_per_rank * topk, nullptr, &pm);
}

int b200moe_ep_combine_peer(void* own_base, const int32_t* pos, int64_t M, int64_t H, int topk, int num_ranks,
                            int64_t rows_per_rank, int32_t epoch, void* out, int32_t* err_word, void* stream) {
  if (M < 0 || H <= 0 || H % 128 != 0 || topk <= 0 || !err_word ||
      num_ranks <= 0 || num_ranks > EpPeerLayout::kMaxRanks || rows_per_rank < 0 || epoch < 1 || !own_base ||
      (M > 0 && (!pos || !out)))
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_ep_combine_peer: bad argument%s");
  if (!aligned16(out)) return fail(B200MOE_ERR_UNSUPPORTED, "b200moe_ep_combine_peer: 16-byte alignment%s");
  const EpPeerLayout lay(rows_per_rank, H, b200moe_ep_row_bytes(H, topk), num_ranks);
  return cuda_status(launch_ep_combine_peer(static_cast<const uint8_t*>(own_base), lay.ret_off(epoch), pos, M, H,
                                            num_ranks, rows_per_rank, epoch, out, err_word, g_peer_wait_ns.load(),
                                            (cudaStream_t)stream),
                     "ep_combine_peer");
}

int64_t b200moe_ep_peer_wait_limit_us(int64_t limit_us) {
  const int64_t previous = (int64_t)(g_peer_wait_ns.load() / 1000);
  if (limit_us > 0) g_peer_wait_ns.store((uint64_t)(limit_us < kPeerWaitMaxUs ? limit_us : kPeerWaitMaxUs) * 1000);
  return previous;
}

int b200moe_router_topk(const void* logits, int logits_bf16, int64_t M, int num_experts, int topk, int scoring,
                        const float* correction_bias, int renormalize, float scaling, float* topk_weights,
                        int32_t* topk_ids, void* stream) {
  int st = check_router("b200moe_router_topk", logits, M, num_experts, topk, scoring, correction_bias, topk_weights,
                        topk_ids);
  if (st) return st;
  return cuda_status(launch_router_topk(logits, logits_bf16, M, num_experts, topk, scoring, correction_bias,
                                        renormalize, scaling, topk_weights, topk_ids, (cudaStream_t)stream),
                     "router_topk");
}

int b200moe_read_error(int32_t* err_word, int32_t* value, int clear, void* stream) {
  if (!err_word || !value) return fail(B200MOE_ERR_INVALID_ARG, "b200moe_read_error: null pointer%s");
  cudaStream_t s = (cudaStream_t)stream;
  int st = cuda_status(cudaMemcpyAsync(value, err_word, sizeof(int32_t), cudaMemcpyDeviceToHost, s), "read_error");
  if (st) return st;
  st = cuda_status(cudaStreamSynchronize(s), "read_error sync");
  if (st) return st;
  if (clear) return cuda_status(cudaMemsetAsync(err_word, 0, sizeof(int32_t), s), "read_error clear");
  return B200MOE_OK;
}

int b200moe_selftest_wait_timeout(int32_t* err_word, int timeout_us, void* stream) {
  if (!err_word || timeout_us <= 0 || timeout_us > 10000000)
    return fail(B200MOE_ERR_INVALID_ARG, "b200moe_selftest_wait_timeout: bad argument%s");
  return cuda_status(launch_wait_timeout_selftest(err_word, (uint64_t)timeout_us * 1000ull, (cudaStream_t)stream),
                     "selftest");
}

}  // extern "C"
