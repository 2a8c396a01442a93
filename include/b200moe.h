/*
 * b200moe: FP8 128x128 block-scaled Mixture-of-Experts layer for NVIDIA B200 (sm_100a).
 *
 * C ABI. Every function takes raw device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an int
 * status: B200MOE_OK (0) or a negative B200MOE_ERR_* code for bad arguments or
 * unsupported shapes (checked on the host, before anything is launched).
 * No function allocates device memory: callers pass outputs and, where needed,
 * a workspace whose size the matching *_workspace_size() call reports.
 *
 * Data-dependent problems found on the device (an expert id outside the
 * expert range, a pipeline wait that timed out) are OR-ed into a caller-owned
 * int32 "device error word" (B200MOE_DEVERR_* bits); read it with
 * b200moe_read_error() after the stream has run.
 *
 * Data types: bf16 = __nv_bfloat16 (passed as void*), fp8 = E4M3FN bytes
 * (uint8_t), scales float32, ids int32.
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200MOE_API __attribute__((visibility("default")))
#else
#define B200MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B200MOE_OK 0
#define B200MOE_ERR_INVALID_ARG (-1)
#define B200MOE_ERR_UNSUPPORTED (-2)
#define B200MOE_ERR_WORKSPACE (-3)
#define B200MOE_ERR_CUDA (-4)

#define B200MOE_DEVERR_BAD_EXPERT_ID 1 /* an id outside [0, num_experts) other than -1 */
#define B200MOE_DEVERR_TIMEOUT 2       /* a bounded pipeline wait gave up */
#define B200MOE_DEVERR_CAPACITY 4      /* routed rows exceeded the given capacity */

/* Library version (major*10000 + minor*100 + patch). */
B200MOE_API int b200moe_version(void);

/* Text for a status code. */
B200MOE_API const char* b200moe_status_string(int status);

/* Message describing the last non-OK status returned on this host thread. */
B200MOE_API const char* b200moe_last_error_message(void);

/* ------------------------------------------------------------------------
 * Routing: moe_align_block_size.
 * Replaces sglang's moe_align_block_size(topk_ids, block_size, num_experts)
 * as called by the reference orchestrator
 * (sglang_integration/aiter.py:95-97, 113-115).
 *
 * topk_ids (M, topk) int32. Entries equal to -1 are dropped silently (the
 * expert-parallel "not on this rank" convention); other ids outside
 * [0, num_experts) are dropped and set B200MOE_DEVERR_BAD_EXPERT_ID.
 * expert_map (nullable, num_experts entries) maps an id to the index of its
 * weights, or to -1 to drop it.
 *
 * Outputs, same meaning as the reference:
 *   sorted_token_ids[sorted_capacity]: flat indices t*topk+j grouped by expert,
 *       each expert padded to a multiple of block_m with the sentinel M*topk.
 *       Order within an expert is ascending flat index (stable).
 *       Every entry past the routed rows is the sentinel.
 *   expert_ids[blocks_capacity]: (mapped) expert of each block_m block; blocks
 *       past num_tokens_post_pad/block_m are -1 (never left uninitialised).
 *   num_tokens_post_pad[1]: total padded rows (device scalar; no host sync).
 * Capacities must be at least b200moe_align_capacity_rows() /
 * b200moe_align_capacity_blocks() (sglang's numel + (E+1)*(block_m-1) sizing).
 * num_experts <= 1024.
 * ---------------------------------------------------------------------- */
B200MOE_API int64_t b200moe_align_capacity_rows(int64_t numel, int num_experts, int block_m);
B200MOE_API int64_t b200moe_align_capacity_blocks(int64_t numel, int num_experts, int block_m);
B200MOE_API int b200moe_align(const int32_t* topk_ids, int64_t M, int topk, int num_experts, int block_m,
                  const int32_t* expert_map, int num_local_experts, int32_t* sorted_token_ids,
                  int64_t sorted_capacity, int32_t* expert_ids, int64_t blocks_capacity,
                  int32_t* num_tokens_post_pad, int32_t* err_word, void* stream);

/* ------------------------------------------------------------------------
 * Router: logits (M, E) f32 (logits_bf16 = 0) or bf16 (1) -> topk_ids and
 * topk_weights (M, topk). Replaces the router kernel in front of the
 * reference's MoE call (aiter topksoftmax, MBR/micro/glm52_fp8_moe.log) and
 * GLM's sigmoid routing (measure_xcd_imbalance.py:50-55: ungrouped top-k of
 * sigmoid(logits) + correction_bias).
 * scoring 0 = softmax: select the top-k softmax probabilities; 1 = sigmoid:
 * select the top-k of sigmoid + correction_bias (nullable). Weights are the
 * unbiased probabilities of the selected experts, divided by their sum when
 * renormalize != 0, times scaling. Ids in descending selection order, equal
 * values broken by the lower id. E <= 1024, topk <= 16.
 * ---------------------------------------------------------------------- */
B200MOE_API int b200moe_router_topk(const void* logits, int logits_bf16, int64_t M, int num_experts, int topk,
                                    int scoring, const float* correction_bias, int renormalize, float scaling,
                                    float* topk_weights, int32_t* topk_ids, void* stream);

/* ------------------------------------------------------------------------
 * Activation quantisation: per_token_group_quant_fp8(x, 128).
 * Replaces sglang's per_token_group_quant_fp8 called at
 * sglang_integration/aiter.py:132-133 and :151-152 (torch form of the same
 * formula: phase5_orchestrator.py:26-32).
 * x (M, K) bf16 with row stride ldx elements; q (M, K) fp8 with row stride ldq;
 * s[m * s_stride_row + g * s_stride_group] = max(amax(x[m, 128g:128g+128])/448, 1e-12);
 * q = e4m3(clamp(x / s, -448, 448)), round to nearest even. K % 128 == 0.
 * ---------------------------------------------------------------------- */
B200MOE_API int b200moe_quant_1x128(const void* x, int64_t M, int64_t K, int64_t ldx, uint8_t* q, int64_t ldq, float* s,
                        int64_t s_stride_row, int64_t s_stride_group, void* stream);

/* ------------------------------------------------------------------------
 * Weight quantisation: per_block_quant_fp8(w, 128, 128)
 * (phase5_orchestrator.py:35-41). w (E, N, K) bf16 contiguous -> q (E, N, K)
 * fp8 and s (E, N/128, K/128) fp32, s = max(block amax/448, 1e-12).
 * ---------------------------------------------------------------------- */
B200MOE_API int b200moe_quant_block128(const void* w, int64_t E, int64_t N, int64_t K, uint8_t* q, float* s, void* stream);

/* ------------------------------------------------------------------------
 * Full layer: replaces _moe_decode_megakernel_full
 * (sglang_integration/aiter.py:74-177) and, for the arguments it supports,
 * the aiter fused_moe call (sglang_integration/aiter.py:459-478) with
 * quant_type=per_128x128, activation=Silu, gate_mode=interleave.
 *
 * hidden (M, H) bf16 row-major; w13 (E_w, 2I, H) fp8 with gate/up rows
 * interleaved (row 2j = gate j, row 2j+1 = up j); w13_scale (E_w, 2I/128, H/128);
 * w2 (E_w, H, I) fp8; w2_scale (E_w, H/128, I/128); topk_weights (M, topk) f32;
 * topk_ids (M, topk) int32; expert_map as in b200moe_align (nullable; then
 * E_w = num_experts). out (M, H) bf16:
 *   out[t] = bf16( sum_j topk_weights[t,j] * W2[e] . q(silu(g) * u) ),
 *   (g, u) = W13[e] . q(hidden[t]), e = expert of slot (t, j);
 * slots whose id is -1 or maps to -1 contribute nothing.
 * Requirements: H % 256 == 0, I % 128 == 0, num_experts <= 1024.
 * workspace: b200moe_layer_workspace_size() bytes, 256-byte aligned; its first
 * 256 bytes (the device error word, then counters that every call leaves at
 * zero) must be zeroed once by the caller, and again after a call reported
 * B200MOE_DEVERR_TIMEOUT.
 * Launches: 4 to 7 (routing, gather + quantise, both GEMM stages, top-k
 * reduce). Small batches (tiles of 16..64 tokens, fewer than 16,384 routed
 * slots, no mixed work lists) can instead run the whole layer as ONE
 * cooperative launch (the reference's deferred single-launch layer,
 * phase8_findings.md:77-81), same results bit for bit:
 * b200moe_set_layer_launch / b200moe_layer_launches below.
 * No host synchronisation: the call can be captured in a CUDA graph.
 * ---------------------------------------------------------------------- */
B200MOE_API size_t b200moe_layer_workspace_size(int64_t M, int64_t H, int64_t I, int num_experts, int num_local_experts,
                                    int topk);
B200MOE_API int b200moe_layer(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
                  const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                  const float* topk_weights, const int32_t* topk_ids, const int32_t* expert_map,
                  int num_local_experts, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Launch policy of b200moe_layer, b200moe_layer_logits and
 * b200moe_layer_quantized (process-wide): 0 (default) = the form measured
 * faster for the shape (so far the separate launches for every shape: the
 * one-launch layer measured 3-4% slower on the GLM decode layer), 1 = the
 * whole layer in one launch wherever it applies, 2 = never. Returns the
 * previous mode, or B200MOE_ERR_INVALID_ARG. */
B200MOE_API int b200moe_set_layer_launch(int mode);
/* Kernel launches one call of those entry points makes for this shape under
 * the current policy (1 = the whole-layer launch); 0 for an empty batch. */
B200MOE_API int b200moe_layer_launches(int64_t M, int64_t H, int64_t I, int num_experts, int num_local_experts,
                                       int topk);

/* Same layer starting from the router: router_logits (M, num_experts) f32
 * (logits_bf16 = 0) or bf16 (1) go through the router of b200moe_router_topk
 * (scoring, correction_bias, renormalize, scaling as there) inside routing's
 * first launch, so the router costs no launch of its own (one launch for the
 * router and routing below 16,384 routed slots, two above, as routing alone).
 * The selected ids and weights are stored to topk_ids / topk_weights (M, topk)
 * for the caller; the result equals b200moe_router_topk followed by
 * b200moe_layer bit for bit. Replaces the router launch in front of the
 * reference's MoE call (aiter topksoftmax, MBR/micro/glm52_fp8_moe.log; GLM's
 * sigmoid routing, measure_xcd_imbalance.py:50-55) and the layer
 * (sglang_integration/aiter.py:74-177). Workspace: b200moe_layer_workspace_size();
 * its first 256 bytes must be zeroed once by the caller (the error word and
 * the router's CTA counter, which every call leaves at zero). */
B200MOE_API int b200moe_layer_logits(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts, int topk,
                                     const void* router_logits, int logits_bf16, int scoring,
                                     const float* correction_bias, int renormalize, float scaling,
                                     const uint8_t* w13, const float* w13_scale, const uint8_t* w2,
                                     const float* w2_scale, const int32_t* expert_map, int num_local_experts,
                                     float* topk_weights, int32_t* topk_ids, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Same layer with pre-quantised activations: hidden_q (M, H) fp8 e4m3 and
 * hidden_scale (M, H/128) f32 from a 1x128 per-token-group quantisation. This
 * is the reference's fp8-input case (sglang_integration/aiter.py:126-130 with
 * a per-group a1_scale, the a1_scale argument of the fused_moe call at :470).
 * Workspace: b200moe_layer_workspace_size(). */
B200MOE_API int b200moe_layer_quantized(const uint8_t* hidden_q, const float* hidden_scale, int64_t M, int64_t H,
                                        int64_t I, int num_experts, int topk, const uint8_t* w13,
                                        const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                                        const float* topk_weights, const int32_t* topk_ids,
                                        const int32_t* expert_map, int num_local_experts, void* out,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Expert parallelism over G ranks: rank r owns experts [r*E/G, (r+1)*E/G).
 * Replaces the dispatch/combine that the reference consumes from DeepEP/Mori
 * (sglang_integration/aiter.py:554-756: tokens arrive with local expert ids,
 * -1 for experts on other ranks, and leave as per-token partial sums).
 *
 * Expert placement (both dispatch forms): replicas == NULL places expert e on
 * rank e / (E/G) only (slots_per_rank 0 or E/G). Otherwise every rank holds
 * slots_per_rank physical experts (slot p = rank * slots_per_rank + local
 * index; slots_per_rank * G >= E) and the device table replicas, E rows of
 * 1 + max_replicas int32, lists for expert e its n >= 1 replicas:
 * [n, p_0, .., p_{n-1}, unused]. This is hot-expert replication (EPLB; the
 * reference's planned "--enable-eplb", moe_placement_glm52_mi355x.md:98-104).
 * A routed slot (t, j) of expert e goes to e's replica on the sending rank
 * `rank` if it has one, else to replica (t*topk + j) mod n; the destination
 * then sees the local index p mod slots_per_rank as the slot's id. Rank r's
 * weights are the logical experts of its slots, in slot order. An id whose
 * table row names no valid slot is dropped and sets B200MOE_DEVERR_BAD_EXPERT_ID.
 *
 * Packed row (b200moe_ep_row_bytes(H, topk) bytes, 16-byte multiple):
 *   [ fp8 row: H bytes | 1x128 scales: H/128 f32 | topk local ids: int32, -1 =
 *     expert not on the destination | topk router weights: f32 | padding ]
 * b200moe_ep_dispatch builds the send buffer from this rank's tokens (quantised
 * with b200moe_quant_1x128): G blocks of rows_per_rank rows, block d holding,
 * in ascending token order, every token with at least one expert on rank d;
 * unused rows carry ids -1. pos[t*G + d] = row of token t in block d or -1;
 * tok_of[d*rows_per_rank + r] = token of that row; counts[d] = rows used.
 * Tokens beyond rows_per_rank for a destination set B200MOE_DEVERR_CAPACITY
 * (rows_per_rank = M never overflows). After an equal-split all-to-all of the
 * G blocks, the receiving rank runs b200moe_layer_packed on all R = G*rows_per_rank
 * received rows (rows without a local expert give zero rows; num_ranks = G sets
 * the expected count of local slots, R*topk/G, which picks the tile size) and sends the
 * (R, H) bf16 result back with a second equal-split all-to-all;
 * b200moe_ep_combine then sums, for each token, the returned rows of the ranks
 * it was sent to, in rank order. No host synchronisation anywhere.
 * ---------------------------------------------------------------------- */
B200MOE_API int64_t b200moe_ep_row_bytes(int64_t H, int topk);
B200MOE_API int b200moe_ep_dispatch(const uint8_t* hidden_q, const float* hidden_scale, const int32_t* topk_ids,
                                    const float* topk_weights, int64_t M, int64_t H, int topk, int num_experts,
                                    int num_ranks, int rank, const int32_t* replicas, int max_replicas,
                                    int slots_per_rank, int64_t rows_per_rank, uint8_t* send_rows, int32_t* pos,
                                    int32_t* tok_of, int32_t* counts, int32_t* err_word, void* stream);
B200MOE_API size_t b200moe_layer_packed_workspace_size(int64_t R, int64_t H, int64_t I, int num_local_experts,
                                                       int topk);
B200MOE_API int b200moe_layer_packed(const uint8_t* rows, int64_t R, int num_ranks, int64_t row_bytes, int64_t H,
                                     int64_t I,
                                     int num_local_experts, int topk, const uint8_t* w13, const float* w13_scale,
                                     const uint8_t* w2, const float* w2_scale, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream);
B200MOE_API int b200moe_ep_combine(const void* returned_rows, const int32_t* pos, int64_t M, int64_t H,
                                   int num_ranks, int64_t rows_per_rank, void* out, void* stream);

/* ------------------------------------------------------------------------
 * The same expert parallelism with the exchange done by the kernels over
 * NVLink peer memory instead of two all-to-alls (one process per GPU; the
 * buffers are shared through CUDA IPC). Same packed rows and results:
 *   b200moe_ep_dispatch_peer   plan + pack, each destination's rows stored
 *                              straight into that rank's receive area (bf16
 *                              `hidden` is quantised 1x128 on the way, or
 *                              hidden_q/hidden_scale copied; pass one); the
 *                              last CTA raises this rank's dispatch flag on
 *                              every rank;
 *   b200moe_layer_packed_peer  waits for the G dispatch flags, runs the layer
 *                              on the received rows; its top-k reduce stores
 *                              each result row straight into the return area
 *                              of the rank the token came from, then raises
 *                              this rank's combine flag on every rank;
 *   b200moe_ep_combine_peer    waits for the G combine flags and sums the
 *                              returned rows in rank order (as
 *                              b200moe_ep_combine).
 * Set-up: each rank allocates its exchange buffer of b200moe_ep_peer_bytes()
 * with b200moe_ep_peer_alloc (zeroed flags; B200MOE_IPC_HANDLE_BYTES bytes of
 * IPC handle out), passes the handle to the other ranks over any host
 * channel, maps theirs with b200moe_ep_peer_open, and builds a DEVICE array of
 * G pointers, peer_bases[g] = rank g's buffer as mapped in this process (its
 * own buffer at g = rank). `epoch` numbers the calls from 1, the same on all
 * ranks; the areas are double-buffered by its parity, which is safe because a
 * rank's call e+2 cannot start before every rank has finished reading e.
 * Flag waits are bounded (B200MOE_DEVERR_TIMEOUT in the error word). At most
 * 64 ranks. Replaces the DeepEP/Mori dispatch/combine pair the reference
 * consumes (sglang_integration/aiter.py:554-756).
 * ---------------------------------------------------------------------- */
#define B200MOE_IPC_HANDLE_BYTES 64
B200MOE_API size_t b200moe_ep_peer_bytes(int64_t rows_per_rank, int64_t H, int topk, int num_ranks);
B200MOE_API int b200moe_ep_peer_alloc(size_t bytes, void** base, void* ipc_handle);
B200MOE_API int b200moe_ep_peer_open(const void* ipc_handle, void** base);
B200MOE_API int b200moe_ep_peer_close(void* base);
B200MOE_API int b200moe_ep_peer_free(void* base);
B200MOE_API int b200moe_ep_dispatch_peer(const void* hidden, const uint8_t* hidden_q, const float* hidden_scale,
                                         const int32_t* topk_ids, const float* topk_weights, int64_t M, int64_t H,
                                         int topk, int num_experts, int num_ranks, int rank,
                                         const int32_t* replicas, int max_replicas, int slots_per_rank,
                                         int64_t rows_per_rank, void* const* peer_bases, void* own_base,
                                         int32_t epoch, int32_t* pos, int32_t* tok_of, int32_t* counts,
                                         int32_t* err_word, void* stream);
B200MOE_API int b200moe_layer_packed_peer(void* own_base, void* const* peer_bases, int num_ranks, int rank,
                                          int64_t rows_per_rank, int32_t epoch, int64_t H, int64_t I,
                                          int num_local_experts, int topk, const uint8_t* w13,
                                          const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                                          void* workspace, size_t workspace_bytes, void* stream);
B200MOE_API int b200moe_ep_combine_peer(void* own_base, const int32_t* pos, int64_t M, int64_t H, int topk,
                                        int num_ranks, int64_t rows_per_rank, int32_t epoch, void* out,
                                        int32_t* err_word, void* stream);
/* Limit of the peer flag waits above, in microseconds, for the whole process
 * (default 10 s: ranks may start a call seconds apart; at most 60 s). Applies
 * to launches made after the call. limit_us <= 0 only queries. Returns the
 * previous limit. A wait that runs out sets B200MOE_DEVERR_TIMEOUT in its
 * error word and the kernel goes on, so a rank whose peer is gone gets an
 * error instead of a hung stream. No counterpart in the reference (its
 * DeepEP/Mori exchange is a library call). */
B200MOE_API int64_t b200moe_ep_peer_wait_limit_us(int64_t limit_us);

/* ------------------------------------------------------------------------
 * b200moe_layer without a workspace argument, for callers that cannot
 * allocate device memory (a fixed memory pool, a host framework that forbids
 * allocation inside an operator). No counterpart in the reference.
 * Same arguments, kernels and result as b200moe_layer; the workspace is a
 * 64 MiB device array inside the library, held by every GPU that loads it
 * until the process exits. Layers whose b200moe_layer_workspace_size()
 * exceeds 64 MiB are rejected with B200MOE_ERR_WORKSPACE (the GLM-5-like
 * decode batch of 64 tokens needs about 43 MB; that layer fits up to 208
 * tokens). The call allocates nothing.
 * The first call on each device looks up the array's device address; make it
 * before any stream capture. All calls on a device share the array and it
 * keeps the last call's contents: calls whose GPU work overlaps (for example
 * on two streams) race. err_out (nullable, device int32) receives this call's
 * device error word (B200MOE_DEVERR_* bits).
 * ---------------------------------------------------------------------- */
B200MOE_API int b200moe_layer_noalloc(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts,
                                      int topk, const uint8_t* w13, const float* w13_scale, const uint8_t* w2,
                                      const float* w2_scale, const float* topk_weights, const int32_t* topk_ids,
                                      const int32_t* expert_map, int num_local_experts, void* out,
                                      int32_t* err_out, void* stream);

/* ------------------------------------------------------------------------
 * Stage-level entry points used by b200moe_layer, exposed for staged callers
 * and tests. They work on the layer's internal expert-sorted row layout:
 * routed rows grouped by expert, each expert padded to a multiple of 16 rows.
 * These replace the reference's kernel launchers
 * moe_decode_megakernel_stage1 (aiter_module/moe_decode_megakernel.py:88-123),
 * ..._stage1_fused(fused_silu) (aiter_module/moe_decode_megakernel_fused.py:125-139)
 * and ..._stage2_fused (aiter_module/moe_decode_megakernel_fused.py:142-157).
 *
 * b200moe_route: the align above with block 16 into sorted_ids (capacity
 * rows_capacity >= b200moe_route_capacity_rows()), plus the GEMM work list:
 * each expert's padded rows cut into chunks of at most tile_tokens rows
 * (16, 32, 64, 128 or 256); chunk_expert/chunk_row0/chunk_rows[chunks_capacity],
 * n_chunks[1] and num_rows[1] (total padded rows) on the device. slot_pos
 * (nullable, M*topk entries) receives the sorted row of every flat slot
 * t*topk+j, or -1 for a dropped slot (for b200moe_combine_reduce). chunk_ready
 * (nullable, chunks_capacity + 2 entries) is zeroed for b200moe_experts and
 * b200moe_experts_fused. route_scratch (nullable) with route_scratch_ints >=
 * b200moe_route_scratch_ints(M*topk, E) entries lets large batches (from
 * 16,384 routed slots) route on several CTAs in two launches (same result);
 * without it one CTA routes everything.
 * ---------------------------------------------------------------------- */
B200MOE_API int64_t b200moe_route_capacity_rows(int64_t numel, int num_local_experts);
B200MOE_API int64_t b200moe_route_capacity_chunks(int64_t numel, int num_local_experts, int tile_tokens);
B200MOE_API int64_t b200moe_route_scratch_ints(int64_t numel, int num_local_experts);
B200MOE_API int b200moe_route(const int32_t* topk_ids, int64_t M, int topk, int num_experts, const int32_t* expert_map,
                  int num_local_experts, int tile_tokens, int32_t* sorted_ids, int64_t rows_capacity,
                  int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows, int64_t chunks_capacity,
                  int32_t* n_chunks, int32_t* num_rows, int32_t* slot_pos, int32_t* chunk_ready,
                  int32_t* route_scratch, int64_t route_scratch_ints, int32_t* err_word, void* stream);

/* Mixed work lists for skewed decode batches (what b200moe_layer does by
 * itself): with tiles of 16..64 tokens, experts with more than heavy_rows
 * padded rows (a skewed router's hot experts) are laid out after all the
 * others and cut into chunks of at most 128 rows in a second list, which
 * b200moe_experts_heavy runs with the token-major stages; the rest form the
 * usual tile_tokens list for b200moe_experts. The device decides per expert
 * after routing: no host synchronisation. counts (4 ints) receives
 * [light chunks, total rows, heavy chunks, first heavy row]; heavy_counters
 * (2 ints) is zeroed for b200moe_experts_heavy; heavy_chunks_capacity >=
 * b200moe_route_capacity_chunks(M*topk, E, 128). Below 16,384 routed slots
 * only (one-CTA routing). b200moe_heavy_rows(M, topk, tile) returns the
 * threshold the layer uses (128), or 0 when the layer does not split (M <=
 * 128: no expert can have more rows; tiles of 128/256; 16,384 slots or more).
 * Replaces nothing in the reference, whose kernels take one tile size per
 * launch (moe_decode_megakernel.py:88-123); sorted_ids keeps its meaning,
 * but the experts' order within it is light experts first. */
B200MOE_API int b200moe_heavy_rows(int64_t M, int topk, int tile_tokens);
B200MOE_API int b200moe_route_mixed(const int32_t* topk_ids, int64_t M, int topk, int num_experts,
                                    const int32_t* expert_map, int num_local_experts, int tile_tokens,
                                    int heavy_rows, int32_t* sorted_ids, int64_t rows_capacity,
                                    int32_t* chunk_expert, int32_t* chunk_row0, int32_t* chunk_rows,
                                    int64_t chunks_capacity, int32_t* heavy_chunk_expert, int32_t* heavy_chunk_row0,
                                    int32_t* heavy_chunk_rows, int64_t heavy_chunks_capacity, int32_t* counts,
                                    int32_t* slot_pos, int32_t* chunk_ready, int32_t* heavy_counters,
                                    int32_t* err_word, void* stream);

/* b200moe_route starting from router logits (the router of b200moe_router_topk
 * fused into routing's first launch; ids and weights stored to topk_ids /
 * topk_weights, then routed): results equal b200moe_router_topk followed by
 * b200moe_route bit for bit. route_scratch (required) holds
 * b200moe_route_logits_scratch_ints(M*topk, E) ints; its first int must be
 * zero before the first call and every call leaves it zero. Replaces the
 * reference's router launch (aiter topksoftmax) and moe_align_block_size. */
B200MOE_API int64_t b200moe_route_logits_scratch_ints(int64_t numel, int num_local_experts);
B200MOE_API int b200moe_route_logits(const void* logits, int logits_bf16, int64_t M, int num_experts, int topk,
                                     int scoring, const float* correction_bias, int renormalize, float scaling,
                                     float* topk_weights, int32_t* topk_ids, const int32_t* expert_map,
                                     int num_local_experts, int tile_tokens, int32_t* sorted_ids,
                                     int64_t rows_capacity, int32_t* chunk_expert, int32_t* chunk_row0,
                                     int32_t* chunk_rows, int64_t chunks_capacity, int32_t* n_chunks,
                                     int32_t* num_rows, int32_t* slot_pos, int32_t* chunk_ready,
                                     int32_t* route_scratch, int64_t route_scratch_ints, int32_t* err_word,
                                     void* stream);

/* Quantise hidden rows into the sorted layout: for every flat slot f with
 * p = slot_pos[f] >= 0 (from b200moe_route), row p of a_q (ld = H) holds
 * q(hidden[f / topk]) and its scales go to a_sT[g * a_s_ld + p] (transposed).
 * Padding rows are not written (a padding row only feeds GEMM outputs that are
 * discarded). a_s_ld >= rows_capacity. From 2,048 routed slots on (topk <= 32)
 * each token is quantised once and stored to all its slot rows; below, every
 * slot row is quantised on its own (same bytes either way). */
B200MOE_API int b200moe_gather_quant(const void* hidden, int64_t M, int64_t H, int topk, const int32_t* slot_pos,
                         int64_t rows_capacity, uint8_t* a_q, float* a_sT, int64_t a_s_ld, void* stream);

/* Copy already quantised rows into the sorted layout: for every flat slot f
 * with p = slot_pos[f] >= 0, row p of a_q (ld = H) = xq[f / topk] (row stride
 * ldxq bytes, 16-byte aligned), its scales xs[t * ldxs + g] to
 * a_sT[g * a_s_ld + p]. Padding rows are not written. The activation path of
 * the layer entries that take quantised rows (b200moe_layer_quantized,
 * b200moe_layer_packed); per token from 2,048 routed slots on, as
 * b200moe_gather_quant. */
B200MOE_API int b200moe_gather_rows(const uint8_t* xq, const float* xs, int64_t ldxq, int64_t ldxs, int64_t M, int64_t H,
                        int topk, const int32_t* slot_pos, int64_t rows_capacity, uint8_t* a_q, float* a_sT,
                        int64_t a_s_ld, void* stream);

/* Stage 1: inter = silu(gate) * up of (a1 . w13^T), re-quantised 1x128 into
 * a2_q (rows_capacity, I) and a2_sT (I/128, a_s_ld). grid_ctas = 0 picks one
 * CTA per SM; any other value fixes the persistent grid (results are
 * bit-identical for every grid). */
B200MOE_API int b200moe_gemm1_silu(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                       const uint8_t* w13, const float* w13_scale, int num_local_experts, int64_t H, int64_t I,
                       const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                       const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens, uint8_t* a2_q,
                       float* a2_sT, int32_t* err_word, int grid_ctas, void* stream);

/* Stage 2: topk_weights[f] * (a2 . w2^T)[p, :] for every sorted row p with
 * f = sorted_ids[p] < M*topk, accumulated in fp32 and stored as a bf16 row of H
 * (the reference rounds this product to bf16 too, aiter.py:164-177). Tiles of 16..64 tokens
 * write it to row f of out_pair (M*topk, H); token-major tiles (128, 256) to
 * row p of out_pair (rows_capacity, H), which keeps a unit's rows together in
 * memory (tiles of 128 store them with TMA: out_pair 16-byte aligned, and the
 * rows of a chunk without a slot, its expert's padding, are written as zeros).
 * Other padding rows and dropped slots are not written. */
B200MOE_API int b200moe_gemm2_combine(const uint8_t* a2_q, const float* a2_sT, int64_t a_s_ld, int64_t rows_capacity,
                          const uint8_t* w2, const float* w2_scale, int num_local_experts, int64_t H, int64_t I,
                          const int32_t* chunk_expert, const int32_t* chunk_row0, const int32_t* chunk_rows,
                          const int32_t* n_chunks, int64_t chunks_capacity, int tile_tokens,
                          const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk,
                          void* out_pair, int32_t* err_word, int grid_ctas, void* stream);

/* Stage 1 and stage 2 in one persistent launch (the reference's fused
 * stage-1 / stage-2 launcher pair, moe_decode_megakernel_fused.py:125-157,
 * as one kernel): same arguments and results as b200moe_gemm1_silu followed
 * by b200moe_gemm2_combine, bit for bit. A stage-2 work unit of a chunk
 * starts as soon as the stage-1 units of that chunk have written their rows,
 * which they count in chunk_ready (zeroed by b200moe_route for this call), so
 * the weight stream does not stop between the stages. Tiles of 16..64 tokens
 * run fused (cooperative launch, one CTA per SM; each CTA takes its next work
 * unit from the counter after the chunks_capacity per-chunk entries of
 * chunk_ready when it is free for one); 128 and 256 run the two stage kernels
 * back to back, whose CTAs take their work units from the two counters after
 * the per-chunk entries. Either way chunk_ready must be the one b200moe_route
 * zeroed for this call: a second call on the same routing needs a new
 * b200moe_route first. */
B200MOE_API int b200moe_experts(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld, int64_t rows_capacity,
                    const uint8_t* w13, const float* w13_scale, const uint8_t* w2, const float* w2_scale,
                    int num_local_experts, int64_t H, int64_t I, const int32_t* chunk_expert,
                    const int32_t* chunk_row0, const int32_t* chunk_rows, const int32_t* n_chunks,
                    int64_t chunks_capacity, int32_t* chunk_ready, int tile_tokens, uint8_t* a2_q, float* a2_sT,
                    const int32_t* sorted_ids, const float* topk_weights, int64_t M, int topk, void* out_pair,
                    int32_t* err_word, int grid_ctas, void* stream);

/* The heavy list of b200moe_route_mixed through the token-major stages
 * (stage 1 then stage 2, units from heavy_counters), writing stage-2 rows by
 * slot into the same out_pair (M*topk rows) as b200moe_experts does for the
 * light list, so one b200moe_combine_reduce (sorted_rows = 0) sums both. */
B200MOE_API int b200moe_experts_heavy(const uint8_t* a1_q, const float* a1_sT, int64_t a_s_ld,
                                      int64_t rows_capacity, const uint8_t* w13, const float* w13_scale,
                                      const uint8_t* w2, const float* w2_scale, int num_local_experts, int64_t H,
                                      int64_t I, const int32_t* heavy_chunk_expert, const int32_t* heavy_chunk_row0,
                                      const int32_t* heavy_chunk_rows, const int32_t* n_heavy_chunks,
                                      int64_t heavy_chunks_capacity, int32_t* heavy_counters, uint8_t* a2_q,
                                      float* a2_sT, const int32_t* sorted_ids, const float* topk_weights, int64_t M,
                                      int topk, void* out_pair, int32_t* err_word, int grid_ctas, void* stream);

/* Everything after b200moe_route for small batches (tiles of 16..64 tokens),
 * in one persistent launch (the single-launch layer the reference deferred,
 * phase8_findings.md:77-81): phase 0 quantises hidden[f / topk] into
 * sorted row slot_pos[f] of a1 for every routed slot f (as
 * b200moe_gather_quant), then both GEMM stages run as in b200moe_experts
 * (stage-2 rows by slot in out_pair, M*topk rows), then the top-k reduce
 * writes out (M, H) bf16 (as b200moe_combine_reduce with sorted_rows = 0).
 * Phases are ordered by device counters after chunk_ready (zeroed by
 * b200moe_route); results equal the separate stages bit for bit. Measured on
 * B200: as fast as the three launches at 64 tokens, 24 us slower at 128, so
 * b200moe_layer keeps the three launches. */
B200MOE_API int b200moe_experts_fused(const void* hidden, int64_t M, int topk, const int32_t* slot_pos, uint8_t* a1_q,
                          float* a1_sT, int64_t a_s_ld, int64_t rows_capacity, const uint8_t* w13,
                          const float* w13_scale, const uint8_t* w2, const float* w2_scale, int num_local_experts,
                          int64_t H, int64_t I, const int32_t* chunk_expert, const int32_t* chunk_row0,
                          const int32_t* chunk_rows, const int32_t* n_chunks, int64_t chunks_capacity,
                          int32_t* chunk_ready, int tile_tokens, uint8_t* a2_q, float* a2_sT,
                          const int32_t* sorted_ids, const float* topk_weights, void* out_pair, void* out,
                          int32_t* err_word, int grid_ctas, void* stream);

/* out[t, :] = bf16( sum_j row_j ) over the slots j with slot_pos[t*topk + j]
 * >= 0 (from b200moe_route), the bf16 rows summed in fp32 in order
 * j = 0..topk-1; row_j is
 * out_pair[slot_pos[t*topk + j]] when sorted_rows is non-zero (token-major
 * tiles), else out_pair[t*topk + j]. Replaces the unpermute of
 * sglang_integration/aiter.py:164-177. */
B200MOE_API int b200moe_combine_reduce(const void* out_pair, const int32_t* slot_pos, int sorted_rows, int64_t M,
                           int topk, int64_t H, void* out, void* stream);

/* ------------------------------------------------------------------------
 * Diagnostics.
 * ---------------------------------------------------------------------- */
/* Copies the device error word to *value (synchronises `stream`); when clear
 * is non-zero the word is reset to 0 afterwards. */
B200MOE_API int b200moe_read_error(int32_t* err_word, int32_t* value, int clear, void* stream);

/* Runs a one-CTA kernel that waits on an mbarrier nothing will complete,
 * with a limit of timeout_us microseconds, and reports the timeout through
 * the error word (B200MOE_DEVERR_TIMEOUT). Exercises the bounded-wait path
 * of the pipelines without faulting or hanging the GPU. */
B200MOE_API int b200moe_selftest_wait_timeout(int32_t* err_word, int timeout_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
