// Instantiations and launcher of the persistent grouped GEMM.
#include <atomic>

#include "launch.h"
#include "moe_gemm.cuh"
#include "moe_gemm_tok.cuh"
#include "moe_gemm_tok2.cuh"

namespace b200moe {

namespace {

int sm_count_cached() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

template <int T, int CS, int EPI>
cudaError_t launch_cfg(const CUtensorMap& tm_w, const CUtensorMap& tm_a, const GemmParams& p,
                       const CUtensorMap& tm_w2, const CUtensorMap& tm_a2, const GemmParams& p2, int grid,
                       cudaStream_t stream) {
  using C = GemmCfg<T, CS>;
  auto kernel = moe_grouped_gemm_kernel<T, CS, EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  if (EPI < EPI_FUSED) {
    kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_w, tm_a, p, tm_w2, tm_a2, p2);
    return cudaGetLastError();
  }
  // Stage-2 units wait for stage-1 units of other CTAs: the whole grid must
  // be resident at once, which a cooperative launch guarantees (or refuses).
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, C::THREADS + 32, C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  const int resident = per_sm * sm_count_cached();
  if (resident <= 0) return cudaErrorCooperativeLaunchTooLarge;
  if (grid > resident) grid = resident;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(C::THREADS + 32, 1, 1);  // + the publisher warp
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  // EPI_FUSED follows the gather launch: launched programmatically, its
  // prologue (barriers, TMEM, tensor maps) overlaps the gather's end. Should
  // the runtime refuse the pair of attributes, the launch goes without it.
  static std::atomic<bool> pdl_ok{true};
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (B200MOE_PDL && EPI == EPI_FUSED && pdl_ok.load()) ? 2 : 1;
  err = cudaLaunchKernelEx(&cfg, kernel, tm_w, tm_a, p, tm_w2, tm_a2, p2);
  if (err != cudaSuccess && cfg.numAttrs == 2) {
    cudaGetLastError();  // clear it, then launch as before
    pdl_ok.store(false);
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, kernel, tm_w, tm_a, p, tm_w2, tm_a2, p2);
  }
  return err;
}

template <int EPI>
cudaError_t launch_tok(const CUtensorMap& tm_w, const CUtensorMap& tm_a, const CUtensorMap& tm_o, const GemmParams& p,
                       int grid, cudaStream_t stream) {
  using C = TokCfgE<EPI>;
  auto kernel = moe_grouped_gemm_tok_kernel<EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  return launch_pdl(kernel, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, tm_w, tm_a, tm_o, p);
}

template <int EPI>
cudaError_t launch_tok2(const CUtensorMap& tm_w, const CUtensorMap& tm_a, const GemmParams& p, int grid,
                        cudaStream_t stream) {
  auto kernel = moe_grouped_gemm_tok2_kernel<EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Tok2Cfg::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  // Pairs that can be resident at once (clusters must fit inside a GPC).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(Tok2Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Tok2Cfg::SMEM_BYTES;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  err = cudaOccupancyMaxActiveClusters(&max_clusters, kernel, &cfg);
  if (err != cudaSuccess) return err;
  int pairs = grid / 2;
  if (max_clusters > 0 && pairs > max_clusters) pairs = max_clusters;
  if (pairs < 1) pairs = 1;
  kernel<<<2 * pairs, Tok2Cfg::THREADS, Tok2Cfg::SMEM_BYTES, stream>>>(tm_w, tm_a, p);
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_epi(int tile_tokens, const CUtensorMap& tm_w, const CUtensorMap& tm_a, const CUtensorMap& tm_o,
                       const GemmParams& p, int grid, cudaStream_t stream) {
  switch (tile_tokens) {
    case 16:
    case 32:
      return launch_cfg<32, 1, EPI>(tm_w, tm_a, p, tm_w, tm_a, p, grid, stream);
    case 64:
      // SiLU epilogue: one column slice (no register spills, measured faster);
      // combine epilogue: two slices (more warps hide its global stores).
      return launch_cfg<64, EPI == EPI_SILU ? 1 : 2, EPI>(tm_w, tm_a, p, tm_w, tm_a, p, grid, stream);
    case 128:
      // Many tokens per expert: routed rows on the MMA M side.
      return launch_tok<EPI>(tm_w, tm_a, tm_o, p, grid, stream);
    case 256:
      // Even more: CTA pairs with a 256-row MMA.
      return launch_tok2<EPI>(tm_w, tm_a, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace

int gemm_tile_rows(int tile_tokens) {
  switch (tile_tokens) {
    case 16:
    case 32:
      return 32;
    case 64:
      return 64;
    case 128:
    case 256:
      return 128;  // per CTA for 256 (pairs)
    default:
      return 0;
  }
}

cudaError_t launch_grouped_gemm_fused(int tile_tokens, const CUtensorMap& tm_w1, const CUtensorMap& tm_a1,
                                      const GemmParams& p1, const CUtensorMap& tm_w2, const CUtensorMap& tm_a2,
                                      const GemmParams& p2, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  // routing in the launch (route_sync set), gather + reduce phases (q0.rows > 0), or neither
  const int epi = p1.route_sync ? EPI_WHOLE : (p1.q0.rows > 0 ? EPI_LAYER : EPI_FUSED);
  switch (tile_tokens) {
    case 16:
    case 32:
      if (epi == EPI_WHOLE) return launch_cfg<32, 1, EPI_WHOLE>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream);
      return epi == EPI_LAYER ? launch_cfg<32, 1, EPI_LAYER>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream)
                              : launch_cfg<32, 1, EPI_FUSED>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream);
    case 64:
      if (epi == EPI_WHOLE) return launch_cfg<64, 1, EPI_WHOLE>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream);
      return epi == EPI_LAYER ? launch_cfg<64, 1, EPI_LAYER>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream)
                              : launch_cfg<64, 1, EPI_FUSED>(tm_w1, tm_a1, p1, tm_w2, tm_a2, p2, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_grouped_gemm(int epi, int tile_tokens, const CUtensorMap& tm_w, const CUtensorMap& tm_a,
                                const CUtensorMap& tm_o, const GemmParams& p, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  if (tile_tokens == 256 && grid < 2) grid = 2;
  if (epi == EPI_SILU) return launch_epi<EPI_SILU>(tile_tokens, tm_w, tm_a, tm_o, p, grid, stream);
  return launch_epi<EPI_COMBINE>(tile_tokens, tm_w, tm_a, tm_o, p, grid, stream);
}

}  // namespace b200moe
