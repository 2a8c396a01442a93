// Instantiations and launcher of the persistent grouped GEMM.
#include "launch.h"
#include "moe_gemm.cuh"
#include "moe_gemm_tok.cuh"

namespace b200moe {

namespace {

template <int T, int CS, int EPI>
cudaError_t launch_cfg(const CUtensorMap& tm_w, const CUtensorMap& tm_a, const GemmParams& p, int grid,
                       cudaStream_t stream) {
  using C = GemmCfg<T, CS>;
  auto kernel = moe_grouped_gemm_kernel<T, CS, EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_w, tm_a, p);
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_tok(const CUtensorMap& tm_w, const CUtensorMap& tm_a, const GemmParams& p, int grid,
                       cudaStream_t stream) {
  auto kernel = moe_grouped_gemm_tok_kernel<EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TokCfg::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  kernel<<<grid, TokCfg::THREADS, TokCfg::SMEM_BYTES, stream>>>(tm_w, tm_a, p);
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_epi(int tile_tokens, const CUtensorMap& tm_w, const CUtensorMap& tm_a, const GemmParams& p,
                       int grid, cudaStream_t stream) {
  switch (tile_tokens) {
    case 16:
    case 32:
      return launch_cfg<32, 1, EPI>(tm_w, tm_a, p, grid, stream);
    case 64:
      // SiLU epilogue: one column slice (no register spills, measured faster);
      // combine epilogue: two slices (more warps hide its global stores).
      return launch_cfg<64, EPI == EPI_SILU ? 1 : 2, EPI>(tm_w, tm_a, p, grid, stream);
    case 128:
      // Many tokens per expert: routed rows on the MMA M side.
      return launch_tok<EPI>(tm_w, tm_a, p, grid, stream);
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
      return 128;
    default:
      return 0;
  }
}

cudaError_t launch_grouped_gemm(int epi, int tile_tokens, const CUtensorMap& tm_w, const CUtensorMap& tm_a,
                                const GemmParams& p, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  if (epi == EPI_SILU) return launch_epi<EPI_SILU>(tile_tokens, tm_w, tm_a, p, grid, stream);
  return launch_epi<EPI_COMBINE>(tile_tokens, tm_w, tm_a, p, grid, stream);
}

}  // namespace b200moe
