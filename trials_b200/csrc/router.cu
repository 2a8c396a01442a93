// Router: scores -> top-k expert ids and weights, one warp per token (the
// arithmetic is route_token_warp in router.cuh, shared with routing's first
// launch when routing starts from logits).
#include "common.cuh"
#include "launch.h"
#include "router.cuh"

namespace b200moe {

namespace {

constexpr int kRouterWarps = 4;

template <int PER>
__global__ void __launch_bounds__(kRouterWarps * 32) router_topk_kernel(const RouterArgs r, int64_t M) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (t >= M) return;
  int id;
  float w;
  route_token_warp<PER>(r, t, lane, id, w);
}

}  // namespace

cudaError_t launch_router_topk(const void* logits, int bf16, int64_t M, int E, int topk, int scoring,
                               const float* bias, int renormalize, float scaling, float* out_w, int32_t* out_ids,
                               cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((M + kRouterWarps - 1) / kRouterWarps);
  const RouterArgs r{logits, bf16, E, topk, scoring, renormalize, bias, scaling, out_w, out_ids};
  switch (router_per_lane(E)) {
    case 8:
      router_topk_kernel<8><<<blocks, kRouterWarps * 32, 0, stream>>>(r, M);
      break;
    case 16:
      router_topk_kernel<16><<<blocks, kRouterWarps * 32, 0, stream>>>(r, M);
      break;
    default:
      router_topk_kernel<32><<<blocks, kRouterWarps * 32, 0, stream>>>(r, M);
  }
  return cudaGetLastError();
}

}  // namespace b200moe
