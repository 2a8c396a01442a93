// Replica choice of the expert-parallel dispatch (plan and pack kernels of
// both exchange forms use it, so they agree on every routed slot).
#pragma once

#include "launch.h"

namespace b200moe {

// Physical slot (rank * slots + local index) that routed slot (t, j) of token
// t with expert id `id` goes to, or -1 (id outside [0, num_experts), or a
// replica table entry outside the G * slots physical slots). With replicas
// the one on the source rank wins (its rows then stay on this GPU); otherwise
// slots rotate over the replicas by t * topk + j, which spreads a hot
// expert's rows evenly over its replicas.
__device__ __forceinline__ int ep_target(const EpPlace& pl, int id, int64_t t, int j, int topk) {
  if (id < 0 || id >= pl.num_experts) return -1;
  if (pl.rep == nullptr) return id;
  const int32_t* r = pl.rep + (int64_t)id * (1 + pl.max_rep);
  const int n = __ldg(r);
  if (n <= 0 || n > pl.max_rep) return -1;
  int p = -1;
  for (int k = 0; k < n; ++k) {
    const int q = __ldg(r + 1 + k);
    if (q / pl.slots == pl.src_rank) {
      p = q;
      break;
    }
  }
  if (p < 0) p = __ldg(r + 1 + (int)((t * topk + j) % n));
  return (p >= 0 && p < pl.G * pl.slots) ? p : -1;
}

}  // namespace b200moe
