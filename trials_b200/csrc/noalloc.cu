// Layer entry point for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc (or any allocator) at
// the point where they run the layer: code running inside a captured or
// replayed CUDA graph region owned by someone else, engines whose memory pool
// is fixed at start-up and must not grow, or plugins whose host framework
// forbids device allocations from inside an operator. They still own the
// inputs and the output, but they have no way to provide the layer's
// workspace. b200moe_layer_noalloc runs the same kernels as b200moe_layer with
// the workspace placed in a file-scope device array instead.
//
// The array is kNoAllocScratchBytes (64 MiB) and every GPU that loads this
// code holds it until the process exits. It covers layers whose
// b200moe_layer_workspace_size() is at most that size, for example the
// GLM-5-like decode batch of 64 tokens (hidden 6144, intermediate 2048,
// 256 experts, top-8) at about 43 MB, and that layer up to 208 tokens;
// larger calls are rejected.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/b200moe.h"
#include "launch.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

}  // namespace

// Shared by every call on a device; keeps the previous call's contents.
static __device__ __align__(256) uint8_t g_layer_scratch[kNoAllocScratchBytes];

// Device address of g_layer_scratch on the current device. In host code the
// symbol name is only a host-side stand-in, so the address is looked up once
// per device with that device current and cached.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return b200moe::record_error(B200MOE_ERR_CUDA, "b200moe_layer_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_layer_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return b200moe::record_error(B200MOE_ERR_CUDA, "b200moe_layer_noalloc: cudaGetSymbolAddress failed");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return B200MOE_OK;
}

extern "C" int b200moe_layer_noalloc(const void* hidden, int64_t M, int64_t H, int64_t I, int num_experts,
                                     int topk, const uint8_t* w13, const float* w13_scale, const uint8_t* w2,
                                     const float* w2_scale, const float* topk_weights, const int32_t* topk_ids,
                                     const int32_t* expert_map, int num_local_experts, void* out,
                                     int32_t* err_out, void* stream) {
  const int E_plan = expert_map ? num_local_experts : num_experts;
  // A zero size means the shape itself is invalid (M < 0, H, I or topk <= 0).
  const size_t need = b200moe_layer_workspace_size(M, H, I, num_experts, E_plan, topk);
  if (need == 0 || E_plan <= 0)
    return b200moe::record_error(B200MOE_ERR_INVALID_ARG, "b200moe_layer_noalloc: bad argument (layer shape)");
  if (need > kNoAllocScratchBytes)
    return b200moe::record_error(B200MOE_ERR_WORKSPACE,
                                 "b200moe_layer_noalloc: layer needs more than the 64 MiB static scratch");
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The device error word is the first 4 bytes of the scratch; it must start
  // at zero for this call's status.
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), s) != cudaSuccess)
    return b200moe::record_error(B200MOE_ERR_CUDA, "b200moe_layer_noalloc: clearing the error word failed");
  st = b200moe_layer(hidden, M, H, I, num_experts, topk, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids,
                     expert_map, num_local_experts, out, scratch, kNoAllocScratchBytes, stream);
  if (st) return st;
  if (err_out != nullptr &&
      cudaMemcpyAsync(err_out, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return b200moe::record_error(B200MOE_ERR_CUDA, "b200moe_layer_noalloc: copying the error word failed");
  return B200MOE_OK;
}
