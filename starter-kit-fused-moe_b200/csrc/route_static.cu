// Routing entry point that allocates nothing.
//
// Some callers may not allocate device memory on the path where they call this
// operator: a TensorRT plugin's enqueue(), an XLA/JAX custom call that only gets
// the buffers its framework planned, or an engine whose memory is carved from a
// pool reserved at start-up and that forbids cudaMalloc (and torch's caching
// allocator) once serving begins. They cannot provide the workspace the other
// entry points take. For them, moe_fp8_route_static runs the same routing
// kernel as moe_fp8_route, with its scratch (the per-expert counters and each
// selection's position inside its expert group) in a fixed array that lives in
// this library's device image:
//
//   * size: 256 counters + 8 positions per token for up to kStaticMaxTokens
//     (16,384) tokens, about 513 KB, held on every GPU that loads this code
//     until the process exits;
//   * the array is shared by every call: the counters are cleared at the start
//     of each call, and calls that overlap on the GPU (two streams, two host
//     threads) race on it and must be serialised by the caller;
//   * the first call on a device looks up the array's device address with that
//     device current (cudaGetSymbolAddress) and caches it; make that first call
//     before capturing a stream into a CUDA graph.
#include <mutex>
#include <string>

#include "moe_fp8.h"
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace {

constexpr int kStaticMaxTokens = 16384;
constexpr int kCounters = moe::kMaxLocalExperts;

// [0, 256): expert counters; [256, 256 + 8 * kStaticMaxTokens): selection positions.
static __device__ __align__(256) int32_t g_route_scratch[kCounters + moe::kTopK * kStaticMaxTokens];

int static_fail(int code, const std::string& msg) {
  moe::set_last_error(msg.c_str());
  return code;
}

// Device address of g_route_scratch on the current device (looked up once per device).
cudaError_t scratch_address(int32_t** out) {
  static std::mutex mu;
  static int32_t* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = static_cast<int32_t*>(p);
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int moe_fp8_route_static(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                         int32_t local_expert_offset, int32_t num_local_experts, float routed_scaling_factor,
                         int32_t* topk_idx, float* topk_weights, void* stream) {
  const int T = num_tokens, E = num_local_experts;
  if (T < 0 || T > kStaticMaxTokens)
    return static_fail(MOE_ERR_INVALID_ARGUMENT, "moe_fp8_route_static: num_tokens must be in [0, " +
                                                     std::to_string(kStaticMaxTokens) + "], got " +
                                                     std::to_string(T));
  if (E < 1 || E > moe::kMaxLocalExperts)
    return static_fail(MOE_ERR_INVALID_ARGUMENT, "moe_fp8_route_static: num_local_experts must be in [1, 256]");
  if (T == 0) return MOE_OK;
  const auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!routing_logits || !topk_idx || !topk_weights || !aligned16(routing_logits) ||
      (routing_bias && !aligned16(routing_bias)))
    return static_fail(MOE_ERR_INVALID_ARGUMENT,
                       "moe_fp8_route_static: logits / outputs must be non-NULL device pointers, "
                       "logits and bias 16-byte aligned");
  int32_t* scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess)
    return static_fail(MOE_ERR_CUDA, std::string("moe_fp8_route_static: cudaGetSymbolAddress: ") +
                                         cudaGetErrorString(e));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the counters must start at zero; the positions are fully rewritten
  e = cudaMemsetAsync(scratch, 0, sizeof(int32_t) * E, st);
  if (e == cudaSuccess)
    e = moe::launch_route(routing_logits, static_cast<const __nv_bfloat16*>(routing_bias), T, local_expert_offset,
                          E, routed_scaling_factor, topk_idx, topk_weights, scratch + kCounters, scratch, nullptr,
                          nullptr, st);
  if (e != cudaSuccess)
    return static_fail(MOE_ERR_CUDA, std::string("moe_fp8_route_static: ") + cudaGetErrorString(e));
  return MOE_OK;
}

}  // extern "C"
