// TVM-FFI binding of the operator for the FlashInfer-Bench harness.
//
// Exports `run` with the destination-passing signature the reference's CUDA
// solution registers (solution/cuda/main.cpp:38-49, exported at :117):
//   run(routing_logits, routing_bias, hidden_states, hidden_states_scale,
//       gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
//       local_expert_offset, routed_scaling_factor, output)
// It validates the DLPack tensors (device, dtype, rank, shapes, contiguity),
// keeps one device workspace per GPU (grown on demand, as the reference keeps
// its scratch cache, solution/cuda/kernel.cu:25-56) and forwards to the C ABI
// moe_fp8_block_scale_run on the caller's TVM-FFI stream. Argument errors raise
// ValueError, failed CUDA work RuntimeError, both carrying the C ABI's message.
#include <cuda_runtime.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <mutex>
#include <string>

#include "moe_fp8.h"

namespace {

using tvm::ffi::TensorView;

struct DeviceWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
DeviceWorkspace g_workspace[64];
std::mutex g_workspace_mutex;

void expect(bool ok, const std::string& what) {
  if (!ok) TVM_FFI_THROW(ValueError) << what;
}

void check_tensor(const TensorView& t, const char* name, int ndim, uint8_t code, int bits, int device) {
  expect(t.device().device_type == kDLCUDA, std::string(name) + " must be a CUDA tensor");
  expect(t.device().device_id == device, std::string(name) + " must be on the same GPU as routing_logits");
  expect(t.ndim() == ndim, std::string(name) + " must have " + std::to_string(ndim) + " dimensions");
  expect(t.dtype().code == code && t.dtype().bits == bits && t.dtype().lanes == 1,
         std::string(name) + " has the wrong dtype");
  expect(t.IsContiguous() && t.byte_offset() == 0, std::string(name) + " must be contiguous");
}

void* workspace_for(int device, size_t need) {
  std::lock_guard<std::mutex> lock(g_workspace_mutex);
  DeviceWorkspace& w = g_workspace[device];
  if (w.bytes < need) {
    if (w.ptr != nullptr) cudaFree(w.ptr);   // synchronises: earlier calls are done with it
    w.ptr = nullptr;
    w.bytes = 0;
    if (cudaMalloc(&w.ptr, need) != cudaSuccess) TVM_FFI_THROW(RuntimeError) << "workspace allocation failed";
    w.bytes = need;
  }
  return w.ptr;
}

void run(TensorView routing_logits, TensorView routing_bias, TensorView hidden_states, TensorView hidden_states_scale,
         TensorView gemm1_weights, TensorView gemm1_weights_scale, TensorView gemm2_weights,
         TensorView gemm2_weights_scale, int32_t local_expert_offset, float routed_scaling_factor,
         TensorView output) {
  expect(routing_logits.device().device_type == kDLCUDA, "routing_logits must be a CUDA tensor");
  const int dev = routing_logits.device().device_id;
  expect(dev >= 0 && dev < 64, "unsupported device id");
  check_tensor(routing_logits, "routing_logits", 2, kDLFloat, 32, dev);
  check_tensor(routing_bias, "routing_bias", 1, kDLBfloat, 16, dev);
  check_tensor(hidden_states, "hidden_states", 2, kDLFloat8_e4m3fn, 8, dev);
  check_tensor(hidden_states_scale, "hidden_states_scale", 2, kDLFloat, 32, dev);
  check_tensor(gemm1_weights, "gemm1_weights", 3, kDLFloat8_e4m3fn, 8, dev);
  check_tensor(gemm1_weights_scale, "gemm1_weights_scale", 3, kDLFloat, 32, dev);
  check_tensor(gemm2_weights, "gemm2_weights", 3, kDLFloat8_e4m3fn, 8, dev);
  check_tensor(gemm2_weights_scale, "gemm2_weights_scale", 3, kDLFloat, 32, dev);
  check_tensor(output, "output", 2, kDLBfloat, 16, dev);

  const int64_t T = routing_logits.size(0), E = gemm1_weights.size(0);
  expect(routing_logits.size(1) == 256, "routing_logits must be [T, 256]");
  expect(routing_bias.size(0) == 256, "routing_bias must be [256]");
  expect(hidden_states.size(0) == T && hidden_states.size(1) == 7168, "hidden_states must be [T, 7168]");
  expect(hidden_states_scale.size(0) == 56 && hidden_states_scale.size(1) == T, "hidden_states_scale must be [56, T]");
  expect(gemm1_weights.size(1) == 4096 && gemm1_weights.size(2) == 7168, "gemm1_weights must be [E, 4096, 7168]");
  expect(gemm1_weights_scale.size(0) == E && gemm1_weights_scale.size(1) == 32 && gemm1_weights_scale.size(2) == 56,
         "gemm1_weights_scale must be [E, 32, 56]");
  expect(gemm2_weights.size(0) == E && gemm2_weights.size(1) == 7168 && gemm2_weights.size(2) == 2048,
         "gemm2_weights must be [E, 7168, 2048]");
  expect(gemm2_weights_scale.size(0) == E && gemm2_weights_scale.size(1) == 56 && gemm2_weights_scale.size(2) == 16,
         "gemm2_weights_scale must be [E, 56, 16]");
  expect(output.size(0) == T && output.size(1) == 7168, "output must be [T, 7168]");
  expect(T <= INT32_MAX && E >= 1 && E <= 256, "unsupported token or expert count");

  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  const size_t need = moe_fp8_workspace_bytes((int32_t)T, (int32_t)E);
  MoeFp8Args a{};
  a.routing_logits = static_cast<const float*>(routing_logits.data_ptr());
  a.routing_bias = routing_bias.data_ptr();
  a.hidden_states = hidden_states.data_ptr();
  a.hidden_states_scale = static_cast<const float*>(hidden_states_scale.data_ptr());
  a.gemm1_weights = gemm1_weights.data_ptr();
  a.gemm1_weights_scale = static_cast<const float*>(gemm1_weights_scale.data_ptr());
  a.gemm2_weights = gemm2_weights.data_ptr();
  a.gemm2_weights_scale = static_cast<const float*>(gemm2_weights_scale.data_ptr());
  a.local_expert_offset = local_expert_offset;
  a.routed_scaling_factor = routed_scaling_factor;
  a.output = output.data_ptr();
  a.num_tokens = (int32_t)T;
  a.num_local_experts = (int32_t)E;
  a.workspace = workspace_for(dev, need);
  a.workspace_bytes = need;
  const int rc = moe_fp8_block_scale_run(&a, TVMFFIEnvGetStream(kDLCUDA, dev));
  if (prev != dev) cudaSetDevice(prev);
  if (rc == MOE_ERR_INVALID_ARGUMENT) TVM_FFI_THROW(ValueError) << moe_fp8_last_error();
  if (rc != MOE_OK) TVM_FFI_THROW(RuntimeError) << moe_fp8_last_error();
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(run, run);
