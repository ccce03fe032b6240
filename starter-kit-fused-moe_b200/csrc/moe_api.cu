// C-ABI layer: argument checks, workspace carving, TMA descriptors and the
// launch sequence route -> permute -> GEMM1 -> GEMM2 -> finalize.
//
// Mirrors the reference's CUDA entry (solution/cuda/main.cpp:38-117: shape and
// dtype checks, then launch on the caller's stream) and its launcher
// (solution/cuda/kernel.cu:60-109), without any host synchronisation: the
// per-expert histogram stays on the device and the GEMM kernels build their
// tile lists from it.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "moe_fp8.h"
#include "moe_common.cuh"
#include "moe_kernels.h"
#include "moe_workspace.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
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

// 2-D byte tensor [rows, cols] (row-major), tile box [box_rows, 128 bytes], 128-byte swizzle.
bool encode_fp8_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                   uint32_t box_cols = 128) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms_of_current_device() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cache[dev] = n;
  return n;
}

int gemm_path(int T);
bool deterministic();

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_workspace(void* ws, size_t bytes, int T, int E) {
  if (!ws) return fail(MOE_ERR_WORKSPACE, "workspace is NULL");
  if (!aligned(ws, 256)) return fail(MOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const size_t need = moe::ws_layout(T, E, deterministic()).total;
  if (bytes < need)
    return fail(MOE_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes, got " +
                                       std::to_string(bytes));
  return MOE_OK;
}

}  // namespace

void moe::set_last_error(const char* msg) { g_last_error = msg; }

extern "C" {

const char* moe_fp8_last_error(void) { return g_last_error.c_str(); }

size_t moe_fp8_workspace_bytes(int32_t max_tokens, int32_t num_local_experts) {
  if (max_tokens < 0 || num_local_experts < 1 || num_local_experts > moe::kMaxLocalExperts) return 0;
  return moe::ws_layout(max_tokens, num_local_experts, deterministic()).total;
}

int32_t moe_fp8_kernels_per_call(int32_t num_tokens) {
  if (num_tokens <= 0) return 0;
  return gemm_path(num_tokens) == 2 ? 4 : 5;
}

int moe_fp8_workspace_view(void* workspace, int32_t T, int32_t E, MoeFp8WorkspaceView* view) {
  if (!workspace || !view || T < 0 || E < 1 || E > moe::kMaxLocalExperts)
    return fail(MOE_ERR_INVALID_ARGUMENT, "bad workspace view request");
  const moe::WsLayout L = moe::ws_layout(T, E);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  view->topk_idx = reinterpret_cast<int32_t*>(w + L.topk_idx);
  view->topk_weights = reinterpret_cast<float*>(w + L.topk_w);
  view->expert_counts = reinterpret_cast<int32_t*>(w + L.counts);
  view->device_error = reinterpret_cast<int32_t*>(w + L.err);
  view->pair_capacity = L.R1;
  return MOE_OK;
}

int moe_fp8_read_device_error(void* workspace, void* stream, int32_t* bits) {
  if (!workspace || !bits) return fail(MOE_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* dev = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + moe::ws_layout(0, 1).err);
  int32_t h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, dev, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dev, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  *bits = h;
  if (h) return fail(MOE_ERR_DEVICE_TIMEOUT, "a kernel gave up on a bounded wait (bits " + std::to_string(h) + ")");
  return MOE_OK;
}

int moe_fp8_route(const float* logits, const void* bias, int32_t T, int32_t offset, int32_t E, float scale,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (T < 0 || E < 1 || E > moe::kMaxLocalExperts) return fail(MOE_ERR_INVALID_ARGUMENT, "bad T or E");
  if (T > 0 && (!logits || !aligned(logits, 16)))
    return fail(MOE_ERR_INVALID_ARGUMENT, "routing_logits must be a 16-byte aligned device pointer");
  if (bias && !aligned(bias, 16)) return fail(MOE_ERR_INVALID_ARGUMENT, "routing_bias must be 16-byte aligned");
  if (int rc = check_workspace(workspace, workspace_bytes, T, E)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const moe::WsLayout L = moe::ws_layout(T, E);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(w + L.counts, 0, sizeof(int32_t) * E, st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing expert counts");
  e = moe::launch_route(logits, static_cast<const __nv_bfloat16*>(bias), T, offset, E, scale,
                        reinterpret_cast<int*>(w + L.topk_idx), reinterpret_cast<float*>(w + L.topk_w),
                        reinterpret_cast<int*>(w + L.pair_pos), reinterpret_cast<int*>(w + L.counts), nullptr, nullptr,
                        st);
  if (e != cudaSuccess) return cuda_fail(e, "routing kernel launch");
  return MOE_OK;
}

}  // extern "C"

namespace {

// Everything one call needs: validated arguments, workspace carve-up, TMA maps.
struct Plan {
  const MoeFp8Args* a;
  moe::WsLayout L;
  int nsm;
  int* counts; int* topk_idx; float* topk_w; int* pair_pos; int* row_token; float* row_weight;
  uint8_t* a1; float* sa1; uint8_t* a2; float* sa2; float* acc; int* err;
  CUtensorMap tmA1, tmB1, tmA2, tmB2, tmO1;
  int path;  // see gemm_path()
  bool det;  // deterministic combine (see moe_fp8_set_deterministic)
  float* pair_out;
  const int* given_idx;    // routed mode: selections made elsewhere [T, 8]
  const float* given_w;
  bool f32_out;            // routed mode without output: fp32 rows stay in the workspace
};

// GEMM kernel families per call:
//   0  128-row tile kernels for both GEMMs
//   1  weight-streaming GEMM1, tile GEMM2
//   2  one weight-streaming launch for GEMM1 and GEMM2 (fused queue)
//   3  weight-streaming GEMM1 and GEMM2 as two launches
// Automatic choice from measured crossovers on B200 (offset-0 routing, 32
// local experts): the fused streaming launch up to 240 tokens, tile kernels above.
std::atomic<int> g_deterministic{-2};
bool deterministic() {
  int d = g_deterministic.load(std::memory_order_relaxed);
  if (d == -2) {
    const char* e = getenv("MOE_DETERMINISTIC");
    d = (e && atoi(e) != 0) ? 1 : 0;
    g_deterministic.store(d, std::memory_order_relaxed);
  }
  return d == 1;
}

std::atomic<int> g_forced_path{-2};
int gemm_path(int T) {
  if (deterministic()) return 0;     // the tile kernels are the ones with an ordered combine
  int f = g_forced_path.load(std::memory_order_relaxed);
  if (f == -2) {
    const char* e = getenv("MOE_GEMM_PATH");
    f = e ? atoi(e) : -1;
    g_forced_path.store(f, std::memory_order_relaxed);
  }
  if (f >= 0 && f <= 3) return f;
  return T <= 240 ? 2 : 0;
}

int make_plan(const MoeFp8Args* a, Plan& p, const int* given_idx = nullptr, const float* given_w = nullptr) {
  if (!a) return fail(MOE_ERR_INVALID_ARGUMENT, "args is NULL");
  const int T = a->num_tokens, E = a->num_local_experts;
  if (T < 0) return fail(MOE_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0");
  if (E < 1 || E > moe::kMaxLocalExperts)
    return fail(MOE_ERR_INVALID_ARGUMENT, "num_local_experts must be in [1, 256]");
  if (T == 0) return MOE_OK;
  const bool routed = given_idx != nullptr;
  if (routed && !given_w) return fail(MOE_ERR_INVALID_ARGUMENT, "topk_weights is NULL");
  if ((!routed && !a->routing_logits) || !a->hidden_states || !a->hidden_states_scale || !a->gemm1_weights ||
      !a->gemm1_weights_scale || !a->gemm2_weights || !a->gemm2_weights_scale || (!routed && !a->output))
    return fail(MOE_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (routed && !a->output && deterministic())
    return fail(MOE_ERR_INVALID_ARGUMENT, "fp32 routed output is not available in deterministic mode");
  p.given_idx = given_idx;
  p.given_w = given_w;
  p.f32_out = routed && !a->output;
  if ((!routed && !aligned(a->routing_logits, 16)) || !aligned(a->hidden_states, 16) ||
      !aligned(a->gemm1_weights, 16) || !aligned(a->gemm2_weights, 16) || !aligned(a->output, 16) ||
      (a->routing_bias && !aligned(a->routing_bias, 16)) || !aligned(a->hidden_states_scale, 16) ||
      !aligned(a->gemm1_weights_scale, 16) || !aligned(a->gemm2_weights_scale, 16))
    return fail(MOE_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  if (int rc = check_workspace(a->workspace, a->workspace_bytes, T, E)) return rc;
  p.a = a;
  p.nsm = num_sms_of_current_device();
  p.det = deterministic();
  p.L = moe::ws_layout(T, E, p.det);
  const moe::WsLayout& L = p.L;
  uint8_t* w = static_cast<uint8_t*>(a->workspace);
  p.counts = reinterpret_cast<int*>(w + L.counts);
  p.topk_idx = reinterpret_cast<int*>(w + L.topk_idx);
  p.topk_w = reinterpret_cast<float*>(w + L.topk_w);
  p.pair_pos = reinterpret_cast<int*>(w + L.pair_pos);
  p.row_token = reinterpret_cast<int*>(w + L.row_token);
  p.row_weight = reinterpret_cast<float*>(w + L.row_weight);
  p.a1 = w + L.a1;
  p.sa1 = reinterpret_cast<float*>(w + L.sa1);
  p.a2 = w + L.a2;
  p.sa2 = reinterpret_cast<float*>(w + L.sa2);
  p.acc = reinterpret_cast<float*>(w + L.out_acc);
  p.err = reinterpret_cast<int*>(w + L.err);
  p.pair_out = p.det ? reinterpret_cast<float*>(w + L.pair_out) : nullptr;
  p.path = gemm_path(T);
  const bool s1 = p.path != 0, s2 = p.path >= 2;
  // the CTA-pair tile kernels load 128 W2 rows per CTA
  const uint32_t w2_box = (s2 || moe::cta_pair_enabled()) ? 128 : 256;
  // streaming kernels: 128-byte boxes, 128-byte swizzle; tile kernels: boxes as wide as their stages
  const uint32_t c1 = s1 ? 128 : moe::kTileStageK1, c2 = s2 ? 128 : moe::kTileStageK2;
  if (!encode_fp8_2d(&p.tmA1, p.a1, moe::kHidden, L.R1, s1 ? 16 : 128, c1) ||
      !encode_fp8_2d(&p.tmB1, a->gemm1_weights, moe::kHidden, (uint64_t)E * moe::kGemm1N, 128, c1) ||
      !encode_fp8_2d(&p.tmA2, p.a2, moe::kInter, 2ull * L.R1, s2 ? 16 : 128, c2) ||
      !encode_fp8_2d(&p.tmB2, a->gemm2_weights, moe::kInter, (uint64_t)E * moe::kHidden, w2_box, c2) ||
      !encode_fp8_2d(&p.tmO1, p.a2, 2 * moe::kInter, L.R1, 32, 64))
    return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return MOE_OK;
}

int launch_stage(const Plan& p, int stage, cudaStream_t st) {
  const MoeFp8Args* a = p.a;
  const int T = a->num_tokens, E = a->num_local_experts;
  cudaError_t e = cudaSuccess;
  switch (stage) {
    case 0:
      // one memset: the call's error word (word 1 of the error area) through the counter block
      e = cudaMemsetAsync(p.err + 1, 0, p.L.counts + moe::WsLayout::kCountersBytes - p.L.err - sizeof(int), st);
      if (e != cudaSuccess) return cuda_fail(e, "clearing expert counts");
      e = moe::launch_route(a->routing_logits, static_cast<const __nv_bfloat16*>(a->routing_bias), T,
                            a->local_expert_offset, E, a->routed_scaling_factor, p.topk_idx, p.topk_w, p.pair_pos,
                            p.counts, (p.path >= 2 || p.det) ? nullptr : p.acc, static_cast<__nv_bfloat16*>(a->output),
                            st, p.given_idx, p.given_w);
      if (e != cudaSuccess) return cuda_fail(e, "routing kernel launch");
      break;
    case 1:
      e = moe::launch_permute(static_cast<const uint8_t*>(a->hidden_states), a->hidden_states_scale, T, E,
                              a->local_expert_offset, p.topk_idx, p.topk_w, p.pair_pos, p.counts, p.L.R1, p.a1,
                              p.sa1, p.row_token, p.row_weight, p.err, p.nsm, st);
      if (e != cudaSuccess) return cuda_fail(e, "permute kernel launch");
      break;
    case 2:
    case 3: {
      if (p.path >= 2) {
        // streaming kernel: path 2 does both GEMMs in stage 2; path 3 one GEMM per stage
        if (p.path == 2 && stage == 3) break;
        uint8_t* w = static_cast<uint8_t*>(a->workspace);
        moe::DecodeArgs d{};
        d.mode = p.path == 2 ? 3 : stage - 1;
        d.E = E;
        d.R1 = p.L.R1;
        d.counts = p.counts;
        d.sa1 = p.sa1;
        d.sa2 = p.sa2;
        d.s13 = a->gemm1_weights_scale;
        d.s2 = a->gemm2_weights_scale;
        d.a2 = p.a2;
        d.row_token = p.row_token;
        d.row_weight = p.row_weight;
        d.out_acc = p.acc;
        d.err = p.err;
        d.queue = reinterpret_cast<int*>(w + p.L.queue());
        d.done1 = reinterpret_cast<int*>(w + p.L.done1());
        d.T = T;
        d.zero_done = reinterpret_cast<int*>(w + p.L.zero_done());
        d.zero_acc = d.mode != 1;            // this launch runs the GEMM2 tiles: it owns the zeroing
        d.prefetch_kb = d.mode != 2 ? 16 : 0;
        d.split_partial = reinterpret_cast<float*>(w + p.L.split_partial);
        d.split_cnt = reinterpret_cast<int*>(w + p.L.split_cnt());
        e = moe::launch_stream_gemm(p.tmA1, p.tmB1, p.tmA2, p.tmB2, d, p.nsm, st);
        if (e != cudaSuccess) return cuda_fail(e, "streaming GEMM launch");
        break;
      }
      if (stage == 2 && p.path == 1) {
        moe::DecodeArgs d{};
        uint8_t* w = static_cast<uint8_t*>(a->workspace);
        d.mode = 1;
        d.E = E;
        d.R1 = p.L.R1;
        d.counts = p.counts;
        d.sa1 = p.sa1;
        d.sa2 = p.sa2;
        d.s13 = a->gemm1_weights_scale;
        d.s2 = a->gemm2_weights_scale;
        d.a2 = p.a2;
        d.err = p.err;
        d.queue = reinterpret_cast<int*>(w + p.L.queue());
        d.done1 = reinterpret_cast<int*>(w + p.L.done1());
        e = moe::launch_stream_gemm(p.tmA1, p.tmB1, p.tmA2, p.tmB2, d, p.nsm, st);
        if (e != cudaSuccess) return cuda_fail(e, "streaming GEMM1 launch");
        break;
      }
      moe::GemmArgs g{};
      g.counts = p.counts;
      g.E = E;
      g.R1 = p.L.R1;
      g.err = p.err;
      g.T = T;
      if (stage == 2) {
        g.sa = p.sa1;
        g.sb = a->gemm1_weights_scale;
        g.a2 = p.a2;
        g.sa2 = p.sa2;
        g.split_partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a->workspace) + p.L.split_partial);
        g.split_cnt = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a->workspace) + p.L.split_cnt());
        g.no_split = p.det;
        e = moe::launch_gemm1(p.tmA1, p.tmB1, p.tmO1, g, p.nsm, st);
      } else {
        g.sa = p.sa2;
        g.sb = a->gemm2_weights_scale;
        g.row_token = p.row_token;
        g.row_weight = p.row_weight;
        g.out_acc = p.acc;
        g.pair_out = p.pair_out;
        g.no_split = p.det;
        e = moe::launch_gemm2(p.tmA2, p.tmB2, g, p.nsm, st);
      }
      if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
      break;
    }
    case 4:
      if (p.f32_out) break;      // routed mode without output: the fp32 rows stay in the workspace
      if (p.det) {
        e = moe::launch_finalize_ordered(p.pair_out, static_cast<__nv_bfloat16*>(a->output), T, p.topk_idx, p.pair_pos,
                                         p.counts, a->local_expert_offset, E, p.err, st);
        if (e != cudaSuccess) return cuda_fail(e, "finalize launch");
        break;
      }
      e = moe::launch_finalize(p.acc, static_cast<__nv_bfloat16*>(a->output), T, p.topk_idx, a->local_expert_offset,
                               E, p.err, st);
      if (e != cudaSuccess) return cuda_fail(e, "finalize launch");
      break;
    default:
      return fail(MOE_ERR_INVALID_ARGUMENT, "stage must be in [0, 4]");
  }
  return MOE_OK;
}

}  // namespace

extern "C" {

int moe_fp8_block_scale_run(const MoeFp8Args* a, void* stream) {
  Plan p{};
  if (int rc = make_plan(a, p)) return rc;
  if (a->num_tokens == 0) return MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int stage = 0; stage < 5; ++stage)
    if (int rc = launch_stage(p, stage, st)) return rc;
  return MOE_OK;
}

int moe_fp8_block_scale_run_routed(const MoeFp8Args* a, const int32_t* topk_idx, const float* topk_weights,
                                   void* stream) {
  if (!topk_idx) return fail(MOE_ERR_INVALID_ARGUMENT, "topk_idx is NULL");
  Plan p{};
  if (int rc = make_plan(a, p, topk_idx, topk_weights)) return rc;
  if (a->num_tokens == 0) return MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int stage = 0; stage < 5; ++stage)
    if (int rc = launch_stage(p, stage, st)) return rc;
  return MOE_OK;
}

int32_t moe_fp8_set_gemm_path(int32_t path) {
  gemm_path(0);  // resolve the environment default once
  const int32_t old = g_forced_path.load(std::memory_order_relaxed);
  if (path >= -1 && path <= 3) g_forced_path.store(path, std::memory_order_relaxed);
  return old;
}

int32_t moe_fp8_gemm_path(int32_t num_tokens) { return gemm_path(num_tokens); }

int32_t moe_fp8_set_cta_pair(int32_t on) { return moe::set_cta_pair(on); }

int32_t moe_fp8_set_deterministic(int32_t on) {
  const int32_t old = deterministic() ? 1 : 0;
  g_deterministic.store(on ? 1 : 0, std::memory_order_relaxed);
  return old;
}

int moe_fp8_quantize_activations(const void* x, int32_t x_is_bf16, int32_t T, void* hidden_states,
                                 float* hidden_states_scale, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID_ARGUMENT, "quantize: num_tokens must be >= 0");
  if (T > 0 && (!x || !hidden_states || !hidden_states_scale || !aligned(x, 16) || !aligned(hidden_states, 16)))
    return fail(MOE_ERR_INVALID_ARGUMENT, "quantize: NULL or misaligned pointer");
  cudaError_t e = moe::launch_quantize(x, x_is_bf16 != 0, T, static_cast<uint8_t*>(hidden_states), hidden_states_scale,
                                       static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "quantize");
}

int moe_fp8_ep_plan(const int32_t* topk_idx, int32_t T, int32_t world, int32_t experts_per_rank, int32_t wave_tokens,
                    int32_t waves, int32_t* send_counts, int32_t* slot, void* stream) {
  if (T < 0 || world < 1 || world > 64 || experts_per_rank < 1 || wave_tokens < 1 || waves < 1 ||
      (long long)wave_tokens * waves < T)
    return fail(MOE_ERR_INVALID_ARGUMENT, "ep_plan: bad sizes (need waves * wave_tokens >= num_tokens)");
  if (!send_counts || (T > 0 && (!topk_idx || !slot))) return fail(MOE_ERR_INVALID_ARGUMENT, "ep_plan: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world * waves, st);
  if (e == cudaSuccess) e = moe::launch_ep_plan(topk_idx, T, world, experts_per_rank, wave_tokens, send_counts, slot, st);
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "ep_plan");
}

int moe_fp8_ep_pack(const float* routing_logits, const void* hidden_states, const float* hidden_states_scale,
                    int32_t T, int32_t world, const int32_t* slot, const int32_t* send_offsets, int32_t wave_tokens,
                    float* send_logits, void* send_hidden, float* send_scales, void* stream) {
  if (T < 0 || world < 1 || world > 64 || wave_tokens < 1) return fail(MOE_ERR_INVALID_ARGUMENT, "ep_pack: bad sizes");
  if (T > 0 && (!aligned(routing_logits, 16) || !aligned(hidden_states, 16) || !aligned(send_logits, 16) ||
                !aligned(send_hidden, 16) || !send_scales || !slot || !send_offsets || !hidden_states_scale))
    return fail(MOE_ERR_INVALID_ARGUMENT, "ep_pack: NULL or misaligned pointer");
  cudaError_t e = moe::launch_ep_pack(routing_logits, static_cast<const uint8_t*>(hidden_states), hidden_states_scale,
                                      T, world, slot, send_offsets, wave_tokens, send_logits,
                                      static_cast<uint8_t*>(send_hidden), send_scales, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "ep_pack");
}

int moe_fp8_ep_scales(const float* token_major_scales, int32_t N, float* hidden_states_scale, void* stream) {
  if (N < 0 || (N > 0 && (!token_major_scales || !hidden_states_scale)))
    return fail(MOE_ERR_INVALID_ARGUMENT, "ep_scales: bad arguments");
  cudaError_t e = moe::launch_ep_scales(token_major_scales, N, hidden_states_scale, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "ep_scales");
}

int moe_fp8_ep_combine(const void* returned_partials, const int32_t* slot, const int32_t* send_offsets,
                       int32_t wave_tokens, int32_t T, int32_t world, void* output, void* stream) {
  if (T < 0 || world < 1 || world > 64 || wave_tokens < 1) return fail(MOE_ERR_INVALID_ARGUMENT, "ep_combine: bad sizes");
  if (T > 0 && (!aligned(returned_partials, 16) || !aligned(output, 16) || !slot || !send_offsets))
    return fail(MOE_ERR_INVALID_ARGUMENT, "ep_combine: NULL or misaligned pointer");
  cudaError_t e = moe::launch_ep_combine(static_cast<const __nv_bfloat16*>(returned_partials), slot, send_offsets,
                                         wave_tokens, T, world, static_cast<__nv_bfloat16*>(output),
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "ep_combine");
}

int moe_fp8_debug_set_waits(uint64_t wait_limit_ns, int32_t gate_extra) {
  if (wait_limit_ns == 0 || gate_extra < 0) return fail(MOE_ERR_INVALID_ARGUMENT, "debug_set_waits: bad arguments");
  cudaError_t e = moe::set_debug_waits_stream(wait_limit_ns, gate_extra);
  if (e == cudaSuccess) e = moe::set_debug_waits_tile(wait_limit_ns, gate_extra);
  if (e == cudaSuccess) e = moe::set_debug_waits_ep(wait_limit_ns, gate_extra);
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "debug_set_waits");
}

// Profiling aid: timeline of the GEMM kernels' CTA 0 (see grouped_gemm.cu).
int moe_fp8_debug_trace(int32_t enable, uint64_t* host, int32_t n) {
  cudaError_t e = enable >= 0 ? moe::set_trace(enable) : moe::read_trace(reinterpret_cast<unsigned long long*>(host), n);
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "trace");
}

int moe_fp8_debug_stream_trace(int32_t enable, uint64_t* host, int32_t n) {
  cudaError_t e = moe::stream_trace(enable, reinterpret_cast<unsigned long long*>(host), n);
  return e == cudaSuccess ? MOE_OK : cuda_fail(e, "trace");
}

int moe_fp8_run_stage(const MoeFp8Args* a, int32_t stage, void* stream) {
  Plan p{};
  if (int rc = make_plan(a, p)) return rc;
  if (a->num_tokens == 0) return MOE_OK;
  return launch_stage(p, stage, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
