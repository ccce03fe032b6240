// Expert-parallel exchange over peer memory (NVLink / NVSwitch), with no host
// synchronisation and no collective library on the data path.
//
// W ranks (one GPU each, W <= 8) each own a symmetric exchange buffer, mapped
// into every peer's address space (CUDA IPC). Rank r holds experts
// [r*epr, (r+1)*epr) and T <= C tokens of its own. One step:
//
//   source r   route its tokens (routing kernel), then ep_dispatch_kernel:
//              for every token slot t < C and every rank d, the token's 8
//              selections (expert id, weight) go to d's receive table at row
//              (r, t) (id -1 past the source's T); if d owns one of the token's
//              experts, the FP8 row (7168 B) and its 56 block scales follow.
//              Plain 16-byte peer stores; the last CTA to finish publishes
//              `epoch` in every peer's dispatch flag [r] (release, system scope).
//   dest d     ep_wait_kernel until all W dispatch flags reach `epoch`; the
//              operator then runs on the W*C received rows with the selections
//              given (moe_fp8_block_scale_run_routed, fp32 rows left in its
//              workspace); ep_return_kernel copies each received row that has
//              a local expert to its source's return area [d][t] (fp32), and
//              the last CTA publishes `epoch` in every source's return flag [d].
//   source r   ep_wait_kernel on the W return flags, then ep_combine_kernel
//              sums each token's partials in ascending rank order in fp32 and
//              rounds once to bf16.
//
// Buffer reuse needs no extra handshake: a source dispatches step k+1 only
// after every rank returned step k, which each rank does only after its
// operator consumed the step-k rows; a rank writes step k+1 returns only after
// every source's step k+1 dispatch arrived, which each source issues only
// after combining step k. All waits are bounded (g_wait_limit_ns); a wait that
// runs out records an error bit and the step's combine writes NaN rows.
//
// The reference has no multi-GPU path; its expert-parallel hook is
// local_expert_offset (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146).
// No TMA is used on peer memory here: every remote access is a plain load or store.
#include <cstring>
#include <string>

#include "moe_common.cuh"
#include "moe_fp8.h"
#include "moe_kernels.h"
#include "moe_workspace.h"

namespace moe {
namespace ep {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 256;
constexpr size_t kHeader = 4096;
// header words (uint32): dispatch flags [0, 64), return flags [64, 128),
// CTA counters [128, 136), error words [136, 138)
constexpr int kFlagDispatch = 0, kFlagReturn = 64, kCounters = 128, kErr = 136;
constexpr int kErrWaitDispatch = 16, kErrWaitReturn = 32;

struct Layout {
  size_t recv_hidden, recv_scale, recv_idx, recv_w, ret, total;
};
__host__ __device__ inline Layout layout(int C, int W) {
  Layout L{};
  const size_t N = (size_t)C * W;
  size_t o = kHeader;
  auto take = [&](size_t b) { size_t r = o; o = (o + b + 1023) / 1024 * 1024; return r; };
  L.recv_hidden = take(N * kHidden);
  L.recv_scale = take(N * kHiddenBlocks * sizeof(float));
  L.recv_idx = take(N * kTopK * sizeof(int));
  L.recv_w = take(N * kTopK * sizeof(float));
  L.ret = take(N * kHidden * sizeof(float));
  L.total = o;
  return L;
}

struct Peers {
  uint8_t* base[kMaxWorld];
};

__device__ __forceinline__ uint32_t* header(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every thread fences its own peer stores; the last CTA of the grid to get here
// publishes `epoch` into word `flag_word + rank` of each destination's header.
__device__ __forceinline__ void publish(uint32_t* counter, const Peers& peers, int W, int flag_word, int rank,
                                        uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < W; ++d) st_release_sys(header(peers.base[d]) + flag_word + rank, epoch);
      atomicExch(counter, 0u);
    }
  }
}

// One warp per token slot t of this source (t < C). Lanes 0-7 hold the
// token's selections; the destination set is the ranks owning at least one.
__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(const int* __restrict__ topk_idx,
                                                               const float* __restrict__ topk_w,
                                                               const uint8_t* __restrict__ hidden,
                                                               const float* __restrict__ hs, int T, int C, int rank,
                                                               int W, int epr, Peers peers, uint32_t epoch) {
  const Layout L = layout(C, W);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* own = peers.base[rank];
  if (blockIdx.x == 0 && threadIdx.x == 0) header(own)[kErr + 1] = 0u;   // this step's error word
  const size_t N = (size_t)C * W;
  for (int t = blockIdx.x * (kThreads / 32) + warp; t < C; t += gridDim.x * (kThreads / 32)) {
    int id = -1;
    float w = 0.f;
    if (lane < kTopK && t < T) {
      id = __ldg(topk_idx + (size_t)t * kTopK + lane);
      w = __ldg(topk_w + (size_t)t * kTopK + lane);
    }
    const uint32_t dbit = (id >= 0 && id < kExperts) ? (1u << (id / epr)) : 0u;
    const uint32_t mask = __reduce_or_sync(0xffffffffu, dbit);
    const size_t row = (size_t)rank * C + t;
    if (lane < kTopK)
      for (int d = 0; d < W; ++d) {
        reinterpret_cast<int*>(peers.base[d] + L.recv_idx)[row * kTopK + lane] = id;
        reinterpret_cast<float*>(peers.base[d] + L.recv_w)[row * kTopK + lane] = w;
      }
    if (!mask) continue;
    constexpr int kPer = kHidden / 16 / 32;   // 14 uint4 per lane
    uint4 v[kPer];
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
#pragma unroll
    for (int i = 0; i < kPer; ++i) v[i] = __ldg(src + lane + 32 * i);
    const float s0 = __ldg(hs + (size_t)lane * T + t);
    const float s1 = lane + 32 < kHiddenBlocks ? __ldg(hs + (size_t)(lane + 32) * T + t) : 0.f;
    uint32_t m = mask;
    while (m) {
      const int d = __ffs(m) - 1;
      m &= m - 1;
      uint4* dst = reinterpret_cast<uint4*>(peers.base[d] + L.recv_hidden + row * kHidden);
#pragma unroll
      for (int i = 0; i < kPer; ++i) dst[lane + 32 * i] = v[i];
      float* sc = reinterpret_cast<float*>(peers.base[d] + L.recv_scale);
      sc[(size_t)lane * N + row] = s0;
      if (lane + 32 < kHiddenBlocks) sc[(size_t)(lane + 32) * N + row] = s1;
    }
  }
  publish(header(own) + kCounters, peers, W, kFlagDispatch, rank, epoch);
}

// Bounded wait until the W flags at `flag_word` of this rank's header reach `epoch`.
__global__ void ep_wait_kernel(uint8_t* own, int W, int flag_word, uint32_t epoch, int code) {
  const int lane = threadIdx.x;
  bool ok = true;
  if (lane < W) {
    const uint32_t* f = header(own) + flag_word + lane;
    if ((int)(ld_acquire_sys(f) - epoch) < 0) {
      const unsigned long long t0 = globaltimer_ns(), limit = g_wait_limit_ns;
      while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if (globaltimer_ns() - t0 > limit) {
          ok = false;
          break;
        }
        __nanosleep(128);
      }
    }
  }
  if (!ok) record_error(reinterpret_cast<int*>(header(own) + kErr), code);
  __threadfence_system();
}

// One warp per received row n = s*C + t: if this rank owns one of its experts,
// the fp32 result row goes back to source s, return row [rank][t].
__global__ void __launch_bounds__(kThreads) ep_return_kernel(const int* __restrict__ topk_idx,
                                                             const float* __restrict__ acc, int C, int offset, int E,
                                                             int rank, int W, Peers peers, uint32_t epoch,
                                                             const int* __restrict__ op_err) {
  const Layout L = layout(C, W);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool failed = *reinterpret_cast<const volatile int*>(op_err + 1) != 0 ||
                      *reinterpret_cast<const volatile uint32_t*>(header(peers.base[rank]) + kErr + 1) != 0u;
  const int N = C * W;
  for (int n = blockIdx.x * (kThreads / 32) + warp; n < N; n += gridDim.x * (kThreads / 32)) {
    const int le = lane < kTopK ? __ldg(topk_idx + (size_t)n * kTopK + lane) - offset : -1;
    if (!__ballot_sync(0xffffffffu, le >= 0 && le < E)) continue;
    const int s = n / C, t = n - s * C;
    const float4* src = reinterpret_cast<const float4*>(acc + (size_t)n * kHidden);
    float4* dst = reinterpret_cast<float4*>(peers.base[s] + L.ret) + ((size_t)rank * C + t) * (kHidden / 4);
    constexpr int kPer = kHidden / 4 / 32;   // 56 float4 per lane
    constexpr int kBatch = 8;
#pragma unroll
    for (int i0 = 0; i0 < kPer; i0 += kBatch) {
      float4 v[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) v[i] = __ldcs(src + lane + 32 * (i0 + i));
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (failed) v[i] = make_float4(NAN, NAN, NAN, NAN);
        dst[lane + 32 * (i0 + i)] = v[i];
      }
    }
  }
  publish(header(peers.base[rank]) + kCounters + 1, peers, W, kFlagReturn, rank, epoch);
}

// One warp per (token, 1024-column chunk): the token's partial rows from the
// ranks owning its experts, summed in ascending rank order, rounded once.
constexpr int kChunk = 1024;
__global__ void __launch_bounds__(kThreads) ep_combine_kernel(const int* __restrict__ topk_idx, int T, int C, int W,
                                                              int epr, const uint8_t* __restrict__ own,
                                                              __nv_bfloat16* __restrict__ out) {
  const Layout L = layout(C, W);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kThreads / 32) + warp;
  if (t >= T) return;
  const int id = lane < kTopK ? __ldg(topk_idx + (size_t)t * kTopK + lane) : -1;
  const uint32_t mask = __reduce_or_sync(0xffffffffu, (id >= 0 && id < kExperts) ? (1u << (id / epr)) : 0u);
  const bool failed = *reinterpret_cast<const volatile uint32_t*>(header(const_cast<uint8_t*>(own)) + kErr + 1) != 0u;
  constexpr int kPer = kChunk / 4 / 32;   // 8 float4 per lane
  float4 a[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int d = 0; d < W; ++d) {
    if (!((mask >> d) & 1)) continue;
    const float4* p = reinterpret_cast<const float4*>(own + L.ret) + ((size_t)d * C + t) * (kHidden / 4) +
                      blockIdx.y * (kChunk / 4);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const float4 v = __ldcs(p + lane + 32 * i);
      a[i].x += v.x;
      a[i].y += v.y;
      a[i].z += v.z;
      a[i].w += v.w;
    }
  }
  __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * kHidden + blockIdx.y * kChunk);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    if (failed) a[i] = make_float4(NAN, NAN, NAN, NAN);
    dst[2 * (lane + 32 * i)] = __floats2bfloat162_rn(a[i].x, a[i].y);
    dst[2 * (lane + 32 * i) + 1] = __floats2bfloat162_rn(a[i].z, a[i].w);
  }
}

int g_nsm[64];
int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && g_nsm[dev]) return g_nsm[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) g_nsm[dev] = n;
  return n;
}

int fail(int code, const std::string& msg) {
  set_last_error(msg.c_str());
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
bool valid_geometry(int C, int W) { return C >= 1 && W >= 1 && W <= kMaxWorld && (long long)C * W <= (1LL << 24); }
int load_peers(void* const* peer_bases, int W, Peers& P) {
  if (!peer_bases) return fail(MOE_ERR_INVALID_ARGUMENT, "ep: peer_bases is NULL");
  for (int d = 0; d < kMaxWorld; ++d) P.base[d] = nullptr;
  for (int d = 0; d < W; ++d) {
    if (!peer_bases[d] || reinterpret_cast<uintptr_t>(peer_bases[d]) % 1024)
      return fail(MOE_ERR_INVALID_ARGUMENT, "ep: peer buffer is NULL or not 1024-byte aligned");
    P.base[d] = static_cast<uint8_t*>(peer_bases[d]);
  }
  return MOE_OK;
}

}  // namespace ep

cudaError_t set_debug_waits_ep(unsigned long long limit_ns, int gate_extra) {
  return set_debug_waits_here(limit_ns, gate_extra);
}

}  // namespace moe

using namespace moe;

extern "C" {

size_t moe_fp8_ep_peer_buffer_bytes(int32_t capacity, int32_t world) {
  if (!ep::valid_geometry(capacity, world)) return 0;
  return ep::layout(capacity, world).total;
}

int moe_fp8_ep_peer_buffer_alloc(int32_t capacity, int32_t world, void** base) {
  if (!base || !ep::valid_geometry(capacity, world)) return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep: bad geometry");
  const size_t bytes = ep::layout(capacity, world).total;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return ep::cuda_fail(e, "ep: buffer allocation");
  }
  *base = p;
  return MOE_OK;
}

int moe_fp8_ep_peer_buffer_free(void* base) {
  cudaError_t e = cudaFree(base);
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep: buffer free");
}

int moe_fp8_ep_peer_ipc_handle(void* base, void* handle) {
  if (!base || !handle) return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep: NULL argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return ep::cuda_fail(e, "ep: cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  return MOE_OK;
}

int moe_fp8_ep_peer_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep: cudaIpcOpenMemHandle");
}

int moe_fp8_ep_peer_ipc_close(void* base) {
  cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep: cudaIpcCloseMemHandle");
}

int moe_fp8_ep_peer_recv_view(void* base, int32_t capacity, int32_t world, MoeFp8EpRecvView* view) {
  if (!base || !view || !ep::valid_geometry(capacity, world))
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep: bad recv view request");
  const ep::Layout L = ep::layout(capacity, world);
  uint8_t* b = static_cast<uint8_t*>(base);
  view->hidden_states = b + L.recv_hidden;
  view->hidden_states_scale = reinterpret_cast<float*>(b + L.recv_scale);
  view->topk_idx = reinterpret_cast<int32_t*>(b + L.recv_idx);
  view->topk_weights = reinterpret_cast<float*>(b + L.recv_w);
  view->num_rows = capacity * world;
  return MOE_OK;
}

int moe_fp8_ep_peer_dispatch(const int32_t* topk_idx, const float* topk_weights, const void* hidden_states,
                             const float* hidden_states_scale, int32_t num_tokens, int32_t capacity, int32_t rank,
                             int32_t world, void* const* peer_bases, uint32_t epoch, void* stream) {
  if (!ep::valid_geometry(capacity, world) || rank < 0 || rank >= world || num_tokens < 0 || num_tokens > capacity ||
      kExperts % world)
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep dispatch: bad sizes (need 0 <= T <= capacity, 256 % world == 0)");
  if (num_tokens > 0 && (!topk_idx || !topk_weights || !hidden_states || !hidden_states_scale ||
                         reinterpret_cast<uintptr_t>(hidden_states) % 16))
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep dispatch: NULL or misaligned pointer");
  ep::Peers P;
  if (int rc = ep::load_peers(peer_bases, world, P)) return rc;
  const int grid = ep::num_sms();
  ep::ep_dispatch_kernel<<<grid, ep::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_idx, topk_weights, static_cast<const uint8_t*>(hidden_states), hidden_states_scale, num_tokens, capacity,
      rank, world, kExperts / world, P, epoch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep dispatch launch");
}

int moe_fp8_ep_peer_wait(void* base, int32_t world, int32_t which, uint32_t epoch, void* stream) {
  if (!base || world < 1 || world > ep::kMaxWorld || (which != 0 && which != 1))
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep wait: bad arguments");
  ep::ep_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(base), world, which == 0 ? ep::kFlagDispatch : ep::kFlagReturn, epoch,
      which == 0 ? ep::kErrWaitDispatch : ep::kErrWaitReturn);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep wait launch");
}

int moe_fp8_ep_peer_return(void* workspace, int32_t num_local_experts, int32_t local_expert_offset, int32_t capacity,
                           int32_t rank, int32_t world, void* const* peer_bases, uint32_t epoch, void* stream) {
  if (!workspace || !ep::valid_geometry(capacity, world) || rank < 0 || rank >= world || num_local_experts < 1 ||
      num_local_experts > kMaxLocalExperts)
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep return: bad arguments");
  ep::Peers P;
  if (int rc = ep::load_peers(peer_bases, world, P)) return rc;
  const int N = capacity * world;
  const WsLayout L = ws_layout(N, num_local_experts);
  const uint8_t* w = static_cast<const uint8_t*>(workspace);
  const int grid = ep::num_sms();
  ep::ep_return_kernel<<<grid, ep::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const int*>(w + L.topk_idx), reinterpret_cast<const float*>(w + L.out_acc), capacity,
      local_expert_offset, num_local_experts, rank, world, P, epoch, reinterpret_cast<const int*>(w + L.err));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep return launch");
}

int moe_fp8_ep_peer_combine(const int32_t* topk_idx, int32_t num_tokens, int32_t capacity, int32_t world,
                            void* base, void* output, void* stream) {
  if (!base || !ep::valid_geometry(capacity, world) || num_tokens < 0 || num_tokens > capacity || kExperts % world)
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep combine: bad arguments");
  if (num_tokens == 0) return MOE_OK;
  if (!topk_idx || !output || reinterpret_cast<uintptr_t>(output) % 16)
    return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep combine: NULL or misaligned pointer");
  ep::ep_combine_kernel<<<dim3((num_tokens + 7) / 8, kHidden / ep::kChunk), ep::kThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(topk_idx, num_tokens, capacity, world,
                                                               kExperts / world, static_cast<const uint8_t*>(base),
                                                               static_cast<__nv_bfloat16*>(output));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MOE_OK : ep::cuda_fail(e, "ep combine launch");
}

int moe_fp8_ep_peer_read_error(void* base, void* stream, int32_t* bits) {
  if (!base || !bits) return ep::fail(MOE_ERR_INVALID_ARGUMENT, "ep: NULL argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* dev = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(base)) + ep::kErr;
  int32_t h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, dev, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dev, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return ep::cuda_fail(e, "ep: reading the error word");
  *bits = h;
  if (h) return ep::fail(MOE_ERR_DEVICE_TIMEOUT, "ep: a wait for a peer ran out (bits " + std::to_string(h) + ")");
  return MOE_OK;
}

}  // extern "C"
