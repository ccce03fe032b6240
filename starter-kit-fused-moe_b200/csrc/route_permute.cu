// Kernel (1) DeepSeek-V3 no-aux routing, kernel (2) permute/gather, and the
// final fp32 -> bf16 pass.
//
// Routing restates the reference's routing step
// (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146,
// "2) No-aux routing"): s = sigmoid(logit), sb = s + bias, group score = sum of
// the two largest sb of each 32-expert group, keep the 4 best groups, pick the
// 8 largest sb among their experts, weight = s / (sum of the 8 s + 1e-20) * scale.
// Unlike solution/triton/current_kernel.py:246-247 no index-dependent tie-break
// is added to the scores: exact ties go to the lower index, everything else is
// decided on the raw fp32 values, so the selected sets equal the reference's.
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

constexpr int kRouteWarps = 4;   // one token per warp, 4 tokens per block (a latency chain: spread it)

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

// Order-preserving map of a float onto uint32 (larger float -> larger key);
// key 0 is below every finite value and marks removed / masked experts.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One warp per token; lane l owns experts 8l..8l+7, so lanes 4g..4g+3 hold group g.
// Each of the 8 selection rounds is one warp max-reduction (redux.sync) of the
// lanes' best keys plus a ballot for the lowest lane holding that key, so
// exact ties resolve to the lower expert index.
// Local selections are counted per block in shared memory and published with
// one global atomic per (block, expert); each selection gets its position
// inside its expert's group (pair_pos), -1 when the expert is not local.
// With `given_idx` set, the selections are not computed: token t's 8 experts
// and weights are read from given_idx / given_w [T, 8] (an id outside
// [0, 256) selects nothing) and only the bookkeeping below runs; this is how a
// rank runs the experts of tokens that other ranks routed.
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(
    const float* __restrict__ logits, const __nv_bfloat16* __restrict__ bias, int T, int offset, int E,
    float scale, int* __restrict__ topk_idx, float* __restrict__ topk_w, int* __restrict__ pair_pos,
    int* __restrict__ counts, float* __restrict__ out_acc, __nv_bfloat16* __restrict__ out,
    const int* __restrict__ given_idx, const float* __restrict__ given_w) {
  __shared__ int hist[kMaxLocalExperts];
  __shared__ int base[kMaxLocalExperts];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  const int t = blockIdx.x * kRouteWarps + warp;
  const bool active = t < T;  // warp-uniform
  float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
  uint4 braw = make_uint4(0, 0, 0, 0);
  if (active && given_idx == nullptr) {
    const float4* lp = reinterpret_cast<const float4*>(logits + (size_t)t * kExperts + lane * 8);
    x0 = __ldg(lp);
    x1 = __ldg(lp + 1);
    if (bias != nullptr) braw = __ldg(reinterpret_cast<const uint4*>(bias + lane * 8));
  }
  __syncthreads();
  int my_le = -1, my_lpos = 0;
  if (active && given_idx != nullptr) {
    if (lane < kTopK) {
      const int sel = __ldg(given_idx + (size_t)t * kTopK + lane);
      const float w = __ldg(given_w + (size_t)t * kTopK + lane);
      topk_idx[(size_t)t * kTopK + lane] = sel;
      topk_w[(size_t)t * kTopK + lane] = w;
      const int le = sel - offset;
      if (sel >= 0 && sel < kExperts && le >= 0 && le < E) {
        my_le = le;
        my_lpos = atomicAdd(&hist[le], 1);
      }
    }
    if (__ballot_sync(0xffffffffu, my_le >= 0) != 0 && out_acc != nullptr) {
      float4* row = reinterpret_cast<float4*>(out_acc + (size_t)t * kHidden);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int c = lane; c < kHidden / 4; c += 32) row[c] = z;
    }
  } else if (active) {
    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&braw);
    float s[8], sb[8];
    float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 bf = __bfloat1622float2(bp[j >> 1]);
      s[j] = sigmoid_ref(x[j]);
      sb[j] = s[j] + ((j & 1) ? bf.y : bf.x);
      if (sb[j] > m1) {
        m2 = m1;
        m1 = sb[j];
      } else if (sb[j] > m2) {
        m2 = sb[j];
      }
    }
    // merge the top-2 of the group's four lanes
#pragma unroll
    for (int d = 1; d <= 2; d <<= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, m1, d);
      const float o2 = __shfl_xor_sync(0xffffffffu, m2, d);
      const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
      m1 = fmaxf(m1, o1);
      m2 = n2;
    }
    const float gscore = m1 + m2;
    const int mygroup = lane >> 2;
    int rank = 0;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const float gs = __shfl_sync(0xffffffffu, gscore, 4 * g);
      rank += (gs > gscore) || (gs == gscore && g < mygroup);
    }
    const bool keep = rank < kTopKGroups;
    uint32_t key[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) key[j] = keep ? order_key(sb[j]) : 0u;

    int sel = 0;
    float s_sel = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      uint32_t lk = 0;
      int lj = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (key[j] > lk) {
          lk = key[j];
          lj = j;
        }
      const uint32_t m = __reduce_max_sync(0xffffffffu, lk);
      const int wl = __ffs(__ballot_sync(0xffffffffu, lk == m)) - 1;
      const int wj = __shfl_sync(0xffffffffu, lj, wl);
      float ws = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == wj) ws = s[j];
      ws = __shfl_sync(0xffffffffu, ws, wl);
      if (lane == wl) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j == wj) key[j] = 0u;
      }
      if (lane == k) {
        sel = wl * 8 + wj;
        s_sel = ws;
      }
    }
    // combine weights from the un-biased sigmoid, summed in selection order
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) sum += __shfl_sync(0xffffffffu, s_sel, k);
    if (lane < kTopK) {
      const float w = (s_sel / (sum + 1e-20f)) * scale;
      topk_idx[(size_t)t * kTopK + lane] = sel;
      topk_w[(size_t)t * kTopK + lane] = w;
      const int le = sel - offset;
      if (le >= 0 && le < E) {
        my_le = le;
        my_lpos = atomicAdd(&hist[le], 1);
      }
    }
    // A token with a local expert gets a zeroed fp32 combine row when out_acc is
    // given (GEMM2 adds into it, finalize rounds it; the streaming GEMM kernel
    // zeroes it itself); a token without one is final already: zero output.
    const bool has_local = __ballot_sync(0xffffffffu, my_le >= 0) != 0;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has_local && out_acc != nullptr) {
      float4* row = reinterpret_cast<float4*>(out_acc + (size_t)t * kHidden);
#pragma unroll 4
      for (int c = lane; c < kHidden / 4; c += 32) row[c] = z;
    } else if (!has_local && out != nullptr) {
      float4* row = reinterpret_cast<float4*>(out + (size_t)t * kHidden);
#pragma unroll 4
      for (int c = lane; c < kHidden / 8; c += 32) row[c] = z;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] = hist[e] ? atomicAdd(&counts[e], hist[e]) : 0;
  __syncthreads();
  if (active && lane < kTopK) pair_pos[(size_t)t * kTopK + lane] = my_le >= 0 ? base[my_le] + my_lpos : -1;
}

// Exclusive scan of align_up(counts[e], 128) over e < E (E <= 256) into off[];
// called by every thread of a 256-thread block.
__device__ void padded_offsets_256(const int* __restrict__ counts, int E, int* off, int* warp_sums) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int v = tid < E ? align_up(counts[tid], 128) : 0;
  int inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += n;
  }
  if (lane == 31) warp_sums[w] = inc;
  __syncthreads();
  int pre = 0;
  for (int i = 0; i < w; ++i) pre += warp_sums[i];
  off[tid] = pre + inc - v;
  __syncthreads();
}

// One warp per token: the token's FP8 row is read once (16-byte loads) and
// written to each of its local pair rows; scales are transposed into the
// row-contiguous [56, R1] layout the GEMM epilogue reads.
__global__ void __launch_bounds__(256) permute_kernel(
    const uint8_t* __restrict__ hidden, const float* __restrict__ hs, int T, int E, int offset,
    const int* __restrict__ topk_idx, const float* __restrict__ topk_w, const int* __restrict__ pair_pos,
    const int* __restrict__ counts, int R1, uint8_t* __restrict__ a1, float* __restrict__ sa1,
    int* __restrict__ row_token, float* __restrict__ row_weight, int* __restrict__ err) {
  __shared__ int off[256];
  __shared__ int warp_sums[8];
  // Let the GEMM kernel become resident now: its prologue (weight prefetch into
  // L2, accumulator zeroing) overlaps routing and this gather; its own
  // griddepcontrol.wait still waits for this grid, which waits for routing.
  pdl_trigger();
  pdl_wait();
  padded_offsets_256(counts, E, off, warp_sums);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * 8 + warp; t < T; t += gridDim.x * 8) {
    int pp = -1, ge = 0;
    float w = 0.f;
    if (lane < kTopK) {
      pp = pair_pos[(size_t)t * kTopK + lane];
      ge = topk_idx[(size_t)t * kTopK + lane];
      w = topk_w[(size_t)t * kTopK + lane];
    }
    const uint32_t any = __ballot_sync(0xffffffffu, pp >= 0);
    if (!any) continue;
    constexpr int kVec = kHidden / 16;  // 448 uint4 per row
    constexpr int kPer = kVec / 32;     // 14 per lane
    uint4 v[kPer];
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
#pragma unroll
    for (int i = 0; i < kPer; ++i) v[i] = __ldg(src + lane + 32 * i);
    const float s0 = lane < kHiddenBlocks ? __ldg(hs + (size_t)lane * T + t) : 0.f;
    const float s1 = lane + 32 < kHiddenBlocks ? __ldg(hs + (size_t)(lane + 32) * T + t) : 0.f;
    uint32_t m = any;
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      const int kpp = __shfl_sync(0xffffffffu, pp, k);
      const int kge = __shfl_sync(0xffffffffu, ge, k);
      const float kw = __shfl_sync(0xffffffffu, w, k);
      const int row = off[kge - offset] + kpp;
      if (!MOE_DCHECK(kge - offset >= 0 && kge - offset < E && row >= 0 && row < R1, err)) continue;
      uint4* dst = reinterpret_cast<uint4*>(a1 + (size_t)row * kHidden);
#pragma unroll
      for (int i = 0; i < kPer; ++i) dst[lane + 32 * i] = v[i];
      if (lane < kHiddenBlocks) sa1[(size_t)lane * R1 + row] = s0;
      if (lane + 32 < kHiddenBlocks) sa1[(size_t)(lane + 32) * R1 + row] = s1;
      if (lane == 0) {
        row_token[row] = t;
        row_weight[row] = kw;
      }
    }
  }
}

// A call whose kernels recorded an error (a bounded wait ran out, or a debug
// index check failed) must not return plausible numbers: its finalize pass
// writes NaN into every row it owns.
__device__ __forceinline__ bool call_failed(const int* err) {
  return *reinterpret_cast<const volatile int*>(err + 1) != 0;
}

// out[t] = bf16(acc[t]) for the tokens with a local expert (the routing kernel
// already wrote zeros for the others). One warp per (token, 1024-column chunk);
// each lane issues all of its loads before converting.
constexpr int kFinalizeChunk = 1024;
__global__ void __launch_bounds__(256) finalize_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ out,
                                                       int T, const int* __restrict__ topk_idx, int offset, int E,
                                                       const int* __restrict__ err) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const int le = lane < kTopK ? __ldg(topk_idx + (size_t)t * kTopK + lane) - offset : -1;
  if (!__ballot_sync(0xffffffffu, le >= 0 && le < E)) return;
  const size_t base = (size_t)t * kHidden + (size_t)blockIdx.y * kFinalizeChunk;
  const float4* src = reinterpret_cast<const float4*>(acc + base);
  uint4* dst = reinterpret_cast<uint4*>(out + base);
  constexpr int kPer = kFinalizeChunk / 8 / 32;  // 4 groups of 8 per lane
  float4 v[2 * kPer];
  const bool failed = call_failed(err);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    v[2 * i] = __ldg(src + 2 * (lane + 32 * i));
    v[2 * i + 1] = __ldg(src + 2 * (lane + 32 * i) + 1);
    if (failed) v[2 * i] = v[2 * i + 1] = make_float4(NAN, NAN, NAN, NAN);
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const float4 a = v[2 * i], b = v[2 * i + 1];
    __nv_bfloat162 r[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                           __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
    dst[lane + 32 * i] = *reinterpret_cast<uint4*>(r);
  }
}

// Deterministic combine: one warp per (token, 1024-column chunk) sums the
// token's pair rows in ascending local-expert order, the order of the
// reference's per-expert accumulation loop (...json:146, step 3), so the
// result does not depend on which GEMM tile finished first.
__global__ void __launch_bounds__(256) finalize_ordered_kernel(const float* __restrict__ pair_out,
                                                               __nv_bfloat16* __restrict__ out, int T,
                                                               const int* __restrict__ topk_idx,
                                                               const int* __restrict__ pair_pos,
                                                               const int* __restrict__ counts, int offset, int E,
                                                               const int* __restrict__ err) {
  __shared__ int off[256];
  __shared__ int warp_sums[8];
  pdl_wait();
  padded_offsets_256(counts, E, off, warp_sums);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const int le = lane < kTopK ? __ldg(topk_idx + (size_t)t * kTopK + lane) - offset : -1;
  const bool local = le >= 0 && le < E;
  const uint32_t lmask = __ballot_sync(0xffffffffu, local);
  if (!lmask) return;
  // rank of this lane's expert among the token's local experts (distinct ids)
  int rank = 0;
  for (int j = 0; j < kTopK; ++j) {
    const int lj = __shfl_sync(0xffffffffu, le, j);
    rank += ((lmask >> j) & 1) && lj < le;
  }
  const int row = local ? off[le] + __ldg(pair_pos + (size_t)t * kTopK + lane) : 0;
  constexpr int kPer = kFinalizeChunk / 4 / 32;   // float4 per lane
  float4 acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int n = __popc(lmask);
  for (int r = 0; r < n; ++r) {
    const int src = __ffs(__ballot_sync(0xffffffffu, local && rank == r)) - 1;
    const int rr = __shfl_sync(0xffffffffu, row, src);
    if (!MOE_DCHECK(rr >= 0 && rr < 8 * T + 128 * E, const_cast<int*>(err))) continue;
    const float4* p = reinterpret_cast<const float4*>(pair_out + (size_t)rr * kHidden + blockIdx.y * kFinalizeChunk);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const float4 v = __ldg(p + lane + 32 * i);
      acc[i].x += v.x;
      acc[i].y += v.y;
      acc[i].z += v.z;
      acc[i].w += v.w;
    }
  }
  __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * kHidden + blockIdx.y * kFinalizeChunk);
  if (call_failed(err))
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = make_float4(NAN, NAN, NAN, NAN);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    dst[2 * (lane + 32 * i)] = __floats2bfloat162_rn(acc[i].x, acc[i].y);
    dst[2 * (lane + 32 * i) + 1] = __floats2bfloat162_rn(acc[i].z, acc[i].w);
  }
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_route(const float* logits, const __nv_bfloat16* bias, int T, int offset, int E, float scale,
                         int* topk_idx, float* topk_w, int* pair_pos, int* counts, float* out_acc,
                         __nv_bfloat16* out, cudaStream_t st, const int* given_idx, const float* given_w) {
  if (T == 0) return cudaSuccess;
  const int grid = (T + kRouteWarps - 1) / kRouteWarps;
  route_kernel<<<grid, kRouteWarps * 32, 0, st>>>(logits, bias, T, offset, E, scale, topk_idx, topk_w, pair_pos,
                                                  counts, out_acc, out, given_idx, given_w);
  return cudaGetLastError();
}

cudaError_t launch_permute(const uint8_t* hidden, const float* hs, int T, int E, int offset, const int* topk_idx,
                           const float* topk_w, const int* pair_pos, const int* counts, int R1, uint8_t* a1,
                           float* sa1, int* row_token, float* row_weight, int* err, int num_sms, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  int grid = (T + 7) / 8;
  if (grid > num_sms * 8) grid = num_sms * 8;
  return launch_kernel(permute_kernel, dim3(grid), dim3(256), 0, st, true, hidden, hs, T, E, offset, topk_idx, topk_w,
                       pair_pos, counts, R1, a1, sa1, row_token, row_weight, err);
}

cudaError_t launch_finalize_ordered(const float* pair_out, __nv_bfloat16* out, int T, const int* topk_idx,
                                    const int* pair_pos, const int* counts, int offset, int E, const int* err,
                                    cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  return launch_kernel(finalize_ordered_kernel, dim3((T + 7) / 8, kHidden / kFinalizeChunk), dim3(256), 0, st, true,
                       pair_out, out, T, topk_idx, pair_pos, counts, offset, E, err);
}

cudaError_t launch_finalize(const float* acc, __nv_bfloat16* out, int T, const int* topk_idx, int offset, int E,
                            const int* err, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  return launch_kernel(finalize_kernel, dim3((T + 7) / 8, kHidden / kFinalizeChunk), dim3(256), 0, st, true, acc, out,
                       T, topk_idx, offset, E, err);
}

}  // namespace moe
