// Expert-parallel exchange kernels: dispatch planning, packing and the
// combine of returned partial outputs.
//
// With W ranks each holding E/W experts (local_expert_offset = rank * E/W, the
// reference's only expert-parallel hook, ...json:146), a token is needed by the
// ranks that own at least one of its 8 selected experts (at most 4 with
// DeepSeek-V3 routing, since the 8 experts come from 4 groups). The source
// rank sends each such rank the token's FP8 row, its 56 block scales and its
// 256 routing logits; the destination re-derives the identical routing from
// the logits, runs the operator over its local experts and returns one bf16
// partial row per received token; the source sums a token's partials in fp32.
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

constexpr int kMaxRanks = 64;

// Tokens are split into waves of `wave_tokens` consecutive tokens; send blocks
// are ordered (wave, destination). slot[t * W + d] = position of token t in
// block (wave(t), d), -1 if d owns none of t's experts;
// send_counts[wave * W + d] = tokens in that block.
__global__ void ep_plan_kernel(const int* __restrict__ topk_idx, int T, int W, int experts_per_rank, int wave_tokens,
                               int* __restrict__ send_counts, int* __restrict__ slot) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int* counts = send_counts + (size_t)(t / wave_tokens) * W;
  uint64_t mask = 0;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    const int d = topk_idx[(size_t)t * kTopK + k] / experts_per_rank;
    if (d >= 0 && d < W) mask |= 1ull << d;
  }
  for (int d = 0; d < W; ++d)
    slot[(size_t)t * W + d] = ((mask >> d) & 1) ? atomicAdd(&counts[d], 1) : -1;
}

// Warp per token: copies the token's FP8 row, logits and scales (token-major)
// into every destination block that needs it.
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const float* __restrict__ logits, const uint8_t* __restrict__ hidden, const float* __restrict__ hs, int T, int W,
    const int* __restrict__ slot, const int* __restrict__ send_off, int wave_tokens, float* __restrict__ s_logits,
    uint8_t* __restrict__ s_hidden, float* __restrict__ s_scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * 8 + warp; t < T; t += gridDim.x * 8) {
    const int* off = send_off + (size_t)(t / wave_tokens) * W;
    constexpr int kPer = kHidden / 16 / 32;  // 14 uint4 per lane
    uint4 v[kPer];
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
#pragma unroll
    for (int i = 0; i < kPer; ++i) v[i] = __ldg(src + lane + 32 * i);
    const float4* lsrc = reinterpret_cast<const float4*>(logits + (size_t)t * kExperts);
    const float4 l0 = __ldg(lsrc + lane), l1 = __ldg(lsrc + lane + 32);
    const float s0 = lane < kHiddenBlocks ? __ldg(hs + (size_t)lane * T + t) : 0.f;
    const float s1 = lane + 32 < kHiddenBlocks ? __ldg(hs + (size_t)(lane + 32) * T + t) : 0.f;
    for (int d = 0; d < W; ++d) {
      const int sl = slot[(size_t)t * W + d];
      if (sl < 0) continue;
      const size_t row = (size_t)off[d] + sl;
      uint4* dst = reinterpret_cast<uint4*>(s_hidden + row * kHidden);
#pragma unroll
      for (int i = 0; i < kPer; ++i) dst[lane + 32 * i] = v[i];
      float4* ldst = reinterpret_cast<float4*>(s_logits + row * kExperts);
      ldst[lane] = l0;
      ldst[lane + 32] = l1;
      if (lane < kHiddenBlocks) s_scale[row * kHiddenBlocks + lane] = s0;
      if (lane + 32 < kHiddenBlocks) s_scale[row * kHiddenBlocks + lane + 32] = s1;
    }
  }
}

// [N, 56] token-major received scales -> [56, N], the operator's layout.
__global__ void ep_scales_kernel(const float* __restrict__ src, int N, float* __restrict__ dst) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)N * kHiddenBlocks) return;
  const int n = (int)(i / kHiddenBlocks), kb = (int)(i % kHiddenBlocks);
  dst[(size_t)kb * N + n] = src[i];
}

// Warp per token: out[t] = bf16(sum over destinations of the returned partial rows), fp32 sum.
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ back, const int* __restrict__ slot,
                                                         const int* __restrict__ send_off, int wave_tokens, int T,
                                                         int W, __nv_bfloat16* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * 8 + warp; t < T; t += gridDim.x * 8) {
    const int* off = send_off + (size_t)(t / wave_tokens) * W;
    // a token has at most 8 destinations (one per selected expert)
    size_t rows[kTopK];
    int nr = 0;
    for (int d = 0; d < W && nr < kTopK; ++d) {
      const int sl = slot[(size_t)t * W + d];
      if (sl >= 0) {
#pragma unroll
        for (int j = 0; j < kTopK; ++j)
          if (j == nr) rows[j] = (size_t)off[d] + sl;
        ++nr;
      }
    }
    constexpr int kPer = kHidden / 8 / 32;  // 28 groups of 8 bf16 per lane
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * kHidden);
    for (int i = 0; i < kPer; ++i) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        if (j < nr) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(back + rows[j] * kHidden) + lane + 32 * i);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h[q]);
            acc[2 * q] += f.x;
            acc[2 * q + 1] += f.y;
          }
        }
      }
      __nv_bfloat162 r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) r[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      dst[lane + 32 * i] = *reinterpret_cast<uint4*>(r);
    }
  }
}

cudaError_t launch_ep_plan(const int* topk_idx, int T, int W, int epr, int wave_tokens, int* send_counts, int* slot,
                           cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  ep_plan_kernel<<<(T + 255) / 256, 256, 0, st>>>(topk_idx, T, W, epr, wave_tokens, send_counts, slot);
  return cudaGetLastError();
}
cudaError_t launch_ep_pack(const float* logits, const uint8_t* hidden, const float* hs, int T, int W, const int* slot,
                           const int* send_off, int wave_tokens, float* s_logits, uint8_t* s_hidden, float* s_scale,
                           cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  ep_pack_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, hidden, hs, T, W, slot, send_off, wave_tokens, s_logits, s_hidden,
                                              s_scale);
  return cudaGetLastError();
}
cudaError_t launch_ep_scales(const float* src, int N, float* dst, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  const size_t n = (size_t)N * kHiddenBlocks;
  ep_scales_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, N, dst);
  return cudaGetLastError();
}
cudaError_t launch_ep_combine(const __nv_bfloat16* back, const int* slot, const int* send_off, int wave_tokens, int T,
                              int W, __nv_bfloat16* out, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  ep_combine_kernel<<<(T + 7) / 8, 256, 0, st>>>(back, slot, send_off, wave_tokens, T, W, out);
  return cudaGetLastError();
}

}  // namespace moe
