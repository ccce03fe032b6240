// Producer-side activation quantiser: x [T, 7168] (bf16 or f32) ->
// e4m3 [T, 7168] + f32 scales [56, T] (token-contiguous), the operator's input
// layout (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:81-88).
//
// Per 1x128 block: s = max(amax, 1e-12) / 448, q = e4m3(x / s) with
// round-to-nearest-even (|x / s| <= 448, so saturation never changes a value).
// The same per-block recipe re-quantises the SwiGLU output in the reference's
// large-batch path (solution/triton/cutlass_gemm1_helper.py:189-205).
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

// One warp per (token, block); lane l holds elements 4l..4l+3 of the block.
template <typename T_IN>
__global__ void __launch_bounds__(256) quantize_kernel(const T_IN* __restrict__ x, int T, uint8_t* __restrict__ q,
                                                       float* __restrict__ scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t unit = (size_t)blockIdx.x * 8 + warp;  // token * 56 + block
  if (unit >= (size_t)T * kHiddenBlocks) return;
  const int t = (int)(unit / kHiddenBlocks), kb = (int)(unit % kHiddenBlocks);
  const size_t off = (size_t)t * kHidden + (size_t)kb * kBlock + 4 * lane;
  float v[4];
  if constexpr (sizeof(T_IN) == 2) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(x + off));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x + off));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  const float s = fmaxf(amax, 1e-12f) / kFp8Max;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(v[i] / s, __NV_SATFINITE, __NV_E4M3);
    packed |= (uint32_t)b << (8 * i);
  }
  reinterpret_cast<uint32_t*>(q + off)[0] = packed;
  if (lane == 0) scale[(size_t)kb * T + t] = s;
}

cudaError_t launch_quantize(const void* x, bool bf16, int T, uint8_t* q, float* scale, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const size_t units = (size_t)T * kHiddenBlocks;
  const unsigned grid = (unsigned)((units + 7) / 8);
  if (bf16)
    quantize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, q, scale);
  else
    quantize_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T, q, scale);
  return cudaGetLastError();
}

}  // namespace moe
