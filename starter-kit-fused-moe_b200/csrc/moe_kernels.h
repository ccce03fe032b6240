// Internal launch interface between the C-ABI layer and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

struct GemmArgs {
  const int* counts;       // [E] pairs per local expert
  int E;                   // local experts
  int R1;                  // pair-row capacity of the workspace
  const float* sa;         // GEMM1: [56, R1] activation scales; GEMM2: [16, 2*R1]
  const float* sb;         // GEMM1: [E, 32, 56] W13 scales;     GEMM2: [E, 56, 16] W2 scales
  uint8_t* a2;             // GEMM1 out: e4m3 [2*R1, 2048]
  float* sa2;              // GEMM1 out: [16, 2*R1]
  const int* row_token;    // GEMM2: token of each pair row
  const float* row_weight; // GEMM2: routing weight of each pair row
  float* out_acc;          // GEMM2 out: f32 [T, 7168]
  float* pair_out;         // GEMM2, deterministic mode: fp32 output row of every pair (no accumulation)
  int no_split;            // deterministic mode: whole tiles only (no K-sliced tails)
  float* split_partial;    // GEMM1: fp32 partial tiles of K-split tail tiles
  int* split_cnt;          // GEMM1: arrivals per split tail tile (zero at launch)
  int* err;                // device error word
  int T;                   // tokens (rows of out_acc), for the debug-build index checks
};

cudaError_t launch_route(const float* logits, const __nv_bfloat16* bias, int T, int offset, int E, float scale,
                         int* topk_idx, float* topk_w, int* pair_pos, int* counts, float* out_acc,
                         __nv_bfloat16* out, cudaStream_t st, const int* given_idx = nullptr,
                         const float* given_w = nullptr);
cudaError_t launch_permute(const uint8_t* hidden, const float* hs, int T, int E, int offset, const int* topk_idx,
                           const float* topk_w, const int* pair_pos, const int* counts, int R1, uint8_t* a1,
                           float* sa1, int* row_token, float* row_weight, int* err, int num_sms, cudaStream_t st);
// Deterministic combine: out[t] = bf16(sum of the token's pair rows of
// pair_out in ascending local-expert order).
// Both finalize passes write NaN rows when the call's error word (err[1]) is set.
cudaError_t launch_finalize_ordered(const float* pair_out, __nv_bfloat16* out, int T, const int* topk_idx,
                                    const int* pair_pos, const int* counts, int offset, int E, const int* err,
                                    cudaStream_t st);
cudaError_t launch_finalize(const float* acc, __nv_bfloat16* out, int T, const int* topk_idx, int offset, int E,
                            const int* err, cudaStream_t st);
// Weight-streaming GEMM kernel (decode_gemm.cu).
struct DecodeArgs {
  int mode;                // 1: GEMM1 tiles, 2: GEMM2 tiles, 3: both in one launch
  int E, R1;
  const int* counts;
  const float* sa1;        // [56, R1]
  float* sa2;              // [16, 2*R1] (written by GEMM1 tiles)
  const float* s13;        // [E, 32, 56]
  const float* s2;         // [E, 56, 16]
  uint8_t* a2;             // e4m3 [2*R1, 2048]
  const int* row_token;
  const float* row_weight;
  float* out_acc;
  int* err;
  int* queue;              // [2]: tile counter, CTA exit counter (zero before the first launch)
  int* done1;              // [E]: finished GEMM1 tile parts per expert (mode 3)
  int T;                   // tokens (rows of out_acc)
  int zero_acc;            // zero out_acc in the prologue (GEMM2 tiles wait for every CTA's part)
  int* zero_done;          // CTAs that finished zeroing (zero before the first launch)
  int prefetch_kb;         // GEMM1 K-blocks per guessed first tile to prefetch into L2 in the prologue
  float* split_partial;    // fp32 partials of K-sliced GEMM1 tiles (null: no slicing)
  int* split_cnt;          // arrivals per K-sliced GEMM1 tile (zero before the first launch)
};
cudaError_t launch_stream_gemm(const CUtensorMap& tmA1, const CUtensorMap& tmW13, const CUtensorMap& tmA2,
                               const CUtensorMap& tmW2, const DecodeArgs& args, int num_sms, cudaStream_t st);
cudaError_t launch_ep_plan(const int* topk_idx, int T, int W, int epr, int wave_tokens, int* send_counts, int* slot,
                           cudaStream_t st);
cudaError_t launch_ep_pack(const float* logits, const uint8_t* hidden, const float* hs, int T, int W, const int* slot,
                           const int* send_off, int wave_tokens, float* s_logits, uint8_t* s_hidden, float* s_scale,
                           cudaStream_t st);
cudaError_t launch_ep_scales(const float* src, int N, float* dst, cudaStream_t st);
cudaError_t launch_ep_combine(const __nv_bfloat16* back, const int* slot, const int* send_off, int wave_tokens, int T,
                              int W, __nv_bfloat16* out, cudaStream_t st);
cudaError_t launch_quantize(const void* x, bool bf16, int T, uint8_t* q, float* scale, cudaStream_t st);
// Test hooks of the bounded waits (one per translation unit with waits).
cudaError_t set_debug_waits_stream(unsigned long long limit_ns, int gate_extra);
cudaError_t set_debug_waits_tile(unsigned long long limit_ns, int gate_extra);
cudaError_t set_debug_waits_ep(unsigned long long limit_ns, int gate_extra);
// Text returned by moe_fp8_last_error() on the calling thread.
void set_last_error(const char* msg);
cudaError_t set_trace(int on);
// Streaming kernel's per-tile timeline (trace builds): enable >= 0 clears it,
// enable < 0 copies n words ([tiles][cta, queue index, claim ns, finish ns]) to host.
cudaError_t stream_trace(int enable, unsigned long long* host, int n);
cudaError_t read_trace(unsigned long long* host, int n);
// tmOut: the GEMM2 operand viewed as [R1, 4096] bytes (hi row | lo row of
// each pair), 32 x 64-byte boxes, 64-byte swizzle; GEMM1 stores its output tiles through it.
cudaError_t launch_gemm1(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmOut,
                         const GemmArgs& args, int num_sms, cudaStream_t st);
// Whether the tile GEMMs run as CTA pairs (256-row tiles over two SMs).
bool cta_pair_enabled();
int set_cta_pair(int on);   // returns the previous setting
cudaError_t launch_gemm2(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& args, int num_sms,
                         cudaStream_t st);

}  // namespace moe
