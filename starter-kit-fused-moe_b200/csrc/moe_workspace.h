// Layout of the operator's device workspace (one contiguous byte buffer owned
// by the caller and reused across calls).
//
// Pair rows: every (token, local expert) selection is one "pair row". Pair rows
// are grouped expert-major and each expert's group is padded to 128 rows so a
// 128-row GEMM tile never straddles two experts. For T tokens and E local
// experts at most min(8, E) * T + 127 * E rows are used; `R1` rounds that up
// to 128.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace moe {

struct WsLayout {
  int T, E, R1;               // tokens, local experts, pair-row capacity
  size_t err;                 // int32 error word (sticky; cleared by the host reader)
  size_t counts;              // int32 [E]   pairs per local expert, then the streaming kernel's
                              //             tile queue [2], per-expert GEMM1 progress [256] and
                              //             the tile GEMM1's split-tile arrival counters [256] and
                              //             the streaming kernel's zeroing counter [1]
  size_t topk_idx;            // int32 [T*8] selected global experts (selection order)
  size_t topk_w;              // f32   [T*8] combine weights
  size_t pair_pos;            // int32 [T*8] position inside the expert's group, -1 if not local
  size_t row_token;           // int32 [R1]  token of each pair row
  size_t row_weight;          // f32   [R1]  combine weight of each pair row
  size_t a1;                  // e4m3  [R1, 7168]   gathered activations
  size_t sa1;                 // f32   [56, R1]     their 1x128 scales (row-contiguous)
  size_t a2;                  // e4m3  [2*R1, 2048] SwiGLU output, two FP8 terms per pair row
  size_t sa2;                 // f32   [16, 2*R1]   their 1x128 scales
  size_t out_acc;             // f32   [T, 7168]    combine accumulator
  size_t split_partial;       // f32   [kMaxSplitUnits, 128*256] tile GEMM1 K-split partial tiles
  size_t pair_out;            // f32   [R1, 7168] per-pair GEMM2 outputs (deterministic mode only)
  size_t total;
  size_t queue() const { return counts + sizeof(int32_t) * 256; }
  size_t done1() const { return counts + sizeof(int32_t) * 258; }
  size_t split_cnt() const { return counts + sizeof(int32_t) * 514; }
  size_t zero_done() const { return counts + sizeof(int32_t) * 770; }
  static constexpr size_t kCountersBytes = sizeof(int32_t) * (256 + 2 + 256 + 256 + 4);
  // Every counter accessor must land inside the block that ws_layout reserves.
  static_assert(sizeof(int32_t) * (770 + 1) <= kCountersBytes, "counter block too small");
  static constexpr int kMaxSplitUnits = 160;
};

inline size_t ws_align(size_t x, size_t a) { return (x + a - 1) / a * a; }

// `deterministic` appends the per-pair output rows of the deterministic
// combine; every other region keeps its offset.
inline WsLayout ws_layout(int T, int E, bool deterministic = false) {
  WsLayout L{};
  L.T = T;
  L.E = E;
  const int k = E < 8 ? E : 8;
  long long rows = (long long)k * T + 127LL * E;
  L.R1 = (int)((rows + 127) / 128 * 128);
  if (L.R1 < 128) L.R1 = 128;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = ws_align(o + bytes, 1024); return r; };
  L.err = take(256);
  L.counts = take(WsLayout::kCountersBytes);
  L.topk_idx = take(sizeof(int32_t) * 8 * (size_t)T);
  L.topk_w = take(sizeof(float) * 8 * (size_t)T);
  L.pair_pos = take(sizeof(int32_t) * 8 * (size_t)T);
  L.row_token = take(sizeof(int32_t) * (size_t)L.R1);
  L.row_weight = take(sizeof(float) * (size_t)L.R1);
  L.a1 = take((size_t)L.R1 * 7168);
  L.sa1 = take(sizeof(float) * 56 * (size_t)L.R1);
  L.a2 = take((size_t)2 * L.R1 * 2048);
  L.sa2 = take(sizeof(float) * 16 * 2 * (size_t)L.R1);
  L.out_acc = take(sizeof(float) * 7168 * (size_t)T);
  L.split_partial = take(sizeof(float) * 128 * 256 * (size_t)WsLayout::kMaxSplitUnits);
  L.pair_out = deterministic ? take(sizeof(float) * 7168 * (size_t)L.R1) : 0;
  L.total = o;
  return L;
}

}  // namespace moe
