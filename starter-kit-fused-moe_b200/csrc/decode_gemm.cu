// Decode-shaped grouped GEMMs (few tokens per expert): weight-streaming
// variants of kernels (3) and (4), same arithmetic as grouped_gemm.cu.
//
// With a handful of tokens per expert the operator is bound by the weight
// bytes. These kernels put the weights on the MMA's M side (128 weight rows per
// instruction) and 16 token rows on N ("swap-AB"):
//   D[w_row, token] = sum_k W[w_row, k] * A[token, k]
// so a pipeline stage is almost all weight bytes (2 KB of activations next to
// 16 or 32 KB of weights) and six to ten stages fit in shared memory, enough
// bytes in flight for one SM to keep its share of HBM bandwidth busy.
// Each K-block's 128x16 fp32 partial lands in its own TMEM slot of a 16- or
// 32-deep ring, so the tensor core runs ahead of the scale promotion instead of
// handing one buffer back and forth.
//
// GEMM1 (MODE 1): per tile (expert, 128 intermediate columns, 16 pair rows),
//   two MMAs per K=32 step: gate rows and up rows of W13 against the same
//   activation rows; promotion by w_scale[row block, kb] * a_scale[token, kb];
//   epilogue SwiGLU and the two-term FP8 re-quantisation of grouped_gemm.cu
//   (1x128 blocks = the 128 columns this tile owns), amax reduced across the
//   tile's 128 threads per token.
// GEMM2 (MODE 2): per tile (expert, 128 output columns, 16 term rows = 8
//   pairs); hi + lo terms summed, times the routing weight, added into the fp32
//   token accumulator (one coalesced 128-byte atomic add per warp and pair).
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {
namespace dec {

constexpr int NTOK = 16;                 // token rows per tile (MMA N)
constexpr int W_TILE = 128 * 128;        // 16 KB of weights per 128-row block and K-block
constexpr int A_TILE = NTOK * 128;       // 2 KB
constexpr int THREADS = 256;             // producer, MMA, 4 promotion warps, 2 spare (scan width)
constexpr int EPI_WARPS = 4;

template <int MODE>
struct Cfg;
template <>
struct Cfg<1> {
  static constexpr int KB = kHiddenBlocks;        // 56
  static constexpr int NT = kInter / 128;         // 16 tiles of 128 intermediate columns
  static constexpr int W_BLOCKS = 2;              // gate + up
  static constexpr int STAGES = 6;
  static constexpr int ROWS_PER_PAIR = 1;
};
template <>
struct Cfg<2> {
  static constexpr int KB = kInterBlocks;         // 16
  static constexpr int NT = kHidden / 128;        // 56 tiles of 128 output columns
  static constexpr int W_BLOCKS = 1;
  static constexpr int STAGES = 10;
  static constexpr int ROWS_PER_PAIR = 2;
};

template <int MODE>
struct Smem {
  static constexpr int STAGE_BYTES = Cfg<MODE>::W_BLOCKS * W_TILE + A_TILE;
  static constexpr int COLS_PER_KB = Cfg<MODE>::W_BLOCKS * NTOK;
  static constexpr int NBUF = 512 / COLS_PER_KB;  // TMEM ring depth in K-blocks
  uint64_t full[Cfg<MODE>::STAGES];
  uint64_t empty[Cfg<MODE>::STAGES];
  uint64_t tfull[NBUF];
  uint64_t tempty[NBUF];
  uint64_t epi_bar[2];
  uint64_t tab_full[2];                    // per-tile scale / token tables, filled by the producer
  uint64_t tab_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
  int warp_sums[8];
  int tile_start[kMaxLocalExperts + 1];
  int tt_cnt[kMaxLocalExperts];
  int row_off[kMaxLocalExperts];
  int cnt[kMaxLocalExperts];
  alignas(16) float sa[2][Cfg<MODE>::KB][NTOK];    // activation scales of the tile's rows (per table slot)
  alignas(16) float sw[2][2][Cfg<MODE>::KB];       // weight block scales: [gate, up][kb] or [w2][kb]
  alignas(16) int tok[2][NTOK / 2];                // GEMM2: token and routing weight of the tile's pairs
  alignas(16) float wgt[2][NTOK / 2];
  float amax[2][EPI_WARPS][NTOK];
};

template <int MODE>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)Cfg<MODE>::STAGES * Smem<MODE>::STAGE_BYTES + sizeof(Smem<MODE>);
}

__device__ __forceinline__ int scan256(int v, int* warp_sums, int& total) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int inc = v;
  if (tid < 256) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += n;
    }
    if (lane == 31) warp_sums[w] = inc;
  }
  __syncthreads();
  int pre = 0, tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int s = warp_sums[i];
    if (i < w) pre += s;
    tot += s;
  }
  total = tot;
  __syncthreads();
  return pre + inc - v;
}

template <int MODE>
__device__ __forceinline__ void decode(const Smem<MODE>& S, int E, int t, int& e, int& nt, int& tt) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (S.tile_start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int local = t - S.tile_start[e];
  nt = local / S.tt_cnt[e];
  tt = local - nt * S.tt_cnt[e];
}

template <int MODE>
__device__ __forceinline__ void set_abort(Smem<MODE>& S, int* err, int code) {
  atomicOr(err, code);
  *reinterpret_cast<volatile int*>(&S.abort_flag) = 1;
}
template <int MODE>
__device__ __forceinline__ bool aborted(const Smem<MODE>& S) {
  return *reinterpret_cast<const volatile int*>(&S.abort_flag) != 0;
}

// Bounded rendezvous of the four promotion warps (one mbarrier phase per use).
template <int MODE>
__device__ __forceinline__ bool epi_sync(Smem<MODE>& S, int& uses, int lane) {
  const int b = uses & 1, phase = (uses >> 1) & 1;
  ++uses;
  __syncwarp();
  if (lane == 0) mbar_arrive(smem_u32(&S.epi_bar[b]));
  return mbar_wait(smem_u32(&S.epi_bar[b]), phase);
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    swap_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     GemmArgs args) {
  using C = Cfg<MODE>;
  using SM = Smem<MODE>;
  constexpr int KB = C::KB, NT = C::NT, STAGES = C::STAGES, NBUF = SM::NBUF;
  constexpr int STAGE_BYTES = SM::STAGE_BYTES, COLS = SM::COLS_PER_KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SM& S = *reinterpret_cast<SM*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.E;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&S.full[s]), 1);
      mbar_init(smem_u32(&S.empty[s]), 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(smem_u32(&S.tfull[b]), 1);
      mbar_init(smem_u32(&S.tempty[b]), EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.epi_bar[b]), EPI_WARPS);
      mbar_init(smem_u32(&S.tab_full[b]), 1);
      mbar_init(smem_u32(&S.tab_empty[b]), EPI_WARPS);
    }
    S.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  {
    const int tid = threadIdx.x;
    const int c = tid < E ? args.counts[tid] : 0;
    const int tt = (c * C::ROWS_PER_PAIR + NTOK - 1) / NTOK;
    int tot0, tot1;
    const int roff = scan256(align_up(c, 128), S.warp_sums, tot0);
    const int tstart = scan256(tt * NT, S.warp_sums, tot1);
    if (tid < E) {
      S.cnt[tid] = c;
      S.tt_cnt[tid] = tt;
      S.row_off[tid] = roff;
      S.tile_start[tid] = tstart;
    }
    if (tid == 0) {
      S.tile_start[E] = tot1;
      S.total_tiles = tot1;
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&S.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;
  const int total = S.total_tiles;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0, tile_iter = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok && !aborted(S); t += gridDim.x) {
        int e, nt, tt;
        decode(S, E, t, e, nt, tt);
        const int arow = C::ROWS_PER_PAIR * S.row_off[e] + tt * NTOK;
        {
          // the tile's scales (and GEMM2 token ids / weights) into table slot p
          const int p = tile_iter & 1;
          if (!mbar_wait(smem_u32(&S.tab_empty[p]), ((tile_iter >> 1) & 1) ^ 1)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            break;
          }
          const uint32_t tb = smem_u32(&S.tab_full[p]);
          constexpr uint32_t kTabBytes = KB * NTOK * 4 + C::W_BLOCKS * KB * 4 + (MODE == 2 ? NTOK * 4 : 0);
          mbar_arrive_expect_tx(tb, kTabBytes);
          const size_t ld_sa = (size_t)C::ROWS_PER_PAIR * args.R1;
          for (int kb = 0; kb < KB; ++kb)
            bulk_load(smem_u32(&S.sa[p][kb][0]), args.sa + kb * ld_sa + arow, NTOK * 4, tb);
          if (MODE == 1) {
            bulk_load(smem_u32(&S.sw[p][0][0]), args.sb + ((size_t)e * 32 + nt) * kHiddenBlocks, KB * 4, tb);
            bulk_load(smem_u32(&S.sw[p][1][0]), args.sb + ((size_t)e * 32 + 16 + nt) * kHiddenBlocks, KB * 4, tb);
          } else {
            bulk_load(smem_u32(&S.sw[p][0][0]), args.sb + ((size_t)e * kHiddenBlocks + nt) * kInterBlocks, KB * 4, tb);
            const int pr = S.row_off[e] + (tt * NTOK) / 2;
            bulk_load(smem_u32(&S.tok[p][0]), args.row_token + pr, NTOK / 2 * 4, tb);
            bulk_load(smem_u32(&S.wgt[p][0]), args.row_weight + pr, NTOK / 2 * 4, tb);
          }
          ++tile_iter;
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES, u = it / STAGES;
          if (!mbar_wait(smem_u32(&S.empty[s]), (u & 1) ^ 1)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&S.full[s]);
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          if (MODE == 1) {
            tma_load_2d(st, &tmW, fb, kb * 128, e * kGemm1N + nt * 128);
            tma_load_2d(st + W_TILE, &tmW, fb, kb * 128, e * kGemm1N + kInter + nt * 128);
          } else {
            tma_load_2d(st, &tmW, fb, kb * 128, e * kHidden + nt * 128);
          }
          tma_load_2d(st + C::W_BLOCKS * W_TILE, &tmA, fb, kb * 128, arow);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, NTOK);
      int it = 0, kt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok && !aborted(S); t += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb, ++it, ++kt) {
          const int s = it % STAGES, u = it / STAGES;
          const int b = kt % NBUF, v = kt / NBUF;
          if (!mbar_wait(smem_u32(&S.tempty[b]), (v & 1) ^ 1) || !mbar_wait(smem_u32(&S.full[s]), u & 1)) {
            set_abort(S, args.err, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t at = st + C::W_BLOCKS * W_TILE;
          const uint32_t d = tmem_base + (uint32_t)(b * COLS);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_e4m3(d, sdesc_sw128(st + kk * 32), sdesc_sw128(at + kk * 32), idesc, kk > 0 ? 1u : 0u);
            if (MODE == 1)
              mma_e4m3(d + NTOK, sdesc_sw128(st + W_TILE + kk * 32), sdesc_sw128(at + kk * 32), idesc,
                       kk > 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(&S.empty[s]));
          mma_commit(smem_u32(&S.tfull[b]));
        }
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ------------------------------------------------------------ promotion + epilogue
    const int q = warp & 3;
    const int r = 32 * q + lane;                          // weight row inside the 128-row block
    const int et = threadIdx.x - 64;                      // 0..127 among promotion threads
    const uint32_t lane_addr = tmem_base + ((uint32_t)(32 * q) << 16);
    int kt = 0, tile_iter = 0, sync_uses = 0;
    for (int t = blockIdx.x; t < total && !aborted(S); t += gridDim.x, ++tile_iter) {
      int e, nt, tt;
      decode(S, E, t, e, nt, tt);
      const int p = tile_iter & 1;
      const int row0 = C::ROWS_PER_PAIR * S.row_off[e] + tt * NTOK;     // first GEMM row of the tile
      const int nvalid = min(NTOK, C::ROWS_PER_PAIR * S.cnt[e] - tt * NTOK);
      if (!mbar_wait(smem_u32(&S.tab_full[p]), (tile_iter >> 1) & 1)) {
        set_abort(S, args.err, kErrTimeoutEpilogue);
        break;
      }
      float g[NTOK], u[NTOK];
#pragma unroll
      for (int i = 0; i < NTOK; ++i) g[i] = u[i] = 0.f;
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb, ++kt) {
        const int b = kt % NBUF, v = kt / NBUF;
        if (!mbar_wait(smem_u32(&S.tfull[b]), v & 1)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        float pg[NTOK], pu[NTOK];
        tmem_ld16(lane_addr + (uint32_t)(b * COLS), pg);
        if (MODE == 1) tmem_ld16(lane_addr + (uint32_t)(b * COLS + NTOK), pu);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.tempty[b]));
        const float swg = S.sw[p][0][kb];
        const float swu = MODE == 1 ? S.sw[p][1][kb] : 0.f;
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          const float sa = S.sa[p][kb][i];
          g[i] = fmaf(pg[i], sa * swg, g[i]);
          if (MODE == 1) u[i] = fmaf(pu[i], sa * swu, u[i]);
        }
      }
      if (!ok) break;

      if (MODE == 1) {
        // C = silu(X2) * X1 for this thread's intermediate column and the tile's tokens
        float am[NTOK];
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          const float x1 = g[i], x2 = u[i];
          g[i] = (x2 / (1.0f + expf(-x2))) * x1;
          am[i] = fabsf(g[i]);
        }
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
          for (int i = 0; i < NTOK; ++i) am[i] = fmaxf(am[i], __shfl_xor_sync(0xffffffffu, am[i], d));
        if (lane < NTOK) {
          float mine = 0.f;
#pragma unroll
          for (int i = 0; i < NTOK; ++i)
            if (i == lane) mine = am[i];
          S.amax[p][q][lane] = mine;
        }
        if (!epi_sync(S, sync_uses, lane)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          break;
        }
        const int col = nt * 128 + r;
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          if (i >= nvalid) break;
          const float amax = fmaxf(fmaxf(S.amax[p][0][i], S.amax[p][1][i]), fmaxf(S.amax[p][2][i], S.amax[p][3][i]));
          const float s_hi = amax / kFp8Max;
          const float inv_hi = amax > 0.f ? kFp8Max / amax : 0.f;
          const __nv_fp8_storage_t hq = __nv_cvt_float_to_fp8(g[i] * inv_hi, __NV_SATFINITE, __NV_E4M3);
          const __half_raw hh = __nv_cvt_fp8_to_halfraw(hq, __NV_E4M3);
          const float hv = __half2float(*reinterpret_cast<const __half*>(&hh));
          const __nv_fp8_storage_t lq =
              __nv_cvt_float_to_fp8((g[i] - hv * s_hi) * (inv_hi * 16.0f), __NV_SATFINITE, __NV_E4M3);
          const size_t prow = (size_t)row0 + i;           // pair row (GEMM1 rows are pair rows)
          args.a2[(2 * prow) * kInter + col] = hq;
          args.a2[(2 * prow + 1) * kInter + col] = lq;
          if (r == 0) {
            float* sa2 = args.sa2 + (size_t)nt * 2 * args.R1 + 2 * prow;
            sa2[0] = s_hi;
            sa2[1] = s_hi * (1.0f / 16.0f);
          }
        }
      } else {
        const int col = nt * 128 + r;
#pragma unroll
        for (int i = 0; i < NTOK / 2; ++i) {
          if (2 * i >= nvalid) break;
          const float v = (g[2 * i] + g[2 * i + 1]) * S.wgt[p][i];
          atomicAdd(args.out_acc + (size_t)S.tok[p][i] * kHidden + col, v);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.tab_empty[p]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

static int g_attr_set[2][64];

template <int MODE>
cudaError_t launch(const CUtensorMap& tmA, const CUtensorMap& tmW, const GemmArgs& args, int num_sms,
                   cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  constexpr size_t bytes = smem_bytes<MODE>();
  static_assert(bytes <= 232448, "shared memory budget");
  if (dev >= 64 || !g_attr_set[MODE - 1][dev]) {
    cudaError_t e = cudaFuncSetAttribute(swap_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) g_attr_set[MODE - 1][dev] = 1;
  }
  swap_gemm_kernel<MODE><<<num_sms, THREADS, bytes, st>>>(tmA, tmW, args);
  return cudaGetLastError();
}

}  // namespace dec

cudaError_t launch_gemm1_decode(const CUtensorMap& tmA, const CUtensorMap& tmW, const GemmArgs& args,
                                int num_sms, cudaStream_t st) {
  return dec::launch<1>(tmA, tmW, args, num_sms, st);
}
cudaError_t launch_gemm2_decode(const CUtensorMap& tmA, const CUtensorMap& tmW, const GemmArgs& args,
                                int num_sms, cudaStream_t st) {
  return dec::launch<2>(tmA, tmW, args, num_sms, st);
}

}  // namespace moe
