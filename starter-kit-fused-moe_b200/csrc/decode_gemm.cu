// Decode-shaped grouped GEMMs (few tokens per expert): weight-streaming
// variants of kernels (3) and (4), same arithmetic as grouped_gemm.cu.
//
// With a handful of tokens per expert the operator is bound by the weight
// bytes. These kernels put the weights on the MMA's M side (128 weight rows per
// instruction) and 16 token rows on N ("swap-AB"):
//   D[w_row, token] = sum_k W[w_row, k] * A[token, k]
// A pipeline stage holds two 128-row weight blocks (32 KB) and 16 activation
// rows (2 KB); six stages keep ~200 KB of weights in flight per SM. Each
// K-block's two 128x16 fp32 partials land in their own 32-column TMEM slot of
// a 16-deep ring, so the tensor core runs ahead of the scale promotion.
//
// Tiles (all: 16 activation rows, two 128-row weight blocks):
//   GEMM1 tile (expert, n1 in 0..15, token tile): W13 gate rows [128 n1, +128)
//     and up rows [2048 + 128 n1, +128); epilogue SwiGLU and the two-term FP8
//     re-quantisation of grouped_gemm.cu over the 128 columns the tile owns.
//   GEMM2 tile (expert, n2 in 0..27, term tile of 8 pairs, K half): W2 rows
//     [256 n2, +256) over half of K; epilogue sums each pair's hi/lo terms,
//     scales by the routing weight and adds into the fp32 token accumulator
//     (the halves' partials simply add; half-size tiles shorten the tail).
// Tiles come from a device-side queue (one atomic counter per launch), so the
// work balances across SMs and, in the fused mode, GEMM2 tiles of an expert
// start as soon as that expert's GEMM1 tiles are done: each GEMM1 tile bumps a
// per-expert counter after its stores; the producer of a GEMM2 tile waits for
// the count (bounded), then fences the async proxy before its TMA reads.
// GEMM1 tiles are queued before all GEMM2 tiles and a CTA only waits on tiles
// already claimed by running CTAs, so the wait cannot deadlock.
#include "moe_common.cuh"
#include "moe_kernels.h"
#include "moe_workspace.h"

namespace moe {
namespace dec {

constexpr int NTOK = 16;                 // activation rows per tile (MMA N)
constexpr int W_TILE = 128 * 128;        // 16 KB: 128 weight rows x one 128-wide K-block
constexpr int A_TILE = NTOK * 128;       // 2 KB
constexpr int STAGE_BYTES = 2 * W_TILE + A_TILE;
constexpr int STAGES = 6;
constexpr int COLS = 2 * NTOK;           // TMEM columns per K-block
constexpr int NBUF = 512 / COLS;         // TMEM ring depth in K-blocks
constexpr int THREADS = 256;             // producer, MMA, 4 promotion warps, 2 spare (scan width)
constexpr int EPI_WARPS = 4;
constexpr int NT1 = kInter / 128;        // 16 GEMM1 tiles per expert and token tile
constexpr int NT2 = kHidden / 256;       // 28 GEMM2 tiles per expert and term tile
constexpr int KB1 = kHiddenBlocks;       // 56
constexpr int KB2 = kInterBlocks;        // 16
constexpr int KS2 = 2;                   // GEMM2 tiles are split in K (partials add into the accumulator)
constexpr int kTileEnd = -1;
constexpr int kMaxKSlices1 = 4;          // GEMM1 K-slices per tile at most (14 K-blocks each)
// partial slices the workspace's split area holds (16 KB each) and tiles its counters cover
constexpr int kMaxSplitSlots = (int)(WsLayout::kMaxSplitUnits * 128 * 256 * 4 / (EPI_WARPS * 2 * NTOK * 32 * 4));
constexpr int kMaxSplitTiles = 256;

struct Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[NBUF];
  uint64_t tempty[NBUF];
  uint64_t epi_bar[2];
  uint64_t tab_full[2];                  // per-tile table, filled by the producer
  uint64_t tab_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  int warp_sums[8];
  int tiles1, tiles2;                    // GEMM1 / GEMM2 tile counts of this launch (GEMM1 K-slices counted)
  int ks1;                               // K-slices per GEMM1 tile (more than one when tiles are scarce)
  int split_last[2];                     // GEMM1: this CTA's slice completed the tile
  int start1[kMaxLocalExperts + 1];      // GEMM1 tile prefix per expert
  int start2[kMaxLocalExperts + 1];
  int tt1[kMaxLocalExperts];             // token tiles per expert (GEMM1) / term tiles (GEMM2)
  int tt2[kMaxLocalExperts];
  int row_off[kMaxLocalExperts];
  int cnt[kMaxLocalExperts];
  int tile_id[2];                        // tile of each table slot (kTileEnd = no more work)
  unsigned long long tile_t0[2];         // claim time of each slot's tile (timeline builds)
  alignas(16) float sa[2][KB1][NTOK];    // activation scales of the tile's rows
  alignas(16) float sw[2][2][KB1];       // weight block scales of the tile's two 128-row blocks
  alignas(16) int tok[2][NTOK / 2];      // GEMM2: token and routing weight of the tile's pairs
  alignas(16) float wgt[2][NTOK / 2];
  float amax[2][EPI_WARPS][NTOK];
};
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + sizeof(Smem);
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Tile {
  int phase;   // 1 or 2
  int e, nt, tt;
  int k0, k1;  // K-blocks of the tile
  int kh;      // GEMM1: K-slice of the tile (0 when GEMM1 tiles are not split)
};

// Optional per-tile timeline (built with -DMOE_GEMM_TRACE): CTA, queue index,
// claim time and finish time (global timer, ns) of every tile.
constexpr int kTileTraceMax = 8192;
__device__ unsigned long long g_tile_trace[kTileTraceMax][4];
__device__ int g_tile_trace_n;
__device__ __forceinline__ void tile_trace(int t, unsigned long long t0) {
#ifdef MOE_GEMM_TRACE
  const int i = atomicAdd(&g_tile_trace_n, 1);
  if (i < kTileTraceMax) {
    g_tile_trace[i][0] = blockIdx.x;
    g_tile_trace[i][1] = (unsigned long long)t;
    g_tile_trace[i][2] = t0;
    g_tile_trace[i][3] = globaltimer_ns();
  }
#endif
}

__device__ __forceinline__ int scan256(int v, int* warp_sums, int& total) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += n;
  }
  if (lane == 31) warp_sums[w] = inc;
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

__device__ __forceinline__ int find_expert(const int* start, int E, int t) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Queue index -> tile. Launch mode 1: GEMM1 only; 2: GEMM2 only; 3: both, GEMM1 first.
__device__ __forceinline__ Tile decode_tile(const Smem& S, int E, int mode, int t) {
  Tile x;
  if (mode == 2) t += S.tiles1;
  if (t < S.tiles1) {
    x.phase = 1;
    x.e = find_expert(S.start1, E, t);
    const int local = t - S.start1[x.e];
    const int ks = S.ks1, kh = local % ks, rest = local / ks;   // the K-slices of a tile are adjacent
    x.nt = rest / S.tt1[x.e];
    x.tt = rest - x.nt * S.tt1[x.e];
    x.kh = kh;
    x.k0 = kh * KB1 / ks;
    x.k1 = (kh + 1) * KB1 / ks;
  } else {
    t -= S.tiles1;
    x.phase = 2;
    x.e = find_expert(S.start2, E, t);
    const int local = t - S.start2[x.e];
    const int kh = local % KS2, rest = local / KS2;    // the K halves of a tile are adjacent in the queue
    x.nt = rest / S.tt2[x.e];
    x.tt = rest - x.nt * S.tt2[x.e];
    x.k0 = kh * (KB2 / KS2);
    x.k1 = x.k0 + KB2 / KS2;
    x.kh = 0;
  }
  return x;
}

__device__ __forceinline__ void set_abort(Smem& S, int* err, int code) {
  record_error(err, code);
  *reinterpret_cast<volatile int*>(&S.abort_flag) = 1;
}
__device__ __forceinline__ bool aborted(const Smem& S) {
  return *reinterpret_cast<const volatile int*>(&S.abort_flag) != 0;
}

// Bounded rendezvous of the four promotion warps (one mbarrier phase per use).
__device__ __forceinline__ bool epi_sync(Smem& S, int& uses, int lane) {
  const int b = uses & 1, phase = (uses >> 1) & 1;
  ++uses;
  __syncwarp();
  if (lane == 0) mbar_arrive(smem_u32(&S.epi_bar[b]));
  return mbar_wait(smem_u32(&S.epi_bar[b]), phase);
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Waits (bounded) until *p >= target with acquire semantics.
__device__ __forceinline__ bool wait_counter(const int* p, int target) {
  if (ld_acquire(p) >= target) return true;
  const unsigned long long t0 = globaltimer_ns(), limit = g_wait_limit_ns;
  while (ld_acquire(p) < target) {
    if (globaltimer_ns() - t0 > limit) return false;
    __nanosleep(64);
  }
  return true;
}

__global__ void __launch_bounds__(THREADS, 1)
    stream_gemm_kernel(const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmW13,
                       const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmW2,
                       DecodeArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem& S = *reinterpret_cast<Smem*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.E, mode = args.mode;

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
      mbar_init(smem_u32(&S.tab_empty[b]), EPI_WARPS + 1);   // promotion warps + MMA thread
    }
    S.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmW13);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmW2);
  }
  // Prologue work that needs nothing from the preceding kernels, so it runs
  // while routing and the gather are still in flight:
  //  * the first K-blocks of the weight tile this CTA will most likely start
  //    with (queue order, every local expert hit once) go into L2, so HBM is
  //    busy from the start;
  //  * this CTA's share of the fp32 combine accumulator is zeroed; GEMM2 tiles
  //    wait until every CTA has done its share.
  if (args.prefetch_kb > 0 && warp == 1 && lane == 0) {
    const int e = blockIdx.x / NT1, nt = blockIdx.x % NT1;
    if (e < E)
      for (int kb = 0; kb < args.prefetch_kb && kb < KB1; ++kb) {
        tma_prefetch_l2_2d(&tmW13, kb * 128, e * kGemm1N + nt * 128);
        tma_prefetch_l2_2d(&tmW13, kb * 128, e * kGemm1N + kInter + nt * 128);
      }
  }
  if (args.zero_acc) {
    const size_t n4 = (size_t)args.T * (kHidden / 4);
    const size_t per = (n4 + gridDim.x - 1) / gridDim.x;
    const size_t b0 = (size_t)blockIdx.x * per, b1 = min(n4, b0 + per);
    float4* acc4 = reinterpret_cast<float4*>(args.out_acc);
    for (size_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) acc4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    __threadfence();
  }
  pdl_trigger();
  pdl_wait();  // the expert histogram and operands come from the preceding kernels
  {
    const int tid = threadIdx.x;
    const int c = tid < E ? args.counts[tid] : 0;
    const int t1 = (c + NTOK - 1) / NTOK;
    const int t2 = (2 * c + NTOK - 1) / NTOK;
    int tot0, tot1, tot2;
    const int roff = scan256(align_up(c, 128), S.warp_sums, tot0);
    const int s1 = scan256(t1 * NT1, S.warp_sums, tot1);
    const int s2 = scan256(t2 * NT2 * KS2, S.warp_sums, tot2);
    // Few GEMM1 tiles (a handful of hit experts): cut each into K-slices so
    // every SM streams weights; the slices meet in a fix-up (the last one to
    // arrive sums the fp32 partials and runs the epilogue).
    int ks1 = 1;
    if (args.split_partial != nullptr && tot1 > 0 && 2 * tot1 <= (int)gridDim.x && tot1 <= kMaxSplitTiles) {
      // at most one round of slices (finer slicing at 4-8 tokens measured no gain)
      ks1 = min(min((int)gridDim.x / tot1, kMaxKSlices1), kMaxSplitSlots / tot1);
      if (ks1 < 2) ks1 = 1;
    }
    if (tid < E) {
      S.cnt[tid] = c;
      S.tt1[tid] = t1;
      S.tt2[tid] = t2;
      S.row_off[tid] = roff;
      S.start1[tid] = s1 * ks1;
      S.start2[tid] = s2;
    }
    if (tid == 0) {
      S.start1[E] = tot1 * ks1;
      S.start2[E] = tot2;
      S.tiles1 = tot1 * ks1;
      S.tiles2 = tot2;
      S.ks1 = ks1;
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&S.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (args.zero_acc && threadIdx.x == 0) atomicAdd(args.zero_done, 1);   // after every thread's fenced zeroing
  const uint32_t tmem_base = S.tmem_base;
  const int total = mode == 1 ? S.tiles1 : mode == 2 ? S.tiles2 : S.tiles1 + S.tiles2;

  if (warp == 0) {
    // ------------------------------------------------------------ producer: tile queue, tables, TMA
    if (lane == 0) {
      int it = 0;
      bool zeroed = !args.zero_acc;
      for (int ti = 0;; ++ti) {
        const int p = ti & 1;
        if (!mbar_wait(smem_u32(&S.tab_empty[p]), ((ti >> 1) & 1) ^ 1)) {
          set_abort(S, args.err, kErrTimeoutProducer);
          break;
        }
        const int t = aborted(S) ? total : atomicAdd(args.queue, 1);
        const uint32_t tb = smem_u32(&S.tab_full[p]);
        if (t >= total) {
          S.tile_id[p] = kTileEnd;
          mbar_arrive(tb);
          break;
        }
        const Tile x = decode_tile(S, E, mode, t);
        if (x.phase == 2 && mode == 3) {
          // GEMM2 reads this expert's SwiGLU rows: wait for all of its GEMM1 tiles
          if (!wait_counter(args.done1 + x.e, EPI_WARPS * NT1 * S.tt1[x.e] + g_gate_extra)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            S.tile_id[p] = kTileEnd;
            mbar_arrive(tb);
            break;
          }
          fence_proxy_async_global();
        }
        if (x.phase == 2 && !zeroed) {
          // GEMM2 adds into the accumulator: every CTA's zeroing must be done
          if (!wait_counter(args.zero_done, (int)gridDim.x)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            S.tile_id[p] = kTileEnd;
            mbar_arrive(tb);
            break;
          }
          zeroed = true;
        }
        S.tile_id[p] = t;
        S.tile_t0[p] = globaltimer_ns();
        const int KB = x.phase == 1 ? KB1 : KB2;
        const size_t ld_sa = x.phase == 1 ? (size_t)args.R1 : 2 * (size_t)args.R1;
        const int nk = x.k1 - x.k0;
        const int arow = (x.phase == 1 ? S.row_off[x.e] : 2 * S.row_off[x.e]) + x.tt * NTOK;
        const float* sa = x.phase == 1 ? args.sa1 : args.sa2;
        const uint32_t bytes = nk * NTOK * 4 + 2 * KB * 4 + (x.phase == 2 ? NTOK * 4 : 0);
        mbar_arrive_expect_tx(tb, bytes);
        for (int kb = x.k0; kb < x.k1; ++kb)
          bulk_load(smem_u32(&S.sa[p][kb][0]), sa + kb * ld_sa + arow, NTOK * 4, tb);
        if (x.phase == 1) {
          bulk_load(smem_u32(&S.sw[p][0][0]), args.s13 + ((size_t)x.e * 32 + x.nt) * KB1, KB1 * 4, tb);
          bulk_load(smem_u32(&S.sw[p][1][0]), args.s13 + ((size_t)x.e * 32 + 16 + x.nt) * KB1, KB1 * 4, tb);
        } else {
          bulk_load(smem_u32(&S.sw[p][0][0]), args.s2 + ((size_t)x.e * kHiddenBlocks + 2 * x.nt) * KB2, KB2 * 4, tb);
          bulk_load(smem_u32(&S.sw[p][1][0]), args.s2 + ((size_t)x.e * kHiddenBlocks + 2 * x.nt + 1) * KB2, KB2 * 4,
                    tb);
          const int pr = S.row_off[x.e] + x.tt * (NTOK / 2);
          bulk_load(smem_u32(&S.tok[p][0]), args.row_token + pr, NTOK / 2 * 4, tb);
          bulk_load(smem_u32(&S.wgt[p][0]), args.row_weight + pr, NTOK / 2 * 4, tb);
        }
        const CUtensorMap* tw = x.phase == 1 ? &tmW13 : &tmW2;
        const CUtensorMap* ta = x.phase == 1 ? &tmA1 : &tmA2;
        const int w0 = x.phase == 1 ? x.e * kGemm1N + x.nt * 128 : x.e * kHidden + x.nt * 256;
        const int w1 = x.phase == 1 ? x.e * kGemm1N + kInter + x.nt * 128 : w0 + 128;
        bool ok = true;
        for (int kb = x.k0; kb < x.k1; ++kb, ++it) {
          const int s = it % STAGES, u = it / STAGES;
          if (!mbar_wait(smem_u32(&S.empty[s]), (u & 1) ^ 1)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&S.full[s]);
          const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(st, tw, fb, kb * 128, w0);
          tma_load_2d(st + W_TILE, tw, fb, kb * 128, w1);
          tma_load_2d(st + 2 * W_TILE, ta, fb, kb * 128, arow);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, NTOK);
      int it = 0, kt = 0;
      for (int ti = 0;; ++ti) {
        const int p = ti & 1;
        if (!mbar_wait(smem_u32(&S.tab_full[p]), (ti >> 1) & 1)) {
          set_abort(S, args.err, kErrTimeoutMma);
          break;
        }
        const int t = S.tile_id[p];
        mbar_arrive(smem_u32(&S.tab_empty[p]));
        if (t == kTileEnd) break;
        const Tile x = decode_tile(S, E, mode, t);
        const int KB = x.k1 - x.k0;
        bool ok = true;
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
          const uint32_t at = st + 2 * W_TILE;
          const uint32_t d = tmem_base + (uint32_t)(b * COLS);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(at + kk * 32);
            mma_e4m3(d, sdesc_sw128(st + kk * 32), ad, idesc, kk > 0 ? 1u : 0u);
            mma_e4m3(d + NTOK, sdesc_sw128(st + W_TILE + kk * 32), ad, idesc, kk > 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(&S.empty[s]));
          mma_commit(smem_u32(&S.tfull[b]));
        }
        if (!ok) break;
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ------------------------------------------------------------ promotion + epilogue
    const int q = warp & 3;
    const int r = 32 * q + lane;                          // weight row inside each 128-row block
    const uint32_t lane_addr = tmem_base + ((uint32_t)(32 * q) << 16);
    int kt = 0, sync_uses = 0;
    for (int ti = 0;; ++ti) {
      const int p = ti & 1;
      if (!mbar_wait(smem_u32(&S.tab_full[p]), (ti >> 1) & 1)) {
        set_abort(S, args.err, kErrTimeoutEpilogue);
        break;
      }
      const int t = S.tile_id[p];
      if (t == kTileEnd) break;
      const Tile x = decode_tile(S, E, mode, t);
      const int nvalid = min(NTOK, (x.phase == 1 ? S.cnt[x.e] : 2 * S.cnt[x.e]) - x.tt * NTOK);
      float g[NTOK], u[NTOK];
#pragma unroll
      for (int i = 0; i < NTOK; ++i) g[i] = u[i] = 0.f;
      bool ok = true;
      for (int kb = x.k0; kb < x.k1; ++kb, ++kt) {
        const int b = kt % NBUF, v = kt / NBUF;
        if (!mbar_wait(smem_u32(&S.tfull[b]), v & 1)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        float p0[NTOK], p1[NTOK];
        tmem_ld16(lane_addr + (uint32_t)(b * COLS), p0);
        tmem_ld16(lane_addr + (uint32_t)(b * COLS + NTOK), p1);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.tempty[b]));
        const float sw0 = S.sw[p][0][kb], sw1 = S.sw[p][1][kb];
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          const float sa = S.sa[p][kb][i];
          g[i] = fmaf(p0[i], sa * sw0, g[i]);
          u[i] = fmaf(p1[i], sa * sw1, u[i]);
        }
      }
      if (!ok) break;

      if (x.phase == 1 && S.ks1 > 1) {
        // K-sliced GEMM1 tile: publish this slice's partial sums; the slice
        // that completes the tile adds the others' and runs the epilogue
        const int ks = S.ks1, base = t - x.kh;                  // queue index of the tile's slice 0
        float* part = args.split_partial;
        const size_t pb = ((size_t)t * EPI_WARPS + q) * (2 * NTOK) * 32 + lane;
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          __stcg(part + pb + (size_t)i * 32, g[i]);
          __stcg(part + pb + (size_t)(NTOK + i) * 32, u[i]);
        }
        __threadfence();
        if (!epi_sync(S, sync_uses, lane)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          break;
        }
        if (q == 0 && lane == 0) {
          const bool last = atomicAdd(args.split_cnt + base / ks, 1) == ks - 1;
          if (last) atomicExch(args.split_cnt + base / ks, 0);   // re-armed for the next launch
          S.split_last[p] = last;
        }
        if (!epi_sync(S, sync_uses, lane)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          break;
        }
        if (S.split_last[p]) {
          __threadfence();
          for (int j = 0; j < ks; ++j) {
            if (j == x.kh) continue;
            const size_t ob = ((size_t)(base + j) * EPI_WARPS + q) * (2 * NTOK) * 32 + lane;
#pragma unroll
            for (int i = 0; i < NTOK; ++i) {
              g[i] += __ldcg(part + ob + (size_t)i * 32);
              u[i] += __ldcg(part + ob + (size_t)(NTOK + i) * 32);
            }
          }
        }
      }
      if (x.phase == 1 && (S.ks1 == 1 || S.split_last[p])) {
        // C = silu(X2) * X1 for this thread's intermediate column and the tile's tokens
        float am[NTOK];
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          const float x1 = g[i], x2 = u[i];
          g[i] = silu_mul(x1, x2);
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
        const int col = x.nt * 128 + r;
        const size_t prow0 = (size_t)S.row_off[x.e] + x.tt * NTOK;
#pragma unroll
        for (int i = 0; i < NTOK; ++i) {
          if (i < nvalid) {
            const float amax =
                fmaxf(fmaxf(S.amax[p][0][i], S.amax[p][1][i]), fmaxf(S.amax[p][2][i], S.amax[p][3][i]));
            const float s_hi = amax / kFp8Max;
            const float inv_hi = amax > 0.f ? kFp8Max / amax : 0.f;
            const __nv_fp8_storage_t hq = __nv_cvt_float_to_fp8(g[i] * inv_hi, __NV_SATFINITE, __NV_E4M3);
            const __half_raw hh = __nv_cvt_fp8_to_halfraw(hq, __NV_E4M3);
            const float hv = __half2float(*reinterpret_cast<const __half*>(&hh));
            const __nv_fp8_storage_t lq =
                __nv_cvt_float_to_fp8((g[i] - hv * s_hi) * (inv_hi * 16.0f), __NV_SATFINITE, __NV_E4M3);
            const size_t prow = prow0 + i;
            args.a2[(2 * prow) * kInter + col] = hq;
            args.a2[(2 * prow + 1) * kInter + col] = lq;
            if (r == 0) {
              float* sa2 = args.sa2 + (size_t)x.nt * 2 * args.R1 + 2 * prow;
              sa2[0] = s_hi;
              sa2[1] = s_hi * (1.0f / 16.0f);
            }
          }
        }
        if (mode == 3) {
          // publish: this warp's part of the expert's SwiGLU rows is written
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(args.done1 + x.e, 1);
        }
      } else if (x.phase == 2) {
        const int col = x.nt * 256 + r;
#pragma unroll
        for (int i = 0; i < NTOK / 2; ++i) {
          if (2 * i < nvalid && MOE_DCHECK(S.tok[p][i] >= 0 && S.tok[p][i] < args.T, args.err)) {
            const float w = S.wgt[p][i];
            float* dst = args.out_acc + (size_t)S.tok[p][i] * kHidden + col;
            atomicAdd(dst, (g[2 * i] + g[2 * i + 1]) * w);
            atomicAdd(dst + 128, (u[2 * i] + u[2 * i + 1]) * w);
          }
        }
      }
      __syncwarp();
      if (q == 0 && lane == 0) tile_trace(t, S.tile_t0[p]);
      if (lane == 0) mbar_arrive(smem_u32(&S.tab_empty[p]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  // the last CTA to leave re-arms the queue, so a launch can be repeated
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(args.queue + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(args.queue, 0);
      atomicExch(args.queue + 1, 0);
      if (args.zero_acc) atomicExch(args.zero_done, 0);
      if (mode == 3)
        for (int e = 0; e < E; ++e) atomicExch(args.done1 + e, 0);
    }
  }
}

static int g_attr_set[64];

}  // namespace dec

cudaError_t set_debug_waits_stream(unsigned long long limit_ns, int gate_extra) {
  return set_debug_waits_here(limit_ns, gate_extra);
}

cudaError_t stream_trace(int enable, unsigned long long* host, int n) {
  if (enable >= 0) {
    static unsigned long long zeros[dec::kTileTraceMax][4];
    const int z = 0;
    cudaError_t e = cudaMemcpyToSymbol(dec::g_tile_trace_n, &z, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(dec::g_tile_trace, zeros, sizeof(zeros));
    return e;
  }
  if (n > dec::kTileTraceMax * 4) n = dec::kTileTraceMax * 4;
  return cudaMemcpyFromSymbol(host, dec::g_tile_trace, sizeof(unsigned long long) * n);
}

cudaError_t launch_stream_gemm(const CUtensorMap& tmA1, const CUtensorMap& tmW13, const CUtensorMap& tmA2,
                               const CUtensorMap& tmW2, const DecodeArgs& args, int num_sms, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !dec::g_attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dec::stream_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)dec::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    if (dev < 64) dec::g_attr_set[dev] = 1;
  }
  return launch_kernel(dec::stream_gemm_kernel, dim3(num_sms), dim3(dec::THREADS), dec::SMEM_BYTES, st, true, tmA1, tmW13,
                       tmA2, tmW2, args);
}

}  // namespace moe
