// Kernels (3) and (4): FP8 block-scale grouped GEMMs on tcgen05.
//
// Both follow the reference's expert loop
// (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146,
// "3) Local expert compute and accumulation"):
//   GEMM1  G1 = A_e W13_e^T (K = 7168), C = silu(G1[:, I:]) * G1[:, :I]
//   GEMM2  O  = C W2_e^T    (K = 2048), output[token] += w * O
// with A, W13, W2 dequantised by their 1x128 / 128x128 fp32 block scales.
//
// One persistent CTA per SM walks a device-built tile list
// (expert, n-tile, m-tile), so no host synchronisation is needed for the
// expert histogram. Inside a CTA, warps specialise:
//   warp 0      TMA producer: A tile 128xSK and B tile 256xSK (FP8, swizzled)
//               per stage into a shared-memory ring (SK = 128: 48 KB stages);
//   warp 1      allocates 512 TMEM columns and issues tcgen05.mma kind::f8f6f4
//               (M=128, N=256, K=32 steps) into one of two TMEM partial
//               accumulators, one partial per 128-wide K-block;
//   warp 11     copies the block scales into shared memory with cp.async
//               (a ring of per-K-block activation-scale slices and per-tile
//               weight-scale rows, plus GEMM2's pair tokens and weights);
//   warps 2-9   promote every K-block's partial into registers with its block
//               scales (acc += partial * sa[row, kb] * sb[n-block, kb]): the
//               scales differ per K-block, so they are applied here, exactly
//               once per 128-wide K-block, while the tensor core already runs
//               the next K-block into the other TMEM buffer;
//   warp 10     (GEMM2) issues the output reductions the epilogue staged.
// Epilogues:
//   GEMM1  SwiGLU, then the 128 outputs of a row are re-quantised to FP8 as
//          two terms (hi = e4m3(c/s), lo = e4m3((c - hi*s)/(s/16)), s = amax/448)
//          stored as two consecutive rows of the GEMM2 operand, each with its
//          own 1x128 scale; GEMM2 sums the pair, so the intermediate keeps
//          about 8 bits of precision while GEMM2 stays on FP8 MMA.
//   GEMM2  sums the hi/lo rows (lane pair shuffle), multiplies by the routing
//          weight and stages the 128-column rows in shared memory; warp 10
//          adds them to the fp32 token accumulator with asynchronous bulk
//          reductions (cp.reduce.async.bulk .add.f32), so the top-k combine
//          happens here, with no separate reduce pass, and overlaps the next
//          tile's main loop.
#include "moe_common.cuh"
#include "moe_kernels.h"
#include "moe_workspace.h"

namespace moe {

// Tiles are 128 rows x 256 columns; block scales change every BK = 128 of K.
// Each GEMM's shared-memory ring moves SK (kTileStageK1/2) of K per stage.
constexpr int BM = 128, BN = 256, BK = 128, MAX_STAGES = 8;
// warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 promotion + epilogue,
// warp 10 GEMM2's output-reduction issuer, warp 11 block-scale loader
constexpr int GEMM_THREADS = 384;
constexpr int STORE_WARP = 10;
constexpr int SCALE_WARP = 11;
constexpr int EPI_WARPS = 8;
constexpr int TMEM_COLS = 512;
constexpr int kScaleRing = 8;        // K-blocks of activation scales in flight
constexpr int kEpiBarrier = 1;       // named barrier of the 8 epilogue warps

struct GemmSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t amax_bar[2];
  uint64_t staged[EPI_WARPS];   // GEMM2: an epilogue warp's rows are staged
  uint64_t sfree[EPI_WARPS];    // GEMM2: the store warp has read them
  int row_tok[EPI_WARPS][16];   // GEMM2: token of each staged row, -1 if none
  uint64_t scfull[kScaleRing];  // activation-scale ring (one 128-row slice per K-block)
  uint64_t scempty[kScaleRing];
  uint64_t tbfull[2];           // per-tile weight scales (+ GEMM2 pair tokens and weights)
  uint64_t tbempty[2];
  alignas(16) float sa_ring[kScaleRing][BM];
  // GEMM1: [0,56) gate-row scales, [64,120) up-row scales.
  // GEMM2: [0,32) scales of output column blocks 2nt and 2nt+1, [64,128) the
  // tile's 64 pair tokens (int), [128,192) their routing weights.
  alignas(16) float tile_buf[2][192];
  int tile_info[2][8];          // the unit's expert, n-tile, m-tile, first pair row, K-blocks [k0, k1),
                                // split slot (-1: whole tile), split tail-tile index
  int units, full_tiles, splits;  // work units: whole tiles, then `splits` K-slices per tail tile
  int split_last[2];            // GEMM1: this CTA completed the split tile
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
  int warp_sums[8];
  int tile_start[kMaxLocalExperts + 1];
  int row_off[kMaxLocalExperts];
  int cnt[kMaxLocalExperts];
  float amax_x[2][2][BM];
};

// Optional timeline of CTA 0 (clock64 per K-block and role), enabled by
// moe_fp8_set_trace(1); slots: 0 promotion wait start, 1 wait end, 2 promotion
// end, 3 MMA wait start, 4 MMA issued, 5 producer slot acquired, 6/7 tile-end
// work start/end (at the tile's last K-block), 8 SwiGLU done, 9 row amax
// exchanged, 10 stores issued (GEMM2: 8 next tile's state loaded, 9 staging
// free, 10 staged, 11 fenced).
constexpr int kTraceKBlocks = 512, kTraceSlots = 16;
__device__ unsigned long long g_trace[kTraceKBlocks * kTraceSlots];
__device__ int g_trace_on;

// The marks are compiled in only with -DMOE_GEMM_TRACE (they cost registers
// in the epilogue's main loop); otherwise the timeline stays zero.
__device__ __forceinline__ void trace_mark(int kt, int slot) {
#ifdef MOE_GEMM_TRACE
  if (blockIdx.x == 0 && kt < kTraceKBlocks && g_trace_on) g_trace[kt * kTraceSlots + slot] = clock64();
#endif
}

template <int MODE>
struct GemmCfg;
template <>
struct GemmCfg<1> {
  static constexpr int KB = kHiddenBlocks;   // 56 K-blocks over H
  static constexpr int NT = kInter / 128;    // 16 n-tiles: 128 gate + 128 up columns each
  static constexpr int ROWS_PER_PAIR = 1;
  static constexpr int SK = kTileStageK1;
  static constexpr int MAX_SPLITS = 6;         // each extra slice costs one partial-tile read in the fix-up
  static constexpr int STAGES = SK == 128 ? 3 : 8;
  // per epilogue warp: its 32 rows' hi and lo 64-byte pieces, two 2 KB boxes
  // in the 64-byte swizzle layout of the output tensor map
  static constexpr int STAGING = EPI_WARPS * 4096;
};
template <>
struct GemmCfg<2> {
  static constexpr int KB = kInterBlocks;    // 16 K-blocks over I
  static constexpr int NT = kHidden / BN;    // 28 n-tiles of 256 output columns
  static constexpr int ROWS_PER_PAIR = 2;    // hi and lo term rows
  static constexpr int SK = kTileStageK2;
  static constexpr int MAX_SPLITS = 4;         // slices of at least 4 K-blocks
  static constexpr int STAGES = SK == 128 ? 3 : 6;
  // per epilogue warp: 16 output rows of 128 fp32 (512 B), 528 B apart so the
  // float4 writes of 8 consecutive lanes fall in at most 2-way bank conflicts
  static constexpr int ROW_STRIDE = 528;
  static constexpr int STAGING = EPI_WARPS * 16 * ROW_STRIDE;
};

// CTA pairs (PAIR): a cluster of two CTAs computes a 256-row tile with
// tcgen05.mma.cta_group::2 (M=256, N=256), issued by the leader (cluster rank
// 0). Each CTA loads its own 128 A rows and half of B (128 rows, N split across
// the pair) and keeps its 128 rows x 256 columns of every K-block's partial in
// its own TMEM, so promotion and epilogue are the single-CTA ones. A stage is
// 32 KB per CTA instead of 48 KB: the operand ingest per SM, the pace-setter of
// the single-CTA kernels, drops by a third and more stages fit.
template <int MODE, bool PAIR>
constexpr int stage_bytes() {
  return (BM + (PAIR ? BN / 2 : BN)) * GemmCfg<MODE>::SK;
}
template <int MODE, bool PAIR>
constexpr int num_stages() {
  return PAIR ? (MODE == 1 ? 5 : 4) : GemmCfg<MODE>::STAGES;
}
template <int MODE, bool PAIR>
constexpr size_t gemm_smem_bytes() {
  return 1024 + (size_t)num_stages<MODE, PAIR>() * stage_bytes<MODE, PAIR>() + GemmCfg<MODE>::STAGING +
         sizeof(GemmSmem);
}
static_assert(gemm_smem_bytes<1, false>() <= 232448 && gemm_smem_bytes<2, false>() <= 232448, "shared memory budget");
static_assert(gemm_smem_bytes<1, true>() <= 232448 && gemm_smem_bytes<2, true>() <= 232448, "shared memory budget");
static_assert(num_stages<1, true>() <= MAX_STAGES && num_stages<2, true>() <= MAX_STAGES, "barrier arrays");
static_assert(GemmCfg<1>::STAGES <= MAX_STAGES && GemmCfg<2>::STAGES <= MAX_STAGES, "barrier arrays");
static_assert(GemmCfg<1>::SK == 128 && GemmCfg<2>::SK == 128, "the CTA-pair tiles assume 128-wide stages");

// ---- cluster / CTA-pair primitives
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_e4m3_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the mbarrier at this offset in both CTAs of the pair when the
// leader's issued tcgen05 operations are done.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   bar), "h"((uint16_t)3)
               : "memory");
}
// Arrive on an mbarrier of the other CTA of the pair (default semantics). The
// epilogue uses it to hand a TMEM buffer back to the leader's MMA after
// tcgen05.wait::ld and tcgen05.fence::before_thread_sync; a cluster-scope
// release here cost ~900 cycles per K-block (measured) and orders nothing the
// tcgen05 fences do not already order.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
static_assert((GemmCfg<1>::SK == 128 || GemmCfg<1>::SK == 64) && (GemmCfg<2>::SK == 128 || GemmCfg<2>::SK == 64),
              "stage K width");

// Block-wide exclusive scan of one int per thread over threads < 256.
__device__ __forceinline__ int block_scan_256(int v, int* warp_sums, int& total) {
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

template <int NT>
__device__ __forceinline__ void decode_tile(const GemmSmem& S, int E, int t, int& e, int& nt, int& mt) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (S.tile_start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int local = t - S.tile_start[e];
  // n-tile fastest: the CTAs of one round share a few A tiles (each read from
  // DRAM once, then from L2 by the expert's NT n-tiles) and sweep the expert's
  // weight rows, which stay in L2 across rounds; with the m-tile fastest an
  // expert holding thousands of rows re-streamed its whole A per n-tile
  // (4x the algorithmic DRAM bytes at 16k tokens, measured)
  mt = local / NT;
  nt = local - mt * NT;
}

// Work units. The tile list is walked round-robin by the persistent CTAs; when
// the last round would be partial (tail = tiles % grid), each tail tile is cut
// into `splits` K-slices so the tail spreads over the whole grid. GEMM2's
// slices simply add their partial outputs; GEMM1's slices meet in a fix-up
// (the last slice to arrive sums the others' fp32 partials and runs the
// epilogue).
struct Unit {
  int tile, k0, k1, slot, tail;   // slot: split index among all split units, -1 for a whole tile
};
__device__ __forceinline__ Unit unit_of(const GemmSmem& S, int u, int KB) {
  Unit x;
  if (u < S.full_tiles) {
    x.tile = u;
    x.k0 = 0;
    x.k1 = KB;
    x.slot = -1;
    x.tail = -1;
  } else {
    const int v = u - S.full_tiles, sp = S.splits;
    const int i = v / sp, j = v - i * sp;
    x.tile = S.full_tiles + i;
    x.k0 = j * KB / sp;
    x.k1 = (j + 1) * KB / sp;
    x.slot = v;
    x.tail = i;
  }
  return x;
}

__device__ __forceinline__ void set_abort(GemmSmem& S, int* err, int code) {
  record_error(err, code);
  *reinterpret_cast<volatile int*>(&S.abort_flag) = 1;
}
__device__ __forceinline__ bool aborted(const GemmSmem& S) {
  return *reinterpret_cast<const volatile int*>(&S.abort_flag) != 0;
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)lo | ((uint32_t)hi << 16);
}
__device__ __forceinline__ float2 unpack_e4m3x2(uint32_t v16) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v16, __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmOut, GemmArgs args) {
  using Cfg = GemmCfg<MODE>;
  constexpr int KB = Cfg::KB, NT = Cfg::NT, STAGES = num_stages<MODE, PAIR>(), SK = Cfg::SK, HS = BK / SK;
  constexpr int A_TILE = BM * SK, B_TILE = (PAIR ? BN / 2 : BN) * SK, STAGE_BYTES = A_TILE + B_TILE;
  constexpr int RB = PAIR ? 2 * BM : BM;   // rows of a tile
  // the pair's rank (0: leader, issues the MMA), the worker index and count (a pair is one worker)
  const int crank = PAIR ? (int)cluster_rank() : 0;
  const int wid = PAIR ? (int)cluster_id() : (int)blockIdx.x;
  const int G = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  GemmSmem& S = *reinterpret_cast<GemmSmem*>(staging + Cfg::STAGING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.E;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&S.full[s]), 1);
      mbar_init(smem_u32(&S.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.tfull[b]), 1);
      mbar_init(smem_u32(&S.tempty[b]), PAIR ? 2 * EPI_WARPS : EPI_WARPS);   // both CTAs' epilogues (leader's copy)
      mbar_init(smem_u32(&S.amax_bar[b]), EPI_WARPS);
    }
    for (int w = 0; w < EPI_WARPS; ++w) {
      mbar_init(smem_u32(&S.staged[w]), 1);
      mbar_init(smem_u32(&S.sfree[w]), 1);
    }
    for (int i = 0; i < kScaleRing; ++i) {
      mbar_init(smem_u32(&S.scfull[i]), 32);     // one cp.async arrival per loader lane
      mbar_init(smem_u32(&S.scempty[i]), EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.tbfull[b]), 33);     // 32 cp.async arrivals + the tile info
      mbar_init(smem_u32(&S.tbempty[b]), EPI_WARPS);
    }
    S.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  pdl_trigger();
  pdl_wait();  // the expert histogram and operands come from the preceding kernels
  // tile list from the device-side expert histogram
  {
    const int tid = threadIdx.x;
    const int c = (tid < E) ? args.counts[tid] : 0;
    const int mt = (c * Cfg::ROWS_PER_PAIR + RB - 1) / RB;
    int tot0, tot1;
    const int roff = block_scan_256(align_up(c, 128), S.warp_sums, tot0);
    const int tstart = block_scan_256(mt * NT, S.warp_sums, tot1);
    if (tid < E) {
      S.cnt[tid] = c;
      S.row_off[tid] = roff;
      S.tile_start[tid] = tstart;
    }
    if (tid == 0) {
      S.tile_start[E] = tot1;
      S.total_tiles = tot1;
      int tail = tot1 % G, sp = 1;
      if (tail > 0) {
        // a pair's two CTAs keep one partial tile each
        sp = min(min(G / tail, Cfg::MAX_SPLITS), (int)(WsLayout::kMaxSplitUnits / ((PAIR ? 2 : 1) * tail)));
        if (sp < 2) sp = 1;
      }
      if (sp == 1 || args.no_split) {
        sp = 1;
        tail = 0;
      }
      S.splits = sp;
      S.full_tiles = tot1 - tail;
      S.units = tot1 - tail + tail * sp;
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      // one warp of each CTA of the pair, same warp id and destination offset
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      tmem_alloc(smem_u32(&S.tmem_base), TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();   // the peer's barriers are initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;
  const int units = S.units;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = wid; u < units && ok && !aborted(S); u += G) {
        const Unit x = unit_of(S, u, KB);
        int e, nt, mt;
        decode_tile<NT>(S, E, x.tile, e, nt, mt);
        const int arow = Cfg::ROWS_PER_PAIR * S.row_off[e] + mt * RB + BM * crank;
        for (int ks = x.k0 * HS; ks < x.k1 * HS; ++ks, ++it) {
          const int s = it % STAGES, u = it / STAGES;
          if (!mbar_wait(smem_u32(&S.empty[s]), (u & 1) ^ 1)) {
            set_abort(S, args.err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          trace_mark(it, 5);
          const uint32_t fb = smem_u32(&S.full[s]);
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_TILE;
          const int x = ks * SK;
          if constexpr (PAIR) {
            // both CTAs' loads complete on the leader's full barrier, which expects both
            const uint32_t fbl = mapa_shared(fb, 0);
            if (crank == 0) mbar_arrive_expect_tx(fb, 2 * STAGE_BYTES);
            tma_load_2d_pair(sa, &tmA, fbl, x, arow);
            if (MODE == 1)   // N split across the pair: leader the 128 gate rows, peer the 128 up rows
              tma_load_2d_pair(sb, &tmB, fbl, x, e * kGemm1N + crank * kInter + nt * 128);
            else
              tma_load_2d_pair(sb, &tmB, fbl, x, e * kHidden + nt * BN + crank * 128);
            continue;
          }
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(sa, &tmA, fb, x, arow);
          if (MODE == 1) {
            tma_load_2d(sb, &tmB, fb, x, e * kGemm1N + nt * 128);
            tma_load_2d(sb + B_TILE / 2, &tmB, fb, x, e * kGemm1N + kInter + nt * 128);
          } else {
            tma_load_2d(sb, &tmB, fb, x, e * kHidden + nt * BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the leader, for a pair)
    if (lane == 0 && crank == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(PAIR ? 2 * BM : BM, BN);
      int it = 0, kt = 0;
      bool ok = true;
      for (int u = wid; u < units && ok && !aborted(S); u += G) {
        const Unit x = unit_of(S, u, KB);
        for (int kb = x.k0; kb < x.k1 && ok; ++kb, ++kt) {
          const int b = kt & 1, v = kt >> 1;
          trace_mark(kt, 3);
          if (!mbar_wait(smem_u32(&S.tempty[b]), (v & 1) ^ 1)) {
            set_abort(S, args.err, kErrTimeoutMma);
            ok = false;
            break;
          }
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
          for (int h = 0; h < HS; ++h, ++it) {                // HS stages per scale block
            const int s = it % STAGES, u = it / STAGES;
            if (!mbar_wait(smem_u32(&S.full[s]), u & 1)) {
              set_abort(S, args.err, kErrTimeoutMma);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t sb = sa + A_TILE;
#pragma unroll
            for (int kk = 0; kk < SK / 32; ++kk) {
              const uint64_t da = SK == 128 ? sdesc_sw128(sa + kk * 32) : sdesc_sw64(sa + kk * 32);
              const uint64_t db = SK == 128 ? sdesc_sw128(sb + kk * 32) : sdesc_sw64(sb + kk * 32);
              if constexpr (PAIR) mma_e4m3_pair(d, da, db, idesc, (h | kk) ? 1u : 0u);
              else mma_e4m3(d, da, db, idesc, (h | kk) ? 1u : 0u);
            }
            if constexpr (PAIR) mma_commit_pair(smem_u32(&S.empty[s]));   // frees the stage in both CTAs
            else mma_commit(smem_u32(&S.empty[s]));
          }
          if (!ok) break;
          if constexpr (PAIR) mma_commit_pair(smem_u32(&S.tfull[b]));
          else mma_commit(smem_u32(&S.tfull[b]));
          trace_mark(kt, 4);
        }
      }
    }
  } else if (warp == SCALE_WARP) {
    // ------------------------------------------------------------ block-scale loader
    // Copies, with 16-byte cp.async whose completion the mbarriers track, each
    // K-block's 128 activation scales into a ring and per tile the weight-scale
    // rows (GEMM2 also the tile's pair tokens and routing weights), so the
    // epilogue reads every scale from shared memory.
    const size_t ld_sa = (size_t)Cfg::ROWS_PER_PAIR * args.R1;
    int kq = 0, j = 0;
    bool ok = true;
    for (int u = wid; u < units && ok && !aborted(S); u += G, ++j) {
      const Unit x = unit_of(S, u, KB);
      int e, nt, mt;
      decode_tile<NT>(S, E, x.tile, e, nt, mt);
      const int arow = Cfg::ROWS_PER_PAIR * S.row_off[e] + mt * RB + BM * crank;
      const int tb = j & 1;
      if (!mbar_wait(smem_u32(&S.tbempty[tb]), ((j >> 1) & 1) ^ 1)) {
        set_abort(S, args.err, kErrTimeoutProducer);
        break;
      }
      float* buf = S.tile_buf[tb];
      if constexpr (MODE == 1) {
        // 14 chunks of 16 B per 56-float row: lanes 0-13 gate row, 14-27 up row
        if (lane < 28) {
          const int row = lane < 14 ? nt : 16 + nt, c = lane < 14 ? lane : lane - 14;
          cp_async16(smem_u32(buf + (lane < 14 ? 0 : 64) + 4 * c),
                     args.sb + ((size_t)e * 32 + row) * kHiddenBlocks + 4 * c);
        }
      } else {
        // 8 chunks of weight scales, 16 of tokens, 16 of weights
        const size_t p0 = (size_t)S.row_off[e] + (mt * RB + BM * crank) / 2;     // this CTA's first pair
        for (int c = lane; c < 40; c += 32) {
          if (c < 8) cp_async16(smem_u32(buf + 4 * c), args.sb + ((size_t)e * kHiddenBlocks + 2 * nt) * kInterBlocks + 4 * c);
          else if (c < 24) cp_async16(smem_u32(buf + 64 + 4 * (c - 8)), args.row_token + p0 + 4 * (c - 8));
          else cp_async16(smem_u32(buf + 128 + 4 * (c - 24)), args.row_weight + p0 + 4 * (c - 24));
        }
      }
      cp_async_mbar_arrive(smem_u32(&S.tbfull[tb]));
      if (lane == 0) {
        S.tile_info[tb][0] = e;
        S.tile_info[tb][1] = nt;
        S.tile_info[tb][2] = mt;
        S.tile_info[tb][3] = S.row_off[e];
        S.tile_info[tb][4] = x.k0;
        S.tile_info[tb][5] = x.k1;
        S.tile_info[tb][6] = x.slot;
        S.tile_info[tb][7] = x.tail;
        mbar_arrive(smem_u32(&S.tbfull[tb]));
      }
      for (int kb = x.k0; kb < x.k1; ++kb, ++kq) {
        const int ss = kq % kScaleRing, su = kq / kScaleRing;
        if (!mbar_wait(smem_u32(&S.scempty[ss]), (su & 1) ^ 1)) {
          set_abort(S, args.err, kErrTimeoutProducer);
          ok = false;
          break;
        }
        cp_async16(smem_u32(&S.sa_ring[ss][4 * lane]), args.sa + (size_t)kb * ld_sa + arow + 4 * lane);
        cp_async_mbar_arrive(smem_u32(&S.scfull[ss]));
      }
    }
    cp_async_wait_all();
  } else if (warp == STORE_WARP) {
    // ------------------------------------------------------------ GEMM2 output reductions
    // For every tile, take each epilogue warp's 16 staged rows and add them to
    // the fp32 token accumulator with asynchronous bulk reductions (lanes 0-15,
    // one 512-byte row each), so the epilogue never waits on the memory system.
    if constexpr (MODE == 2) {
      int j = 0;
      for (int u = wid; u < units && !aborted(S); u += G, ++j) {
        const Unit x = unit_of(S, u, KB);
        int e, nt, mt;
        decode_tile<NT>(S, E, x.tile, e, nt, mt);
        bool ok = true;
        for (int w = 0; w < EPI_WARPS && ok; ++w) {
          if (!mbar_wait(smem_u32(&S.staged[w]), j & 1)) {
            set_abort(S, args.err, kErrTimeoutEpilogue);
            ok = false;
            break;
          }
          const int tok = lane < 16 ? S.row_tok[w][lane] : -1;
          if (tok >= 0 && MOE_DCHECK(tok < args.T, args.err)) {
            const uint8_t* row = staging + (size_t)(w * 16 + lane) * Cfg::ROW_STRIDE;
            if (args.pair_out != nullptr) {
              // deterministic mode: the pair's own row (staged row `lane` of epilogue
              // warp w is pair 16 * quadrant + lane of the tile), written once
              const size_t prow = (size_t)S.row_off[e] + (mt * RB + BM * crank) / 2 + 16 * ((w + 2) & 3) + lane;
              bulk_store(args.pair_out + prow * kHidden + nt * BN + 128 * (w >> 2), smem_u32(row), 128 * sizeof(float));
            } else {
              float* dst = args.out_acc + (size_t)tok * kHidden + nt * BN + 128 * (w >> 2);
              bulk_reduce_add_f32(dst, smem_u32(row), 128 * sizeof(float));
            }
            bulk_commit();
          }
          bulk_wait_read_all();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&S.sfree[w]));
        }
        if (!ok) break;
      }
      bulk_wait_all();                   // reductions complete before the CTA exits
    }
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    const int ew = warp - 2;
    const int q = warp & 3;          // TMEM lane quadrant this warp may access
    const int g = ew >> 2;           // column half
    const int r = 32 * q + lane;     // row inside the tile
    const uint32_t lane_addr = tmem_base + ((uint32_t)(32 * q) << 16);
    int kt = 0, tile_iter = 0, amax_iter = 0;
    for (int u = wid; u < units && !aborted(S); u += G, ++tile_iter) {
      // the scale loader publishes the decoded tile with the tile's scales
      const int tb = tile_iter & 1;
      const float* tbuf = S.tile_buf[tb];
      if (warp == 4 && lane == 0) trace_mark(kt, 12);
      if (!mbar_wait(smem_u32(&S.tbfull[tb]), (tile_iter >> 1) & 1)) {
        set_abort(S, args.err, kErrTimeoutEpilogue);
        break;
      }
      // only the K range is live through the main loop; the rest of the tile's
      // description is read after it (registers are the epilogue's limit)
      const int k0 = S.tile_info[tb][4], k1 = S.tile_info[tb][5];
      if (warp == 4 && lane == 0) trace_mark(kt, 13);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      bool ok = true;
      for (int kb = k0; kb < k1; ++kb) {
        {
          const int b = kt & 1, v = kt >> 1;
          if (warp == 4 && lane == 0) trace_mark(kt, 0);
          if (!mbar_wait(smem_u32(&S.tfull[b]), v & 1)) {
            set_abort(S, args.err, kErrTimeoutEpilogue);
            ok = false;
            break;
          }
          const int ss = kt % kScaleRing;
          if (!mbar_wait(smem_u32(&S.scfull[ss]), (kt / kScaleRing) & 1)) {
            set_abort(S, args.err, kErrTimeoutEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          if (warp == 4 && lane == 0) trace_mark(kt, 1);
          const float sa = S.sa_ring[ss][r];
          const float f0 = sa * (MODE == 1 ? tbuf[kb] : tbuf[16 * g + kb]);
          const float f1 = MODE == 1 ? sa * tbuf[64 + kb] : f0;
          const uint32_t base = lane_addr + (uint32_t)(b * BN);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            // MODE 1: chunks 0-3 = gate columns 64g.., chunks 4-7 = up columns 128+64g..
            const int col0 = MODE == 1 ? (c < 4 ? 64 * g + 16 * c : 128 + 64 * g + 16 * (c - 4)) : 128 * g + 16 * c;
            float p0[16];
            tmem_ld16(base + col0, p0);
            tmem_ld_wait();
            const float f = c < 4 ? f0 : f1;
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[16 * c + i] = fmaf(p0[i], f, acc[16 * c + i]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&S.tempty[b]), 0));   // the leader's MMA waits
            else mbar_arrive(smem_u32(&S.tempty[b]));
            mbar_arrive(smem_u32(&S.scempty[ss]));
          }
          if (warp == 4 && lane == 0) trace_mark(kt, 2);
          ++kt;
        }
      }
      if (!ok) break;
      if (warp == 4 && lane == 0) trace_mark(kt - 1, 6);
      // GEMM2's pair token and weight are the last reads of this tile's scale
      // buffer; release it before the output work (whose global stores the
      // release would otherwise wait for)
      const int e = S.tile_info[tb][0], nt = S.tile_info[tb][1], mt = S.tile_info[tb][2];
      const int row_off_e = S.tile_info[tb][3];
      const int slot = S.tile_info[tb][6], tail_i = S.tile_info[tb][7];
      const int row_in_expert = mt * RB + BM * crank + r;     // GEMM row inside the expert's group
      const bool valid = row_in_expert < Cfg::ROWS_PER_PAIR * S.cnt[e];
      // a pair tile's second half can start past the expert's 128-row padded group
      // (GEMM1 groups are 128-aligned; GEMM2 term groups are 256-aligned): that
      // CTA's rows belong to the next group and must not be stored
      const bool beyond = mt * RB + BM * crank >= Cfg::ROWS_PER_PAIR * align_up(S.cnt[e], 128);
      const float w_pair = MODE == 2 ? tbuf[128 + (r >> 1)] : 0.f;
      const int tok_pair = MODE == 2 ? reinterpret_cast<const int*>(tbuf)[64 + (r >> 1)] : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.tbempty[tb]));

      if constexpr (MODE == 1) {
        if (slot >= 0) {
          // K-split tail tile: publish this slice's fp32 partial; the slice
          // that arrives last sums all of them and runs the epilogue.
          const int sp = S.splits;
          float4* part = reinterpret_cast<float4*>(args.split_partial);
          const int pslot = PAIR ? 2 * slot + crank : slot;   // each CTA of a pair keeps its own half
          const size_t base = (size_t)pslot * (EPI_WARPS * 32 * 32) + (size_t)ew * 32 * 32 + lane;
#pragma unroll
          for (int j4 = 0; j4 < 32; ++j4)
            __stcg(part + base + 32 * j4, make_float4(acc[4 * j4], acc[4 * j4 + 1], acc[4 * j4 + 2], acc[4 * j4 + 3]));
          __threadfence();
          named_barrier_sync(kEpiBarrier, EPI_WARPS * 32);
          if (ew == 0 && lane == 0)
            S.split_last[tb] = atomicAdd(args.split_cnt + (PAIR ? 2 * tail_i + crank : tail_i), 1) == sp - 1;
          named_barrier_sync(kEpiBarrier, EPI_WARPS * 32);
          if (!S.split_last[tb]) continue;
          __threadfence();
          const int first = slot - (slot % sp);
          for (int o = first; o < first + sp; ++o) {
            if (o == slot) continue;
            const size_t ob = (size_t)(PAIR ? 2 * o + crank : o) * (EPI_WARPS * 32 * 32) + (size_t)ew * 32 * 32 + lane;
#pragma unroll
            for (int j4 = 0; j4 < 32; ++j4) {
              const float4 v = __ldcg(part + ob + 32 * j4);
              acc[4 * j4] += v.x;
              acc[4 * j4 + 1] += v.y;
              acc[4 * j4 + 2] += v.z;
              acc[4 * j4 + 3] += v.w;
            }
          }
        }
        // SwiGLU: C = silu(X2) * X1 with X1 = gate half (cols < I), X2 = up half
        float amax = 0.f;
        if (valid) {                     // rows past the expert's count hold no data
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float c = silu_mul(acc[j], acc[64 + j]);
            acc[j] = c;
            amax = fmaxf(amax, fabsf(c));
          }
        }
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 8);
        // exchange the row maximum with the warp that holds the other 64 columns
        const int xb = amax_iter & 1;
        S.amax_x[xb][g][r] = amax;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.amax_bar[xb]));
        if (!mbar_wait(smem_u32(&S.amax_bar[xb]), (amax_iter >> 1) & 1)) {
          set_abort(S, args.err, kErrTimeoutEpilogue);
          break;
        }
        amax = fmaxf(amax, S.amax_x[xb][g ^ 1][r]);
        ++amax_iter;
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 9);
        // two-term quantisation, staged in the store boxes' 64-byte swizzle
        // (16-byte chunk c of row l sits at chunk c ^ ((l >> 1) & 3)), then
        // written by two TMA tensor stores per warp (rows past the expert's
        // count fill padding rows whose GEMM2 outputs are discarded)
        uint8_t* box_hi = staging + (size_t)ew * 4096;
        uint8_t* box_lo = box_hi + 2048;
        if (lane == 0) bulk_wait_read_all();                  // previous tile's boxes have been read
        __syncwarp();
        const float s_hi = amax / kFp8Max;
        const float inv_hi = amax > 0.f ? kFp8Max / amax : 0.f;
        const float s_lo = s_hi * (1.0f / 16.0f);
        const float inv_lo = inv_hi * 16.0f;
        const int sw = (lane >> 1) & 3;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int m4 = 0; m4 < 4; ++m4) {
            const int j4 = 4 * k + m4;
            float c[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] = acc[4 * j4 + i];
            hi[m4] = pack_e4m3x4(c[0] * inv_hi, c[1] * inv_hi, c[2] * inv_hi, c[3] * inv_hi);
            const float2 h01 = unpack_e4m3x2(hi[m4] & 0xffffu);
            const float2 h23 = unpack_e4m3x2(hi[m4] >> 16);
            lo[m4] = pack_e4m3x4((c[0] - h01.x * s_hi) * inv_lo, (c[1] - h01.y * s_hi) * inv_lo,
                                 (c[2] - h23.x * s_hi) * inv_lo, (c[3] - h23.y * s_hi) * inv_lo);
          }
          const int off = lane * 64 + ((k ^ sw) << 4);
          *reinterpret_cast<uint4*>(box_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(box_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && !beyond && MOE_DCHECK(row_off_e + mt * RB + BM * crank + 32 * q + 32 <= args.R1, args.err)) {
          const int y = row_off_e + mt * RB + BM * crank + 32 * q;   // pair row of the warp's first row
          tma_store_2d(&tmOut, smem_u32(box_hi), nt * 128 + 64 * g, y);
          tma_store_2d(&tmOut, smem_u32(box_lo), kInter + nt * 128 + 64 * g, y);
          bulk_commit();
        }
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 10);
        if (valid && g == 0) {
          const size_t prow = (size_t)row_off_e + row_in_expert;  // pair row
          float* sa2 = args.sa2 + (size_t)nt * 2 * args.R1 + 2 * prow;
          sa2[0] = s_hi;
          sa2[1] = s_lo;
        }
      } else {
        // combine: (hi row + lo row) * routing weight. Lanes 2p and 2p+1 hold
        // the two 64-column halves of pair p's 128-column output row; the warp
        // stages its 16 rows in shared memory for the store warp
        const int odd = lane & 1;
        const float w = w_pair;
        const int token = tok_pair;
        uint8_t* wstage = staging + (size_t)ew * 16 * Cfg::ROW_STRIDE;
        float* hrow = reinterpret_cast<float*>(wstage + (size_t)(lane >> 1) * Cfg::ROW_STRIDE + odd * 256);
        if (!mbar_wait(smem_u32(&S.sfree[ew]), (tile_iter & 1) ^ 1)) {   // previous tile's rows read
          set_abort(S, args.err, kErrTimeoutEpilogue);
          break;
        }
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 9);
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          float o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = 4 * j4 + i;
            const float a = acc[j], bb = acc[64 + j];
            const float send = odd ? a : bb;
            const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const float mine = odd ? bb : a;
            o[i] = (mine + recv) * w;
          }
          reinterpret_cast<float4*>(hrow)[j4] = make_float4(o[0], o[1], o[2], o[3]);
        }
        if (!odd) S.row_tok[ew][lane >> 1] = valid ? token : -1;
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 10);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.staged[ew]));
        if (warp == 4 && lane == 0) trace_mark(kt - 1, 11);
      }
      if (warp == 4 && lane == 0) trace_mark(kt - 1, 7);
    }
  }

  if (MODE == 1 && warp >= 2 && warp < 2 + EPI_WARPS && lane == 0) bulk_wait_all();   // output tiles written
  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the other may still signal its barriers
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

static int g_smem_set[2][2][64];
static int g_clusters[2][64];

// CTA-pair tile kernels: off unless $MOE_CTA_PAIR=1 at first use or moe_fp8_set_cta_pair(1).
int g_cta_pair = -1;
int set_cta_pair(int on) {
  const int old = cta_pair_enabled() ? 1 : 0;
  g_cta_pair = on ? 1 : 0;
  return old;
}
bool cta_pair_enabled() {
  if (g_cta_pair < 0) {
    const char* e = getenv("MOE_CTA_PAIR");
    g_cta_pair = (e && atoi(e) == 1) ? 1 : 0;
  }
  return g_cta_pair == 1;
}

template <int MODE, bool PAIR>
cudaError_t launch_gemm_t(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmOut,
                          const GemmArgs& args, int num_sms, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = grouped_gemm_kernel<MODE, PAIR>;
  const size_t smem = gemm_smem_bytes<MODE, PAIR>();
  if (dev >= 64 || !g_smem_set[MODE - 1][PAIR][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) g_smem_set[MODE - 1][PAIR][dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int nattr = 1;
  int grid = num_sms;
  if (PAIR) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    nattr = 2;
    // as many pairs as can be resident at once (a persistent grid must not wait for a second wave)
    int clusters = dev < 64 ? g_clusters[MODE - 1][dev] : 0;
    if (clusters == 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(num_sms & ~1);
      q.blockDim = dim3(GEMM_THREADS);
      q.dynamicSmemBytes = smem;
      q.attrs = &attr[1];
      q.numAttrs = 1;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, kern, &q);
      if (e != cudaSuccess || clusters < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
      clusters = min(clusters, num_sms / 2);
      if (dev < 64) g_clusters[MODE - 1][dev] = clusters;
    }
    grid = 2 * clusters;
  }
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmOut, args);
}

cudaError_t set_debug_waits_tile(unsigned long long limit_ns, int gate_extra) {
  return set_debug_waits_here(limit_ns, gate_extra);
}

cudaError_t set_trace(int on) {
  cudaError_t e = cudaMemcpyToSymbol(g_trace_on, &on, sizeof(int));
  if (e == cudaSuccess && on) {
    static unsigned long long zeros[kTraceKBlocks * kTraceSlots];
    e = cudaMemcpyToSymbol(g_trace, zeros, sizeof(zeros));
  }
  return e;
}
cudaError_t read_trace(unsigned long long* host, int n) {
  if (n > kTraceKBlocks * kTraceSlots) n = kTraceKBlocks * kTraceSlots;
  return cudaMemcpyFromSymbol(host, g_trace, sizeof(unsigned long long) * n);
}

cudaError_t launch_gemm1(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmOut,
                         const GemmArgs& args, int num_sms, cudaStream_t st) {
  return cta_pair_enabled() ? launch_gemm_t<1, true>(tmA, tmB, tmOut, args, num_sms, st)
                            : launch_gemm_t<1, false>(tmA, tmB, tmOut, args, num_sms, st);
}
cudaError_t launch_gemm2(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& args, int num_sms,
                         cudaStream_t st) {
  // GEMM2 stores no tiles
  return cta_pair_enabled() ? launch_gemm_t<2, true>(tmA, tmB, tmA, args, num_sms, st)
                            : launch_gemm_t<2, false>(tmA, tmB, tmA, args, num_sms, st);
}

}  // namespace moe
