// Shared constants and sm_100a primitives (mbarrier, TMA, tcgen05) for the
// DeepSeek-V3 FP8 block-scale fused-MoE kernels.
//
// Geometry is fixed by the operator definition
// (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:11-56):
// H = 7168, I = 2048, 256 routed experts in 8 groups, top-8, 128-wide FP8 blocks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace moe {

constexpr int kHidden = 7168;           // H
constexpr int kInter = 2048;            // I
constexpr int kGemm1N = 2 * kInter;     // 4096 (gate rows, then up rows)
constexpr int kExperts = 256;           // routed experts (global)
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kTopKGroups = 4;
constexpr int kBlock = 128;             // quantisation block edge
constexpr int kHiddenBlocks = kHidden / kBlock;   // 56
constexpr int kInterBlocks = kInter / kBlock;     // 16
// K width of one shared-memory stage of the 128-row tile GEMMs (128: 128-byte
// swizzle, one stage per scale block; 64: 64-byte swizzle, two stages per
// block). The tensor maps of those GEMMs are built with the same box width.
constexpr int kTileStageK1 = 128;   // GEMM1
constexpr int kTileStageK2 = 128;   // GEMM2
constexpr float kFp8Max = 448.f;
constexpr int kMaxLocalExperts = 256;

// Error bits written to the device error word.
constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutEpilogue = 4;

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// Set when a kernel found an index outside its buffer (debug builds only,
// -DMOE_DEBUG); the access is skipped.
constexpr int kErrIndex = 8;

// The device error area (first 256 bytes of the workspace): word 0 is sticky
// (cleared only by the host reader), word 1 covers the current call (cleared
// with the call's counters); the finalize pass reads word 1.
__device__ __forceinline__ void record_error(int* err, int code) {
  atomicOr(err, code);
  atomicOr(err + 1, code);
}

// Test hooks, one copy per translation unit (set from the host through
// moe_fp8_debug_set_waits): the wait limit, and an amount added to the
// streaming kernel's GEMM2 gate target so that a test can make that wait run
// out on purpose. Defaults: 2 s, 0.
static __device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
static __device__ int g_gate_extra = 0;
static inline cudaError_t set_debug_waits_here(unsigned long long limit_ns, int gate_extra) {
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_gate_extra, &gate_extra, sizeof(gate_extra));
  return e;
}

#ifdef MOE_DEBUG
// Debug builds check computed indices before the access they guard.
#define MOE_DCHECK(cond, err) ((cond) ? true : (record_error((err), kErrIndex), false))
#else
#define MOE_DCHECK(cond, err) true
#endif

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// g_wait_limit_ns (2 s) and returns false (the caller records an error and unwinds).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns(), limit = g_wait_limit_ns;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit) return false;
  }
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion counted on `bar`.
// x (the innermost coordinate, in bytes for FP8) is always a multiple of 128.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled bulk tensor store shared -> global, tracked by the issuing
// thread's bulk async-group (x a multiple of 16 bytes, y >= 0).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

// L2 prefetch of one tensor-map box (no shared memory involved).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* m, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y)
               : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// 1-D bulk reduction shared -> global: dst[i] += src[i] over `bytes` of fp32
// (16-byte aligned addresses, size a multiple of 16), tracked by the issuing
// thread's bulk async-group. The generic-proxy writes of src must be made
// visible to the async proxy first (fence_proxy_async_smem).
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(dst)),
               "r"(src), "r"(bytes)
               : "memory");
}
// 1-D bulk copy shared -> global (16-byte aligned, size a multiple of 16),
// tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's bulk groups have finished reading their shared-memory sources.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src))
               : "memory");
}
// The mbarrier receives one arrival once all of this thread's earlier cp.async
// copies have completed (the arrival is part of the barrier's initial count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Named barrier over `count` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row core groups 1024 bytes apart.
// Fields: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version=1 [46,48),
// base offset [49,52) = 0 (tiles are 1024-byte aligned), layout [61,64) = 2 (SW128).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;              // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;    // SBO
  d |= (uint64_t)1 << 46;              // version
  d |= (uint64_t)2 << 61;              // SWIZZLE_128B
  return d;
}

// SwiGLU of one intermediate column: silu(x2) * x1 = x2 / (1 + e^-x2) * x1,
// with the hardware exponential and the approximate division (a few ulp; for
// x2 -> -inf the quotient goes to 0, for x2 -> +inf it is x2).
__device__ __forceinline__ float silu_mul(float x1, float x2) {
  return __fdividef(x2, 1.0f + __expf(-x2)) * x1;
}

// Same for the 64-byte swizzle canonical layout: rows of 64 bytes, 8-row core
// groups 512 bytes apart, layout type 4 (SW64); tiles 512-byte aligned.
__device__ __forceinline__ uint64_t sdesc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;              // LBO (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;     // SBO
  d |= (uint64_t)1 << 46;              // version
  d |= (uint64_t)4 << 61;              // SWIZZLE_64B
  return d;
}

// Instruction descriptor for kind::f8f6f4 with e4m3 A and B, f32 accumulator,
// both operands K-major. N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4)                        // D format f32
         | (0u << 7) | (0u << 10)         // A, B = e4m3
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ programmatic dependent launch
// Lets the next kernel on the stream start launching (its prologue overlaps this kernel).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the preceding kernel on the stream has completed and its writes are visible
// (a no-op when this kernel was launched without the programmatic-serialization attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with programmatic stream serialization (PDL) when `pdl` is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

}  // namespace moe
