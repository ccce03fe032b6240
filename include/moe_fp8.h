/*
 * C-ABI of the B200 (sm_100a) DeepSeek-V3 FP8 block-scale fused-MoE operator.
 *
 * Drop-in for the operator `moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048`
 * of LudensCS/starter-kit-fused-moe. All tensor pointers are device pointers;
 * nothing here takes a framework type. Calls are asynchronous on the given
 * CUDA stream and never synchronise the host (except moe_fp8_read_device_error).
 */
#ifndef MOE_FP8_H_
#define MOE_FP8_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARGUMENT 1   /* bad shape, null pointer, misaligned pointer */
#define MOE_ERR_WORKSPACE 2          /* workspace missing or too small */
#define MOE_ERR_CUDA 3               /* a CUDA runtime / driver call failed */
#define MOE_ERR_DEVICE_TIMEOUT 4     /* a kernel gave up on a bounded wait (see moe_fp8_read_device_error) */

/*
 * Arguments of one operator call, in the reference's order.
 * Replaces the 11-argument DPS entry point
 *   run(routing_logits, routing_bias, hidden_states, hidden_states_scale,
 *       gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
 *       local_expert_offset, routed_scaling_factor, output)
 * of solution/cuda/main.cpp:38-49 (TVM-FFI export at main.cpp:117) and
 * solution/triton/current_kernel.py:1913-1925; shapes and dtypes as in
 * resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:57-145.
 */
typedef struct MoeFp8Args {
  const float* routing_logits;        /* f32  [T, 256] */
  const void* routing_bias;           /* bf16 [256], or NULL for all-zero bias */
  const void* hidden_states;          /* e4m3 [T, 7168] */
  const float* hidden_states_scale;   /* f32  [56, T] (token-contiguous) */
  const void* gemm1_weights;          /* e4m3 [E, 4096, 7168] */
  const float* gemm1_weights_scale;   /* f32  [E, 32, 56] */
  const void* gemm2_weights;          /* e4m3 [E, 7168, 2048] */
  const float* gemm2_weights_scale;   /* f32  [E, 56, 16] */
  int32_t local_expert_offset;        /* first global expert held here */
  float routed_scaling_factor;        /* 2.5 for DeepSeek-V3 */
  void* output;                       /* bf16 [T, 7168], fully overwritten */
  int32_t num_tokens;                 /* T >= 0 */
  int32_t num_local_experts;          /* E: 32 in the reference; 1..256 accepted */
  void* workspace;                    /* device scratch, >= moe_fp8_workspace_bytes(T, E) */
  size_t workspace_bytes;
} MoeFp8Args;

/*
 * Runs routing -> permute -> GEMM1+SwiGLU -> GEMM2+combine on `stream`
 * (a cudaStream_t; NULL = legacy default stream).
 * Replaces solution/cuda/kernel.cu:60-109 (launch_moe_cuda) behind main.cpp:38.
 */
int moe_fp8_block_scale_run(const MoeFp8Args* args, void* stream);

/* Launches one stage of moe_fp8_block_scale_run on its own: 0 routing,
 * 1 permute, 2 GEMM1+SwiGLU, 3 GEMM2+combine, 4 fp32 -> bf16 output. Each stage
 * reads what the earlier stages left in the workspace, so a stage can be
 * re-run and timed alone after one full call with the same arguments (GEMM2
 * adds into the accumulator that stage 0 clears). With GEMM path 2 stage 2
 * runs both GEMMs and stage 3 launches nothing. A profiling aid; the
 * reference's stages are the separate launches of solution/cuda/pure_moe.cu:589-661. */
int moe_fp8_run_stage(const MoeFp8Args* args, int32_t stage, void* stream);

/* The operator with the routing already made (expert parallelism: the rows a
 * rank received from other ranks, with the selections their sources made):
 * topk_idx / topk_weights [T, 8] replace routing_logits and routing_bias, which
 * may be NULL (an id outside [0, 256) selects nothing). With args->output
 * NULL the rounding pass is skipped: each row that has a local expert keeps
 * its fp32 result in the workspace's combine accumulator (moe_fp8_ep_peer_return
 * reads it there); not available in deterministic mode. Follows the expert
 * loop of the definition's reference (...json:146, step 3) for given
 * selections. */
int moe_fp8_block_scale_run_routed(const MoeFp8Args* args, const int32_t* topk_idx, const float* topk_weights,
                                   void* stream);

/* GEMM kernel family used for a call with `num_tokens` tokens:
 *   0  128-row tile kernels for both GEMMs (prefill shapes),
 *   1  weight-streaming GEMM1 + tile GEMM2,
 *   2  one weight-streaming launch doing GEMM1 and GEMM2 (decode shapes),
 *   3  weight-streaming GEMM1 and GEMM2 as two launches.
 * Automatic choice: 2 up to 240 tokens, 0 above. Plays the role of
 * the reference's token-count path selection (solution/triton/current_kernel.py:1812-1813, :2022). */
int32_t moe_fp8_gemm_path(int32_t num_tokens);

/* Forces a GEMM kernel family for every call (0..3), or -1 for the automatic
 * choice ($MOE_GEMM_PATH sets the initial value). Returns the previous setting. */
int32_t moe_fp8_set_gemm_path(int32_t path);

/* Deterministic combine (1) or the default fast combine (0); returns the
 * previous setting ($MOE_DETERMINISTIC sets the initial value). When on, every
 * call uses the 128-row tile kernels without K-sliced tiles, GEMM2 writes each
 * (token, expert) output row once, and the final pass sums a token's rows in
 * ascending local-expert order (the reference's accumulation order,
 * ...json:146 step 3), so repeated calls give bit-identical outputs. The
 * workspace then also holds those rows: moe_fp8_workspace_bytes reports the
 * size for the current setting. Plays the role of the reference's ordered
 * gather-reduce (cutlass_large_path.py:140-179). */
int32_t moe_fp8_set_deterministic(int32_t on);

/* Run the 128-row tile GEMMs as CTA pairs (1) or single CTAs (0, the default;
 * also $MOE_CTA_PAIR=1 at load); returns the previous setting. A pair is a
 * two-CTA cluster computing a 256-row tile with tcgen05.mma.cta_group::2: each
 * CTA loads its own 128 rows of activations and half of the weight tile (32 KB
 * per K-block instead of 48 KB), the leader issues the MMA, and each CTA
 * promotes and stores its own 128 rows. Same results within the parity bar;
 * not faster on this workload (see the design notes), hence off. Takes effect
 * for later calls; the workspace is unchanged. The reference's CuTe K13 kernel
 * shares operand tiles across a (1, 4) cluster instead
 * (solution/triton/cutlass_gemm1_helper.py:326-333). */
int32_t moe_fp8_set_cta_pair(int32_t on);

/* Workspace bytes for up to `max_tokens` tokens and `num_local_experts` experts.
 * The reference keeps an equivalent op-owned cache (solution/cuda/kernel.cu:25-56,
 * solution/triton/current_kernel.py:186-208); here the caller owns it. */
size_t moe_fp8_workspace_bytes(int32_t max_tokens, int32_t num_local_experts);

/* Routing only (kernel 1): writes topk ids / weights / per-expert counts into
 * the workspace, readable through moe_fp8_workspace_view. Follows the routing
 * step of the definition's reference (...json:146) and replaces
 * solution/triton/current_kernel.py:211-314 (_routing_topk_kernel). */
int moe_fp8_route(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                  int32_t local_expert_offset, int32_t num_local_experts, float routed_scaling_factor,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Device pointers into a workspace holding the state of the last call made
 * with the same (num_tokens, num_local_experts). Exposes what the reference
 * keeps in its internal buffers (topk ids / weights and per-expert counts of
 * solution/triton/current_kernel.py:1307-1502). */
typedef struct MoeFp8WorkspaceView {
  int32_t* topk_idx;       /* [T, 8] selected global experts, descending biased score */
  float* topk_weights;     /* [T, 8] combine weights */
  int32_t* expert_counts;  /* [E] local pairs per expert */
  int32_t* device_error;   /* sticky error bits of the kernels' bounded waits */
  int32_t pair_capacity;   /* padded pair-row capacity */
} MoeFp8WorkspaceView;
int moe_fp8_workspace_view(void* workspace, int32_t num_tokens, int32_t num_local_experts,
                           MoeFp8WorkspaceView* view);

/* Reads (and clears) the sticky device error word of a workspace; synchronises
 * `stream`. Returns MOE_OK, or MOE_ERR_DEVICE_TIMEOUT with *bits set (1: a
 * producer wait, 2: an MMA wait, 4: an epilogue wait ran out; 8: a debug-build
 * index check failed). Every kernel that records an error also marks the
 * current call, and that call's finalize pass writes NaN into the output rows
 * it owns, so a failed call never returns plausible numbers even when nobody
 * reads this word. The reference checks CUDA errors after its launches
 * (solution/cuda/kernel.cu:19-23). */
int moe_fp8_read_device_error(void* workspace, void* stream, int32_t* bits);

/* Test hook for the bounded waits (affects every later launch in this process
 * on the current device): `wait_limit_ns` replaces the 2 s limit of every
 * device-side wait (the expert-parallel flag waits included), and `gate_extra` is added to the target of the streaming
 * kernel's GEMM2 gate (the count of finished GEMM1 tiles it waits for), so a
 * test can make that wait run out without faulting anything. Restore with
 * (2000000000, 0). Returns MOE_OK or MOE_ERR_INVALID_ARGUMENT / MOE_ERR_CUDA.
 * Replaces nothing in the reference (its kernels have no bounded waits). */
int moe_fp8_debug_set_waits(uint64_t wait_limit_ns, int32_t gate_extra);

/* Routing without a workspace, for callers that may not allocate device
 * memory where they call this operator (a TensorRT plugin's enqueue, an XLA
 * custom call limited to the buffers its framework planned, a serving engine
 * that reserved its memory pool at start-up and forbids cudaMalloc afterwards).
 * Same kernel and results as moe_fp8_route; writes topk_idx [T, 8] and
 * topk_weights [T, 8] (device pointers). Its scratch (per-expert counters and
 * selection positions) is a fixed array inside this library's device image:
 * up to 16,384 tokens (larger T is rejected with MOE_ERR_INVALID_ARGUMENT),
 * about 513 KB held on every GPU that loads the library until exit. Every call
 * shares that array (the counters are cleared at the start of each call), so
 * calls that overlap on the GPU race and must be serialised by the caller. The
 * first call on a device looks up the array's address and should come before
 * any stream capture. No counterpart in the reference. */
int moe_fp8_route_static(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                         int32_t local_expert_offset, int32_t num_local_experts, float routed_scaling_factor,
                         int32_t* topk_idx, float* topk_weights, void* stream);

/* Producer-side activation quantiser: x [T, 7168] (bf16 if x_is_bf16, else f32)
 * -> hidden_states e4m3 [T, 7168] and hidden_states_scale f32 [56, T], the
 * operator's input layout (...json:81-88). Per 1x128 block s = max(amax,
 * 1e-12)/448 and q = e4m3(x/s), round to nearest even. The reference uses the
 * same recipe to re-quantise the SwiGLU output (cutlass_gemm1_helper.py:189-205). */
int moe_fp8_quantize_activations(const void* x, int32_t x_is_bf16, int32_t num_tokens, void* hidden_states,
                                 float* hidden_states_scale, void* stream);

/* ---- Expert parallelism (W ranks, each holding experts [r*E/W, (r+1)*E/W) and
 * calling moe_fp8_block_scale_run with local_expert_offset = r*E/W). The
 * reference has no multi-GPU path; its only hook is local_expert_offset
 * (...json:146). These kernels do the data movement around the all-to-alls
 * that the caller runs (NCCL / torch.distributed). Tokens are processed in
 * waves of `wave_tokens` consecutive tokens so that the exchange of one wave
 * can overlap the grouped GEMMs of another; send blocks are ordered
 * (wave, destination) and `send_offsets` [waves * W] is the exclusive scan of
 * `send_counts` in that order.
 *   plan     topk_idx [T, 8] -> send_counts [waves * W] (cleared first; every
 *            rank must use the same `waves`, and waves * wave_tokens >= T) and
 *            slot [T, W] (position of a token in its (wave, destination) block,
 *            -1 if that rank owns none of its experts).
 *   pack     logits [S, 256] f32, FP8 rows [S, 7168], scales [S, 56] f32
 *            (token-major for transport) into the send blocks.
 *   scales   received token-major scales [N, 56] -> [56, N] for the operator.
 *   combine  partial outputs returned into the send layout, bf16 [S, 7168] ->
 *            output [T, 7168] bf16, each token's partials summed in fp32. */
int moe_fp8_ep_plan(const int32_t* topk_idx, int32_t num_tokens, int32_t world, int32_t experts_per_rank,
                    int32_t wave_tokens, int32_t waves, int32_t* send_counts, int32_t* slot, void* stream);
int moe_fp8_ep_pack(const float* routing_logits, const void* hidden_states, const float* hidden_states_scale,
                    int32_t num_tokens, int32_t world, const int32_t* slot, const int32_t* send_offsets,
                    int32_t wave_tokens, float* send_logits, void* send_hidden, float* send_scales, void* stream);
int moe_fp8_ep_scales(const float* token_major_scales, int32_t num_tokens, float* hidden_states_scale, void* stream);
int moe_fp8_ep_combine(const void* returned_partials, const int32_t* slot, const int32_t* send_offsets,
                       int32_t wave_tokens, int32_t num_tokens, int32_t world, void* output, void* stream);

/* ---- Expert parallelism over peer memory (one GPU per rank, W <= 8 ranks on
 * one NVLink/NVSwitch node, 256 % W == 0). No host synchronisation and no
 * collective library on the data path: each rank owns an exchange buffer that
 * every peer maps (CUDA IPC), and the kernels move rows with plain peer stores
 * and publish (epoch) flags; every wait is bounded. One step on rank r, with
 * `epoch` increased by one per step on every rank and T <= capacity tokens:
 *   1. moe_fp8_route (E = 256) of the rank's tokens, then
 *      moe_fp8_ep_peer_dispatch: selections (expert id, weight) of every token
 *      slot to every rank, FP8 row + 56 scales to the ranks owning one of its
 *      experts, then flags.
 *   2. moe_fp8_ep_peer_wait(which = 0), then moe_fp8_block_scale_run_routed on
 *      the W * capacity received rows (moe_fp8_ep_peer_recv_view) with
 *      output = NULL and local_expert_offset = r * 256 / W, then
 *      moe_fp8_ep_peer_return (fp32 rows back to their sources, then flags).
 *   3. moe_fp8_ep_peer_wait(which = 1), then moe_fp8_ep_peer_combine: each
 *      token's partials summed in fp32 in ascending rank order, rounded once.
 * A wait that runs out sets a bit in the buffer's error word (16: dispatch
 * wait, 32: return wait; moe_fp8_ep_peer_read_error) and the step's combine
 * writes NaN rows. The reference has no multi-GPU path; its only
 * expert-parallel hook is local_expert_offset (...json:146). */
typedef struct MoeFp8EpRecvView {
  void* hidden_states;          /* e4m3 [W * capacity, 7168], row s * capacity + t */
  float* hidden_states_scale;   /* f32 [56, W * capacity] */
  int32_t* topk_idx;            /* [W * capacity, 8] global expert ids, -1 past a source's tokens */
  float* topk_weights;          /* [W * capacity, 8] */
  int32_t num_rows;             /* W * capacity */
} MoeFp8EpRecvView;
size_t moe_fp8_ep_peer_buffer_bytes(int32_t capacity, int32_t world);
int moe_fp8_ep_peer_buffer_alloc(int32_t capacity, int32_t world, void** base);
int moe_fp8_ep_peer_buffer_free(void* base);
/* 64-byte CUDA IPC handle of a buffer, and its mapping in another process. */
int moe_fp8_ep_peer_ipc_handle(void* base, void* handle);
int moe_fp8_ep_peer_ipc_open(const void* handle, void** base);
int moe_fp8_ep_peer_ipc_close(void* base);
int moe_fp8_ep_peer_recv_view(void* base, int32_t capacity, int32_t world, MoeFp8EpRecvView* view);
/* peer_bases: host array of the W ranks' buffer addresses as mapped in this process. */
int moe_fp8_ep_peer_dispatch(const int32_t* topk_idx, const float* topk_weights, const void* hidden_states,
                             const float* hidden_states_scale, int32_t num_tokens, int32_t capacity, int32_t rank,
                             int32_t world, void* const* peer_bases, uint32_t epoch, void* stream);
/* which = 0: the W dispatch flags, 1: the W return flags of this rank's buffer. */
int moe_fp8_ep_peer_wait(void* base, int32_t world, int32_t which, uint32_t epoch, void* stream);
/* workspace: the one moe_fp8_block_scale_run_routed used for the W * capacity received rows. */
int moe_fp8_ep_peer_return(void* workspace, int32_t num_local_experts, int32_t local_expert_offset,
                           int32_t capacity, int32_t rank, int32_t world, void* const* peer_bases, uint32_t epoch,
                           void* stream);
int moe_fp8_ep_peer_combine(const int32_t* topk_idx, int32_t num_tokens, int32_t capacity, int32_t world,
                            void* base, void* output, void* stream);
int moe_fp8_ep_peer_read_error(void* base, void* stream, int32_t* bits);

/* Text of the last error on the calling thread (the reference raises the
 * equivalent message through TVM_FFI_ICHECK, solution/cuda/main.cpp:20-34). */
const char* moe_fp8_last_error(void);

/* Number of kernels moe_fp8_block_scale_run launches for a given token count
 * (the reference's launch sequence is solution/cuda/pure_moe.cu:564-662). */
int32_t moe_fp8_kernels_per_call(int32_t num_tokens);

#ifdef __cplusplus
}
#endif
#endif /* MOE_FP8_H_ */
