"""Seeded synthetic inputs for the DeepSeek-V3 FP8 block-scale MoE operator.

The operator's inputs (shapes, dtypes and the transposed activation-scale
layout) follow the definition
`resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:57-135`.
The contest's own workloads are not available, so seeded synthetic tensors with
the benchmark's distributions stand in for them:

* routing_logits  f32  [T, 256]          ~ N(0, 1)
* routing_bias    bf16 [256]             ~ N(0, 0.1)
* hidden_states   e4m3 [T, 7168]         N(0, 1) quantised per 1x128 block,
  hidden_states_scale f32 [56, T]        scale = amax / 448 (token-contiguous)
* gemm1_weights   e4m3 [E, 4096, 7168]   N(0, 1/sqrt(7168)) per 128x128 block,
  gemm1_weights_scale f32 [E, 32, 56]
* gemm2_weights   e4m3 [E, 7168, 2048]   N(0, 1/sqrt(2048)) per 128x128 block,
  gemm2_weights_scale f32 [E, 56, 16]

Generation order is fixed (logits, bias, hidden, W13 expert by expert, W2
expert by expert) so that a CPU generator with a given seed always yields the
same tensors; the golden fixtures depend on that.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

H = 7168
I = 2048
E_GLOBAL = 256
E_LOCAL = 32
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
BLOCK = 128
FP8_MAX = 448.0
ROUTED_SCALING_FACTOR = 2.5
SKEW_LOCAL_EXPERTS = (0, 8, 16, 24)
SKEW_BIAS = 3.0


@dataclass
class MoeInputs:
    routing_logits: torch.Tensor
    routing_bias: torch.Tensor
    hidden_states: torch.Tensor
    hidden_states_scale: torch.Tensor
    gemm1_weights: torch.Tensor
    gemm1_weights_scale: torch.Tensor
    gemm2_weights: torch.Tensor
    gemm2_weights_scale: torch.Tensor
    local_expert_offset: int
    routed_scaling_factor: float

    def args(self):
        """The ten inputs in the reference's positional order."""
        return (self.routing_logits, self.routing_bias, self.hidden_states,
                self.hidden_states_scale, self.gemm1_weights, self.gemm1_weights_scale,
                self.gemm2_weights, self.gemm2_weights_scale,
                self.local_expert_offset, self.routed_scaling_factor)

    @property
    def T(self) -> int:
        return int(self.routing_logits.shape[0])

    def to(self, device) -> "MoeInputs":
        mv = lambda t: t.to(device)
        return MoeInputs(mv(self.routing_logits), mv(self.routing_bias), mv(self.hidden_states),
                         mv(self.hidden_states_scale), mv(self.gemm1_weights),
                         mv(self.gemm1_weights_scale), mv(self.gemm2_weights),
                         mv(self.gemm2_weights_scale), self.local_expert_offset,
                         self.routed_scaling_factor)


def quantize_rows_1x128(x: torch.Tensor):
    """x f32 [T, K] -> (e4m3 [T, K], f32 scales [K/128, T]) with scale = amax/448."""
    T, K = x.shape
    xb = x.view(T, K // BLOCK, BLOCK)
    amax = xb.abs().amax(dim=2).clamp_min(1e-12)
    s = amax / FP8_MAX
    q = (xb / s.unsqueeze(2)).to(torch.float8_e4m3fn).view(T, K)
    return q, s.t().contiguous()


def quantize_block_128x128(w: torch.Tensor):
    """w f32 [N, K] -> (e4m3 [N, K], f32 scales [N/128, K/128]) with scale = amax/448."""
    N, K = w.shape
    wb = w.view(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    amax = wb.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / FP8_MAX
    q = (wb / s[:, None, :, None]).to(torch.float8_e4m3fn).view(N, K)
    return q, s.contiguous()


@torch.no_grad()
def make_inputs(T: int, seed: int = 0, device: str = "cpu", num_local_experts: int = E_LOCAL,
                local_expert_offset: int = 0, skewed: bool = False,
                weight_experts: int | None = None) -> MoeInputs:
    """Build one seeded input set.

    `num_local_experts` experts of weights are generated (the first
    `weight_experts` of them when given, the rest are copies, which keeps large
    expert counts cheap to build for tests that only check properties).
    `skewed=True` sets the routing bias of local experts {0, 8, 16, 24} to +3.
    """
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    logits = torch.randn(T, E_GLOBAL, generator=g, device=dev, dtype=torch.float32)
    bias_f = torch.randn(E_GLOBAL, generator=g, device=dev, dtype=torch.float32) * 0.1
    if skewed:
        for le in SKEW_LOCAL_EXPERTS:
            bias_f[local_expert_offset + le] = SKEW_BIAS
    bias = bias_f.to(torch.bfloat16)
    hid = torch.randn(T, H, generator=g, device=dev, dtype=torch.float32)
    hq, hs = quantize_rows_1x128(hid)
    del hid

    E = num_local_experts
    n_gen = E if weight_experts is None else min(E, weight_experts)
    w13 = torch.empty(E, 2 * I, H, dtype=torch.float8_e4m3fn, device=dev)
    s13 = torch.empty(E, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=dev)
    std1 = 1.0 / math.sqrt(H)
    for e in range(n_gen):
        w = torch.randn(2 * I, H, generator=g, device=dev, dtype=torch.float32) * std1
        w13[e], s13[e] = quantize_block_128x128(w)
    w2 = torch.empty(E, H, I, dtype=torch.float8_e4m3fn, device=dev)
    s2 = torch.empty(E, H // BLOCK, I // BLOCK, dtype=torch.float32, device=dev)
    std2 = 1.0 / math.sqrt(I)
    for e in range(n_gen):
        w = torch.randn(H, I, generator=g, device=dev, dtype=torch.float32) * std2
        w2[e], s2[e] = quantize_block_128x128(w)
    for e in range(n_gen, E):
        w13[e].copy_(w13[e % n_gen]); s13[e].copy_(s13[e % n_gen])
        w2[e].copy_(w2[e % n_gen]); s2[e].copy_(s2[e % n_gen])
    return MoeInputs(logits, bias, hq, hs, w13, s13, w2, s2,
                     int(local_expert_offset), float(ROUTED_SCALING_FACTOR))
