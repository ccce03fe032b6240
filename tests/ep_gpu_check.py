"""Multi-GPU expert-parallel check (run by tests/test_gpu_ep.py under torchrun).

Every rank builds the same 256-expert weights (seeded), keeps its shard of
256/W experts, runs ep_forward on its own seeded tokens over NCCL, and compares
the result with the single-GPU operator over all 256 experts on the same tokens
(the single-GPU path is itself checked against the CPU oracle). Prints one
line per rank; exits non-zero on a mismatch.
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__ as ge  # noqa: E402


def main():
    T = int(os.environ.get("EP_CHECK_TOKENS", "200"))
    waves = int(os.environ.get("EP_CHECK_WAVES", "3"))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    pkg = ge.load_package()
    import fused_moe_b200.ep as ep
    full = pkg.inputs.make_inputs(8, seed=0, device="cuda", num_local_experts=256, weight_experts=16)
    x = pkg.inputs.make_inputs(T, seed=100 + rank, device="cuda", weight_experts=1)
    epr = 256 // world
    sl = slice(rank * epr, (rank + 1) * epr)
    stats = {}
    out = ep.ep_forward(x.routing_logits, full.routing_bias, x.hidden_states, x.hidden_states_scale,
                        full.gemm1_weights[sl], full.gemm1_weights_scale[sl], full.gemm2_weights[sl],
                        full.gemm2_weights_scale[sl], 2.5, stats=stats, waves=waves)
    ref = pkg.run(x.routing_logits, full.routing_bias, x.hidden_states, x.hidden_states_scale, full.gemm1_weights,
                  full.gemm1_weights_scale, full.gemm2_weights, full.gemm2_weights_scale, 0, 2.5)
    torch.cuda.synchronize()
    err = (out.float() - ref.float()).abs()
    bad = err > 1e-2 + 2e-2 * ref.float().abs()
    ok = not bool(bad.any()) and pkg.read_device_error() == 0
    print(f"EP_CHECK rank={rank} world={world} T={T} waves={waves} sent={stats['sent_tokens']} received={stats['received_tokens']} "
          f"max_abs_err={err.max().item():.3e} bad={int(bad.sum())} ok={ok}", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
