"""Multi-GPU expert-parallel check (run by tests/test_gpu_ep.py under torchrun).

Every rank builds the same 256-expert weights (seeded, every expert distinct),
keeps its shard of 256/W experts and runs its own seeded tokens through

* the peer-memory transport (PeerExpertParallel: CUDA IPC buffers, peer stores,
  epoch flags), two steps in a row, the second on fewer tokens;
* the collective transport (ep_forward over NCCL, 3 waves).

A sample of each rank's tokens is checked against the CPU oracle over all 256
experts (fp32 sum over every expert, rounded once) at the parity bar, and the
two transports must agree. Prints one line per rank; exits non-zero on a
mismatch.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__ as ge  # noqa: E402


def check(got, ref):
    err = np.abs(got - ref)
    bad = ~(err <= 1e-2 + 2e-2 * np.abs(ref))
    return float(err.max()), int(bad.sum())


def main():
    T = int(os.environ.get("EP_CHECK_TOKENS", "200"))
    n_sample = int(os.environ.get("EP_CHECK_SAMPLE", "12"))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    pkg = ge.load_package()
    O = ge.load_oracle()
    import fused_moe_b200.ep as ep
    full = pkg.inputs.make_inputs(8, seed=0, device="cuda", num_local_experts=256)
    x = pkg.inputs.make_inputs(T, seed=100 + rank, device="cuda", num_local_experts=1)
    epr = 256 // world
    sl = slice(rank * epr, (rank + 1) * epr)
    shard = (full.gemm1_weights[sl], full.gemm1_weights_scale[sl], full.gemm2_weights[sl], full.gemm2_weights_scale[sl])
    peer = ep.PeerExpertParallel(rank, world, T)
    outs = []
    for n in (T, T // 2 + 1):                       # two steps: buffers reused, fewer tokens the second time
        idx = torch.arange(n, device="cuda")
        outs.append(peer.forward(x.routing_logits[idx], full.routing_bias, x.hidden_states[idx],
                                 x.hidden_states_scale[:, idx].contiguous(), *shard, 2.5))
    torch.cuda.synchronize()
    perr = peer.read_error()
    coll = ep.ep_forward(x.routing_logits, full.routing_bias, x.hidden_states, x.hidden_states_scale, *shard, 2.5,
                         waves=3)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, T // 2], np.random.default_rng(rank).choice(T, n_sample, replace=False)]))
    r = torch.from_numpy(rows).cuda()
    ref = O.moe_forward(x.routing_logits[r], full.routing_bias, x.hidden_states[r],
                        x.hidden_states_scale[:, r].contiguous(), full.gemm1_weights, full.gemm1_weights_scale,
                        full.gemm2_weights, full.gemm2_weights_scale, 0, 2.5)
    e1, b1 = check(outs[0][r].float().cpu().numpy(), ref)
    half = rows[rows < T // 2 + 1]
    e2, b2 = check(outs[1][torch.from_numpy(half).cuda()].float().cpu().numpy(), ref[rows < T // 2 + 1])
    ec, bc = check(coll[r].float().cpu().numpy(), ref)
    agree = bool(torch.allclose(outs[0].float(), coll.float(), atol=1e-2, rtol=2e-2))
    ok = b1 == 0 and b2 == 0 and bc == 0 and perr == 0 and agree and pkg.read_device_error() == 0
    print(f"EP_CHECK rank={rank} world={world} T={T} sampled={len(rows)} peer_max_abs_err={e1:.3e} "
          f"peer_step2_max_abs_err={e2:.3e} collective_max_abs_err={ec:.3e} bad={b1 + b2 + bc} "
          f"transports_agree={agree} ok={ok}", flush=True)
    dist.barrier()
    peer.close()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
