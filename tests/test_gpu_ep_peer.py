"""GPU, one device: the peer-memory expert-parallel exchange with W ranks
emulated in one process (W = 2, 4, 8).

Every emulated rank gets its own exchange buffer on this GPU and the peer table
lists all W of them, so the same kernels and flag protocol run as across W
GPUs. Phases are run rank by rank in stream order (every rank's dispatch, then
every rank's compute, then every rank's combine), so no kernel ever waits on a
kernel that has not been launched before it. Two steps with different ragged
splits of one token pool (one rank gets no tokens) check buffer reuse: stale
rows of the first step must not leak into the second.

Expected values: the CPU oracle over all 256 experts (distinct weights) for the
whole token pool, summed in fp32 and rounded once, which is what the expert-
parallel result must equal within the parity bar. Also: a flag wait that runs
out (20 ms limit, a flag nothing sets) reports its bit and the combine writes
NaN instead of numbers.
"""
import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu

POOL = 72
CAPACITY = 72


@pytest.fixture(scope="module")
def pool(pkg, oracle):
    """256-expert weights, a pool of tokens and the oracle's output for it."""
    full = pkg.inputs.make_inputs(POOL, seed=2024, device="cuda", num_local_experts=256)
    ref = oracle.moe_forward(*full.args())
    yield full, ref
    del full
    torch.cuda.empty_cache()


def _splits(world, step):
    """Ragged token ranges per rank; step 1 leaves the last rank empty."""
    if step == 0:
        cuts = np.linspace(0, POOL, world + 1).astype(int)
    else:
        w = np.arange(world, 0, -1, dtype=float)
        w[-1] = 0.0
        cuts = np.concatenate([[0], np.cumsum(w / w.sum() * POOL)]).round().astype(int)
        cuts[-1] = POOL
    return [(int(a), int(b)) for a, b in zip(cuts[:-1], cuts[1:])]


def _make_ranks(pkg, world):
    import fused_moe_b200.ep as ep
    K = ep.LibraryPeerBackend(pkg)
    bases = [K.alloc(CAPACITY, world) for _ in range(world)]
    ranks = [ep.PeerExpertParallel(r, world, CAPACITY, peer_bases=bases, backend=K, base=bases[r])
             for r in range(world)]
    return K, bases, ranks


def _step(ranks, full, spans, shards):
    for r, (a, b) in enumerate(spans):
        idx = torch.arange(a, b, device="cuda")
        ranks[r].dispatch(full.routing_logits[idx], full.routing_bias, full.hidden_states[idx],
                          full.hidden_states_scale[:, idx].contiguous(), 2.5)
    for r in range(len(ranks)):
        ranks[r].compute(*shards[r], 2.5)
    return [ranks[r].combine(device="cuda") for r in range(len(ranks))]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange_emulated_ranks_match_oracle(world, pkg, pool):
    full, ref = pool
    epr = 256 // world
    shards = [(full.gemm1_weights[r * epr:(r + 1) * epr], full.gemm1_weights_scale[r * epr:(r + 1) * epr],
               full.gemm2_weights[r * epr:(r + 1) * epr], full.gemm2_weights_scale[r * epr:(r + 1) * epr])
              for r in range(world)]
    K, bases, ranks = _make_ranks(pkg, world)
    try:
        for step in range(2):
            spans = _splits(world, step)
            outs = _step(ranks, full, spans, shards)
            torch.cuda.synchronize()
            for r, (a, b) in enumerate(spans):
                assert ranks[r].read_error() == 0
                assert outs[r].shape == (b - a, 7168)
                if b > a:
                    err = assert_close(outs[r].float().cpu().numpy(), ref[a:b], what=f"W={world} step {step} rank {r}")
                    print(f"W={world} step={step} rank={r} tokens={b - a} max_abs_err={err:.3e}")
        assert pkg.read_device_error() == 0
    finally:
        for rk in ranks:
            rk.close()


def test_peer_wait_runs_out_and_combine_reports_it(pkg, pool):
    full, _ = pool
    lib = pkg.load_library()
    K, bases, ranks = _make_ranks(pkg, 2)
    try:
        rk = ranks[0]
        idx = torch.arange(0, 8, device="cuda")
        rk.dispatch(full.routing_logits[idx], full.routing_bias, full.hidden_states[idx],
                    full.hidden_states_scale[:, idx].contiguous(), 2.5)
        # rank 1 never dispatches and never returns: both waits of rank 0 run out
        assert lib.moe_fp8_debug_set_waits(20_000_000, 0) == 0
        try:
            K.wait(rk, 0)
            out = rk.combine(device="cuda")
            torch.cuda.synchronize()
        finally:
            assert lib.moe_fp8_debug_set_waits(2_000_000_000, 0) == 0
        bits = rk.read_error()
        assert bits & 16 and bits & 32, f"expected both wait bits, got {bits}"
        assert torch.isnan(out.float()).all()
    finally:
        for r in ranks:
            r.close()
