import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import __graft_entry__ as ge  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"
ATOL, RTOL = 1e-2, 2e-2   # output tolerance stated by the operator's acceptance bar


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return ge.load_package()


@pytest.fixture(scope="session")
def oracle():
    return ge.load_oracle()


def load_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return {k: z[k] for k in z.files}


def assert_close(got, ref, atol=ATOL, rtol=RTOL, what="output"):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape
    err = np.abs(got - ref)
    bad = ~(err <= atol + rtol * np.abs(ref))
    assert not bad.any(), (f"{what}: {bad.sum()} / {bad.size} elements outside atol {atol} / rtol {rtol}; "
                           f"max abs err {err.max():.4e}")
    return float(err.max()) if err.size else 0.0


def same_selection(idx_a, idx_b, sb):
    """Row-wise: are two top-8 selections the same set, up to exact ties in sb?"""
    a = np.sort(idx_a, axis=1)
    b = np.sort(idx_b, axis=1)
    same = (a == b).all(axis=1)
    for t in np.nonzero(~same)[0]:
        va = np.sort(sb[t, idx_a[t]])
        vb = np.sort(sb[t, idx_b[t]])
        same[t] = np.array_equal(va, vb)
    return same


def sampled_rows(oracle, x, n=160, seed=1234):
    """Token rows to check a large call on (the operator is token-wise): every
    token with >= 4 local experts (at most n // 2 of them), the first and last
    token, and a seeded random draw up to n rows. Returns (rows int64 numpy,
    MoeInputs of those tokens on the CPU, with the same weights)."""
    import torch
    from dataclasses import replace
    logits = oracle.to_np(x.routing_logits)
    bias = oracle.to_np(x.routing_bias)
    idx, _ = oracle.route(logits, bias, x.routed_scaling_factor)
    E = int(x.gemm1_weights.shape[0])
    le = idx - int(x.local_expert_offset)
    nloc = ((le >= 0) & (le < E)).sum(axis=1)
    T = logits.shape[0]
    heavy = np.nonzero(nloc >= 4)[0][: n // 2]
    rng = np.random.default_rng(seed)
    rest = rng.choice(T, size=min(T, n), replace=False)
    rows = np.unique(np.concatenate([heavy, [0, T - 1], rest]))[:n]
    r = torch.from_numpy(rows).to(x.routing_logits.device)
    xs = replace(x, routing_logits=x.routing_logits[r], hidden_states=x.hidden_states[r],
                 hidden_states_scale=x.hidden_states_scale[:, r].contiguous())
    return rows, xs
