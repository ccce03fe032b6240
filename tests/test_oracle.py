"""CPU: the oracle (numpy + C restatements) against golden vectors produced by
running the reference's own PyTorch implementation (tests/golden/make_golden.py)."""
import hashlib
import json

import numpy as np
import pytest
import torch

from cases import FULL_CASES, ROUTING_CASES, routing_case
from conftest import assert_close, load_golden, same_selection


def _checksum(t):
    t = t.contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()[:16]


def _sorted_with_weights(idx, w):
    p = np.argsort(idx, axis=1)
    return np.take_along_axis(idx, p, 1), np.take_along_axis(w, p, 1)


@pytest.mark.parametrize("name", ROUTING_CASES)
def test_routing_restatements_match_reference(name, oracle):
    import build_oracle
    g = load_golden(name)
    logits, bias = routing_case(name)
    meta = json.loads(str(g["meta"]))
    assert meta["checksums"]["routing_logits"] == _checksum(logits), "routing input generator drifted"
    bias_f = bias.float().numpy()
    for impl in ("numpy", "c"):
        if impl == "numpy":
            idx, w = oracle.route(logits.numpy(), bias_f, 2.5)
        else:
            idx, w = build_oracle.routing(logits.numpy(), bias_f, 2.5)
        si, sw = _sorted_with_weights(idx, w)
        assert (si == g["topk_idx"]).all(), f"{impl}: selection differs from the reference"
        np.testing.assert_allclose(sw, g["topk_weights"], rtol=1e-6, atol=1e-7)


def test_c_and_numpy_routing_agree_on_ties(oracle):
    import build_oracle
    logits, bias = routing_case("routing_adversarial")
    a, wa = oracle.route(logits.numpy(), bias.float().numpy(), 2.5)
    b, wb = build_oracle.routing(logits.numpy(), bias.float().numpy(), 2.5)
    assert (a == b).all()      # both break exact ties towards the lower index, in selection order
    np.testing.assert_allclose(wa, wb, rtol=1e-6)


@pytest.mark.parametrize("name", list(FULL_CASES))
def test_oracle_output_matches_reference(name, pkg, oracle):
    T, seed, skewed = FULL_CASES[name]
    g = load_golden(name)
    x = pkg.inputs.make_inputs(T, seed=seed, skewed=skewed)
    meta = json.loads(str(g["meta"]))
    for k, v in meta["checksums"].items():
        assert _checksum(getattr(x, k)) == v, f"input generator drifted on {k}"
    idx, w = oracle.route(oracle.to_np(x.routing_logits), oracle.to_np(x.routing_bias), 2.5)
    assert (np.sort(idx, 1) == g["topk_idx"]).all()
    out = oracle.moe_forward(*x.args(), routing=(idx, w))
    ref = torch.from_numpy(g["output_bf16"]).view(torch.bfloat16).float().numpy()
    # the restatement sums fp32 products in another order: at most one bf16 ulp apart
    assert_close(out, ref, atol=1e-3, rtol=8e-3, what=name)
    assert (out == ref).mean() > 0.99


def test_tie_aware_selection_helper():
    sb = np.zeros((1, 256), np.float32)
    assert same_selection(np.arange(8)[None], np.arange(8, 16)[None], sb).all()
    sb[0, :8] = 1
    assert not same_selection(np.arange(8)[None], np.arange(8, 16)[None], sb).all()


@pytest.mark.parametrize("scale", [1e-3, 1.0, 300.0])
def test_quantize_restatement_matches_torch(scale, pkg, oracle):
    """The numpy activation quantiser equals the input generator's torch conversion, bit for bit."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(40, 7168, generator=g) * scale
    x[1, :128] = 0.0                     # all-zero block
    x[2, 5] = -0.0
    for xx in (x, x.to(torch.bfloat16).float()):
        q, s = pkg.inputs.quantize_rows_1x128(xx)
        q2, s2 = oracle.quantize_rows(xx.numpy())
        assert np.array_equal(s.numpy(), s2)
        assert np.array_equal(q.view(torch.uint8).numpy(), q2)
