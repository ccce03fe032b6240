"""GPU: the routing entry point that allocates nothing (moe_fp8_route_static).

It exists for callers that may not allocate device memory where they call
the operator (a TensorRT plugin's enqueue, an XLA custom call restricted to its
planned buffers, a serving engine that forbids cudaMalloc once its pool is
reserved), so they cannot hand over the workspace the other entry points take.
Its scratch lives in a fixed array inside the library. This test calls it
through the C ABI twice in a row, on two different inputs, and checks each
result against the workspace-based moe_fp8_route: ids identical, weights within
the routing tolerance used elsewhere (rtol 1e-6). The first call is also
checked directly against the reference's own routing of the same tokens (the
golden vectors made by running the operator definition's reference). It also
checks that a token count above the array's limit is rejected.
"""
import ctypes

import numpy as np
import pytest
import torch

from cases import routing_case
from conftest import load_golden, same_selection

pytestmark = pytest.mark.gpu

MAX_TOKENS = 16384


def _route_with_workspace(pkg, logits, bias, offset, E):
    idx, w, _ = pkg.route(logits, bias, offset, E, 2.5)
    return idx.cpu().numpy(), w.cpu().numpy()


def _route_static(pkg, logits, bias, offset, E):
    lib = pkg.load_library()
    T = logits.shape[0]
    idx = torch.full((T, 8), -7, dtype=torch.int32, device="cuda")
    w = torch.full((T, 8), -7.0, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.moe_fp8_route_static(ctypes.c_void_p(logits.data_ptr()),
                                  ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                                  T, offset, E, ctypes.c_float(2.5), ctypes.c_void_p(idx.data_ptr()),
                                  ctypes.c_void_p(w.data_ptr()), stream)
    assert rc == 0, lib.moe_fp8_last_error()
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


def test_static_routing_matches_workspace_routing_twice(pkg):
    cases = [("routing_T4096_seed12_skewed", 0, 32), ("routing_T16384_seed11", 96, 64)]
    for name, offset, E in cases:          # two calls in a row, different sizes and offsets
        logits, bias = routing_case(name)
        logits, bias = logits.cuda(), bias.cuda()
        ref_idx, ref_w = _route_with_workspace(pkg, logits, bias, offset, E)
        idx, w = _route_static(pkg, logits, bias, offset, E)
        assert (idx == ref_idx).all(), f"{name}: expert ids differ"
        np.testing.assert_allclose(w, ref_w, rtol=1e-6, atol=1e-7)
        if name == "routing_T4096_seed12_skewed":
            g = load_golden(name)
            s = 1.0 / (1.0 + np.exp(-logits.cpu().numpy().astype(np.float32)))
            sb = (s + bias.float().cpu().numpy()[None]).astype(np.float32)
            same = same_selection(idx, g["topk_idx"].astype(np.int64), sb)
            assert same.all(), f"{(~same).sum()} tokens select a different set than the reference"
            exact = (np.sort(idx, 1) == g["topk_idx"]).all(1)
            p = np.argsort(idx, 1)
            np.testing.assert_allclose(np.take_along_axis(w, p, 1)[exact], g["topk_weights"][exact],
                                       rtol=1e-6, atol=1e-7)


def test_static_routing_rejects_too_many_tokens(pkg):
    lib = pkg.load_library()
    logits = torch.zeros(16, 256, device="cuda")
    out_i = torch.zeros(16, 8, dtype=torch.int32, device="cuda")
    out_w = torch.zeros(16, 8, device="cuda")
    rc = lib.moe_fp8_route_static(ctypes.c_void_p(logits.data_ptr()), None, MAX_TOKENS + 1, 0, 32,
                                  ctypes.c_float(2.5), ctypes.c_void_p(out_i.data_ptr()),
                                  ctypes.c_void_p(out_w.data_ptr()), None)
    assert rc == 1
    assert b"16384" in lib.moe_fp8_last_error()
