"""GPU: failures are visible, and nothing here faults a GPU.

* A bounded device wait that runs out: the test hook moe_fp8_debug_set_waits
  shortens every wait to 20 ms and raises the target of the streaming kernel's
  GEMM2 gate (the count of finished GEMM1 tiles of an expert) past anything the
  kernel can reach. The call must come back (no hang), report the producer-wait
  bit through moe_fp8_read_device_error, and write NaN into every output row it
  owns instead of plausible numbers; the next normal call must be parity-clean.
  The reference's equivalent error path is its CUDA_CHECK after each launch
  (solution/cuda/kernel.cu:19-23).
* The -DMOE_DEBUG build (libmoe_b200_debug.so) checks every computed index
  before the access it guards; on correct inputs it records nothing and gives
  the same results as the release build.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu

WAIT_LIMIT_NS = 2_000_000_000


def _local_rows(oracle, x):
    idx, _ = oracle.route(oracle.to_np(x.routing_logits), oracle.to_np(x.routing_bias), 2.5)
    le = idx - int(x.local_expert_offset)
    return ((le >= 0) & (le < x.gemm1_weights.shape[0])).any(axis=1)


def test_gate_wait_runs_out_and_the_call_reports_it(pkg, oracle):
    lib = pkg.load_library()
    x = pkg.inputs.make_inputs(64, seed=61, device="cuda")
    old = pkg.set_gemm_path(2)
    try:
        assert pkg.read_device_error() == 0
        assert lib.moe_fp8_debug_set_waits(20_000_000, 1 << 24) == 0
        try:
            out = pkg.run(*x.args())
            torch.cuda.synchronize()
        finally:
            assert lib.moe_fp8_debug_set_waits(WAIT_LIMIT_NS, 0) == 0
        bits = pkg.read_device_error()
        assert bits & 1, f"expected the producer-wait bit, got {bits}"
        local = torch.from_numpy(_local_rows(oracle, x)).cuda()
        assert local.any()
        assert torch.isnan(out[local].float()).all(), "a timed-out call returned numbers"
        assert (out[~local] == 0).all()
        # the next normal call on the same workspace is clean
        out2 = pkg.run(*x.args())
        torch.cuda.synchronize()
        assert pkg.read_device_error() == 0
        assert_close(out2.float().cpu().numpy(), oracle.moe_forward(*x.args()), what="after a timed-out call")
    finally:
        pkg.set_gemm_path(old)


def test_debug_set_waits_rejects_bad_arguments(pkg):
    lib = pkg.load_library()
    assert lib.moe_fp8_debug_set_waits(0, 0) == 1
    assert lib.moe_fp8_debug_set_waits(WAIT_LIMIT_NS, -1) == 1


@pytest.fixture
def debug_build(pkg):
    """Route pkg.run through the index-checking library for the test's duration."""
    path = pkg.LIB_PATH.with_name("libmoe_b200_debug.so")
    if not path.exists():
        pytest.fail("libmoe_b200_debug.so is not built (build.py --debug, or __graft_entry__.build())")
    dbg = pkg.load_library(path)
    saved = pkg._lib
    pkg._lib = dbg
    pkg._ws.clear()
    try:
        yield dbg
    finally:
        pkg._lib = saved
        pkg._ws.clear()
        torch.cuda.empty_cache()


@pytest.mark.parametrize("path,T,skewed", [(2, 40, False), (0, 600, True), (1, 64, False), (3, 17, False)])
def test_debug_build_checks_pass_on_valid_inputs(path, T, skewed, debug_build, pkg, oracle):
    x = pkg.inputs.make_inputs(T, seed=70 + T, device="cuda", skewed=skewed)
    old = debug_build.moe_fp8_set_gemm_path(path)
    try:
        out = pkg.run(*x.args())
        torch.cuda.synchronize()
    finally:
        debug_build.moe_fp8_set_gemm_path(old)
    assert pkg.read_device_error() == 0
    assert_close(out.float().cpu().numpy(), oracle.moe_forward(*x.args()), what=f"debug build path {path}")


def test_debug_build_deterministic_combine(debug_build, pkg, oracle):
    x = pkg.inputs.make_inputs(200, seed=9, device="cuda")
    old = debug_build.moe_fp8_set_deterministic(1)
    try:
        pkg._ws.clear()
        out = pkg.run(*x.args())
        torch.cuda.synchronize()
    finally:
        debug_build.moe_fp8_set_deterministic(old)
    assert pkg.read_device_error() == 0
    assert_close(out.float().cpu().numpy(), oracle.moe_forward(*x.args()), what="debug build deterministic")
