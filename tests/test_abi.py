"""CPU: the C-ABI library loads and exports every symbol include/moe_fp8.h
declares; argument checks that need no GPU behave like the reference's."""
import ctypes
import re

import pytest
import torch

from conftest import ROOT


def _declared_functions():
    txt = (ROOT / "include" / "moe_fp8.h").read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(moe_[a-z0-9_]+)\s*\(", txt, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared_functions()
    assert "moe_fp8_block_scale_run" in names and "moe_fp8_workspace_bytes" in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/moe_fp8.h but not exported"
    assert set(_declared_functions()) <= set(pkg.EXPORTED_SYMBOLS) | {"moe_fp8_block_scale_run"}


def test_workspace_size_monotonic(pkg):
    lib = pkg.load_library()
    sizes = [lib.moe_fp8_workspace_bytes(t, 32) for t in (0, 1, 16, 4096, 16384)]
    assert all(a <= b for a, b in zip(sizes, sizes[1:]))
    assert lib.moe_fp8_workspace_bytes(16, 0) == 0 and lib.moe_fp8_workspace_bytes(16, 257) == 0
    # T=16384: 8*T + 127*E pair rows of activations, two FP8 terms of intermediate, fp32 accumulator
    assert sizes[-1] < 3 * 2**30


def test_kernels_per_call(pkg):
    lib = pkg.load_library()
    assert lib.moe_fp8_kernels_per_call(0) == 0
    assert lib.moe_fp8_kernels_per_call(16) == 4        # routing, permute, fused streaming GEMMs, finalize
    assert lib.moe_fp8_kernels_per_call(4096) == 5
    assert [lib.moe_fp8_gemm_path(t) for t in (1, 96, 240, 241, 4096)] == [2, 2, 2, 0, 0]


def test_invalid_arguments_rejected_before_any_launch(pkg):
    lib = pkg.load_library()
    a = pkg.MoeFp8Args()
    a.num_tokens, a.num_local_experts = 4, 0
    assert lib.moe_fp8_block_scale_run(ctypes.byref(a), None) == 1
    assert b"num_local_experts" in lib.moe_fp8_last_error()
    a.num_local_experts = 32
    assert lib.moe_fp8_block_scale_run(ctypes.byref(a), None) == 1        # NULL tensors
    a.num_tokens = -1
    assert lib.moe_fp8_block_scale_run(ctypes.byref(a), None) == 1
    a.num_tokens = 0
    assert lib.moe_fp8_block_scale_run(ctypes.byref(a), None) == 0        # T = 0 is a no-op
    assert lib.moe_fp8_block_scale_run(None, None) == 1


def test_run_raises_without_cuda(pkg):
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    x = torch.zeros(1, 256)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.run(x, None, x, x, x, x, x, x, 0, 2.5)


def test_no_cpu_fallback_in_product_sources():
    """The product package never imports the oracle."""
    for p in (ROOT / "starter-kit-fused-moe_b200").rglob("*.py"):
        assert "moe_oracle" not in p.read_text() and "oracle/" not in p.read_text(), p


def test_deterministic_switch_and_workspace(pkg):
    lib = pkg.load_library()
    base = lib.moe_fp8_workspace_bytes(64, 32)
    old = pkg.set_deterministic(True)
    try:
        assert lib.moe_fp8_gemm_path(16) == 0                      # tile kernels only
        assert lib.moe_fp8_workspace_bytes(64, 32) >= base + 64 * 7168 * 4
    finally:
        pkg.set_deterministic(old)
    assert lib.moe_fp8_workspace_bytes(64, 32) == base
