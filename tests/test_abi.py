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


def test_routed_run_argument_checks(pkg):
    """moe_fp8_block_scale_run_routed rejects missing selections and the fp32
    routed output in deterministic mode before launching anything."""
    lib = pkg.load_library()
    f = lib.moe_fp8_block_scale_run_routed
    f.argtypes = [ctypes.POINTER(pkg.MoeFp8Args), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    a = pkg.MoeFp8Args()
    a.num_tokens, a.num_local_experts = 4, 32
    assert f(ctypes.byref(a), None, None, None) == 1
    assert b"topk_idx" in lib.moe_fp8_last_error()
    fake = ctypes.c_void_p(256)                      # never dereferenced: the checks fail first
    assert f(ctypes.byref(a), fake, None, None) == 1
    assert b"topk_weights" in lib.moe_fp8_last_error()
    a.hidden_states = a.hidden_states_scale = a.gemm1_weights = a.gemm1_weights_scale = 256
    a.gemm2_weights = a.gemm2_weights_scale = 256
    old = pkg.set_deterministic(True)
    try:
        assert f(ctypes.byref(a), fake, fake, None) == 1
        assert b"deterministic" in lib.moe_fp8_last_error()
    finally:
        pkg.set_deterministic(old)
    a.num_tokens = 0
    assert f(ctypes.byref(a), fake, fake, None) == 0     # T = 0 is a no-op


def test_peer_exchange_geometry_checks(pkg):
    """Exchange-buffer sizes and the argument checks of the peer-memory entries
    (no device memory is touched)."""
    lib = pkg.load_library()
    nb = lib.moe_fp8_ep_peer_buffer_bytes
    nb.argtypes, nb.restype = [ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t
    assert nb(0, 2) == 0 and nb(16, 0) == 0 and nb(16, 9) == 0      # W <= 8
    b2, b8 = nb(8192, 2), nb(8192, 8)
    # rows of 7168 FP8 bytes + 56 scales + 8 ids + 8 weights, and fp32 return rows, per (source, slot)
    per_row = 7168 + 56 * 4 + 8 * 4 + 8 * 4 + 7168 * 4
    assert b2 >= 2 * 8192 * per_row and b8 >= 8 * 8192 * per_row and b8 < 8 * 8192 * per_row + 2 ** 20
    d = lib.moe_fp8_ep_peer_dispatch
    d.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int32] * 4 + [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    peers = (ctypes.c_void_p * 2)(1024, 2048)
    assert d(None, None, None, None, 9, 8, 0, 2, peers, 1, None) == 1           # T > capacity
    assert d(None, None, None, None, 4, 8, 0, 3, peers, 1, None) == 1           # 256 % 3 != 0
    assert d(None, None, None, None, 4, 8, 2, 2, peers, 1, None) == 1           # rank >= world
    assert d(None, None, None, None, 4, 8, 0, 2, peers, 1, None) == 1           # NULL token tensors
    w = lib.moe_fp8_ep_peer_wait
    w.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p]
    assert w(None, 2, 0, 1, None) == 1 and w(ctypes.c_void_p(1024), 2, 2, 1, None) == 1
