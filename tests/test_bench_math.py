"""CPU: bench.py's roofline arithmetic (no GPU): algorithmic bytes per call and
per kernel, and t_bound = max(bytes / HBM peak, FLOPs / FP8 peak)."""
import bench


def test_algorithmic_bytes_match_the_stated_formula():
    # 17 hit experts, 65 pairs at T=64: weights + scales of each hit expert, per-token I/O, one counter block
    b = bench.algorithmic_bytes(64, 65, 17)
    assert b == 17 * (2 * 2048 * 7168 + 32 * 56 * 4 + 7168 * 2048 + 56 * 16 * 4) + 64 * (1024 + 7168 + 224 + 14336) + 512
    # the streaming kernel's bytes (GEMM1 + GEMM2) for the same call: 753.6 MB
    assert abs(bench.gemm1_bytes(65, 17) + bench.gemm2_bytes(65, 17) - 753_623_008) < 1e6


def test_rooflines_pick_the_binding_unit():
    hbm, fp8 = 6500.0, 3000.0                      # GB/s, TFLOP/s
    p = {"gemm1_kernel": {"us": 100.0, "bytes": 1.3e9, "useful_flops": 1e11},
         "gemm2_kernel": {"us": 100.0, "bytes": 1e8, "useful_flops": 2.4e11}}
    bench.add_rooflines(p, hbm, fp8)
    g1, g2 = p["gemm1_kernel"], p["gemm2_kernel"]
    assert g1["bound"] == "hbm" and abs(g1["t_bound_us"] - 200.0) < 1e-6 and abs(g1["frac"] - 2.0) < 1e-9
    assert g2["bound"] == "tensor" and abs(g2["t_bound_us"] - 80.0) < 1e-6 and abs(g2["frac"] - 0.8) < 1e-9
    assert abs(g2["tensor_frac_of_fp8_peak"] - 0.8) < 1e-9
