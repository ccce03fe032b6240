"""Benchmark of the B200 FP8 block-scale fused MoE (DeepSeek-V3 shapes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference] [--no-sweep]

One step = one operator call on one batch of T tokens (default T=64: the
decode configuration of the benchmark, 32 local experts, local_expert_offset 0).
`value` is device time per call (CUDA events, inputs resident in HBM, L2
flushed between calls); `e2e` is the same call through the public `run(...)`
with the step's inputs copied from pinned host memory and the output copied
back inside the timed region. With N > 1 ranks (torchrun) the workload is the
expert-parallel configuration: 8192 tokens per rank over 256 experts sharded
256/N per GPU, exchanged over peer memory; the max over ranks is reported.
`--impl reference` times the CPU reference path (the numpy oracle restating
the definition's PyTorch reference) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

import __graft_entry__ as ge

H, I = 7168, 2048
FLOPS_PER_PAIR = 2 * H * 2 * I + 2 * I * H                 # 88,080,384
W13_BYTES = 2 * I * H + 32 * 56 * 4                          # per expert, with scales
W2_BYTES = H * I + 56 * 16 * 4
TOKEN_IO_BYTES = 256 * 4 + H + 56 * 4 + H * 2                # logits, hidden, scales, bf16 output
L2_FLUSH_BYTES = 256 << 20
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the fused
# streaming kernel on the default workload (seed-0 inputs, T=64), from one
# `ncu --set full --clock-control none -k regex:stream_gemm_kernel -s 2 -c 1`
# capture of `python bench.py --steps 3 --warmup 3 --no-sweep --no-cpu-baseline`.
# Other token counts have no capture, so their `traffic` is reported as null.
STREAM_TRAFFIC_BYTES_T64 = 764_299_520 + 7_048_192


def load_peaks():
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def measure_fp8_peak(seconds=2.0):
    """Dense FP8 tensor throughput of this GPU, measured live with the vendor
    library: torch._scaled_mm (cuBLASLt) e4m3 x e4m3 -> bf16 at 8192^3, per-tensor
    scales. Returns (burst TFLOP/s: best of 10 timed calls, sustained TFLOP/s:
    back-to-back calls for `seconds`)."""
    n = 8192
    a = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
    one = torch.ones((), device="cuda")
    mm = lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    for _ in range(5):
        mm()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        mm()
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    flop = 2.0 * n ** 3
    reps = max(10, int(seconds * 1e3 / best))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        mm()
    e1.record()
    e1.synchronize()
    sustained = flop * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
    del a, b
    torch.cuda.empty_cache()
    return flop / (best * 1e-3) / 1e12, sustained


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    ~2 ms while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.samples = []        # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self._stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, rs))
                    except Exception:
                        pass
                    time.sleep(0.002)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        sm = [s[0] for s in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


class Op:
    """One configured operator call through the C ABI, plus stage-wise timing."""

    def __init__(self, pkg, x):
        import ctypes
        self.pkg, self.x, self.ctypes = pkg, x, ctypes
        self.T = x.T
        self.E = int(x.gemm1_weights.shape[0])
        self.out = torch.empty(self.T, H, dtype=torch.bfloat16, device="cuda")
        self.ws = pkg.workspace(self.T, self.E, torch.device("cuda", torch.cuda.current_device()))
        p = pkg._ptr
        self.args = pkg.MoeFp8Args(p(x.routing_logits), p(x.routing_bias), p(x.hidden_states),
                                   p(x.hidden_states_scale), p(x.gemm1_weights), p(x.gemm1_weights_scale),
                                   p(x.gemm2_weights), p(x.gemm2_weights_scale), x.local_expert_offset,
                                   x.routed_scaling_factor, p(self.out), self.T, self.E, p(self.ws),
                                   self.ws.numel())
        self.lib = pkg.load_library()

    def __call__(self):
        rc = self.lib.moe_fp8_block_scale_run(self.ctypes.byref(self.args), self.pkg._stream_handle(None))
        assert rc == 0, self.lib.moe_fp8_last_error()

    def stage(self, s):
        rc = self.lib.moe_fp8_run_stage(self.ctypes.byref(self.args), s, self.pkg._stream_handle(None))
        assert rc == 0, self.lib.moe_fp8_last_error()

    def routing_stats(self):
        _, _, counts = self.pkg.workspace_tensors(self.ws, self.T, self.E)
        c = counts.cpu().numpy()
        return int(c.sum()), int((c > 0).sum())


def timed(fn, n, flush):
    """Per-call device times (ms) with CUDA events; L2 flushed outside each timed interval."""
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for a, b in evs:
        flush.add_(1)
        a.record(st)
        fn()
        b.record(st)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def algorithmic_bytes(T, pairs, hit):
    return hit * (W13_BYTES + W2_BYTES) + T * TOKEN_IO_BYTES + 512


def gemm1_bytes(pairs, hit):
    # W13 tiles of the hit experts + gathered activation rows/scales + two-term FP8 intermediate out
    return hit * W13_BYTES + pairs * (H + 56 * 4) + pairs * 2 * (I + 16 * 4)


def gemm2_bytes(pairs, hit):
    # W2 tiles of the hit experts + two-term intermediate rows/scales in + fp32 accumulator adds
    return hit * W2_BYTES + pairs * 2 * (I + 16 * 4) + pairs * H * 4 * 2


def pinned_staging(tensors, align=256):
    """One pinned host byte buffer holding `tensors` (each at a 256-byte aligned
    offset), its device twin, and device views shaped like the tensors."""
    offs, n = [], 0
    for t in tensors:
        n = (n + align - 1) // align * align
        offs.append(n)
        n += t.numel() * t.element_size()
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    for t, o in zip(tensors, offs):
        b = t.detach().contiguous().cpu().view(torch.uint8).reshape(-1)
        host[o:o + b.numel()].copy_(b)
    dev = torch.empty(n, dtype=torch.uint8, device="cuda")
    views = [dev[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(tensors, offs)]
    return host, dev, views


def cpu_reference_time(O, x, dequant_all=True):
    """Seconds for one call of the CPU reference path: the numpy restatement of
    the definition's PyTorch reference, dequantising every local expert first as
    the reference does, with BLAS on all host cores."""
    xc = x.to("cpu")
    t0 = time.perf_counter()
    O.moe_forward(*xc.args(), dequant_all=dequant_all)
    return time.perf_counter() - t0


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else os.cpu_count()
    except Exception:
        return os.cpu_count()


def run_reference_arm(a, world, rank):
    """CPU reference path on the host cores, on this arm's workload.

    N=1: the T-token decode call (32 local experts) through the numpy
    restatement of the definition's PyTorch reference, which dequantises all
    local experts first as the reference does; every step is one full call.
    BASELINE config 0 (T=16) is timed once alongside and reported in `config0`.
    N>1: the expert-parallel job (N x 8192 tokens over 256 experts) needs tens of
    fp32 TFLOP per step on the CPU; it is not timed, and no scaled estimate is
    reported (an `unavailable` line)."""
    if rank != 0:
        return
    if world > 1:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"CPU reference of the {world} x {a.ep_tokens}-token expert-parallel step is not timed: "
                          f"~{world * a.ep_tokens * 8 * FLOPS_PER_PAIR / 1e12:.0f} fp32 TFLOP per step on the host "
                          "cores takes minutes, and no scaled estimate is reported"}), flush=True)
        return
    pkg = ge.load_package()
    O = ge.load_oracle()
    x = pkg.inputs.make_inputs(a.tokens, seed=0, num_local_experts=32)
    workload = f"decode T={a.tokens} tokens per GPU, E_local=32, local_expert_offset=0"
    times = []
    for i in range(a.warmup + a.steps):
        dt = cpu_reference_time(O, x)
        if i >= a.warmup:
            times.append(dt)
    us = statistics.median(times) * 1e6
    x0 = pkg.inputs.make_inputs(16, seed=0)
    t0 = statistics.median([cpu_reference_time(O, x0) for _ in range(3)]) * 1e6
    cores = blas_threads()
    line = {"metric": "fused_moe_us_per_call", "value": us, "unit": "us", "n_gpus": world, "steps": len(times),
            "warmup": a.warmup, "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, benchmark distributions)",
            "impl": "reference",
            "config": {"workload": workload, "parallelism": "cpu"},
            "config0": {"workload": "BASELINE config 0: T=16, 32 local experts, seed 0", "us_per_call": t0,
                        "calls": 3},
            "cpu_baseline": {"value": us, "unit": "us", "cores": cores, "kind": "port",
                             "sample": f"one full operator call per step at T={a.tokens} (numpy restatement of the "
                                       "definition's PyTorch reference; all 32 local experts dequantised to fp32 "
                                       "first, as the reference does)"},
            "e2e": {"value": us, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ep_bench(a, world, rank):
    """expert parallel over `world` GPUs, 256/world experts per
    rank, `--ep-tokens` tokens per rank, peer-memory dispatch and combine
    (ep.PeerExpertParallel: CUDA IPC buffers over NVLink, device-side flags, no
    host synchronisation inside a step)."""
    import torch.distributed as dist
    pkg = ge.load_package()
    import fused_moe_b200.ep as ep
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    T = a.ep_tokens
    epr = 256 // world
    full = pkg.inputs.make_inputs(8, seed=0, device="cuda", num_local_experts=256)   # every expert distinct
    sl = slice(rank * epr, (rank + 1) * epr)
    shard = tuple(t[sl].contiguous() for t in (full.gemm1_weights, full.gemm1_weights_scale, full.gemm2_weights,
                                                full.gemm2_weights_scale))
    bias = full.routing_bias
    x = pkg.inputs.make_inputs(T, seed=100 + rank, device="cuda", num_local_experts=1)
    peer = ep.PeerExpertParallel(rank, world, T)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    marks = []

    def step():
        return peer.forward(x.routing_logits, bias, x.hidden_states, x.hidden_states_scale, *shard, 2.5,
                            output=out, marks=marks)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    assert peer.read_error() == 0
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    marks.clear()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        per = timed(step, a.steps, flush)
    barrier(world)
    torch.cuda.synchronize()
    ms = max_over_ranks(sum(per), world) / a.steps
    # per-phase device times of this rank (median over the timed steps)
    names = ("route+dispatch", "wait dispatch", "local experts (routed operator)", "return", "wait return+combine")
    k = len(names) + 1
    phases = {n: statistics.median([marks[i * k + j].elapsed_time(marks[i * k + j + 1]) * 1e3
                                    for i in range(a.steps)]) for j, n in enumerate(names)}
    pairs = peer.K.pairs(peer)
    info = [None] * world
    dist.all_gather_object(info, {"pairs": pairs, "phases_us": phases})
    # end to end: this rank's inputs from pinned host memory, its output back
    pin = lambda t: t.cpu().pin_memory()
    h_in = [pin(t) for t in (x.routing_logits, x.hidden_states, x.hidden_states_scale)]
    d_in = [torch.empty_like(t, device="cuda") for t in h_in]
    h_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        for d, h in zip(d_in, h_in):
            d.copy_(h, non_blocking=True)
        o = peer.forward(d_in[0], bias, d_in[1], d_in[2], *shard, 2.5, output=out)
        h_out.copy_(o, non_blocking=True)

    e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(sum(timed(e2e_step, a.steps, flush)), world) / a.steps
    # parity outside the timed region: sampled tokens of this rank against the CPU oracle over all 256 experts
    O = ge.load_oracle()
    out_chk = step().clone()
    torch.cuda.synchronize()
    rows = np.unique(np.random.default_rng(rank).choice(T, 6, replace=False))
    r = torch.from_numpy(rows).cuda()
    ref = O.moe_forward(x.routing_logits[r], bias, x.hidden_states[r], x.hidden_states_scale[:, r].contiguous(),
                        full.gemm1_weights, full.gemm1_weights_scale, full.gemm2_weights, full.gemm2_weights_scale,
                        0, 2.5)
    got = out_chk[r].float().cpu().numpy()
    err = np.abs(got - ref)
    bad = int((~(err <= 1e-2 + 2e-2 * np.abs(ref))).sum())
    par = [None] * world
    dist.all_gather_object(par, (float(err.max()), bad, int(rows.size), peer.read_error()))
    fp8_burst, fp8_sustained = measure_fp8_peak()
    peer.close()
    pr = [i["pairs"] for i in info]
    tot_pairs = sum(pr)
    per_gpu_tflops = tot_pairs / world * FLOPS_PER_PAIR / (ms * 1e-3) / 1e12
    t_bound = max(pr) * FLOPS_PER_PAIR / (fp8_sustained * 1e12)          # busiest rank's MMA work at peak
    line = {
        "metric": "fused_moe_us_per_call", "value": ms * 1e3, "unit": "us", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8_e4m3 (fp32 accumulate)",
        "data": "synthetic (seeded, benchmark distributions; random-init weights, 256 distinct experts)",
        "config": {"workload": f"expert parallel: {T} tokens per GPU, 256 experts ({epr} per GPU, "
                               f"local_expert_offset = {epr}*rank), peer-memory dispatch and combine over NVLink",
                   "tokens_per_rank": T, "experts_per_rank": epr, "parallelism": f"ep{world}",
                   "transport": "CUDA IPC peer stores + device flags (no host sync, no collective on the data path)",
                   "l2": "flushed (256 MB write) between timed calls"},
        "tflops_per_gpu": per_gpu_tflops,
        "tflops_total": per_gpu_tflops * world,
        "pairs_per_rank": {"min": min(pr), "max": max(pr), "mean": tot_pairs / world, "all": pr},
        "phases_us": {"rank0": info[0]["phases_us"],
                      "max_over_ranks": {n: max(i["phases_us"][n] for i in info) for n in names}},
        "roofline": {"kernel": "whole expert-parallel step, per GPU (busiest rank's local (token, expert) pairs at "
                               "the sustained FP8 peak)",
                     "bound": "tensor", "achieved": per_gpu_tflops, "peak": fp8_sustained, "unit": "TFLOP/s",
                     "frac": t_bound / (ms * 1e-3), "frac_mean_rank": per_gpu_tflops / fp8_sustained,
                     "peak_kind": "measured in this run: torch._scaled_mm e4m3 8192^3, 2 s loop",
                     "traffic": None},
        "parity": {"vs": "CPU oracle over all 256 experts (fp32 sum, rounded once)",
                   "sampled_tokens_per_rank": par[0][2], "max_abs_err": max(p[0] for p in par),
                   "elements_outside_tolerance": sum(p[1] for p in par), "device_errors": sum(p[3] for p in par),
                   "tolerance": "atol 1e-2 + rtol 2e-2"},
        "e2e": {"value": e2e_ms * 1e3, "unit": "us",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in h_in),
                "d2h_bytes_per_step": h_out.numel() * h_out.element_size()},
        "gpu_launches": a.steps * 10,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


GEMM1_FLOPS_PER_PAIR = 2 * H * 2 * I
GEMM2_FLOPS_PER_PAIR = 2 * I * H


def sweep_point(pkg, T, skewed, seed, flush, hbm_peak, n=5, warm=3, E=32):
    """One operator call configuration: whole-call time, per-GEMM stage-alone
    times, and each against its roofline t_bound = max(bytes / HBM peak,
    useful FLOPs / FP8 peak) (frac = t_bound / t)."""
    x = pkg.inputs.make_inputs(T, seed=seed, device="cuda", skewed=skewed, num_local_experts=E)
    op = Op(pkg, x)
    for _ in range(warm):
        op()
    t = statistics.median(timed(op, n, flush))
    pairs, hit = op.routing_stats()
    path = pkg.gemm_path(T)
    g1 = statistics.median(timed(lambda: op.stage(2), n, flush))
    g2 = statistics.median(timed(lambda: op.stage(3), n, flush)) if path != 2 else 0.0
    b = algorithmic_bytes(T, pairs, hit)
    fl = pairs * FLOPS_PER_PAIR
    def roof(bytes_, flops, ms):
        return {"us": ms * 1e3, "bytes": bytes_, "useful_flops": flops, "tflops": flops / (ms * 1e-3) / 1e12}

    res = {"T": T, "skewed": skewed, "local_experts": E, "us_per_call": t * 1e3, "pairs": pairs, "hit_experts": hit,
           "tflops": fl / (t * 1e-3) / 1e12, "hbm_gbs": b / (t * 1e-3) / 1e9,
           "hbm_frac_of_measured": b / (t * 1e-3) / 1e9 / hbm_peak,
           "roofline_call": roof(b, fl, t)}
    if path == 2:
        res["fused_stream_kernel"] = roof(gemm1_bytes(pairs, hit) + gemm2_bytes(pairs, hit), fl, g1)
    else:
        res["gemm1_kernel"] = roof(gemm1_bytes(pairs, hit), pairs * GEMM1_FLOPS_PER_PAIR, g1)
        res["gemm2_kernel"] = roof(gemm2_bytes(pairs, hit), pairs * GEMM2_FLOPS_PER_PAIR, g2)
        res["gemm2_kernel"]["mma_flops"] = 2 * pairs * GEMM2_FLOPS_PER_PAIR   # hi + lo terms of the intermediate
    del op, x
    torch.cuda.empty_cache()
    return res


def add_rooflines(point, hbm_peak, fp8_peak):
    """Fill in each kernel entry of a sweep point: t_bound = max(bytes / HBM peak,
    useful FLOPs / FP8 peak), frac = t_bound / t, and the tensor fraction."""
    hbm, fp8 = hbm_peak * 1e9, fp8_peak * 1e12
    for k, v in point.items():
        if isinstance(v, dict) and "useful_flops" in v:
            tb = max(v["bytes"] / hbm, v["useful_flops"] / fp8)
            t = v["us"] * 1e-6
            v.update({"t_bound_us": tb * 1e6, "bound": "hbm" if v["bytes"] / hbm >= v["useful_flops"] / fp8 else "tensor",
                      "frac": tb / t, "tensor_frac_of_fp8_peak": v["useful_flops"] / t / fp8})
    return point


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--skewed", action="store_true", help="BASELINE config 3 routing bias (+3 on 4 local experts)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-tokens", type=int, default=8192, help="tokens per rank in the multi-GPU (EP) run")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)
    world, rank, local = dist_setup() if a.impl == "ours" else (int(os.environ.get("WORLD_SIZE", "1")),
                                                                 int(os.environ.get("RANK", "0")), 0)
    if a.impl == "reference":
        run_reference_arm(a, world, rank)
        return

    if world > 1:
        run_ep_bench(a, world, rank)
        import torch.distributed as dist
        dist.destroy_process_group()
        return

    pkg = ge.load_package()
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    T = a.tokens
    x = pkg.inputs.make_inputs(T, seed=rank, device="cuda", skewed=a.skewed)
    op = Op(pkg, x)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    for _ in range(a.warmup):
        op()
    torch.cuda.synchronize()
    assert pkg.read_device_error() == 0

    # ---- timed region: K calls, inputs resident, L2 flushed between calls
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        per_call = timed(op, a.steps, flush)
    barrier(world)
    torch.cuda.synchronize()
    total_ms = max_over_ranks(sum(per_call), world)
    ms_per_step = total_ms / a.steps
    pairs, hit = op.routing_stats()

    # ---- dominant kernel timed alone on the same stream: the fused weight-streaming
    # GEMM1+GEMM2 launch (decode sizes) or GEMM1 (larger calls)
    path = pkg.gemm_path(T)
    g1 = timed(lambda: op.stage(2), a.steps, flush)
    g1_ms = statistics.median(g1)
    if path == 2:
        kname = "stream_gemm_kernel (GEMM1+SwiGLU+GEMM2+combine, one launch)"
        g1_bytes = gemm1_bytes(pairs, hit) + gemm2_bytes(pairs, hit)
    else:
        kname = ("stream_gemm_kernel" if path in (1, 3) else "grouped_gemm_kernel<1>") + " (GEMM1+SwiGLU)"
        g1_bytes = gemm1_bytes(pairs, hit)
    g1_achieved = g1_bytes / (g1_ms * 1e-3) / 1e9

    # ---- end to end through the public run(...) with host buffers: the step's
    # inputs (logits, bias, FP8 hidden rows, scales) are staged in one pinned
    # host buffer and moved with one host->device copy, as a serving loop would;
    # run(...) gets device views into that buffer (each 256-byte aligned)
    h_in, d_in_buf, d_in = pinned_staging((x.routing_logits, x.routing_bias, x.hidden_states,
                                           x.hidden_states_scale))
    h_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    d_out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def e2e_step():
        d_in_buf.copy_(h_in, non_blocking=True)
        pkg.run(d_in[0], d_in[1], d_in[2], d_in[3], x.gemm1_weights, x.gemm1_weights_scale, x.gemm2_weights,
                x.gemm2_weights_scale, x.local_expert_offset, x.routed_scaling_factor, output=d_out)
        h_out.copy_(d_out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_times = timed(e2e_step, a.steps, flush)
    e2e_ms = max_over_ranks(sum(e2e_times), world) / a.steps
    h2d = h_in.numel()
    d2h = h_out.numel() * h_out.element_size()

    line = {
        "metric": "fused_moe_us_per_call", "value": ms_per_step * 1e3, "unit": "us", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_per_step, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp8_e4m3 (fp32 accumulate)",
        "data": "synthetic (seeded, benchmark distributions; random-init weights)",
        "config": {"workload": f"{'decode' if pkg.gemm_path(T) == 2 else 'prefill'} T={T} tokens per GPU, "
                               f"E_local=32, local_expert_offset=0{', skewed bias' if a.skewed else ''}",
                   "tokens": T, "local_experts": 32, "pairs": pairs, "hit_experts": hit,
                   "parallelism": "replicas" if world > 1 else "single",
                   "l2": "flushed (256 MB write) between timed calls; weights also exceed L2"},
        "tflops": pairs * FLOPS_PER_PAIR / (ms_per_step * 1e-3) / 1e12,
        "hbm_gbs_whole_call": algorithmic_bytes(T, pairs, hit) / (ms_per_step * 1e-3) / 1e9,
        "roofline": {"kernel": kname, "bound": "hbm",
                     "achieved": g1_achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": g1_achieved / hbm_peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": g1_bytes, "launch_us": g1_ms * 1e3,
                     "traffic": STREAM_TRAFFIC_BYTES_T64 if (T == 64 and path == 2) else None},

        "e2e": {"value": e2e_ms * 1e3, "unit": "us", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": a.steps * int(pkg.load_library().moe_fp8_kernels_per_call(T)),
        "clocks": clk.summary(),
    }
    del op
    if rank == 0 and world == 1 and not a.no_sweep:
        sw = []
        # decode points, BASELINE configs 2 and 3, and the expert-parallel workload of one
        # rank run on a single GPU holding all 256 experts (the like-for-like base of the EP lines);
        # prefill points use the FP8 burst peak (each kernel is timed alone, milliseconds long)
        for (tt, sk, e) in ((1, False, 32), (8, False, 32), (32, False, 32), (4096, False, 32), (16384, True, 32),
                            (8192, False, 256)):
            sw.append(sweep_point(pkg, tt, sk, 0 if e == 32 else 100, flush, hbm_peak, E=e))
        line["sweep"] = sw
    # the FP8 peak is measured after every timed region: its seconds of dense GEMM
    # leave the power limiter engaged for a while
    fp8_burst, fp8_sustained = measure_fp8_peak()
    line["peaks"] = {"hbm_gbs": hbm_peak, "hbm_kind": peak_kind, "fp8_tflops_burst": fp8_burst,
                     "fp8_tflops_sustained": fp8_sustained,
                     "fp8_how": "measured in this run after the timed regions: torch._scaled_mm e4m3 8192^3 "
                                "(cuBLASLt), best of 10 / 2 s loop"}
    for p in line.get("sweep", []):
        add_rooflines(p, hbm_peak, fp8_burst)
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        O = ge.load_oracle()
        dt = cpu_reference_time(O, x)
        line["cpu_baseline"] = {"value": dt * 1e6, "unit": "us", "cores": blas_threads(), "kind": "port",
                                "sample": f"one full operator call at T={T} (numpy restatement of the "
                                          "definition's PyTorch reference, all local experts dequantised first)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
