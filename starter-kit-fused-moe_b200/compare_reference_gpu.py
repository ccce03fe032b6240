"""Time the reference solution's own GPU path beside this operator (one GPU).

    python starter-kit-fused-moe_b200/compare_reference_gpu.py --reference-dir DIR [--tokens 1,8,64,4096,16384s]

DIR is a directory holding the reference's `solution/triton/*.py`
(`current_kernel.py` and the CuTe-DSL helpers it imports). For each token count
(suffix `s`: the skewed bias of BASELINE config 3) both `run` entry points get
the same seeded inputs and a destination-passing output; each is timed with
CUDA events after 3 warm-up calls, L2 flushed (256 MB write) before every timed
call, median of 10, and the two outputs are compared. One JSON line per token
count. A measurement aid only: nothing in the operator imports it. The
reference's CuTe GEMM shares operand tiles across a thread-block cluster, so
run this on one GPU only, never inside a multi-GPU job.
"""
from __future__ import annotations

import argparse
import json
import pathlib
import statistics
import sys

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", required=True)
    ap.add_argument("--tokens", default="1,8,64,4096,16384s")
    a = ap.parse_args()
    root = pathlib.Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(pathlib.Path(a.reference_dir).resolve()))
    import __graft_entry__ as ge
    pkg = ge.load_package()
    import current_kernel as ck
    took = {}
    orig = ck._run_cutlass_large_path

    def wrap(*args, **kw):
        r = orig(*args, **kw)
        took["cute"] = bool(r)
        return r

    ck._run_cutlass_large_path = wrap
    flush = torch.empty(256 << 18, dtype=torch.float32, device="cuda")

    def timeit(fn, n=10, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(n):
            flush.add_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    for tok in a.tokens.split(","):
        skewed = tok.endswith("s")
        T = int(tok.rstrip("s"))
        x = pkg.inputs.make_inputs(T, seed=0, device="cuda", skewed=skewed)
        out_o = torch.empty(T, 7168, dtype=torch.bfloat16, device="cuda")
        out_r = torch.empty_like(out_o)
        r = {"T": T, "skewed": skewed, "ours_us": timeit(lambda: pkg.run(*x.args(), output=out_o))}
        took.clear()
        ck.run(*x.args(), output=out_r)
        torch.cuda.synchronize()
        r["ref_path"] = "cute_k13" if took.get("cute") else "triton"
        r["ref_us"] = timeit(lambda: ck.run(*x.args(), output=out_r))
        d = (out_o.float() - out_r.float()).abs()
        r["max_abs_diff"] = d.max().item()
        r["frac_outside_atol1e-2_rtol2e-2"] = (~(d <= 1e-2 + 2e-2 * out_o.float().abs())).float().mean().item()
        print(json.dumps(r), flush=True)
        del x
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
