"""Generate golden vectors by running the reference operator itself.

Runs only where the reference checkout is present (the build container):
    python tests/golden/make_golden.py --ref-root DIR [--only name,name]

It execs the `reference` source of the operator definition
(`resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146`)
unmodified on CPU, on seeded inputs (`inputs.make_inputs` / `cases.routing_case`),
and records

* the bf16 output (as raw int16) of whole-operator cases, and
* the routing result (`topk_idx`, per-token combine weights) read from the
  reference function's own local variables when it returns (or, for the
  routing-only cases, the moment its routing step is complete),

together with checksums of the inputs so the tests can tell if the input
generator ever drifts. Outputs land in this directory as .npz files.
"""
from __future__ import annotations

import argparse
import gc
import hashlib
import inspect
import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "starter-kit-fused-moe_b200"))
sys.path.insert(0, str(HERE))
import inputs as gen  # noqa: E402
from cases import FULL_CASES, ROUTING_CASES, routing_case  # noqa: E402

DEF_JSON = "resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json"
KEEP = ("topk_idx", "weights")


class _StopAfterRouting(Exception):
    pass


def load_reference(ref_root: pathlib.Path):
    src = json.loads((ref_root / DEF_JSON).read_text())["reference"]
    ns: dict = {}
    exec(compile(src, "<definition reference>", "exec"), ns)
    return ns["run"]


def run_traced(fn, args, stop_after_routing=False):
    """Run fn(*args); capture `topk_idx` and `weights` from its frame."""
    captured = {}
    code = inspect.unwrap(fn).__code__

    def local_tracer(frame, event, arg):
        if event == "return" or (stop_after_routing and event == "line" and "output" in frame.f_locals):
            loc = frame.f_locals
            captured.update({k: loc[k].clone() for k in KEEP if k in loc})
            if event == "line":
                raise _StopAfterRouting()
        return local_tracer

    def global_tracer(frame, event, arg):
        return local_tracer if frame.f_code is code else None

    sys.settrace(global_tracer)
    try:
        result = fn(*args)
    except _StopAfterRouting:
        result = None
    finally:
        sys.settrace(None)
    return result, captured


def checksum(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()[:16]


def routing_arrays(loc):
    topk = loc["topk_idx"].to(torch.int64)
    w = torch.gather(loc["weights"], 1, topk)
    # canonical order: ascending expert id (selection sets are what is compared)
    idx_sorted, perm = torch.sort(topk, dim=1)
    return idx_sorted.to(torch.int16).numpy(), torch.gather(w, 1, perm).numpy().astype(np.float32)


def input_checksums(x):
    return {k: checksum(getattr(x, k)) for k in
            ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
             "gemm1_weights_scale", "gemm2_weights_scale")}


def make_full_case(ref, name, T, seed, skewed=False):
    x = gen.make_inputs(T, seed=seed, skewed=skewed)
    out, loc = run_traced(ref, list(x.args()))
    idx, w = routing_arrays(loc)
    np.savez_compressed(
        HERE / f"{name}.npz",
        output_bf16=out.view(torch.int16).numpy(), topk_idx=idx, topk_weights=w,
        meta=json.dumps(dict(T=T, seed=seed, skewed=skewed, local_expert_offset=0,
                             routed_scaling_factor=x.routed_scaling_factor,
                             checksums=input_checksums(x))))
    print(name, "done", tuple(out.shape))
    del x, out, loc
    gc.collect()


def make_routing_case(ref, name, logits, bias):
    """Routing-only golden: the reference is stopped right after its routing step."""
    T = logits.shape[0]
    E = gen.E_LOCAL
    # placeholders of the right shapes: the reference asserts them, routing ignores them
    hq = torch.zeros(T, gen.H, dtype=torch.float8_e4m3fn)
    hs = torch.ones(gen.H // 128, T)
    w13 = torch.zeros(E, 2 * gen.I, gen.H, dtype=torch.float8_e4m3fn)
    s13 = torch.ones(E, 32, 56)
    w2 = torch.zeros(E, gen.H, gen.I, dtype=torch.float8_e4m3fn)
    s2 = torch.ones(E, 56, 16)
    _, loc = run_traced(ref, [logits, bias, hq, hs, w13, s13, w2, s2, 0, 2.5], stop_after_routing=True)
    idx, w = routing_arrays(loc)
    np.savez_compressed(HERE / f"{name}.npz", topk_idx=idx, topk_weights=w,
                        meta=json.dumps(dict(T=T, checksums=dict(routing_logits=checksum(logits),
                                                                 routing_bias=checksum(bias)))))
    print(name, "done", T)
    del loc
    gc.collect()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", required=True, help="checkout of the reference repository")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    ref = load_reference(pathlib.Path(a.ref_root))
    todo = a.only.split(",") if a.only else list(FULL_CASES) + list(ROUTING_CASES)
    for name in todo:
        if name in FULL_CASES:
            T, seed, skewed = FULL_CASES[name]
            make_full_case(ref, name, T, seed, skewed=skewed)
        else:
            logits, bias = routing_case(name)
            make_routing_case(ref, name, logits, bias)


if __name__ == "__main__":
    main()
