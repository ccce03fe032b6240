"""Build the C routing oracle (test infrastructure) into oracle/_build/.

    python oracle/build_oracle.py

`routing(logits, bias, scale)` loads it through ctypes. The reference has no
C/C++ code for this path that compiles on its own (its CUDA solution needs a
GPU and TVM-FFI; the operator's ground truth is the definition's PyTorch
`reference`), so there is no `oracle/_ref` build: the restatements here are
pinned against golden vectors produced by running that PyTorch reference.
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "routing_oracle.c"
LIB = HERE / "_build" / "librouting_oracle.so"


def build(force: bool = False) -> pathlib.Path:
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    subprocess.run(["gcc", "-O2", "-fno-fast-math", "-ffp-contract=off", "-shared", "-fPIC", str(SRC),
                    "-o", str(LIB), "-lm"], check=True)
    return LIB


_lib = None


def routing(logits: np.ndarray, bias: np.ndarray | None, scale: float):
    """(topk_idx int32 [T, 8], weights f32 [T, 8]) in selection order."""
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
    x = np.ascontiguousarray(logits, dtype=np.float32)
    T = x.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    idx = np.zeros((T, 8), np.int32)
    w = np.zeros((T, 8), np.float32)
    P = ctypes.c_void_p
    _lib.route_tokens.argtypes = [P, P, ctypes.c_int, ctypes.c_float, P, P]
    _lib.route_tokens(x.ctypes.data, None if b is None else b.ctypes.data, T, float(scale),
                      idx.ctypes.data, w.ctypes.data)
    return idx, w


if __name__ == "__main__":
    print(build(force=True))
