"""Build the sm_100a shared library `libmoe_b200.so` in-tree with nvcc.

    python starter-kit-fused-moe_b200/build.py [-v] [--debug]

Every .cu file under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked into one shared library
next to this file, so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libmoe_b200.so"
OBJ = HERE / "_build"


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    return LIB.exists() and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in _deps())


def build(debug: bool = False, verbose: bool = False, force: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIB
    OBJ.mkdir(exist_ok=True)
    flags = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             "-O3", "--expt-relaxed-constexpr", "-I", str(INCLUDE)]
    if debug:
        flags += ["-DMOE_DEBUG"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    srcs = sorted(CSRC.glob("*.cu"))

    def compile_one(s):
        o = OBJ / (s.stem + ".o")
        r = subprocess.run([nvcc(), *flags, "-c", str(s), "-o", str(o)], capture_output=True, text=True)
        return s, o, r

    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, srcs))
    objs = []
    for s, o, r in results:
        if verbose or r.returncode:
            sys.stderr.write(f"--- {s.name}\n{r.stdout}{r.stderr}")
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {s.name}")
        objs.append(str(o))
    tmp = LIB.with_name(LIB.name + ".tmp")
    r = subprocess.run([nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *objs,
                        "-lcudart"], capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(debug=a.debug, verbose=a.verbose, force=True))
