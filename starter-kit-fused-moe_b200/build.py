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
# -DMOE_DEBUG build: every kernel checks its computed indices before the
# accesses they guard and records error bit 8 instead of touching memory out of
# range (compute-sanitizer is closed on the GPU pool, so this is the bounds check).
DEBUG_LIB = HERE / "libmoe_b200_debug.so"
DEBUG_OBJ = HERE / "_build_debug"


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date(lib: pathlib.Path = LIB) -> bool:
    return lib.exists() and all(lib.stat().st_mtime >= d.stat().st_mtime for d in _deps())


def build(debug: bool = False, verbose: bool = False, force: bool = False) -> pathlib.Path:
    """Build libmoe_b200.so, or with `debug` the index-checking libmoe_b200_debug.so."""
    lib_path, obj_dir = (DEBUG_LIB, DEBUG_OBJ) if debug else (LIB, OBJ)
    if not force and up_to_date(lib_path):
        return lib_path
    obj_dir.mkdir(exist_ok=True)
    flags = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             "-O3", "--expt-relaxed-constexpr", "-I", str(INCLUDE)]
    if debug:
        flags += ["-DMOE_DEBUG"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    srcs = sorted(CSRC.glob("*.cu"))

    def compile_one(s):
        o = obj_dir / (s.stem + ".o")
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
    tmp = lib_path.with_name(lib_path.name + ".tmp")
    r = subprocess.run([nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *objs,
                        "-lcudart"], capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, lib_path)
    return lib_path


TVM_SRC = HERE / "tvm_ffi" / "moe_tvm_ffi.cc"
TVM_LIB = HERE / "libmoe_b200_tvm_ffi.so"


def tvm_ffi_paths():
    """(include dir, lib dir) of the installed apache-tvm-ffi package, or None."""
    try:
        import tvm_ffi
    except ImportError:
        return None
    root = pathlib.Path(tvm_ffi.__file__).parent
    inc, lib = root / "include", root / "lib"
    return (inc, lib) if (inc / "tvm" / "ffi" / "function.h").exists() and (lib / "libtvm_ffi.so").exists() else None


def build_tvm_ffi(force: bool = False) -> pathlib.Path | None:
    """Build the TVM-FFI binding (`run`, the FlashInfer-Bench entry) over libmoe_b200.so.
    Returns None when apache-tvm-ffi is not installed."""
    paths = tvm_ffi_paths()
    if paths is None:
        return None
    lib = build()
    if not force and TVM_LIB.exists() and TVM_LIB.stat().st_mtime >= max(TVM_SRC.stat().st_mtime, lib.stat().st_mtime):
        return TVM_LIB
    inc, tlib = paths
    cuda = pathlib.Path(nvcc()).parent.parent
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-fPIC", "-shared", str(TVM_SRC), "-o", str(TVM_LIB),
           "-I", str(inc), "-I", str(INCLUDE), "-I", str(cuda / "include"),
           "-L", str(HERE), "-lmoe_b200", "-L", str(tlib), "-ltvm_ffi", "-L", str(cuda / "lib64"), "-lcudart",
           "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + str(tlib), "-Wl,-rpath," + str(cuda / "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("TVM-FFI binding build failed")
    return TVM_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(debug=a.debug, verbose=a.verbose, force=True))
    if not a.debug:
        print(build_tvm_ffi(force=True))
