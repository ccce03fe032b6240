"""Pack the operator as a FlashInfer-Bench CUDA solution (``solution.json``).

The reference submits its kernels to the FlashInfer-Bench harness as a
Solution document (``scripts/pack_solution.py:34-84``, format in
``README.md:227-279``): name, definition, author, a build spec and the source
files. This writes the same document for this package: every CUDA source and
header of the library, the C-ABI header, and the TVM-FFI binding as
``main.cpp`` whose ``run`` has the reference's destination-passing signature.
All includes are by file name, so the flat source list compiles as one
directory. The tcgen05 kernels need the harness to compile for sm_100a.

Usage: python pack_solution.py [--out solution.json] [--name NAME] [--author AUTHOR]
"""
from __future__ import annotations

import argparse
import json
import pathlib
import re

HERE = pathlib.Path(__file__).resolve().parent
DEFINITION = "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
ENTRY_FILE = "main.cpp"


def source_files() -> list[tuple[str, pathlib.Path]]:
    """(name in the solution, file) for every source the harness must compile."""
    csrc = HERE / "csrc"
    files = [(p.name, p) for p in sorted(csrc.iterdir()) if p.suffix in (".cu", ".cuh", ".h")]
    files.append(("moe_fp8.h", HERE.parent / "include" / "moe_fp8.h"))
    files.append((ENTRY_FILE, HERE / "tvm_ffi" / "moe_tvm_ffi.cc"))
    return files


def pack(name: str = "fused-moe-b200", author: str = "fused-moe-b200", definition: str = DEFINITION) -> dict:
    sources = [{"path": n, "content": p.read_text()} for n, p in source_files()]
    names = {s["path"] for s in sources}
    for s in sources:                      # the flat layout must be closed under #include "..."
        for inc in re.findall(r'#include\s+"([^"]+)"', s["content"]):
            if inc not in names:
                raise RuntimeError(f"{s['path']} includes {inc}, which is not packed")
    return {
        "name": name,
        "definition": definition,
        "author": author,
        "spec": {
            "language": "cuda",
            "target_hardware": ["cuda"],
            "entry_point": f"{ENTRY_FILE}::run",
            "dependencies": [],
            "destination_passing_style": True,
            "binding": "tvm-ffi",
        },
        "sources": sources,
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="solution.json")
    ap.add_argument("--name", default="fused-moe-b200")
    ap.add_argument("--author", default="fused-moe-b200")
    a = ap.parse_args()
    doc = pack(a.name, a.author)
    pathlib.Path(a.out).write_text(json.dumps(doc, indent=2))
    print(f"{a.out}: {len(doc['sources'])} sources, entry {doc['spec']['entry_point']}")


if __name__ == "__main__":
    main()
