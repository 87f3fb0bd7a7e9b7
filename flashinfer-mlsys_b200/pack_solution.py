"""Pack the library into a contest ``solution.json``, the document that the
reference's scripts/pack_solution.py:34-81 writes with flashinfer_bench's
``pack_solution_from_files`` from config.toml (config.toml:1-8):

    {"name", "definition", "author",
     "spec": {"language": "cuda", "target_hardware": ["cuda"],
              "entry_point": "kernel.cu::kernel", "dependencies": [],
              "destination_passing_style": true, "binding": "torch"},
     "sources": [{"path": ..., "content": ...}, ...]}

The spec fields follow the harness's documented solution format
(README.md:236-279: DPS on by default, binding "torch" or "tvm-ffi"); the
reference's own packer sets no binding (scripts/pack_solution.py:56-62), which
its notes say the torch extension needs (notes/cuda_changes_and_plan.md:5-18).
Sources are flat: ``kernel.cu`` (the entry of the chosen binding: this
package's solution/kernel.cu for "torch", solution/kernel_tvm_ffi.cu for
"tvm-ffi"), every .cu/.cuh/.h of csrc/ and the C-ABI header moe_fp8_ds.h.
The harness's builder compiles every .cu of the directory and must target
sm_100a only (the kernels use tcgen05 and TMA): ``-gencode
arch=compute_100a,code=sm_100a``, which for tvm_ffi's builder means
TVM_FFI_CUDA_ARCH_LIST="10.0a".

flashinfer_bench itself (third-party, not vendored by the reference) is not
needed to write or read the document.

    python -m flashinfer-mlsys_b200.pack_solution [-o solution.json] [--name N] [--author A] [--binding torch|tvm-ffi]
"""
from __future__ import annotations

import argparse
import json
import os

from . import build as _build

DEFINITION = "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
ENTRY_FILE = "kernel.cu"
HERE = os.path.dirname(os.path.abspath(__file__))
ENTRY_SOURCES = {"torch": "kernel.cu", "tvm-ffi": "kernel_tvm_ffi.cu"}


def source_files(binding: str = "torch") -> list[tuple[str, str]]:
    """(path inside the solution, file on disk), entry point first."""
    if binding not in ENTRY_SOURCES:
        raise ValueError(f"binding must be one of {sorted(ENTRY_SOURCES)}, got {binding!r}")
    files = [(ENTRY_FILE, os.path.join(HERE, "solution", ENTRY_SOURCES[binding]))]
    files += [(f, os.path.join(_build.CSRC, f)) for f in _build.SOURCES + _build.HEADERS]
    files.append(("moe_fp8_ds.h", os.path.join(_build.INCLUDE, "moe_fp8_ds.h")))
    return files


def pack(name: str = "moe-fp8-ds-b200", author: str = "flashinfer-mlsys_b200", binding: str = "torch") -> dict:
    sources = []
    for path, disk in source_files(binding):
        with open(disk, encoding="utf-8") as f:
            sources.append({"path": path, "content": f.read()})
    return {
        "name": name,
        "definition": DEFINITION,
        "author": author,
        "spec": {
            "language": "cuda",
            "target_hardware": ["cuda"],
            "entry_point": f"{ENTRY_FILE}::kernel",
            "dependencies": [],
            "destination_passing_style": True,
            "binding": binding,
        },
        "sources": sources,
    }


def extract(solution: dict, out_dir: str) -> list[str]:
    """Write the sources of a packed solution under out_dir; returns the .cu
    files (what a builder compiles). Paths must stay inside out_dir."""
    os.makedirs(out_dir, exist_ok=True)
    root = os.path.realpath(out_dir)
    cu = []
    for s in solution["sources"]:
        dst = os.path.realpath(os.path.join(root, s["path"]))
        if os.path.commonpath([root, dst]) != root:
            raise ValueError(f"source path escapes the solution directory: {s['path']}")
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        with open(dst, "w", encoding="utf-8") as f:
            f.write(s["content"])
        if dst.endswith(".cu"):
            cu.append(dst)
    return cu


def main() -> None:
    ap = argparse.ArgumentParser(description="Pack the sm_100a MoE library into a contest solution.json")
    ap.add_argument("-o", "--output", default="solution.json")
    ap.add_argument("--name", default="moe-fp8-ds-b200")
    ap.add_argument("--author", default="flashinfer-mlsys_b200")
    ap.add_argument("--binding", default="torch", choices=sorted(ENTRY_SOURCES))
    args = ap.parse_args()
    sol = pack(args.name, args.author, args.binding)
    with open(args.output, "w", encoding="utf-8") as f:
        json.dump(sol, f, indent=2)
    print(f"Solution packed: {args.output} ({len(sol['sources'])} sources, entry {sol['spec']['entry_point']})")


if __name__ == "__main__":
    main()
