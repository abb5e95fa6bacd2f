"""Packs the operators as flashinfer-bench Solution JSON files.

    python -m karnbirkhera-mlsys2026-dsa_sparse_attention_b200.fib.pack [-o DIR] [--which attention|indexer|both]

Replaces the reference's scripts/pack_solution.py (which packs solution/cuda/
as a CUDA solution with the torch binding, config.toml:1-10).  A Solution here
has the layout of the reference's solution.json (name, definition, author,
spec{language, target_hardware, entry_point, dependencies,
destination_passing_style}, sources[{path, content}], description), with
language "python": kernel.py (solution_kernel.py) compiles the packed CUDA
sources for sm_100a itself, since the harness's CUDA builders take no compile
flags.  The sources are packed flat (the CUDA files include the C-ABI header
by name).  `unpack` writes a Solution's sources into a directory, the way the
harness extracts it.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tomllib

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(HERE)
REPO_DIR = os.path.dirname(PKG_DIR)
CONFIG = os.path.join(HERE, "config.toml")

# packed path -> file in this repository
FILES = {
    "kernel.py": os.path.join(HERE, "solution_kernel.py"),
    "dsa_capi.cu": os.path.join(PKG_DIR, "csrc", "dsa_capi.cu"),
    "dsa_split_sm100.cu": os.path.join(PKG_DIR, "csrc", "dsa_split_sm100.cu"),
    "dsa_noalloc.cu": os.path.join(PKG_DIR, "csrc", "dsa_noalloc.cu"),
    "dsa_indexer_sm100.cu": os.path.join(PKG_DIR, "csrc", "dsa_indexer_sm100.cu"),
    "dsa_common.cuh": os.path.join(PKG_DIR, "csrc", "dsa_common.cuh"),
    "dsa_sm100_ptx.cuh": os.path.join(PKG_DIR, "csrc", "dsa_sm100_ptx.cuh"),
    "dsa_sparse_attention.h": os.path.join(REPO_DIR, "include", "dsa_sparse_attention.h"),
}
OPERATORS = ("attention", "indexer")


def load_config() -> dict:
    with open(CONFIG, "rb") as f:
        return tomllib.load(f)


def solution(which: str) -> dict:
    """The Solution JSON object for one operator ("attention" or "indexer")."""
    if which not in OPERATORS:
        raise ValueError(f"unknown operator {which!r}; expected one of {OPERATORS}")
    cfg = load_config()
    op = cfg[which]
    sources = []
    for path, src in FILES.items():
        with open(src, encoding="utf-8") as f:
            sources.append({"path": path, "content": f.read()})
    return {
        "name": op["name"],
        "definition": op["definition"],
        "author": cfg["author"],
        "spec": {
            "language": "python",
            "target_hardware": ["NVIDIA_B200"],
            "entry_point": op["entry_point"],
            "dependencies": [],
            "destination_passing_style": bool(op.get("destination_passing_style", True)),
        },
        "sources": sources,
        "description": ("B200 (sm_100a) tcgen05 kernels behind a C ABI; kernel.py compiles the packed CUDA "
                        "sources with nvcc on first use and calls them through ctypes."),
    }


def write(which: str, out_dir: str) -> str:
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, f"{which}_solution.json")
    with open(path, "w", encoding="utf-8") as f:
        json.dump(solution(which), f, indent=2)
    return path


def unpack(sol: dict, dest_dir: str) -> list[str]:
    """Write a Solution's sources into dest_dir; returns the written paths."""
    out = []
    for s in sol["sources"]:
        rel = os.path.normpath(s["path"])
        if rel.startswith("..") or os.path.isabs(rel):
            raise ValueError(f"source path escapes the solution directory: {s['path']}")
        p = os.path.join(dest_dir, rel)
        os.makedirs(os.path.dirname(p) or dest_dir, exist_ok=True)
        with open(p, "w", encoding="utf-8") as f:
            f.write(s["content"])
        out.append(p)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--out", default=".", help="output directory")
    ap.add_argument("--which", choices=OPERATORS + ("both",), default="both")
    args = ap.parse_args(argv)
    for which in (OPERATORS if args.which == "both" else (args.which,)):
        print(write(which, args.out))


if __name__ == "__main__":
    sys.exit(main())
