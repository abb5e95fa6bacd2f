"""Recipe: compile the reference's naive top-k indexer into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The product never imports, links or runs anything
under oracle/.

What it builds
    oracle/_ref/dsa_ref_topk.so — a Python extension module compiled straight
    from the reference source where it lies
    (methodology/reference/topk_kernel_naive.cu: two small CUDA kernels, a
    page dequant-gather and the index translation, around torch::matmul and
    at::topk).  nvcc compiles the .cu for sm_100a, g++ links it against
    libtorch.  No reference source is copied into this repository.

The module exposes the reference's DPS entry point
    dsa_ref_topk.launch_topk_c(q_index_fp8, k_index_cache_fp8, weights,
                               seq_lens, block_table, topk_indices)
and needs a GPU: tests/test_indexer_ref_gpu.py runs it on the GPU box to pin
oracle/dsa_indexer_oracle.py (and the library) against the reference's own
outputs.  Inputs given to it must have every block-table entry inside the pool
(the reference reads them unchecked, topk_kernel_naive.cu:37-38).

The reference tree is only present in the development container; on the GPU
box the prebuilt .so (git-ignored, carried with the working tree) is used.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
# The reference tree: DSA_REFERENCE_ROOT, else a directory named "reference"
# beside this repository's root.
REF_ROOT = os.environ.get("DSA_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
TOPK_SRC = os.path.join(REF_ROOT, "methodology", "reference", "topk_kernel_naive.cu")
MODULE = "dsa_ref_topk"


def ref_module_path() -> str:
    return os.path.join(OUT_DIR, MODULE + ".so")


def build_ref_indexer(force: bool = False, verbose: bool = False) -> str | None:
    """Compile topk_kernel_naive.cu for sm_100a.  Returns the .so path, or None
    when the reference tree is absent (GPU box) and no prebuilt module exists."""
    out = ref_module_path()
    if not os.path.exists(TOPK_SRC):
        return out if os.path.exists(out) else None
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(TOPK_SRC):
        return out
    import torch
    import torch.utils.cpp_extension as ce  # noqa: WPS433 (heavy import kept local)

    os.makedirs(OUT_DIR, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], "/usr/local/cuda/include"]
    obj = os.path.join(OUT_DIR, MODULE + ".o")
    nvcc = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
            "-DTORCH_API_INCLUDE_EXTENSION_H", "--expt-relaxed-constexpr"]
    nvcc += [f"-I{p}" for p in inc]
    nvcc += ["-c", TOPK_SRC, "-o", obj]
    libdirs = ce.library_paths(device_type="cuda") + ["/usr/local/cuda/lib64"]
    link = ["g++", "-shared", obj, "-o", out]
    link += [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    link += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    for cmd in (nvcc, link):
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    os.remove(obj)
    return out


def load_ref_indexer():
    """Import the compiled reference module, or return None if it is absent."""
    path = ref_module_path()
    if not os.path.exists(path):
        return None
    import importlib.util
    import torch  # noqa: F401  (the module links libtorch; import torch first)
    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    p = build_ref_indexer(force="--force" in sys.argv, verbose=True)
    print(p)
