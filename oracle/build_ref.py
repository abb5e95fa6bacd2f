"""Recipe: compile the reference's own naive kernel for CPU into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The product never imports, links or runs anything
under oracle/.

What it builds
    oracle/_ref/dsa_ref_naive.so — a Python extension module compiled straight
    from the reference source where it lies
    (methodology/checkpoints/kernel_naive.cu, 77 lines of ATen calls that the
    reference records as matching the contest's Python reference with zero error
    on all 23 workloads).  `g++ -x c++` compiles the .cu file as C++; the only
    addition is the force-included oracle/ref_cpu_shim.h, which turns the
    file's CUDAGuard (kernel_naive.cu:31) into a no-op so the ATen calls run on
    CPU tensors.  No reference source is copied into this repository.

The built module exposes the reference's DPS entry point
    dsa_ref_naive.launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache,
                                            sparse_indices, sm_scale, output, lse)
and is used (a) to pin oracle/dsa_oracle.py, (b) to make the golden fixtures in
tests/golden/, and (c) as the timed CPU reference arm of bench.py.

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
NAIVE_SRC = os.path.join(REF_ROOT, "methodology", "checkpoints", "kernel_naive.cu")
MODULE = "dsa_ref_naive"


def ref_module_path() -> str:
    return os.path.join(OUT_DIR, MODULE + ".so")


def build_ref(force: bool = False, verbose: bool = False) -> str | None:
    """Compile kernel_naive.cu for CPU.  Returns the .so path, or None when the
    reference tree is absent (GPU box) and no prebuilt module exists."""
    out = ref_module_path()
    if not os.path.exists(NAIVE_SRC):
        return out if os.path.exists(out) else None
    if (not force and os.path.exists(out)
            and os.path.getmtime(out) >= os.path.getmtime(NAIVE_SRC)
            and os.path.getmtime(out) >= os.path.getmtime(os.path.join(HERE, "ref_cpu_shim.h"))):
        return out
    import torch.utils.cpp_extension as ce  # noqa: WPS433 (heavy import kept local)

    os.makedirs(OUT_DIR, exist_ok=True)
    inc = ce.include_paths() + [sysconfig.get_paths()["include"], "/usr/local/cuda/include"]
    libdirs = ce.library_paths()
    import torch
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-x", "c++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-include", os.path.join(HERE, "ref_cpu_shim.h")]
    cmd += [f"-I{p}" for p in inc]
    cmd += [NAIVE_SRC, "-o", out]
    cmd += [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def load_ref():
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
    p = build_ref(force="--force" in sys.argv, verbose=True)
    print(p)
