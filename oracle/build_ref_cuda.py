"""Recipe: compile the reference's own optimised CUDA kernel into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The product never imports, links or runs anything
under oracle/.

What it builds
    oracle/_ref/dsa_ref_cuda.so — a Python extension module compiled straight
    from the reference's shipped solution where it lies
    (solution/cuda/kernel.cu: the split-KV kernel with its fused last-arrival
    reduce and the pybind export of launch_sparse_attention_c).  nvcc compiles
    the .cu for sm_100a, g++ links it against libtorch.  No reference source is
    copied into this repository.

The module exposes the reference's DPS entry point
    dsa_ref_cuda.launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache,
                                           sparse_indices, sm_scale, output, lse)
and needs a GPU.  It is the same-box comparison for the operator:
tests/test_ref_cuda_gpu.py checks it against a CPU restatement of its
algorithm and against the operator's oracle, and bench.py's reference arm
times it (key `ref_cuda`).  What it accepts:
  * num_tokens <= 8 only — its split plan needs kv_per_split <= 128
    (solution/cuda/kernel.cu:634-641, :688-691) and rejects larger batches;
  * every index in [-1, num_pages * 64): its copies read the row of any index
    >= 0 unchecked (kernel.cu:146-151), and its barrier waits spin without a
    bound (kernel.cu:105-116), so only valid inputs are ever given to it.
Its scratch and counters are process-global and sized for one device
(kernel.cu:643-671): use it on one device per process.

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
KERNEL_SRC = os.path.join(REF_ROOT, "solution", "cuda", "kernel.cu")
MODULE = "dsa_ref_cuda"
MAX_TOKENS = 8


def ref_module_path() -> str:
    return os.path.join(OUT_DIR, MODULE + ".so")


def build_ref_cuda(force: bool = False, verbose: bool = False) -> str | None:
    """Compile solution/cuda/kernel.cu for sm_100a.  Returns the .so path, or
    None when the reference tree is absent (GPU box) and no prebuilt module
    exists."""
    out = ref_module_path()
    if not os.path.exists(KERNEL_SRC):
        return out if os.path.exists(out) else None
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(KERNEL_SRC):
        return out
    import torch
    import torch.utils.cpp_extension as ce  # noqa: WPS433 (heavy import kept local)

    os.makedirs(OUT_DIR, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], "/usr/local/cuda/include"]
    obj = os.path.join(OUT_DIR, MODULE + ".o")
    nvcc = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
            "-DTORCH_API_INCLUDE_EXTENSION_H", "--expt-relaxed-constexpr"]
    nvcc += [f"-I{p}" for p in inc]
    nvcc += ["-c", KERNEL_SRC, "-o", obj]
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


def load_ref_cuda():
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
    p = build_ref_cuda(force="--force" in sys.argv, verbose=True)
    print(p)
