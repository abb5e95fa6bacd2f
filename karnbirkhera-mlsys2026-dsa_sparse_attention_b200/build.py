"""Build recipe for libdsa_b200.so — the sm_100a kernels behind the C ABI in
include/dsa_sparse_attention.h.

One nvcc invocation per translation unit, then one link, all in-tree so the
built library travels with the working tree.  The CUDA runtime is linked
SHARED so that the library and PyTorch use the same runtime instance (one
current-device state per thread, one primary context).

    python -m <package>.build            (or __graft_entry__.build())
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_NAME = "libdsa_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["dsa_capi.cu", "dsa_split_sm100.cu", "dsa_noalloc.cu", "dsa_indexer_sm100.cu"]
HEADERS = ["dsa_common.cuh", "dsa_sm100_ptx.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-v", "-cudart", "shared"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _needs_rebuild() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    deps.append(os.path.join(REPO_DIR, "include", "dsa_sparse_attention.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link libdsa_b200.so."""
    if not force and not _needs_rebuild():
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    inc = ["-I", os.path.join(REPO_DIR, "include"), "-I", CSRC]
    objs = []
    for src in SOURCES:
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *inc, "-c", os.path.join(CSRC, src), "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or res.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cuda_lib = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "shared", "-o", tmp, *objs,
           "-Xlinker", f"-rpath={cuda_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        raise RuntimeError("link of libdsa_b200.so failed")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


HOST_SRC = os.path.join(CSRC, "dsa_host_binding.cpp")
HOST_NAME = "_dsa_host"
HOST_BUILD_DIR = os.path.join(PKG_DIR, "_build", "host")
HOST_PATH = os.path.join(PKG_DIR, HOST_NAME + ".so")


def build_host(force: bool = False, verbose: bool = False) -> str:
    """Compile the C++ fast path of launch_sparse_attention_c (a PyTorch C++
    extension: argument checks on at::Tensor, then the C ABI) into the package
    directory as _dsa_host.so.  Only the package's own loader imports it, by
    path, so nothing is compiled at run time."""
    if not force and os.path.exists(HOST_PATH) and os.path.getmtime(HOST_PATH) >= max(
            os.path.getmtime(HOST_SRC), os.path.getmtime(os.path.abspath(__file__))):
        return HOST_PATH
    from torch.utils.cpp_extension import load
    os.makedirs(HOST_BUILD_DIR, exist_ok=True)
    load(name=HOST_NAME, sources=[HOST_SRC], extra_cflags=["-O2"], build_directory=HOST_BUILD_DIR,
         with_cuda=True, verbose=verbose)
    built = os.path.join(HOST_BUILD_DIR, HOST_NAME + ".so")
    if not os.path.exists(built):
        raise RuntimeError(f"build of {HOST_NAME} produced no {built}")
    tmp = HOST_PATH + ".tmp"
    shutil.copyfile(built, tmp)
    os.replace(tmp, HOST_PATH)
    return HOST_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_host(force="--force" in sys.argv, verbose="-v" in sys.argv))
