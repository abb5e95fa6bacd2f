"""The C-ABI library loads and exports every function include/*.h declares.
No compute calls: these run without a GPU."""
import ctypes
import glob
import os
import re

import pytest

from tests.conftest import REPO, submodule


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(dsa_\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("dsa_sparse_attention_fwd", "dsa_sparse_attention_workspace_size",
                 "dsa_sparse_attention_read_errors", "dsa_status_string"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib_mod = submodule("_lib")
    assert os.path.exists(lib_mod.LIB_PATH), "build the library first (__graft_entry__.build())"
    lib = ctypes.CDLL(lib_mod.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    # and the Python binding knows every one of them
    assert set(declared_functions()) <= set(lib_mod.SIGNATURES)


def test_status_strings_and_version():
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    assert lib_mod.status_string(0) == "DSA_OK"
    assert lib_mod.status_string(5) == "DSA_ERR_BAD_INDEX"
    assert lib_mod.status_string(99) == "DSA_ERR_UNKNOWN"
    assert lib.dsa_sparse_attention_abi_version() == 1004


def test_invalid_arguments_rejected_before_any_device_work():
    """Null / misaligned pointers and bad counts fail with INVALID_ARGUMENT on
    the host (no device is touched)."""
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    f = lib.dsa_sparse_attention_fwd
    null = None
    assert f(null, null, null, null, null, 0, 1, 0.1, null, null, null, 0, null) == 0  # N=0 is a no-op
    assert f(null, null, null, null, null, -1, 1, 0.1, null, null, null, 0, null) == lib_mod.DSA_ERR_INVALID_ARGUMENT
    assert f(null, null, null, null, null, 4, 1, 0.1, null, null, null, 0, null) == lib_mod.DSA_ERR_INVALID_ARGUMENT
    odd = 0x1001
    assert f(odd, odd, odd, odd, odd, 4, 1, 0.1, odd, odd, odd, 1 << 30, null) == lib_mod.DSA_ERR_INVALID_ARGUMENT
    assert f(16, 16, 16, 16, 16, 4, 0, 0.1, 16, 16, 16, 1 << 30, null) == lib_mod.DSA_ERR_INVALID_ARGUMENT
    assert f(16, 16, 16, 16, 16, 4, 1, float("nan"), 16, 16, 16, 1 << 30, null) == lib_mod.DSA_ERR_INVALID_ARGUMENT


def test_paged_entry_rejects_bad_block_table_arguments():
    """The page-table-native entry point checks its extra arguments on the
    host too: a null or misaligned block table or row map, and empty or
    oversized table shapes fail with INVALID_ARGUMENT before any device work."""
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    f = lib.dsa_sparse_attention_fwd_paged
    inv = lib_mod.DSA_ERR_INVALID_ARGUMENT
    a = 16   # a 16-byte aligned stand-in address; rejected before it is dereferenced

    def call(bt=a, rows=4, maxp=8, seq=None, n=4):
        return f(a, a, a, a, bt, rows, maxp, seq, a, n, 1, 0.1, a, a, a, 1 << 30, None)

    assert call(n=0) == 0                     # no tokens: a no-op, like the slot-id entry point
    assert call(bt=None) == inv
    assert call(bt=a + 2) == inv              # block table must be 4-byte aligned
    assert call(rows=0) == inv
    assert call(maxp=0) == inv
    assert call(maxp=(2**31 - 1) // 64 + 1) == inv   # positions are int32
    assert call(seq=a + 1) == inv             # misaligned row map


def test_operator_fails_loudly_without_library(monkeypatch, tmp_path):
    lib_mod = submodule("_lib")
    monkeypatch.setattr(lib_mod, "_lib", None)
    monkeypatch.setattr(lib_mod, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        lib_mod.load()


def test_host_binding_is_built_and_loads():
    """The C++ fast path of launch_sparse_attention_c (csrc/dsa_host_binding.cpp)
    is built in-tree, imports by path and exports its two functions."""
    att = submodule("attention")
    host = att._load_host()
    assert host, "_dsa_host.so is missing: run build.build_host()"
    assert callable(host.fwd) and callable(host.set_fwd)


@pytest.mark.parametrize("batch,max_pages", [(1, 1), (3, 7), (64, 512), (4096, 1), (5, 1100)])
def test_indexer_workspace_layout(batch, max_pages):
    """Header (256 B) + counter region (8 KB), the fp32 scores, each row's key
    range (2 x u32), then the score split plan, 16-byte aligned: a 16-byte
    header, 1028 u32 fractions and 1024 16-byte log entries (host-only call)."""
    lib = submodule("_lib").load()
    plan_bytes = 16 + 4 * (1024 + 4) + 16 * 1024
    keys_end = 256 + 8192 + batch * max_pages * 64 * 4 + batch * 8
    want = ((keys_end + 15) & ~15) + plan_bytes
    assert lib.dsa_topk_indexer_workspace_size(batch, max_pages) == want
    assert lib.dsa_topk_indexer_workspace_size(0, max_pages) == lib.dsa_topk_indexer_workspace_size(1, max_pages)
    assert lib.dsa_topk_indexer_workspace_size(batch, 0) == 0
    assert lib.dsa_topk_indexer_workspace_size(-1, max_pages) == 0


def test_process_wide_switches_return_ok():
    """The switches only set process-wide flags (no device work)."""
    lib = submodule("_lib").load()
    for f in (lib.dsa_topk_indexer_set_calibrated_plan, lib.dsa_sparse_attention_set_cluster_merge):
        assert f(0) == 0
        assert f(1) == 0
