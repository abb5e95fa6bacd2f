"""ctypes binding of libdsa_b200.so (the C ABI in include/dsa_sparse_attention.h).

The library is built in-tree by build.py.  There is no fallback: if the
library is missing or fails to load, importing the package's operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libdsa_b200.so")

# dsa_status values (include/dsa_sparse_attention.h)
DSA_OK = 0
DSA_ERR_INVALID_ARGUMENT = 1
DSA_ERR_UNSUPPORTED_DEVICE = 2
DSA_ERR_WORKSPACE_TOO_SMALL = 3
DSA_ERR_CUDA = 4
DSA_ERR_BAD_INDEX = 5
DSA_ERR_DEVICE_TIMEOUT = 6
DEVICE_ERR_BAD_INDEX = 0x1
DEVICE_ERR_TIMEOUT = 0x2

# Every symbol the header declares, with its ctypes signature.
_VP = ctypes.c_void_p
SIGNATURES = {
    "dsa_sparse_attention_workspace_size": (ctypes.c_size_t, [ctypes.c_int64]),
    "dsa_sparse_attention_fwd": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_float, _VP, _VP, _VP, ctypes.c_size_t, _VP]),
    "dsa_sparse_attention_fwd_profiled": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int64,
                                                         ctypes.c_int64, ctypes.c_float, _VP, _VP, _VP,
                                                         ctypes.c_size_t, _VP, ctypes.POINTER(_VP)]),
    "dsa_sparse_attention_fwd_paged": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64,
                                                      _VP, _VP, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                                      _VP, _VP, _VP, ctypes.c_size_t, _VP]),
    "dsa_sparse_attention_fwd_fp8": (ctypes.c_int, [_VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64,
                                                    ctypes.c_float, _VP, _VP, _VP, ctypes.c_size_t, _VP]),
    "dsa_sparse_attention_fwd_fp8_paged": (ctypes.c_int, [_VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64, _VP,
                                                          _VP, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _VP,
                                                          _VP, _VP, ctypes.c_size_t, _VP]),
    "dsa_sparse_attention_read_errors": (ctypes.c_int, [_VP, _VP, ctypes.POINTER(ctypes.c_uint32)]),
    "dsa_sparse_attention_fwd_noalloc": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64,
                                                        ctypes.c_float, _VP, _VP, _VP]),
    "dsa_topk_indexer_workspace_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "dsa_topk_indexer_fwd": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                            _VP, _VP, ctypes.c_size_t, _VP]),
    "dsa_sparse_attention_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "dsa_sparse_attention_test_hold": (ctypes.c_int, [ctypes.c_int]),
    "dsa_sparse_attention_set_cluster_merge": (ctypes.c_int, [ctypes.c_int]),
    "dsa_topk_indexer_set_calibrated_plan": (ctypes.c_int, [ctypes.c_int]),
    "dsa_sparse_attention_noalloc_read_errors": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "dsa_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "dsa_sparse_attention_abi_version": (ctypes.c_int, []),
}

_lib = None
_lock = threading.Lock()


class DsaError(RuntimeError):
    """Raised when the operator rejects its arguments or the device reports an
    error.  `status` is the dsa_status code."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        name = status_string(status) if _lib is not None else str(status)
        super().__init__(f"{name}{': ' + what if what else ''}")


def load():
    """Load (once) and return the ctypes handle of libdsa_b200.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                              "(nvcc, sm_100a). There is no CPU fallback.")
        import torch  # noqa: F401  -- load torch's CUDA runtime first so both share it
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().dsa_status_string(int(status)).decode()


def check(status: int, what: str = "") -> None:
    if status != DSA_OK:
        raise DsaError(status, what)
