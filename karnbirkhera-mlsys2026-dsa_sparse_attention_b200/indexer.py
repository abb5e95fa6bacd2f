"""Host-side mirror of the reference's top-k indexer entry point.

The reference's naive indexer exports
``launch_topk_c(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)``
(methodology/reference/topk_kernel_naive.cu:65-119, definition
dsa_topk_indexer_fp8_h64_d128_topk2048_ps64).  The same call, and a
value-returning ``topk_indexer(...)``, run here on libdsa_b200.so through its C
ABI (dsa_topk_indexer_fwd): a tcgen05 fp8 scoring kernel, whose CTAs split
the rows' positions by a plan calibrated on the previous calls, and a top-k
kernel (a histogram of the row's scores in value bins, then a direct ranking
of the keys at and above the threshold bin; radix passes for rows outside
its limits).

Argument checks are on the host (dtype, shape, contiguity, device); a bad
block-table entry or an oversized seq_len found on the device is reported by
``check_errors()`` (or ``check=True``), like the attention's bad indices.
The workspace (scores, key ranges, the split plan) is one per device: calls
whose work may overlap on the GPU (different streams, no ordering) race on
it, so keep them on one stream or order them.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

HEADS = 64
DIM = 128
PAGE_BYTES = 8448
TOPK = 2048

_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}


def _workspace(dev: torch.device, batch: int, max_pages: int) -> torch.Tensor:
    lib = _lib.load()
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    need = int(lib.dsa_topk_indexer_workspace_size(max(batch, 1), max_pages))
    if need == 0:
        raise _lib.DsaError(_lib.DSA_ERR_INVALID_ARGUMENT, f"no workspace for batch {batch}, max pages {max_pages}")
    with _lock:
        ws = _workspaces.get(idx)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = ws
        return ws


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def _check(q, kc, w, sl, bt, out=None):
    def req(cond, msg):
        if not cond:
            raise _lib.DsaError(_lib.DSA_ERR_INVALID_ARGUMENT, (msg() if callable(msg) else msg))

    named = {"q_index_fp8": q, "k_index_cache": kc, "weights": w, "seq_lens": sl, "block_table": bt}
    if out is not None:
        named["topk_indices"] = out
    for name, t in named.items():
        req(isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous(), lambda: f"{name} must be a contiguous CUDA tensor")
        req(t.device == q.device, lambda: f"{name} is on {t.device}, q_index_fp8 on {q.device}")
    req(q.dtype in (torch.uint8, torch.float8_e4m3fn) and q.dim() == 3 and tuple(q.shape[1:]) == (HEADS, DIM),
        lambda: f"q_index_fp8 must be fp8 e4m3 (or its bytes) [B, 64, 128], got {q.dtype} {tuple(q.shape)}")
    b = q.shape[0]
    req(kc.element_size() == 1 and kc.dim() >= 1 and kc.numel() == kc.shape[0] * PAGE_BYTES,
        lambda: f"k_index_cache must be [num_pages, ...] of 8448-byte pages, got {kc.dtype} {tuple(kc.shape)}")
    req(w.dtype == torch.float32 and tuple(w.shape) == (b, HEADS), lambda: f"weights must be fp32 [B, 64], got {tuple(w.shape)}")
    req(sl.dtype == torch.int32 and tuple(sl.shape) == (b,), lambda: f"seq_lens must be int32 [B], got {tuple(sl.shape)}")
    req(bt.dtype == torch.int32 and bt.dim() == 2 and bt.shape[0] == b and bt.shape[1] >= 1,
        lambda: f"block_table must be int32 [B, max_num_pages], got {tuple(bt.shape)}")
    if out is not None:
        req(out.dtype == torch.int32 and tuple(out.shape) == (b, TOPK),
            lambda: f"topk_indices must be int32 [B, 2048], got {tuple(out.shape)}")
    return b


def launch_topk_c(q_index_fp8, k_index_cache, weights, seq_lens, block_table, topk_indices, *,
                  check: bool = False, stream: torch.cuda.Stream | None = None):
    """Destination-passing entry point with the reference's argument order
    (methodology/reference/topk_kernel_naive.cu:65-71): writes topk_indices."""
    b = _check(q_index_fp8, k_index_cache, weights, seq_lens, block_table, topk_indices)
    if b == 0:
        return
    lib = _lib.load()
    dev = q_index_fp8.device
    ws = _workspace(dev, b, block_table.shape[1])
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        st = lib.dsa_topk_indexer_fwd(_as_bytes(q_index_fp8).data_ptr(), k_index_cache.data_ptr(), weights.data_ptr(),
                                      seq_lens.data_ptr(), block_table.data_ptr(), b, block_table.shape[1],
                                      k_index_cache.shape[0], topk_indices.data_ptr(), ws.data_ptr(), ws.numel(),
                                      s.cuda_stream)
    _lib.check(st, "dsa_topk_indexer_fwd")
    if check:
        check_errors(dev, s)


def topk_indexer(q_index_fp8, k_index_cache, weights, seq_lens, block_table, *, check: bool = False):
    """Value-returning form: topk_indices int32 [B, 2048]."""
    out = torch.empty((q_index_fp8.shape[0], TOPK), dtype=torch.int32, device=q_index_fp8.device)
    launch_topk_c(q_index_fp8, k_index_cache, weights, seq_lens, block_table, out, check=check)
    return out


def check_errors(device=None, stream: torch.cuda.Stream | None = None) -> int:
    """Synchronise, read and clear the indexer workspace's device error word;
    raise DsaError on a bad block-table entry / seq_len or a timeout."""
    import ctypes
    lib = _lib.load()
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        ws = _workspaces.get(idx)
    if ws is None:
        return 0
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    flags = ctypes.c_uint32(0)
    with torch.cuda.device(idx):
        st = lib.dsa_sparse_attention_read_errors(ws.data_ptr(), s.cuda_stream, ctypes.byref(flags))
    if st != _lib.DSA_OK:
        raise _lib.DsaError(st, f"device flags 0x{flags.value:x}")
    return flags.value
