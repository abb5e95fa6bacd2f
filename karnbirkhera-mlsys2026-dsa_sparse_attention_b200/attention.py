"""Host-side mirror of the reference's operator interface.

The reference exports one destination-passing entry point,
``launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
sm_scale, output, lse)`` (solution/cuda/kernel.cu:673-681, :726-729, selected by
config.toml:8-10), and the contest's value-returning form
``kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale) ->
(output, lse)``.  Both are provided here with the same argument meaning; the
work is done by libdsa_b200.so through its C ABI.

Differences from the reference launcher, all on the safe side:
  * arguments are checked (dtype, shape, contiguity, device, alignment) and a
    bad call raises DsaError (a RuntimeError, like the reference's TORCH_CHECK);
  * any num_tokens >= 0 is accepted (the reference rejects num_tokens >= 9,
    kernel.cu:688-691);
  * the scratch workspace is per device (the reference's is process-global,
    kernel.cu:646-671).  Every call on a device uses it, so calls whose work
    may overlap on the GPU (issued on different streams with no ordering
    between them) race on it: keep them on one stream or order them with
    events, or call the C ABI with a workspace of its own per stream;
  * indices outside [-1, num_pages*64) are detected on the device; call
    ``check_device_errors()`` (or pass ``check=True``) to raise on them.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _lib

NUM_HEADS = 16
CKV_DIM = 512
KPE_DIM = 64
PAGE_SIZE = 64
TOPK = 2048

_ws_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}
_CHECK_ALWAYS = os.environ.get("DSA_CHECK_ERRORS", "0") == "1"


_ws_need: dict[tuple[int, int], int] = {}


def workspace_for(device: torch.device, num_tokens: int) -> torch.Tensor:
    """Zero-initialised per-device workspace, grown on demand and kept for the
    life of the process (the C ABI never needs it cleared again)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return _workspace_on(idx, num_tokens)


def _workspace_on(idx: int, num_tokens: int) -> torch.Tensor:
    key = (idx, max(int(num_tokens), 1))
    need = _ws_need.get(key)
    if need is None:
        lib = _lib.load()
        with torch.cuda.device(idx):
            need = int(lib.dsa_sparse_attention_workspace_size(key[1]))
        if need == 0:
            raise _lib.DsaError(_lib.DSA_ERR_CUDA, "cannot query the device for the workspace size")
        _ws_need[key] = need
    ws = _workspaces.get(idx)
    if ws is not None and ws.numel() >= need:
        return ws
    with _ws_lock:
        ws = _workspaces.get(idx)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = ws
        return ws


def _bad(msg: str):
    raise _lib.DsaError(_lib.DSA_ERR_INVALID_ARGUMENT, msg)


# (name, dtype, shape with None for N / P) of each argument
_SPECS = (("q_nope", torch.bfloat16, ("N", NUM_HEADS, CKV_DIM), "bf16 [N,16,512]"),
          ("q_pe", torch.bfloat16, ("N", NUM_HEADS, KPE_DIM), "bf16 [N,16,64]"),
          ("ckv_cache", torch.bfloat16, ("P", PAGE_SIZE, CKV_DIM), "bf16 [P,64,512]"),
          ("kpe_cache", torch.bfloat16, ("P", PAGE_SIZE, KPE_DIM), "bf16 [P,64,64]"),
          ("sparse_indices", torch.int32, ("N", TOPK), "int32 [N,2048]"),
          ("output", torch.bfloat16, ("N", NUM_HEADS, CKV_DIM), "bf16 [N,16,512]"),
          ("lse", torch.float32, ("N", NUM_HEADS), "fp32 [N,16]"))


_shapes: dict[tuple[int, int], tuple] = {}
_MAX_TOKENS = 1 << 24   # the C ABI's num_tokens limit


def _checked(tensors):
    """Validate the arguments and return (data pointers, N, P, device index).
    Messages are only formatted for a failing check, and each tensor's
    attributes are read once, so a good call costs a few reads per tensor."""
    ptrs = []
    dev = -2
    for spec, t in zip(_SPECS, tensors):
        if not isinstance(t, torch.Tensor):
            _bad(f"{spec[0]} must be a torch.Tensor")
        d = t.get_device()   # -1 for a CPU tensor
        if d < 0:
            _bad(f"{spec[0]} must be a CUDA tensor")
        if not t.is_contiguous():
            _bad(f"{spec[0]} must be contiguous")
        ptr = t.data_ptr()
        if ptr & 15:
            _bad(f"{spec[0]} must be 16-byte aligned")
        if dev == -2:
            dev = d
        elif d != dev:
            _bad(f"{spec[0]} is on {t.device}, q_nope on {tensors[0].device}")
        ptrs.append(ptr)
    qs, cs = tensors[0].shape, tensors[2].shape
    n = qs[0] if len(qs) == 3 else -1
    p = cs[0] if len(cs) == 3 else -1
    wants = _shapes.get((n, p))
    if wants is None:
        wants = tuple(tuple(n if d == "N" else p if d == "P" else d for d in spec[2]) for spec in _SPECS)
        if len(_shapes) < 4096:
            _shapes[(n, p)] = wants
    for (name, dtype, _, what), t, want in zip(_SPECS, tensors, wants):
        if t.dtype != dtype or t.shape != want:
            _bad(f"{name} must be {what}, got {t.dtype} {tuple(t.shape)}")
    return ptrs, n, p, dev


try:   # the current stream's handle without building a Stream object
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:   # pragma: no cover - older torch
    def _raw_stream(idx):
        return torch.cuda.current_stream(idx).cuda_stream


_host = None   # the C++ fast path (module), False once known to be absent
_host_lock = threading.Lock()


def _load_host():
    """The in-tree C++ fast path of launch_sparse_attention_c
    (csrc/dsa_host_binding.cpp, built by build.build_host): the same checks
    on at::Tensor and one call of the C ABI, a few microseconds less host
    time per call than the checks here.  Imported by path (nothing is
    compiled at run time) and handed the C ABI function of the library this
    package loaded; when it is absent the calls take the path below, which
    runs the same kernel."""
    global _host
    with _host_lock:
        if _host is None:
            _host = False
            path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_dsa_host.so")
            if os.path.exists(path):
                import importlib.util
                spec = importlib.util.spec_from_file_location("_dsa_host", path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                mod.set_fwd(ctypes.cast(_lib.load().dsa_sparse_attention_fwd, ctypes.c_void_p).value)
                _host = mod
    return _host


def _scalar(sm_scale) -> float:
    if isinstance(sm_scale, torch.Tensor):
        return float(sm_scale.item())
    return float(sm_scale)


def launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse,
                              *, check: bool = False, stream: torch.cuda.Stream | None = None):
    """Destination-passing entry point with the reference's argument order
    (solution/cuda/kernel.cu:673-681).  Writes `output` and `lse` in place on
    the current (or given) CUDA stream."""
    host = _host if _host is not None else _load_host()
    if host and stream is None:
        # C++ checks and launch; any failed check (-1) falls through to the
        # checks below, which raise with the message
        try:
            idx = q_nope.get_device() if q_nope.dim() == 3 else -1
            n = q_nope.shape[0]
        except (AttributeError, TypeError):
            idx = -1
        if idx >= 0 and 0 < n <= _MAX_TOKENS:
            try:
                st = host.fwd(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, _scalar(sm_scale), output, lse,
                              _workspace_on(idx, n))
            except TypeError:   # an argument that is not a tensor
                st = -1
            if st >= 0:
                _lib.check(st, "dsa_sparse_attention_fwd")
                if check or _CHECK_ALWAYS:
                    check_device_errors(q_nope.device, None)
                return
    ptrs, n, p, idx = _checked((q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, output, lse))
    lib = _lib.load()
    if n == 0:
        return
    ws = _workspace_on(idx, n)
    raw = stream.cuda_stream if stream is not None else _raw_stream(idx)
    args = (ptrs[0], ptrs[1], ptrs[2], ptrs[3], ptrs[4], n, p, _scalar(sm_scale), ptrs[5], ptrs[6],
            ws.data_ptr(), ws.numel(), raw)
    if idx == torch.cuda.current_device():
        st = lib.dsa_sparse_attention_fwd(*args)
    else:
        with torch.cuda.device(idx):
            st = lib.dsa_sparse_attention_fwd(*args)
    _lib.check(st, "dsa_sparse_attention_fwd")
    if check or _CHECK_ALWAYS:
        check_device_errors(q_nope.device, stream)


def kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, *, check: bool = False):
    """Value-returning entry point: returns (output bf16 [N,16,512], lse fp32 [N,16])."""
    n = q_nope.shape[0]
    output = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.empty((n, NUM_HEADS), dtype=torch.float32, device=q_nope.device)
    launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse,
                              check=check)
    return output, lse


def _check_paged(block_table, positions, seq_of_token, n):
    def req(cond, msg):
        if not cond:
            raise _lib.DsaError(_lib.DSA_ERR_INVALID_ARGUMENT, (msg() if callable(msg) else msg))

    for name, t in (("block_table", block_table), ("positions", positions), ("seq_of_token", seq_of_token)):
        if t is None and name == "seq_of_token":
            continue
        req(isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous() and t.dtype == torch.int32,
            lambda: f"{name} must be a contiguous int32 CUDA tensor")
    req(block_table.dim() == 2 and block_table.shape[0] >= 1 and block_table.shape[1] >= 1,
        lambda: f"block_table must be [num_rows, max_num_pages], got {tuple(block_table.shape)}")
    req(tuple(positions.shape) == (n, TOPK), lambda: f"positions must be int32 [N,2048], got {tuple(positions.shape)}")
    req(positions.data_ptr() % 16 == 0, "positions must be 16-byte aligned")
    if seq_of_token is not None:
        req(tuple(seq_of_token.shape) == (n,), lambda: f"seq_of_token must be int32 [N], got {tuple(seq_of_token.shape)}")


def launch_sparse_attention_paged(q_nope, q_pe, ckv_cache, kpe_cache, block_table, positions, sm_scale, output,
                                  lse, *, seq_of_token=None, check: bool = False,
                                  stream: torch.cuda.Stream | None = None):
    """Page-table-native form of launch_sparse_attention_c: the 2048 selected
    keys of token t are positions in its sequence, translated on the device
    through row seq_of_token[t] (t when None) of `block_table`
    ([num_rows, max_num_pages] int32, physical page ids) as
    slot = block_table[row][pos // 64] * 64 + pos % 64 -- the translation the
    reference runs as a separate step (methodology/reference/
    topk_kernel_naive.cu:52-62).  Positions of -1 are padding."""
    ptrs, n, p, idx = _checked((q_nope, q_pe, ckv_cache, kpe_cache, positions, output, lse))
    _check_paged(block_table, positions, seq_of_token, n)
    lib = _lib.load()
    if n == 0:
        return
    ws = _workspace_on(idx, n)
    raw = stream.cuda_stream if stream is not None else _raw_stream(idx)
    args = (ptrs[0], ptrs[1], ptrs[2], ptrs[3], block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
            seq_of_token.data_ptr() if seq_of_token is not None else None, ptrs[4], n, p, _scalar(sm_scale),
            ptrs[5], ptrs[6], ws.data_ptr(), ws.numel(), raw)
    if idx == torch.cuda.current_device():
        st = lib.dsa_sparse_attention_fwd_paged(*args)
    else:
        with torch.cuda.device(idx):
            st = lib.dsa_sparse_attention_fwd_paged(*args)
    _lib.check(st, "dsa_sparse_attention_fwd_paged")
    if check or _CHECK_ALWAYS:
        check_device_errors(q_nope.device, stream)


def kernel_paged(q_nope, q_pe, ckv_cache, kpe_cache, block_table, positions, sm_scale, *, seq_of_token=None,
                 check: bool = False):
    """Value-returning page-table-native entry point: (output, lse)."""
    n = q_nope.shape[0]
    output = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.empty((n, NUM_HEADS), dtype=torch.float32, device=q_nope.device)
    launch_sparse_attention_paged(q_nope, q_pe, ckv_cache, kpe_cache, block_table, positions, sm_scale, output,
                                  lse, seq_of_token=seq_of_token, check=check)
    return output, lse


def check_device_errors(device=None, stream: torch.cuda.Stream | None = None) -> int:
    """Synchronise, read and clear the device error word of `device`'s
    workspace; raise DsaError if an index was out of range or a pipeline wait
    timed out.  Returns the raw flags (0 when clean)."""
    lib = _lib.load()
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _ws_lock:
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
