"""FP8 KV cache variant of the attention operator.

The reference has no FP8 KV form (it rejects FP8 KV as outside its definition,
methodology/optimization_log.md:1205).  The cache format here is the 656-byte
MLA row: per slot, 512 ckv values as fp8 e4m3, 4 fp32 scales (scale j for ckv
values [128 j, 128 j + 128)), then the 64 rope values as bf16 —
``kv_cache_fp8 [num_pages, 64, 656] uint8``.  Dequantised
``ckv = bf16_rn(float(e4m3) * scale)``; the operator then computes exactly what
``kernel`` computes on the dequantised cache (bit for bit), reading 656 bytes
per selected key instead of 1152.

    kv = quantize_kv_fp8(ckv_cache, kpe_cache)
    output, lse = kernel_fp8(q_nope, q_pe, kv, sparse_indices, sm_scale)
"""
from __future__ import annotations

import torch

from . import _lib
from .attention import (CKV_DIM, KPE_DIM, NUM_HEADS, PAGE_SIZE, TOPK, _CHECK_ALWAYS, _check_paged, _scalar,
                        check_device_errors, workspace_for)

FP8_ROW_BYTES = 656
FP8_SCALE_OFFSET = 512
FP8_ROPE_OFFSET = 528
E4M3_MAX = 448.0


def quantize_kv_fp8(ckv_cache: torch.Tensor, kpe_cache: torch.Tensor) -> torch.Tensor:
    """bf16 ckv [P,64,512] and kpe [P,64,64] -> kv_cache_fp8 [P,64,656] uint8.
    Each group of 128 ckv values of a slot gets scale = amax / 448 (a zero
    group gets scale 1) and values e4m3_rn(x / scale); kpe is kept in bf16."""
    p = ckv_cache.shape[0]
    x = ckv_cache.float().reshape(p, PAGE_SIZE, 4, 128)
    amax = x.abs().amax(dim=-1)
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (x / scale[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    out = torch.empty((p, PAGE_SIZE, FP8_ROW_BYTES), dtype=torch.uint8, device=ckv_cache.device)
    out[..., :FP8_SCALE_OFFSET] = q.view(torch.uint8).reshape(p, PAGE_SIZE, CKV_DIM)
    out[..., FP8_SCALE_OFFSET:FP8_ROPE_OFFSET] = scale.contiguous().view(torch.uint8).reshape(p, PAGE_SIZE, 16)
    out[..., FP8_ROPE_OFFSET:] = kpe_cache.contiguous().view(torch.uint8).reshape(p, PAGE_SIZE, 2 * KPE_DIM)
    return out


def dequantize_kv_fp8(kv_cache_fp8: torch.Tensor):
    """kv_cache_fp8 [P,64,656] -> (ckv bf16 [P,64,512], kpe bf16 [P,64,64]),
    the values the operator computes with."""
    p = kv_cache_fp8.shape[0]
    raw = kv_cache_fp8.reshape(p, PAGE_SIZE, FP8_ROW_BYTES)
    vals = raw[..., :FP8_SCALE_OFFSET].contiguous().view(torch.float8_e4m3fn).float().reshape(p, PAGE_SIZE, 4, 128)
    scale = raw[..., FP8_SCALE_OFFSET:FP8_ROPE_OFFSET].contiguous().view(torch.float32).reshape(p, PAGE_SIZE, 4)
    ckv = (vals * scale[..., None]).to(torch.bfloat16).reshape(p, PAGE_SIZE, CKV_DIM)
    kpe = raw[..., FP8_ROPE_OFFSET:].contiguous().view(torch.bfloat16).reshape(p, PAGE_SIZE, KPE_DIM)
    return ckv, kpe


def _check_fp8_args(q_nope, q_pe, kv_cache_fp8, sparse_indices, output, lse):
    def req(cond, msg):
        if not cond:
            raise _lib.DsaError(_lib.DSA_ERR_INVALID_ARGUMENT, (msg() if callable(msg) else msg))

    tensors = {"q_nope": q_nope, "q_pe": q_pe, "kv_cache_fp8": kv_cache_fp8, "sparse_indices": sparse_indices,
               "output": output, "lse": lse}
    for name, t in tensors.items():
        req(isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous(), lambda: f"{name} must be a contiguous CUDA tensor")
        req(t.data_ptr() % 16 == 0, lambda: f"{name} must be 16-byte aligned")
        req(t.device == q_nope.device, lambda: f"{name} is on {t.device}, q_nope on {q_nope.device}")
    n = q_nope.shape[0] if q_nope.dim() == 3 else -1
    req(q_nope.dtype == torch.bfloat16 and tuple(q_nope.shape) == (n, NUM_HEADS, CKV_DIM),
        lambda: f"q_nope must be bf16 [N,16,512], got {q_nope.dtype} {tuple(q_nope.shape)}")
    req(q_pe.dtype == torch.bfloat16 and tuple(q_pe.shape) == (n, NUM_HEADS, KPE_DIM),
        lambda: f"q_pe must be bf16 [N,16,64], got {q_pe.dtype} {tuple(q_pe.shape)}")
    p = kv_cache_fp8.shape[0] if kv_cache_fp8.dim() == 3 else -1
    req(kv_cache_fp8.element_size() == 1 and tuple(kv_cache_fp8.shape) == (p, PAGE_SIZE, FP8_ROW_BYTES),
        lambda: f"kv_cache_fp8 must be 1-byte [P,64,656], got {kv_cache_fp8.dtype} {tuple(kv_cache_fp8.shape)}")
    req(sparse_indices.dtype == torch.int32 and tuple(sparse_indices.shape) == (n, TOPK),
        lambda: f"indices must be int32 [N,2048], got {sparse_indices.dtype} {tuple(sparse_indices.shape)}")
    req(output.dtype == torch.bfloat16 and tuple(output.shape) == (n, NUM_HEADS, CKV_DIM),
        lambda: f"output must be bf16 [N,16,512], got {output.dtype} {tuple(output.shape)}")
    req(lse.dtype == torch.float32 and tuple(lse.shape) == (n, NUM_HEADS),
        lambda: f"lse must be fp32 [N,16], got {lse.dtype} {tuple(lse.shape)}")
    return n, p


def _call(fn_name, args, dev, s, check):
    lib = _lib.load()
    fn = getattr(lib, fn_name)
    if dev.index == torch.cuda.current_device():
        st = fn(*args)
    else:
        with torch.cuda.device(dev):
            st = fn(*args)
    _lib.check(st, fn_name)
    if check or _CHECK_ALWAYS:
        check_device_errors(dev, s)


def launch_sparse_attention_fp8_c(q_nope, q_pe, kv_cache_fp8, sparse_indices, sm_scale, output, lse, *,
                                  check: bool = False, stream: torch.cuda.Stream | None = None):
    """Destination-passing FP8-cache form of launch_sparse_attention_c."""
    n, p = _check_fp8_args(q_nope, q_pe, kv_cache_fp8, sparse_indices, output, lse)
    if n == 0:
        return
    dev = q_nope.device
    ws = workspace_for(dev, n)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    args = (q_nope.data_ptr(), q_pe.data_ptr(), kv_cache_fp8.data_ptr(), sparse_indices.data_ptr(), n, p,
            _scalar(sm_scale), output.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), s.cuda_stream)
    _call("dsa_sparse_attention_fwd_fp8", args, dev, s, check)


def kernel_fp8(q_nope, q_pe, kv_cache_fp8, sparse_indices, sm_scale, *, check: bool = False):
    """Value-returning FP8-cache entry point: (output bf16 [N,16,512], lse fp32 [N,16])."""
    n = q_nope.shape[0]
    output = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.empty((n, NUM_HEADS), dtype=torch.float32, device=q_nope.device)
    launch_sparse_attention_fp8_c(q_nope, q_pe, kv_cache_fp8, sparse_indices, sm_scale, output, lse, check=check)
    return output, lse


def launch_sparse_attention_fp8_paged(q_nope, q_pe, kv_cache_fp8, block_table, positions, sm_scale, output, lse, *,
                                      seq_of_token=None, check: bool = False,
                                      stream: torch.cuda.Stream | None = None):
    """Page-table-native FP8-cache form (block table and positions as in
    launch_sparse_attention_paged)."""
    n, p = _check_fp8_args(q_nope, q_pe, kv_cache_fp8, positions, output, lse)
    _check_paged(block_table, positions, seq_of_token, n)
    if n == 0:
        return
    dev = q_nope.device
    ws = workspace_for(dev, n)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    args = (q_nope.data_ptr(), q_pe.data_ptr(), kv_cache_fp8.data_ptr(), block_table.data_ptr(),
            block_table.shape[0], block_table.shape[1], seq_of_token.data_ptr() if seq_of_token is not None else None,
            positions.data_ptr(), n, p, _scalar(sm_scale), output.data_ptr(), lse.data_ptr(), ws.data_ptr(),
            ws.numel(), s.cuda_stream)
    _call("dsa_sparse_attention_fwd_fp8_paged", args, dev, s, check)


def kernel_fp8_paged(q_nope, q_pe, kv_cache_fp8, block_table, positions, sm_scale, *, seq_of_token=None,
                     check: bool = False):
    """Value-returning page-table-native FP8-cache entry point: (output, lse)."""
    n = q_nope.shape[0]
    output = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.empty((n, NUM_HEADS), dtype=torch.float32, device=q_nope.device)
    launch_sparse_attention_fp8_paged(q_nope, q_pe, kv_cache_fp8, block_table, positions, sm_scale, output, lse,
                                      seq_of_token=seq_of_token, check=check)
    return output, lse
