"""B200-native (sm_100a) DSA sparse MLA attention operator.

Definition dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64: 16 heads, a
512-wide compressed KV and a 64-wide rope key, 2048 selected slots per query
token from 64-slot pages.  Drop-in for the reference's entry points:

    kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale) -> (output, lse)
    launch_sparse_attention_c(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse)

page-table-native forms that translate positions through a block table on
the device: kernel_paged(...) and launch_sparse_attention_paged(...), and the
top-k indexer upstream of them (definition
dsa_topk_indexer_fp8_h64_d128_topk2048_ps64): topk_indexer(...) and
launch_topk_c(...); and the FP8 KV cache variant (656-byte rows, fp8.py):
kernel_fp8(...), launch_sparse_attention_fp8_c(...), kernel_fp8_paged(...),
quantize_kv_fp8(...).

The package directory name contains dashes; import it with
``importlib.import_module("karnbirkhera-mlsys2026-dsa_sparse_attention_b200")``.
"""
from .attention import (CKV_DIM, KPE_DIM, NUM_HEADS, PAGE_SIZE, TOPK, check_device_errors, kernel, kernel_paged,
                        launch_sparse_attention_c, launch_sparse_attention_paged, workspace_for)
from ._lib import DsaError
from .fp8 import (dequantize_kv_fp8, kernel_fp8, kernel_fp8_paged, launch_sparse_attention_fp8_c,
                  launch_sparse_attention_fp8_paged, quantize_kv_fp8)
from .indexer import launch_topk_c, topk_indexer

__all__ = ["kernel", "launch_sparse_attention_c", "kernel_paged", "launch_sparse_attention_paged",
           "topk_indexer", "launch_topk_c", "kernel_fp8", "launch_sparse_attention_fp8_c", "kernel_fp8_paged",
           "launch_sparse_attention_fp8_paged", "quantize_kv_fp8", "dequantize_kv_fp8", "check_device_errors", "workspace_for", "DsaError",
           "NUM_HEADS", "CKV_DIM", "KPE_DIM", "PAGE_SIZE", "TOPK"]
