"""CPU oracle for the DSA top-k indexer — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, as the checker or the timed CPU baseline; the product path never
calls it.

Definition dsa_topk_indexer_fp8_h64_d128_topk2048_ps64, restated from the
reference's naive kernel methodology/reference/topk_kernel_naive.cu:65-111
(with its helpers :22-62).  Pinned on the GPU: the reference's naive indexer
mixes CUDA kernels with ATen calls and has no CPU build, and it ships no
fixtures or tests, so oracle/build_ref_indexer.py compiles it from its source
for sm_100a and tests/test_indexer_ref_gpu.py checks this restatement (and the
library) against its outputs on the GPU box.

  * q_index_fp8 [B, 64, 128] fp8 e4m3, used as fp32 (:78 `.to(kFloat32)`);
  * the index-key cache is paged: a page is 8448 bytes = 64 rows of 128 fp8
    (8192 B) followed by the 64 rows' fp32 scales (256 B) (:16-20);
    K[row] = fp8(row) * scale(row) in fp32 (dequant_gather_kernel, :28-49);
  * for batch row b with seq_len sl > 0 (:92-93): the sequence's pages are
    block_table[b][0 .. ceil(sl/64)) (:94-96, :101); K = its first sl rows (:103);
    scores = q[b] @ K^T  [64, sl] (:104);
    final = sum_h relu(scores[h]) * weights[b][h]  [sl] (:105-106);
    top min(2048, sl) positions by final, largest first, sorted (:106 at::topk);
    position -> slot id through the block table:
    block_table[b][pos >> 6] * 64 + (pos & 63) (translate_indices_kernel, :52-62);
  * every other entry of topk_indices is -1 (:77 `fill_(-1)`); sl <= 0 leaves
    the row all -1 (:93).

Ties: at::topk does not specify the order of equal scores; this oracle (and
the CUDA kernel) put the lower position first.  Because summation order
differs between implementations, tests compare selections with a tolerance on
the score at the selection boundary rather than index by index.
"""
from __future__ import annotations

import torch

NUM_HEADS = 64
HEAD_DIM = 128
PAGE_SIZE = 64
PAGE_DATA_BYTES = 8192
PAGE_BYTES = 8448
TOPK = 2048


def dequant_pages(k_cache_u8: torch.Tensor, pages: torch.Tensor) -> torch.Tensor:
    """Rows of the given pages as fp32 [len(pages) * 64, 128] (fp8 * scale)."""
    pg = k_cache_u8[pages.long()]                                           # [P, 8448] uint8
    data = pg[:, :PAGE_DATA_BYTES].reshape(-1, PAGE_SIZE, HEAD_DIM)
    vals = data.contiguous().view(torch.float8_e4m3fn).float()             # [P, 64, 128]
    scales = pg[:, PAGE_DATA_BYTES:].contiguous().view(torch.float32)       # [P, 64]
    return (vals * scales[:, :, None]).reshape(-1, HEAD_DIM)


def indexer_scores(q_index_fp8, k_cache_u8, weights, seq_len: int, block_row) -> torch.Tensor:
    """final[sl] for one batch row (q_index_fp8 [64, 128] as uint8)."""
    npages = (seq_len + PAGE_SIZE - 1) // PAGE_SIZE
    K = dequant_pages(k_cache_u8, block_row[:npages])[:seq_len]            # [sl, 128]
    q = q_index_fp8.contiguous().view(torch.float8_e4m3fn).float()         # [64, 128]
    scores = q @ K.t()                                                      # [64, sl]
    return (torch.relu(scores) * weights.float()[:, None]).sum(0)


def topk_indexer_oracle(q_index_fp8, k_index_cache, weights, seq_lens, block_table):
    """topk_indices [B, 2048] int32 (slot ids, -1 padded), plus the per-row
    final scores (list of fp32 tensors) for tolerance-aware comparisons."""
    q = q_index_fp8.cpu()
    kc = k_index_cache.cpu().reshape(k_index_cache.shape[0], -1)
    w = weights.cpu()
    sls = seq_lens.cpu().tolist()
    bt = block_table.cpu()
    B = q.shape[0]
    out = torch.full((B, TOPK), -1, dtype=torch.int32)
    finals = []
    for b in range(B):
        sl = int(sls[b])
        if sl <= 0:
            finals.append(torch.empty(0))
            continue
        final = indexer_scores(q[b], kc, w[b], sl, bt[b])
        finals.append(final)
        k = min(TOPK, sl)
        # largest first; equal scores by lower position (stable sort on -score)
        order = torch.sort(-final, stable=True).indices[:k]
        pages = bt[b][order >> 6].to(torch.int64)
        out[b, :k] = (pages * PAGE_SIZE + (order & (PAGE_SIZE - 1))).to(torch.int32)
    return out, finals
