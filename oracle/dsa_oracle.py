"""CPU oracle for DSA sparse MLA attention — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline.  The product path never calls it.

It restates the reference's naive ATen kernel,
methodology/checkpoints/kernel_naive.cu:21-72, in PyTorch fp32 on CPU.  That
kernel is recorded by the reference as matching the contest definition's
Python `run()` with zero abs/rel error on all 23 workloads
(methodology/CLAUDE.md:301-310).  The semantics it pins:

  * fixed shapes: 16 heads, ckv width 512, kpe width 64, page size 64,
    top-k 2048 (kernel_naive.cu:14-18);
  * a sparse index is a flat slot id, slot = page * 64 + offset, i.e. a row of
    the cache viewed as [num_pages * 64, width] (kernel_naive.cu:38-39);
  * index -1 is padding and is skipped (kernel_naive.cu:48-50);
  * logits = (q_nope . ckv[slot] + q_pe . kpe[slot]) * sm_scale, in fp32
    (kernel_naive.cu:59-61);
  * lse is the BASE-2 log-sum-exp of the scaled logits (kernel_naive.cu:66);
  * output = softmax(logits) @ ckv[slots], rounded to bf16 (kernel_naive.cu:68-70);
  * a token with no valid index gets output 0 and lse -inf (kernel_naive.cu:43-44).

Parity is pinned two ways (tests/test_oracle.py): against the reference's own
naive kernel compiled for CPU from its source (oracle/build_ref.py), and
against the committed golden fixtures in tests/golden/ that the same compiled
reference produced.
"""
from __future__ import annotations

import math

import torch

NUM_HEADS = 16
CKV_DIM = 512
KPE_DIM = 64
PAGE_SIZE = 64
TOPK = 2048
INV_LN2 = 1.0 / math.log(2.0)


def sparse_attention_oracle(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale):
    """Value-returning form: returns (output bf16 [N,16,512], lse fp32 [N,16]).

    Follows kernel_naive.cu:21-72 step for step.  The only deviation is that
    the cache rows are cast to fp32 AFTER the gather instead of casting the
    whole cache first (kernel_naive.cu:38-39): the cast is exact and
    element-wise, so the result is identical while the CPU cost no longer
    scales with the pool size.
    """
    n = q_nope.shape[0]
    output = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16)
    lse = torch.empty((n, NUM_HEADS), dtype=torch.float32)
    launch_sparse_attention_oracle(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
                                   sm_scale, output, lse)
    return output, lse


def dequantize_kv_fp8(kv_cache_fp8):
    """FP8 KV rows [P, 64, 656] bytes -> (ckv bf16 [P, 64, 512], kpe bf16 [P, 64, 64]).

    The FP8 variant's format (the reference defines no FP8 KV form): per slot,
    bytes [0, 512) are ckv as fp8 e4m3, bytes [512, 528) four fp32 scales
    (scale j covers ckv values [128 j, 128 j + 128)), bytes [528, 656) the 64
    rope values as bf16.  ckv = bf16_rn(float(e4m3) * scale_j) in fp32."""
    raw = kv_cache_fp8.cpu().contiguous()
    p = raw.shape[0]
    ckv = torch.empty((p, 64, 512), dtype=torch.bfloat16)
    for j in range(4):
        vals = raw[:, :, 128 * j:128 * (j + 1)].contiguous().view(torch.float8_e4m3fn).to(torch.float32)
        scale = raw[:, :, 512 + 4 * j:516 + 4 * j].contiguous().view(torch.float32)   # [P, 64, 1]
        ckv[:, :, 128 * j:128 * (j + 1)] = (vals * scale).to(torch.bfloat16)
    kpe = raw[:, :, 528:656].contiguous().view(torch.bfloat16)
    return ckv, kpe


def sparse_attention_fp8_oracle(q_nope, q_pe, kv_cache_fp8, sparse_indices, sm_scale):
    """The FP8 variant's semantics: the attention above on the dequantised cache."""
    ckv, kpe = dequantize_kv_fp8(kv_cache_fp8)
    return sparse_attention_oracle(q_nope, q_pe, ckv, kpe, sparse_indices, sm_scale)


def launch_sparse_attention_oracle(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
                                   sm_scale, output, lse):
    """Destination-passing form with the reference's argument order
    (kernel_naive.cu:21-29)."""
    kc_all = ckv_cache.reshape(-1, CKV_DIM)          # kernel_naive.cu:38
    kp_all = kpe_cache.reshape(-1, KPE_DIM)          # kernel_naive.cu:39
    scale = float(sm_scale)                          # kernel_naive.cu:33 (fp32 scalar)
    scale32 = torch.tensor(scale, dtype=torch.float32)
    output.zero_()                                   # kernel_naive.cu:43
    lse.fill_(float("-inf"))                         # kernel_naive.cu:44
    for t in range(q_nope.shape[0]):                 # kernel_naive.cu:46
        indices = sparse_indices[t]
        valid = indices[indices.ne(-1)]              # kernel_naive.cu:48-50
        if valid.numel() == 0:                       # kernel_naive.cu:51
            continue
        tok = valid.to(torch.long)                   # kernel_naive.cu:53
        kc = kc_all.index_select(0, tok).float()     # kernel_naive.cu:54
        kp = kp_all.index_select(0, tok).float()     # kernel_naive.cu:55
        qn = q_nope[t].float()                       # kernel_naive.cu:56
        qp = q_pe[t].float()                         # kernel_naive.cu:57
        logits = qn @ kc.t() + qp @ kp.t()           # kernel_naive.cu:59-60
        logits_scaled = logits * scale32             # kernel_naive.cu:61
        lse[t].copy_(torch.logsumexp(logits_scaled, -1) * INV_LN2)   # kernel_naive.cu:66
        attn = torch.softmax(logits_scaled, -1)      # kernel_naive.cu:68
        output[t].copy_((attn @ kc).to(torch.bfloat16))              # kernel_naive.cu:69-70
    return output, lse


def reference_cuda_splits(num_tokens):
    """Splits per token of the reference's shipped CUDA kernel:
    clamp(132 // N, 1, 64) (solution/cuda/kernel.cu:634-641)."""
    return max(1, min(64, 132 // max(num_tokens, 1)))


def reference_cuda_oracle(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale):
    """CPU restatement of the reference's shipped CUDA kernel's algorithm
    (solution/cuda/kernel.cu), which is NOT the operator's semantics when a
    token has more than 32 splits; used only to pin that kernel's GPU output.

      * S = reference_cuda_splits(N) splits of ceil(2048 / S) consecutive index
        slots per token (kernel.cu:634-641, :686-687, :206-207);
      * per split: natural-log-domain online softmax over its valid keys,
        m_s = max logit, l_s = sum exp(logit - m_s), o_s = sum exp(logit - m_s)
        ckv (kernel.cu:307-388; computed here exactly, not in 4-key batches,
        which differs by rounding only); an empty split gives (-inf, 0, 0);
      * the fused reduce of the last-arriving split (kernel.cu:430-509) reads
        the per-split (m, l) with one lane per split, `lane_id <
        splits_per_token` over 32 lanes (:439-441, :452-456), so only splits
        0..31 enter m_global and l_global; the output loop runs over all S
        splits but takes each weight with __shfl_sync(.., scale_s, s_iter)
        (:475), which for s_iter >= 32 returns lane s_iter % 32's weight.
        With S <= 32 (N >= 5) this is the exact split-KV combine; with S > 32
        (N <= 4) splits 32.. are left out of l and lse and mis-weighted in the
        output.
    Returns (output bf16 [N,16,512], lse fp32 [N,16])."""
    n = q_nope.shape[0]
    S = reference_cuda_splits(n)
    kvps = (TOPK + S - 1) // S
    kc_all = ckv_cache.reshape(-1, CKV_DIM)
    kp_all = kpe_cache.reshape(-1, KPE_DIM)
    scale = torch.tensor(float(sm_scale), dtype=torch.float32)
    output = torch.zeros((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16)
    lse = torch.full((n, NUM_HEADS), float("-inf"), dtype=torch.float32)
    for t in range(n):
        idx = sparse_indices[t].to(torch.long)
        valid = idx.ne(-1)
        safe = torch.where(valid, idx, torch.zeros_like(idx))        # -1 reads row 0, then masked (:146-151)
        kc = kc_all.index_select(0, safe).float()
        kp = kp_all.index_select(0, safe).float()
        logits = (q_nope[t].float() @ kc.t() + q_pe[t].float() @ kp.t()) * scale    # [16, 2048]
        logits = torch.where(valid[None, :], logits, torch.full_like(logits, float("-inf")))
        pad = S * kvps - TOPK
        lg = torch.cat([logits, torch.full((NUM_HEADS, pad), float("-inf"))], 1).view(NUM_HEADS, S, kvps)
        vv = torch.cat([kc, torch.zeros((pad, CKV_DIM))], 0).view(S, kvps, CKV_DIM)
        m_s = lg.max(-1).values                                     # [16, S]
        safe_m = torch.where(torch.isinf(m_s), torch.zeros_like(m_s), m_s)
        p = torch.exp(lg - safe_m[..., None])                       # exp(-inf) = 0 for masked keys
        l_s = p.sum(-1)                                             # [16, S]
        o_s = torch.einsum("hsk,skd->hsd", p, vv)                   # [16, S, 512]
        lanes = min(S, 32)
        m_g = m_s[:, :lanes].max(-1).values                         # :439-446
        w = torch.where(torch.isinf(m_g)[:, None], torch.zeros((NUM_HEADS, lanes)),
                        torch.exp(m_s[:, :lanes] - m_g[:, None]))   # :452-456 (exp(-inf) = 0)
        l_g = (l_s[:, :lanes] * w).sum(-1)                          # :457-461
        wt = w[:, [s % 32 for s in range(S)]]                       # __shfl_sync wraps lanes (:475)
        o = (wt[..., None] * o_s).sum(1)                            # :474-492
        empty = l_g == 0
        inv_l = torch.where(empty, torch.zeros_like(l_g), 1.0 / l_g)
        output[t] = (o * inv_l[:, None]).to(torch.bfloat16)       # :496-507
        lse[t] = torch.where(empty, torch.full_like(l_g, float("-inf")),
                             m_g * 1.4426950408889634 + torch.log2(l_g))   # :508-510
    return output, lse


def compact_pool(ckv_cache, kpe_cache, sparse_indices):
    """Gather only the rows the indices touch into a dense pool and remap the
    indices onto it (-1 stays -1).  Result-identical input for the oracle when
    the real pool is too large for host memory; returns
    (ckv [R,1,512]... as [ceil(R/64),64,512], kpe likewise, remapped indices)."""
    idx = sparse_indices.to(torch.long)
    valid = idx.ne(-1)
    uniq, inv = torch.unique(idx[valid], return_inverse=True)
    rows = uniq.numel()
    pages = max(1, (rows + PAGE_SIZE - 1) // PAGE_SIZE)
    kc_all = ckv_cache.reshape(-1, CKV_DIM)
    kp_all = kpe_cache.reshape(-1, KPE_DIM)
    ckv = torch.zeros((pages * PAGE_SIZE, CKV_DIM), dtype=ckv_cache.dtype, device=ckv_cache.device)
    kpe = torch.zeros((pages * PAGE_SIZE, KPE_DIM), dtype=kpe_cache.dtype, device=kpe_cache.device)
    ckv[:rows] = kc_all.index_select(0, uniq)
    kpe[:rows] = kp_all.index_select(0, uniq)
    remap = torch.full_like(idx, -1)
    remap[valid] = inv
    return (ckv.view(pages, PAGE_SIZE, CKV_DIM), kpe.view(pages, PAGE_SIZE, KPE_DIM),
            remap.to(torch.int32))


def translate_block_table(block_table, positions, num_pages, seq_of_token=None):
    """Positions within each token's sequence -> flat slot ids, the
    translation the reference runs as its own step after top-k selection
    (methodology/reference/topk_kernel_naive.cu:52-62, with phys_idx = the
    sequence's block_table row, :96-109): slot = block_table[row][pos >> 6] * 64
    + (pos & 63), row = seq_of_token[t] (t when None).

    The reference translates only selected positions of valid sequences; this
    restatement also defines the other inputs the library accepts: -1 stays
    padding, and a position outside the row, a row outside the table or a page
    outside [0, num_pages) becomes -1 as well (the library reports those as bad
    indices).  Returns (slots int32 [N, 2048], bad bool [N, 2048])."""
    pos = positions.to(torch.int64).cpu()
    bt = block_table.to(torch.int64).cpu()
    n = pos.shape[0]
    rows = (torch.arange(n, dtype=torch.int64) if seq_of_token is None
            else seq_of_token.to(torch.int64).cpu())
    row_ok = (rows >= 0) & (rows < bt.shape[0])
    pidx = pos >> 6
    in_row = (pos >= 0) & (pidx < bt.shape[1]) & row_ok[:, None]
    page = torch.full_like(pos, -1)
    r = rows.clamp(0, bt.shape[0] - 1)[:, None].expand_as(pos)
    page[in_row] = bt[r[in_row], pidx[in_row]]
    ok = in_row & (page >= 0) & (page < num_pages)
    slots = torch.where(ok, page * PAGE_SIZE + (pos & (PAGE_SIZE - 1)), torch.full_like(pos, -1))
    bad = (~ok) & (pos != -1)
    return slots.to(torch.int32), bad
