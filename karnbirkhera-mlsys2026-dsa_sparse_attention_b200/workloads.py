"""Seeded synthetic inputs for the five benchmark configurations.

The reference's own workloads (23 decode cases, num_tokens 1..8) live in an
external dataset that is not available; these generators stand in for it with
the shapes, value distributions and index patterns the benchmark
configurations name.  Everything is drawn from a seeded torch.Generator on the
requested device, so a (config, seed, device type) triple always yields the
same tensors.

  cfg 1  4 tokens, 128-page pool, indices uniform without replacement over 8192 slots
  cfg 2  64 tokens, one 512-page sequence each, pages = a permutation of a 32768-page pool
  cfg 3  128 tokens, context ~ U[256, 4096], short rows padded with -1
  cfg 4  4096 tokens over one 131072-slot cache, token t draws from [0, 2048+t), half from the last 4096
  cfg 5  1024 tokens = 256 sequences x 4, 131072 slots per sequence, ~60% of a sequence's indices shared

Values are N(0,1) in bf16; sm_scale = 1/sqrt(192).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

NUM_HEADS = 16
CKV_DIM = 512
KPE_DIM = 64
PAGE_SIZE = 64
TOPK = 2048
SM_SCALE = 1.0 / math.sqrt(192.0)
BYTES_PER_KEY = (CKV_DIM + KPE_DIM) * 2           # 1152 gathered bytes per valid index
FLOPS_PER_KEY = NUM_HEADS * (CKV_DIM + KPE_DIM + CKV_DIM) * 2   # 34816


@dataclass
class Workload:
    name: str
    q_nope: torch.Tensor
    q_pe: torch.Tensor
    ckv_cache: torch.Tensor
    kpe_cache: torch.Tensor
    sparse_indices: torch.Tensor
    sm_scale: float = SM_SCALE
    meta: dict = field(default_factory=dict)

    @property
    def num_tokens(self) -> int:
        return self.q_nope.shape[0]

    @property
    def num_pages(self) -> int:
        return self.ckv_cache.shape[0]

    def valid_keys(self) -> int:
        """Number of non-padding index slots (the algorithmic gather count)."""
        return int((self.sparse_indices != -1).sum().item())

    def gathered_bytes(self) -> int:
        return self.valid_keys() * BYTES_PER_KEY

    def flops(self) -> int:
        return self.valid_keys() * FLOPS_PER_KEY

    def args(self):
        return (self.q_nope, self.q_pe, self.ckv_cache, self.kpe_cache, self.sparse_indices, self.sm_scale)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(int(seed))
    return g


def randn_bf16(shape, gen: torch.Generator, device, chunk: int = 1 << 27) -> torch.Tensor:
    """N(0,1) bf16 tensor, generated in chunks so huge pools never need an
    fp32 copy of the whole tensor."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    flat = out.view(-1)
    for s in range(0, flat.numel(), chunk):
        e = min(flat.numel(), s + chunk)
        flat[s:e] = torch.randn(e - s, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    return out


def _queries(n: int, gen, device):
    return randn_bf16((n, NUM_HEADS, CKV_DIM), gen, device), randn_bf16((n, NUM_HEADS, KPE_DIM), gen, device)


def _cache(pages: int, gen, device):
    return randn_bf16((pages, PAGE_SIZE, CKV_DIM), gen, device), randn_bf16((pages, PAGE_SIZE, KPE_DIM), gen, device)


def sample_without_replacement(rows: int, n: int, k: int, gen, device) -> torch.Tensor:
    """[rows, k] int64: for each row, k distinct values of [0, n) in random order."""
    keys = torch.rand((rows, n), generator=gen, device=device)
    return keys.topk(k, dim=1).indices


def translate(page_table: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Sequence positions -> global slot ids through a page table
    ([rows, pages_per_seq] -> slot = page_table[pos // 64] * 64 + pos % 64)."""
    pages = torch.gather(page_table, 1, positions // PAGE_SIZE)
    return (pages * PAGE_SIZE + positions % PAGE_SIZE).to(torch.int32)


def make_uniform(num_tokens: int, num_pages: int, seed: int = 0, device="cpu", pad: int = 0,
                 name: str = "uniform") -> Workload:
    """Generic case: indices uniform without replacement over the whole pool.
    If the pool has fewer than 2048 slots every slot is taken once and the row
    is padded with -1; `pad` extra trailing slots of each row are set to -1."""
    g = _gen(seed, device)
    q_nope, q_pe = _queries(num_tokens, g, device)
    ckv, kpe = _cache(num_pages, g, device)
    slots = num_pages * PAGE_SIZE
    take = min(TOPK, slots)
    idx = torch.full((num_tokens, TOPK), -1, dtype=torch.int32, device=device)
    if num_tokens:
        idx[:, :take] = sample_without_replacement(num_tokens, slots, take, g, device).to(torch.int32)
    if pad:
        idx[:, TOPK - pad:] = -1
    return Workload(name, q_nope, q_pe, ckv, kpe, idx, SM_SCALE, {"seed": seed})


def config1(seed: int = 1, device="cpu") -> Workload:
    w = make_uniform(4, 128, seed=seed, device=device, name="cfg1_decode_n4_p128")
    w.meta.update(config=1)
    return w


def config2(seed: int = 2, device="cpu", num_tokens: int = 64, pages_per_seq: int = 512,
            pool_pages: int | None = None) -> Workload:
    """One sequence per token; the pool's pages are a random permutation shared
    out 512 per sequence (pool_pages defaults to num_tokens * 512 = 32768)."""
    g = _gen(seed, device)
    pool = pool_pages if pool_pages is not None else num_tokens * pages_per_seq
    if pool < num_tokens * pages_per_seq:
        # reduced pool for profiling: sequences reuse pages cyclically
        table = torch.randperm(pool, generator=g, device=device)
        table = table.repeat((num_tokens * pages_per_seq + pool - 1) // pool)[: num_tokens * pages_per_seq]
    else:
        table = torch.randperm(pool, generator=g, device=device)[: num_tokens * pages_per_seq]
    table = table.view(num_tokens, pages_per_seq)
    q_nope, q_pe = _queries(num_tokens, g, device)
    ckv, kpe = _cache(pool, g, device)
    pos = sample_without_replacement(num_tokens, pages_per_seq * PAGE_SIZE, TOPK, g, device)
    idx = translate(table, pos)
    # page-table-native form of the same problem: token t reads row t
    return Workload("cfg2_decode_n64_seq32k", q_nope, q_pe, ckv, kpe, idx, SM_SCALE,
                    {"config": 2, "seed": seed, "pool_pages": pool,
                     "block_table": table.to(torch.int32).contiguous(), "positions": pos.to(torch.int32).contiguous(),
                     "seq_of_token": None})


def decode_batches(w: Workload, count: int, seed: int = 0):
    """`count` further decode batches over a config-2 workload's pool: fresh
    queries and fresh positions of each token's own sequence, mapped through
    the workload's page table.  Returns [(q_nope, q_pe, sparse_indices)]."""
    table = w.meta["block_table"].long()
    device = w.q_nope.device
    g = _gen(seed, device)
    out = []
    for _ in range(count):
        q_nope, q_pe = _queries(w.num_tokens, g, device)
        pos = sample_without_replacement(w.num_tokens, table.shape[1] * PAGE_SIZE, TOPK, g, device)
        out.append((q_nope, q_pe, translate(table, pos)))
    return out


def config3(seed: int = 3, device="cpu", num_tokens: int = 128) -> Workload:
    g = _gen(seed, device)
    ctx = torch.randint(256, 4097, (num_tokens,), generator=g, device=device)
    pages = (ctx + PAGE_SIZE - 1) // PAGE_SIZE
    pool = int(pages.sum().item())
    perm = torch.randperm(pool, generator=g, device=device)
    q_nope, q_pe = _queries(num_tokens, g, device)
    ckv, kpe = _cache(pool, g, device)
    idx = torch.full((num_tokens, TOPK), -1, dtype=torch.int32, device=device)
    off = 0
    for t in range(num_tokens):
        c = int(ctx[t].item())
        p = int(pages[t].item())
        table = perm[off:off + p].view(1, p)
        off += p
        take = min(c, TOPK)
        pos = sample_without_replacement(1, c, take, g, device)
        idx[t, :take] = translate(table, pos)[0]
    return Workload("cfg3_ragged_n128", q_nope, q_pe, ckv, kpe, idx, SM_SCALE,
                    {"config": 3, "seed": seed, "ctx": ctx.tolist()})


def config4(seed: int = 4, device="cpu", num_tokens: int = 4096, cache_tokens: int = 131072) -> Workload:
    """Prefill-shaped chunk: token t draws 2048 distinct positions from
    [0, 2048+t), min(1024, #old) of them from the positions older than the
    last 4096 and the rest from the last 4096."""
    g = _gen(seed, device)
    pages = cache_tokens // PAGE_SIZE
    table = torch.randperm(pages, generator=g, device=device).view(1, pages)
    q_nope, q_pe = _queries(num_tokens, g, device)
    ckv, kpe = _cache(pages, g, device)
    t = torch.arange(num_tokens, device=device)
    w = TOPK + t                                   # visible positions per token
    win_start = (w - 4096).clamp(min=0)            # start of the recent window
    n_old = win_start.clamp(max=1024)
    span = TOPK + num_tokens
    pos = torch.arange(span, device=device).view(1, span)
    keys = torch.rand((num_tokens, span), generator=g, device=device)
    recent_keys = torch.where((pos >= win_start.view(-1, 1)) & (pos < w.view(-1, 1)), keys, -1.0)
    old_keys = torch.where(pos < win_start.view(-1, 1), keys, -1.0)
    recent = recent_keys.topk(TOPK, dim=1).indices
    old = old_keys.topk(1024, dim=1).indices
    # row: the first (2048 - n_old) recent picks, then n_old old picks
    j = torch.arange(TOPK, device=device).view(1, TOPK)
    n_recent = (TOPK - n_old).view(-1, 1)
    old_part = torch.gather(old, 1, (j - n_recent).clamp(min=0, max=1023))
    chosen = torch.where(j < n_recent, recent, old_part)
    idx = translate(table.expand(num_tokens, pages), chosen)
    return Workload("cfg4_prefill_n4096_cache128k", q_nope, q_pe, ckv, kpe, idx, SM_SCALE,
                    {"config": 4, "seed": seed, "page_table": table[0]})


CFG5_SEQS = 256
CFG5_TOKENS_PER_SEQ = 4
CFG5_SEQ_TOKENS = 131072
CFG5_SHARED = 1229     # ~60% of 2048


def config5(seed: int = 5, device="cpu", seq_begin: int = 0, seq_end: int = CFG5_SEQS,
            seq_tokens: int = CFG5_SEQ_TOKENS) -> Workload:
    """Batch-sharded decode.  Sequences [seq_begin, seq_end) of the 256; each
    sequence's pages, queries and positions come from a generator seeded by
    (seed, sequence id), so any sharding of the sequences over ranks produces
    exactly the same per-token problems.  The local pool holds only the
    selected sequences' pages (a random permutation of them)."""
    nseq = seq_end - seq_begin
    pps = seq_tokens // PAGE_SIZE
    pool = nseq * pps
    gl = _gen(seed * 1000003 + seq_begin, device)
    table = torch.randperm(pool, generator=gl, device=device).view(nseq, pps)
    ckv = torch.empty((pool, PAGE_SIZE, CKV_DIM), dtype=torch.bfloat16, device=device)
    kpe = torch.empty((pool, PAGE_SIZE, KPE_DIM), dtype=torch.bfloat16, device=device)
    n = nseq * CFG5_TOKENS_PER_SEQ
    q_nope = torch.empty((n, NUM_HEADS, CKV_DIM), dtype=torch.bfloat16, device=device)
    q_pe = torch.empty((n, NUM_HEADS, KPE_DIM), dtype=torch.bfloat16, device=device)
    idx = torch.empty((n, TOPK), dtype=torch.int32, device=device)
    positions = torch.empty((n, TOPK), dtype=torch.int32, device=device)
    for i, s in enumerate(range(seq_begin, seq_end)):
        g = _gen(seed * 7919 + s, device)
        c, k = _cache(pps, g, device)           # this sequence's pages, in sequence order
        ckv[table[i]] = c
        kpe[table[i]] = k
        a, b = i * CFG5_TOKENS_PER_SEQ, (i + 1) * CFG5_TOKENS_PER_SEQ
        q_nope[a:b], q_pe[a:b] = _queries(CFG5_TOKENS_PER_SEQ, g, device)
        shared = sample_without_replacement(1, seq_tokens, CFG5_SHARED, g, device)
        keys = torch.rand((CFG5_TOKENS_PER_SEQ, seq_tokens), generator=g, device=device)
        keys[:, shared[0]] = -1.0
        own = keys.topk(TOPK - CFG5_SHARED, dim=1).indices
        pos = torch.cat([shared.expand(CFG5_TOKENS_PER_SEQ, -1), own], dim=1)
        idx[a:b] = translate(table[i:i + 1].expand(CFG5_TOKENS_PER_SEQ, pps), pos)
        positions[a:b] = pos.to(torch.int32)
    # page-table-native form: local sequence i is block-table row i, shared by its 4 tokens
    seq_of_token = torch.arange(nseq, dtype=torch.int32, device=device).repeat_interleave(CFG5_TOKENS_PER_SEQ)
    return Workload("cfg5_sharded_decode_n1024", q_nope, q_pe, ckv, kpe, idx, SM_SCALE,
                    {"config": 5, "seed": seed, "seq_begin": seq_begin, "seq_end": seq_end,
                     "seq_tokens": seq_tokens, "block_table": table.to(torch.int32).contiguous(),
                     "positions": positions, "seq_of_token": seq_of_token})


def make_config(cfg: int, device="cpu", seed: int | None = None, **kw) -> Workload:
    fns = {1: config1, 2: config2, 3: config3, 4: config4, 5: config5}
    fn = fns[int(cfg)]
    if seed is None:
        return fn(device=device, **kw)
    return fn(seed=seed, device=device, **kw)


# ---------------------------------------------------------------------------
# DSA top-k indexer (dsa_topk_indexer_fp8_h64_d128_topk2048_ps64), the operator
# that produces sparse_indices upstream.  Seeded synthetic inputs of the
# definition's shapes: fp8 e4m3 queries [B, 64, 128] and index keys, pages of
# 8448 bytes (64 rows x 128 fp8, then the 64 rows' fp32 scales), fp32 head
# weights [B, 64], int32 seq_lens [B] and block_table [B, max_pages].
# ---------------------------------------------------------------------------
IDX_HEADS = 64
IDX_DIM = 128
IDX_PAGE_BYTES = 8448
IDX_PAGE_DATA_BYTES = 8192


@dataclass
class IndexerWorkload:
    name: str
    q_index_fp8: torch.Tensor     # uint8 [B, 64, 128] (fp8 e4m3 bytes)
    k_index_cache: torch.Tensor   # uint8 [pages, 8448]
    weights: torch.Tensor         # fp32 [B, 64]
    seq_lens: torch.Tensor        # int32 [B]
    block_table: torch.Tensor     # int32 [B, max_pages]
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return self.q_index_fp8.shape[0]

    def args(self):
        return (self.q_index_fp8, self.k_index_cache, self.weights, self.seq_lens, self.block_table)

    def key_bytes(self) -> int:
        """Index-key bytes one call must read: 132 bytes per position in range."""
        return int(self.seq_lens.clamp(min=0).sum().item()) * (IDX_DIM + 4)


def _fp8_bytes(shape, gen, device, scale=1.0) -> torch.Tensor:
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * scale
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def make_indexer(seq_lens, max_pages: int, seed: int = 0, device="cpu", pool_pages: int | None = None,
                 name: str = "indexer") -> IndexerWorkload:
    """Row b's pages are a random slice of a permuted pool (pool_pages defaults
    to batch * max_pages, so rows own disjoint pages); block-table entries past
    a row's seq_len point into the pool too (the operator must not use them)."""
    g = _gen(seed, device)
    sl = torch.as_tensor(seq_lens, dtype=torch.int32, device=device)
    B = sl.shape[0]
    pool = pool_pages if pool_pages is not None else B * max_pages
    perm = torch.randperm(pool, generator=g, device=device)
    table = perm.repeat((B * max_pages + pool - 1) // pool)[: B * max_pages].view(B, max_pages).to(torch.int32)
    q = _fp8_bytes((B, IDX_HEADS, IDX_DIM), g, device)
    cache = torch.empty((pool, IDX_PAGE_BYTES), dtype=torch.uint8, device=device)
    cache[:, :IDX_PAGE_DATA_BYTES] = _fp8_bytes((pool, IDX_PAGE_DATA_BYTES), g, device)
    scales = torch.rand((pool, PAGE_SIZE), generator=g, device=device) * 0.2 + 0.05
    cache[:, IDX_PAGE_DATA_BYTES:] = scales.contiguous().view(torch.uint8).view(pool, -1)
    w = torch.randn((B, IDX_HEADS), generator=g, device=device) * 0.1
    return IndexerWorkload(name, q, cache, w, sl, table.contiguous(),
                           {"seed": seed, "max_pages": max_pages, "pool_pages": pool})


def indexer_small(seed: int = 11, device="cpu") -> IndexerWorkload:
    """CPU-runnable case: 4 rows of 1000..8192 positions."""
    return make_indexer([1000, 2048, 5000, 8192], 128, seed=seed, device=device, name="indexer_small")


def indexer_edges(seed: int = 12, device="cpu") -> IndexerWorkload:
    """Sequence lengths at every boundary: empty, one position, page and tile
    edges, fewer / exactly / more than 2048 positions."""
    return make_indexer([0, 1, 63, 64, 65, 127, 128, 129, 2047, 2048, 2049, 4097], 72, seed=seed, device=device,
                        name="indexer_edges")


def indexer_long(seed: int = 14, device="cpu") -> IndexerWorkload:
    """Rows longer than the top-k kernel keeps in shared memory (32768
    positions): 40000 and 70000 positions in 1100-page tables."""
    return make_indexer([40000, 70000], 1100, seed=seed, device=device, name="indexer_long")


def indexer_ties(seed: int = 15, device="cpu") -> IndexerWorkload:
    """Exact ties at the selection threshold: pages whose keys are all zero
    score exactly 0 (weights are non-negative).
      row 0: 2880 positions, 15 zero pages (960 zeros, 1920 positive): 128 of
             the zeros are selected -- the lowest positions;
      row 1: 4096 positions, 40 zero pages (2560 zeros): 512 zeros selected;
      row 2: 3000 positions with all-zero weights: positions 0..2047;
      row 3: 10000 positions with all-zero weights (more ties than the top-k
             kernel lists as candidates): positions 0..2047."""
    w = make_indexer([2880, 4096, 3000, 10000], 160, seed=seed, device=device, name="indexer_ties")
    w.weights.abs_()
    w.weights[2:].zero_()
    for row, first, count in ((0, 5, 15), (1, 3, 40)):
        pages = w.block_table[row, first:first + count].long()
        w.k_index_cache[pages, :IDX_PAGE_DATA_BYTES] = 0
    w.meta.update(zero_pages={0: (5, 15), 1: (3, 40)})
    return w


def indexer_ragged(seed: int = 16, device="cpu", batch: int = 64, max_len: int = 32768) -> IndexerWorkload:
    """Serving-batch decode with ragged sequences: 64 rows whose lengths are
    uniform in [1024, max_len] (seeded), in max_len-position block tables."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1024, max_len + 1, (batch,), generator=g).tolist()
    pages = (max_len + PAGE_SIZE - 1) // PAGE_SIZE
    return make_indexer(lens, pages, seed=seed, device=device, name=f"indexer_ragged_b{batch}_s{max_len // 1024}k")


def indexer_decode(seed: int = 13, device="cpu", batch: int = 64, seq_len: int = 32768) -> IndexerWorkload:
    """Serving-batch decode paired with attention config 2: 64 rows, each a
    32768-position sequence (512 pages) of a permuted 32768-page pool (277 MB)."""
    pages = (seq_len + PAGE_SIZE - 1) // PAGE_SIZE
    return make_indexer([seq_len] * batch, pages, seed=seed, device=device, name="indexer_decode_b64_s32k")
