"""Properties of the seeded benchmark generators (CPU, reduced sizes where the
full configuration is too large for a unit test)."""
import torch

from tests.conftest import submodule

W = submodule("workloads")


def _rows_unique(idx):
    for r in idx:
        v = r[r != -1]
        assert v.unique().numel() == v.numel(), "indices must be drawn without replacement"


def test_config1_shape_and_range():
    w = W.config1()
    assert tuple(w.q_nope.shape) == (4, 16, 512) and tuple(w.q_pe.shape) == (4, 16, 64)
    assert tuple(w.ckv_cache.shape) == (128, 64, 512) and tuple(w.kpe_cache.shape) == (128, 64, 64)
    assert w.sparse_indices.dtype == torch.int32 and tuple(w.sparse_indices.shape) == (4, 2048)
    assert int(w.sparse_indices.min()) >= 0 and int(w.sparse_indices.max()) < 8192
    _rows_unique(w.sparse_indices)
    assert abs(w.sm_scale - 192 ** -0.5) < 1e-12
    assert w.gathered_bytes() == 4 * 2048 * 1152


def test_generators_are_deterministic():
    a, b = W.config1(), W.config1()
    for k in ("q_nope", "q_pe", "ckv_cache", "kpe_cache", "sparse_indices"):
        assert torch.equal(getattr(a, k), getattr(b, k))
    assert not torch.equal(W.config1(seed=99).sparse_indices, a.sparse_indices)


def test_config2_sequences_own_their_pages():
    w = W.config2(num_tokens=8, pages_per_seq=32)
    idx = w.sparse_indices.long()
    pages = idx // 64
    _rows_unique(w.sparse_indices)
    seen = [set(p.tolist()) for p in pages]
    for i in range(len(seen)):
        assert len(seen[i]) <= 32
        for j in range(i):
            assert not (seen[i] & seen[j]), "each token reads only its own sequence's pages"


def test_config3_ragged_padding():
    w = W.config3(num_tokens=16)
    ctx = w.meta["ctx"]
    for t, c in enumerate(ctx):
        row = w.sparse_indices[t]
        nvalid = int((row != -1).sum())
        assert nvalid == min(c, 2048)
        assert bool((row[:nvalid] != -1).all()) and bool((row[nvalid:] == -1).all())
    _rows_unique(w.sparse_indices)


def test_config4_causal_local_heavy():
    n = 3000
    w = W.config4(num_tokens=n, cache_tokens=8192)
    _rows_unique(w.sparse_indices)
    assert w.valid_keys() == n * 2048
    table = w.meta["page_table"].long()
    inv = torch.empty_like(table)
    inv[table] = torch.arange(table.numel())
    slots = w.sparse_indices.long()
    pos = inv[slots // 64] * 64 + slots % 64
    t = torch.arange(n).view(-1, 1)
    assert bool((pos < 2048 + t).all()), "token t only sees positions < 2048 + t"
    recent = (pos >= (2048 + t - 4096)).sum(dim=1)
    assert bool((recent >= 1024).all()), "at least half of the picks come from the last 4096 positions"
    assert int(recent[-1]) == 2048 - min(1024, 2048 + n - 1 - 4096)


def test_config5_sharing_and_sharding_identity():
    sh = submodule("sharding")
    full = W.config5(seq_begin=0, seq_end=4, seq_tokens=4096)
    assert full.num_tokens == 16
    idx = full.sparse_indices.long()
    inter = len(set(idx[0].tolist()) & set(idx[1].tolist()))
    # 1229 shared picks, plus chance overlap of the two tokens' 819 own picks
    # among the remaining 4096-1229 positions (~234 expected at this reduced size)
    chance = 819 * 819 / (4096 - 1229)
    assert 1229 <= inter <= 1229 + 1.5 * chance, f"tokens of one sequence share ~60% of indices, got {inter}"
    parts = [sh.shard_config5(2, r, num_seqs=4, seq_tokens=4096) for r in range(2)]
    assert sum(p.num_tokens for p in parts) == 16
    # queries are identical regardless of the sharding
    assert torch.equal(torch.cat([p.q_nope for p in parts]), full.q_nope)
    # gathered rows are identical (slot ids differ, data does not)
    for r, p in enumerate(parts):
        a = r * 8
        rows_local = p.ckv_cache.reshape(-1, 512)[p.sparse_indices.long()]
        rows_full = full.ckv_cache.reshape(-1, 512)[full.sparse_indices[a:a + 8].long()]
        assert torch.equal(rows_local, rows_full)


def test_row_range_partitions():
    sh = submodule("sharding")
    for n in (1, 7, 64, 256, 1024):
        for world in (1, 2, 3, 4, 8):
            spans = [sh.row_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b


def test_block_table_form_translates_to_the_slot_ids():
    """Configs 2 and 5 also carry their page-table-native form (block table,
    positions, row of each token); translating it with the oracle's restatement
    of the reference's translate step gives exactly the slot ids."""
    from oracle.dsa_oracle import translate_block_table
    for w in (W.config2(num_tokens=8, pages_per_seq=32), W.config5(seq_begin=3, seq_end=7, seq_tokens=4096)):
        m = w.meta
        slots, bad = translate_block_table(m["block_table"], m["positions"], w.num_pages, m["seq_of_token"])
        assert not bad.any()
        assert torch.equal(slots, w.sparse_indices)


def test_decode_batches_stay_in_each_tokens_sequence():
    """The benchmark's rotating decode batches draw fresh distinct positions of
    each token's own sequence and map them through the workload's page table."""
    w = W.config2(num_tokens=4, pages_per_seq=32, pool_pages=128)
    batches = W.decode_batches(w, 2, seed=3)
    table = w.meta["block_table"]
    for q_nope, q_pe, idx in batches:
        assert q_nope.shape == w.q_nope.shape and q_pe.shape == w.q_pe.shape
        assert idx.shape == (4, 2048) and idx.dtype == torch.int32
        for r in range(4):
            pages = set(table[r].tolist())
            assert all(int(x) // 64 in pages for x in idx[r])
            assert len(set(idx[r].tolist())) == 2048
    assert not torch.equal(batches[0][2], batches[1][2])
