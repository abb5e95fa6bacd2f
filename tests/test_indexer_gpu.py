"""GPU parity of the top-k indexer (dsa_topk_indexer_fwd) against the CPU oracle.

The selection is compared as sets of slot ids per row.  Scores are fp32 sums
over 64 heads whose rounding differs between the tensor-core fp8 products and
the oracle's fp32 matmul, so a position may swap with another only when both
scores lie within SCORE_TOL (relative to the row's largest |score|) of the
selection boundary; the returned order must be non-increasing in the oracle's
score within the same tolerance.  Rows with at most 2048 positions must
return every position.
"""
import pytest
import torch

from oracle.dsa_indexer_oracle import topk_indexer_oracle
from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")
SCORE_TOL = 2e-3


def to_dev(w):
    return W.IndexerWorkload(w.name, *(t.cuda() for t in w.args()), dict(w.meta))


def check_rows(out, ref, finals, w, rows=None):
    bt = w.block_table.cpu().long()
    out, ref = out.cpu(), ref.cpu()
    rows = range(out.shape[0]) if rows is None else rows
    swaps = 0
    for b in rows:
        sl = int(w.seq_lens[b])
        k = min(sl, 2048) if sl > 0 else 0
        assert torch.all(out[b, k:] == -1), f"row {b}: entries after {k} must be -1"
        if k == 0:
            continue
        got = out[b, :k]
        assert torch.all(got >= 0), f"row {b}: a selected entry is -1"
        # slot -> position through this row's table
        pos_of = {int(bt[b, pi]) * 64 + o: pi * 64 + o for pi in range((sl + 63) // 64) for o in range(64)}
        gpos = torch.tensor([pos_of[int(s)] for s in got])
        assert len(set(gpos.tolist())) == k, f"row {b}: duplicate selections"
        f = finals[b]
        scale = float(f.abs().max()) + 1e-30
        sc = f[gpos]
        # order: non-increasing within tolerance
        assert torch.all(sc[1:] <= sc[:-1] + SCORE_TOL * scale), f"row {b}: order is not by descending score"
        if k == sl:
            assert set(gpos.tolist()) == set(range(sl)), f"row {b}: short row must return every position"
            continue
        kth = torch.sort(f, descending=True).values[k - 1]
        rset = set(int(s) for s in ref[b, :k])
        for s, pos in zip(got.tolist(), gpos.tolist()):
            if s not in rset:
                swaps += 1
                assert abs(float(f[pos]) - float(kth)) <= SCORE_TOL * scale, \
                    f"row {b}: position {pos} (score {float(f[pos]):.5f}) is not near the boundary {float(kth):.5f}"
    return swaps


def test_small_rows_against_oracle(dsa):
    w = W.indexer_small()
    ref, finals = topk_indexer_oracle(*w.args())
    wd = to_dev(w)
    out = dsa.topk_indexer(*wd.args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    swaps = check_rows(out, ref, finals, w)
    assert swaps <= 4


def test_sequence_length_edges(dsa):
    """Empty rows, single positions, page and tile boundaries, 2047 / 2048 /
    2049 positions (short rows return everything, sorted)."""
    w = W.indexer_edges()
    ref, finals = topk_indexer_oracle(*w.args())
    out = dsa.topk_indexer(*to_dev(w).args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    check_rows(out, ref, finals, w)
    assert torch.all(out[0].cpu() == -1)


def test_decode_batch_sampled_rows(dsa):
    """The serving-size case (64 rows x 32768 positions): all rows run, 6 are
    checked against the oracle."""
    w = W.indexer_decode()
    rows = [0, 13, 27, 40, 51, 63]
    sub = W.IndexerWorkload(w.name, w.q_index_fp8[rows], w.k_index_cache, w.weights[rows], w.seq_lens[rows],
                            w.block_table[rows])
    ref, finals = topk_indexer_oracle(*sub.args())
    out = dsa.topk_indexer(*to_dev(w).args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    swaps = check_rows(out[rows], ref, finals, sub)
    assert swaps <= 6


def test_long_rows_keys_from_l2(dsa):
    """Rows past the shared-memory key capacity (40000 and 70000 positions)."""
    w = W.indexer_long()
    ref, finals = topk_indexer_oracle(*w.args())
    out = dsa.topk_indexer(*to_dev(w).args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    swaps = check_rows(out, ref, finals, w)
    assert swaps <= 4


def test_threshold_ties_take_lowest_positions(dsa):
    """Exact ties at the k-th score are broken by position, like the oracle's
    stable sort: the selected zero-score positions (the tail of each row)
    must be exactly the oracle's, in increasing position order."""
    w = W.indexer_ties()
    ref, finals = topk_indexer_oracle(*w.args())
    out = dsa.topk_indexer(*to_dev(w).args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    check_rows(out, ref, finals, w)
    out = out.cpu()
    for b, zeros_taken in ((0, 128), (1, 512), (2, 2048), (3, 2048)):
        n_zero = int((finals[b] == 0).sum())
        assert n_zero >= zeros_taken
        tail = slice(2048 - zeros_taken, 2048)
        assert torch.equal(out[b, tail], ref[b, tail]), f"row {b}: tied positions differ from the oracle's"


def test_bad_block_table_entries_reported(dsa):
    w = W.indexer_small()
    bt = w.block_table.clone()
    bt[1, 3] = w.k_index_cache.shape[0] + 5      # page outside the pool, inside row 1's 2048 positions
    bt[2, 10] = -7
    wd = to_dev(W.IndexerWorkload(w.name, w.q_index_fp8, w.k_index_cache, w.weights, w.seq_lens, bt))
    out = dsa.topk_indexer(*wd.args())
    torch.cuda.synchronize()
    with pytest.raises(dsa.DsaError) as ei:
        dsa.indexer.check_errors()
    assert "BAD_INDEX" in str(ei.value)
    assert dsa.indexer.check_errors() == 0
    o = out.cpu()
    # row 1 has 2048 positions: the 64 on the bad page are not returned
    assert int((o[1] >= 0).sum()) == 2048 - 64
    assert not torch.any((o[2] // 64) == -7)


def test_workspace_reused_across_shapes(dsa):
    """One cached workspace serves calls of different (batch, max_pages)
    shapes: the rows' key ranges move with the layout and must be cleared on
    a change (a stale range would only widen the bins, but the results must
    not depend on call history)."""
    for w in (W.indexer_small(), W.indexer_edges(), W.indexer_small(seed=21), W.indexer_ties()):
        ref, finals = topk_indexer_oracle(*w.args())
        out = dsa.topk_indexer(*to_dev(w).args())
        torch.cuda.synchronize()
        assert dsa.indexer.check_errors() == 0
        check_rows(out, ref, finals, w)
