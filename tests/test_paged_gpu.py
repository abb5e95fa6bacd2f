"""GPU parity of the page-table-native entry point (dsa_sparse_attention_fwd_paged).

The paged form translates positions through a block table on the device.  It
must give exactly the results of the slot-id form on the translated slots
(the same rows reach the same kernel, so the comparison is bitwise), and the
oracle's result on those slots within the contest tolerance (output element
fails iff |err| > 1e-2 and |err| > 1e-2 * |ref|; lse within 1e-3).  The
translation itself is the oracle's restatement of the reference's translate
step (oracle/dsa_oracle.py: translate_block_table).
"""
import pytest
import torch

from oracle.dsa_oracle import compact_pool, sparse_attention_oracle, translate_block_table
from tests.conftest import assert_lse_close, assert_output_close, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")


def paged(dsa, w, block_table, positions, seq_of_token=None):
    out, lse = dsa.kernel_paged(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, block_table, positions, w.sm_scale,
                                seq_of_token=seq_of_token)
    torch.cuda.synchronize()
    return out, lse


def slot_ids(dsa, w, idx):
    out, lse = dsa.kernel(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, idx, w.sm_scale)
    torch.cuda.synchronize()
    return out, lse


def oracle(w, idx, tokens=None):
    sel = slice(None) if tokens is None else tokens
    ckv, kpe, idx_c = compact_pool(w.ckv_cache, w.kpe_cache, idx[sel])
    return sparse_attention_oracle(w.q_nope[sel].cpu(), w.q_pe[sel].cpu(), ckv.cpu(), kpe.cpu(), idx_c.cpu(),
                                   w.sm_scale)


def test_config2_paged_equals_slot_ids(dsa):
    """Benchmark config 2 (one 512-page sequence per token, pages a permutation
    of the pool): block table row t serves token t."""
    w = W.config2(device="cuda")
    bt, pos = w.meta["block_table"], w.meta["positions"]
    out_p, lse_p = paged(dsa, w, bt, pos)
    assert dsa.check_device_errors() == 0
    out_s, lse_s = slot_ids(dsa, w, w.sparse_indices)
    assert torch.equal(out_p, out_s) and torch.equal(lse_p, lse_s)
    sel = torch.arange(0, 64, 9)
    ro, rl = oracle(w, w.sparse_indices, sel)
    assert_output_close(out_p[sel], ro)
    assert_lse_close(lse_p[sel], rl)


def test_config5_row_map_shared_by_tokens(dsa):
    """Config 5 form: 4 tokens per sequence share one block-table row
    (seq_of_token), 16 sequences of 16384 positions."""
    w = W.config5(seq_begin=0, seq_end=16, seq_tokens=16384, device="cuda")
    m = w.meta
    out_p, lse_p = paged(dsa, w, m["block_table"], m["positions"], m["seq_of_token"])
    assert dsa.check_device_errors() == 0
    out_s, lse_s = slot_ids(dsa, w, w.sparse_indices)
    assert torch.equal(out_p, out_s) and torch.equal(lse_p, lse_s)
    ro, rl = oracle(w, w.sparse_indices)
    assert_output_close(out_p, ro)
    assert_lse_close(lse_p, rl)


def test_padding_and_bad_entries(dsa):
    """-1 padding, positions beyond a row, unmapped (-1) and out-of-pool pages,
    a token whose row is outside the table and a fully padded token: bad
    entries are masked like padding and reported as BAD_INDEX."""
    n, pages, max_pages = 7, 48, 40
    w = W.make_uniform(n, pages, seed=11, device="cuda")
    g = torch.Generator(device="cpu").manual_seed(11)
    bt = torch.stack([torch.randperm(pages, generator=g)[:max_pages] for _ in range(6)]).to(torch.int32)
    bt[1, 3] = -1                    # unmapped page
    bt[2, 5] = pages + 3             # page outside the pool
    pos = torch.stack([torch.randperm(max_pages * 64, generator=g)[:2048] for _ in range(n)]).to(torch.int32)
    pos[0, 100:900] = -1             # padding
    pos[3, 7] = max_pages * 64 + 5   # beyond the row
    pos[4, 9] = -3                   # negative, not the sentinel
    pos[5] = -1                      # fully padded token
    seq = torch.tensor([0, 1, 2, 3, 4, 5, 9], dtype=torch.int32)   # token 6: row 9 is outside the 6-row table
    slots, bad = translate_block_table(bt, pos, pages, seq)
    assert bad.any(dim=1).tolist() == [False, True, True, True, True, False, True]
    bt_d, pos_d, seq_d = bt.cuda(), pos.cuda(), seq.cuda()
    out_p, lse_p = paged(dsa, w, bt_d, pos_d, seq_d)
    with pytest.raises(dsa.DsaError) as ei:
        dsa.check_device_errors()
    assert "BAD_INDEX" in str(ei.value)
    assert dsa.check_device_errors() == 0
    out_s, lse_s = slot_ids(dsa, w, slots.cuda())
    assert dsa.check_device_errors() == 0
    assert torch.equal(out_p, out_s) and torch.equal(lse_p, lse_s)
    ro, rl = oracle(w, slots.cuda())
    assert_output_close(out_p, ro)
    assert_lse_close(lse_p, rl)
    assert torch.all(out_p[5] == 0) and torch.all(torch.isneginf(lse_p[5]))
    assert torch.all(out_p[6] == 0) and torch.all(torch.isneginf(lse_p[6]))


@pytest.mark.parametrize("n", [1, 3, 9, 17, 150])
def test_paged_plan_shapes(dsa, n):
    """Token counts that give every plan shape (tokens over many CTAs, CTAs
    over several tokens, the two-block-ahead prefetch crossing token ends)."""
    pages, max_pages = 48, 32
    w = W.make_uniform(n, pages, seed=300 + n, device="cuda")
    g = torch.Generator(device="cpu").manual_seed(n)
    rows = max(1, n // 2)
    bt = torch.stack([torch.randperm(pages, generator=g)[:max_pages] for _ in range(rows)]).to(torch.int32)
    pos = torch.stack([torch.randperm(max_pages * 64, generator=g)[:2048] for _ in range(n)]).to(torch.int32)
    pos[:, -(n * 13) % 700:] = -1
    seq = (torch.arange(n) % rows).to(torch.int32)
    slots, bad = translate_block_table(bt, pos, pages, seq)
    assert not bad.any()
    out_p, lse_p = paged(dsa, w, bt.cuda(), pos.cuda(), seq.cuda())
    assert dsa.check_device_errors() == 0
    out_s, lse_s = slot_ids(dsa, w, slots.cuda())
    assert torch.equal(out_p, out_s) and torch.equal(lse_p, lse_s)
