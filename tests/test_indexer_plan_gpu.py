"""The indexer's score split: CTA g takes the active tiles (those with
positions) between the cumulative fractions frac[g] and frac[g + 1] of the
call's total, from the calibrated plan (the previous call's measured CTA
rates) or g / grid.  Any partition must give bitwise the same scores, hence
the same top-k.

The plan lives at the end of the indexer workspace (16-byte aligned after the
rows' key ranges): a header (magic, 0, grid, 0), then grid + 1 uint32
fractions of 2^31.  These tests read it, and write partitions of their own
into it, to cover splits the calibration would not produce (empty CTAs, one
CTA with every tile).
"""
import pytest
import torch

from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")
MAGIC = 0x4E414C50
ONE = 1 << 31
RECORDS = 256 + 1024 * 2 * 4   # workspace header + counter region


def plan_offset(batch, max_pages):
    row_keys = RECORDS + batch * max_pages * 64 * 4
    return (row_keys + batch * 8 + 15) & ~15


def launch_shape(w):
    """(tiles, grid) of the score launch: two pages per tile, two CTAs per SM."""
    batch, max_pages = w.block_table.shape
    tiles = batch * ((max_pages + 1) // 2)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return tiles, min(tiles, 2 * sms)


def plan_words(dsa, w, n):
    ws = dsa.indexer._workspaces[torch.cuda.current_device()]
    off = plan_offset(*w.block_table.shape)
    return ws[off:off + 16 + 4 * n].view(torch.int32)


def read_plan(dsa, w, grid):
    words = plan_words(dsa, w, grid + 1).cpu().long() & 0xffffffff
    return words[:4].tolist(), words[4:4 + grid + 1]


def write_plan(dsa, w, grid, frac):
    as_i32 = [f - (1 << 32) if f >= (1 << 31) else f for f in [MAGIC, 0, grid, 0] + list(frac)]
    plan_words(dsa, w, grid + 1)[:] = torch.tensor(as_i32, dtype=torch.int32)


def run(dsa, w):
    out = dsa.topk_indexer(*w.args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    return out


@pytest.fixture
def plan_switch(dsa):
    lib = dsa._lib.load()
    yield lib.dsa_topk_indexer_set_calibrated_plan
    lib.dsa_topk_indexer_set_calibrated_plan(1)


def ragged(n_rows, max_pages, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(0, max_pages * 64 + 1, (n_rows,), generator=g).tolist()
    return W.make_indexer(lens, max_pages, seed=seed, device="cuda", name=f"ragged{n_rows}")


@pytest.mark.parametrize("shape", ["uniform", "ragged", "ragged_long"])
def test_repeated_calls_bitwise_and_plan_valid(dsa, plan_switch, shape):
    """The first call takes the equal split, later ones the plan (rows up to
    32768 positions: the two-CTA top-k; longer: the one-CTA top-k, whose
    extra CTA updates the plan)."""
    w = {"uniform": lambda: W.indexer_decode(batch=16, seq_len=16384, device="cuda"),
         "ragged": lambda: ragged(40, 256, 31),
         "ragged_long": lambda: ragged(6, 1100, 32)}[shape]()
    plan_switch(0)
    ref = run(dsa, w)
    plan_switch(1)
    _, grid = launch_shape(w)
    for i in range(6):
        out = run(dsa, w)
        assert torch.equal(out, ref), f"call {i}: the planned split changed the result"
        h, f = read_plan(dsa, w, grid)
        assert h[0] == MAGIC and h[2] == grid, h
        assert int(f[0]) == 0 and int(f[-1]) == ONE
        assert torch.all(f[1:] >= f[:-1])


def test_any_partition_gives_the_same_result(dsa, plan_switch):
    """Partitions written into the plan: one CTA with every tile, every other
    CTA empty, a random monotone split, and the equal split shifted."""
    w = W.indexer_decode(batch=8, seq_len=8192, device="cuda")
    w.seq_lens[3] = 1000    # a ragged row among full ones
    w.seq_lens[5] = 0
    plan_switch(0)
    ref = run(dsa, w)
    plan_switch(1)
    run(dsa, w)   # lays out this shape's plan region
    _, grid = launch_shape(w)
    g = torch.Generator().manual_seed(3)
    cuts = torch.sort(torch.randint(0, ONE + 1, (grid - 1,), generator=g)).values
    parts = {
        "first_takes_all": [0] + [ONE] * grid,
        "last_takes_all": [0] * grid + [ONE],
        "every_other_empty": [2 * (i // 2) * ONE // grid for i in range(grid)] + [ONE],
        "random": [0] + cuts.tolist() + [ONE],
        "shifted": [0] + [min(ONE, i * ONE // grid + (1 << 20)) for i in range(1, grid)] + [ONE],
    }
    for name, frac in parts.items():
        assert len(frac) == grid + 1 and all(a <= b for a, b in zip(frac, frac[1:]))
        write_plan(dsa, w, grid, frac)
        out = run(dsa, w)
        assert torch.equal(out, ref), f"partition {name} changed the result"


def test_plan_carries_over_between_shapes(dsa, plan_switch):
    """Shapes alternating on one workspace: a plan made on one shape is used
    by the next call of any shape with the same grid (other grids take g /
    grid); results stay bitwise those of the first call of each shape."""
    plan_switch(1)
    shapes = [W.indexer_small(device="cuda"), W.indexer_edges(device="cuda"),
              W.indexer_decode(batch=4, seq_len=4096, device="cuda")]
    first = [run(dsa, w) for w in shapes]
    for _ in range(3):
        for w, f in zip(shapes, first):
            assert torch.equal(run(dsa, w), f)
            assert torch.equal(run(dsa, w), f)


def test_same_layout_new_lengths(dsa, plan_switch):
    """A plan made on ragged rows applied to full rows of the same table
    layout and back: the fractions are of each call's own active tiles, so
    every call is split over its own rows."""
    full = W.indexer_decode(batch=16, seq_len=16384, device="cuda")
    rag = ragged(16, 256, 33)
    plan_switch(0)
    refs = [run(dsa, full), run(dsa, rag)]
    plan_switch(1)
    for i in range(8):
        w = (full, rag)[i % 2]
        assert torch.equal(run(dsa, w), refs[i % 2]), f"call {i}"


@pytest.mark.parametrize("rows", [4096, 4100])
def test_many_rows_split(dsa, plan_switch, rows):
    """4096 rows: the largest batch split over active tiles (the rows'
    lengths fit a pipeline stage); 4100: the equal split of tile indices,
    no plan.  Sampled rows against the oracle, and bitwise the same with the
    plan on and off."""
    from oracle.dsa_indexer_oracle import topk_indexer_oracle
    from tests.test_indexer_gpu import check_rows
    g = torch.Generator().manual_seed(rows)
    lens = torch.randint(0, 129, (rows,), generator=g).tolist()
    w = W.make_indexer(lens, 2, seed=rows, device="cpu", name=f"rows{rows}")
    wd = W.IndexerWorkload(w.name, *(t.cuda() for t in w.args()), dict(w.meta))
    plan_switch(0)
    ref = run(dsa, wd)
    plan_switch(1)
    for _ in range(3):
        assert torch.equal(run(dsa, wd), ref)
    sample = [0, 1, 17, rows // 2, rows - 2, rows - 1]
    sub = W.IndexerWorkload(w.name, w.q_index_fp8[sample], w.k_index_cache, w.weights[sample], w.seq_lens[sample],
                            w.block_table[sample])
    ro, finals = topk_indexer_oracle(*sub.args())
    check_rows(ref[sample], ro, finals, sub)
