"""The indexer's calibrated score plan: the score kernel's tile ranges come
from the previous call's measured CTA rates, and any partition of the tiles
must give bitwise the same scores, hence the same top-k.

The plan lives at the end of the indexer workspace (16-byte aligned after the
rows' key ranges): a header (magic, tiles, grid, 0), then grid + 1 uint32
bounds.  These tests read it, and write partitions of their own into it, to
cover ranges the calibration would not produce (empty CTAs, one CTA with
every tile).
"""
import pytest
import torch

from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")
MAGIC = 0x4E414C50
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
    tiles, grid = launch_shape(w)
    for i in range(6):
        out = run(dsa, w)
        assert torch.equal(out, ref), f"call {i}: the planned split changed the result"
        hdr = plan_words(dsa, w, grid + 1)
        h = hdr[:4].tolist()
        assert h[0] == MAGIC and h[1] == tiles and h[2] == grid, h
        b = hdr[4:4 + grid + 1].long()
        assert int(b[0]) == 0 and int(b[-1]) == tiles
        assert torch.all(b[1:] >= b[:-1])


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
    tiles, grid = launch_shape(w)
    g = torch.Generator().manual_seed(3)
    cuts = torch.sort(torch.randint(0, tiles + 1, (grid - 1,), generator=g)).values
    parts = {
        "first_takes_all": [0] + [tiles] * grid,
        "last_takes_all": [0] * grid + [tiles],
        "every_other_empty": [min(tiles, 2 * (i // 2) * tiles // grid) for i in range(grid)] + [tiles],
        "random": [0] + cuts.tolist() + [tiles],
        "shifted": [0] + [min(tiles, (i * tiles) // grid + 3) for i in range(1, grid)] + [tiles],
    }
    for name, bounds in parts.items():
        assert len(bounds) == grid + 1 and all(a <= b for a, b in zip(bounds, bounds[1:]))
        words = plan_words(dsa, w, grid + 1)
        words[:4] = torch.tensor([MAGIC, tiles, grid, 0], dtype=torch.int32)
        words[4:4 + grid + 1] = torch.tensor(bounds, dtype=torch.int32)
        out = run(dsa, w)
        assert torch.equal(out, ref), f"partition {name} changed the result"


def test_plan_of_another_shape_is_not_used(dsa, plan_switch):
    """Shapes alternating on one workspace: each call's plan is tagged with
    its tile count and grid, and a call of another shape takes the equal
    split; results stay bitwise those of the first call of each shape."""
    plan_switch(1)
    shapes = [W.indexer_small(device="cuda"), W.indexer_edges(device="cuda"),
              W.indexer_decode(batch=4, seq_len=4096, device="cuda")]
    first = [run(dsa, w) for w in shapes]
    for _ in range(3):
        for w, f in zip(shapes, first):
            assert torch.equal(run(dsa, w), f)
            assert torch.equal(run(dsa, w), f)
