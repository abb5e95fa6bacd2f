"""Host-side checks of the static work plan (csrc/dsa_common.cuh).

The kernel computes the plan's floor divisions in double precision
(`plan_div`), the host in 64-bit integers.  These tests restate both in
Python (numpy float64 division is IEEE correctly rounded, like the GPU's
div.rn.f64) and check that they agree over the whole argument range the host
accepts (num_tokens <= 2^24, grid <= 1024), and that the plan's ranges tile
the blocks, so every CTA boundary maps to the right owner.
"""
import numpy as np
import pytest

BLOCKS_PER_TOKEN = 16
MAX_TOKENS = 1 << 24
MAX_GRID = 1024


def div_device(num, den):
    return np.floor(np.asarray(num, dtype=np.int64).astype(np.float64) /
                    np.float64(den)).astype(np.int64)


def range_begin(b, total, grid):
    return (np.asarray(b, dtype=np.int64) * total) // grid


def owner(g, total, grid):
    return ((np.asarray(g, dtype=np.int64) + 1) * grid - 1) // total


@pytest.mark.parametrize("tokens,grid", [(1, 16), (4, 64), (9, 144), (64, 148), (128, 148), (300, 148),
                                         (4096, 148), (1 << 20, 1024), (MAX_TOKENS, 1024),
                                         (MAX_TOKENS - 1, 1021), (12345677, 997)])
def test_device_division_matches_integer_plan(tokens, grid):
    total = tokens * BLOCKS_PER_TOKEN
    grid = min(grid, total)
    b = np.arange(grid + 1, dtype=np.int64)
    assert np.array_equal(div_device(b * total, grid), range_begin(b, total, grid))
    # owners of every range boundary and of its neighbours, plus random blocks
    starts = range_begin(b[:-1], total, grid)
    rng = np.random.default_rng(tokens ^ grid)
    g = np.unique(np.concatenate([starts, np.maximum(starts - 1, 0), np.minimum(starts + 1, total - 1),
                                  rng.integers(0, total, size=4096), [total - 1]]))
    assert np.array_equal(div_device((g + 1) * grid - 1, total), owner(g, total, grid))


@pytest.mark.parametrize("tokens,grid", [(1, 16), (5, 80), (64, 148), (300, 148), (4096, 148)])
def test_ranges_tile_the_blocks_and_owners_agree(tokens, grid):
    total = tokens * BLOCKS_PER_TOKEN
    grid = min(grid, total)
    begins = range_begin(np.arange(grid + 1), total, grid)
    assert begins[0] == 0 and begins[-1] == total
    assert np.all(np.diff(begins) >= 1)          # no empty range while grid <= total
    g = np.arange(total)
    own = owner(g, total, grid)
    assert np.all(begins[own] <= g) and np.all(g < begins[own + 1])
