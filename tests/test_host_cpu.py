"""Host-side DUST configuration on CPU: the recipe's draw counts at the two tracks' scales and the
split of those draws over ranks."""
import pytest


def total(rec):
    return sum(rec.writers) + sum(rec.hidden) + sum(rec.hubs) + rec.embedding + sum(rec.local.values())


def test_recipe_draw_counts():
    """train/val/run.py:41-71 (Recipe, recipe): the 16k Adam cell (val track) and its 0.3125 scaling (speedrun track);
    counts round to multiples of 64 with at least 64 per block."""
    from noise_b200.dust import recipe
    full = recipe(1.0)
    assert full.writers == [256] * 8 and full.hidden == [512] * 8 and full.hubs == [512] * 8
    assert full.embedding == 2048
    assert full.local == dict(q=384, v=384, gate=128, k=1664, ve=4608)
    assert total(full) == 19_456
    speed = recipe(0.3125)
    assert total(speed) == 5_440
    assert all(c % 64 == 0 and c >= 64 for c in speed.writers + speed.hidden + speed.hubs + list(speed.local.values()))
    assert (full.nrep, full.lr, full.warmdown, full.betas) == (16, 0.003, 0.3, (0.7, 0.95))


@pytest.mark.parametrize('world', [1, 2, 4, 8])
def test_recipe_splits_over_ranks(world):
    """Every block's draws and the 8 mixing-scalar draws divide evenly over 1, 2, 4 and 8 ranks."""
    from noise_b200.dust import recipe
    for scale in (1.0, 0.3125):
        rec = recipe(scale)
        counts = rec.writers + rec.hidden + rec.hubs + [rec.embedding] + list(rec.local.values())
        assert all(k % world == 0 for k in counts) and 8 % world == 0


def test_units_that_fit_is_the_library_chunking():
    """The host sizes its workspace from the library's own chunk query: the chunk's workspace fits
    the budget, the number of chunks is the fewest that any fitting chunk allows, the chunks are
    equal, and the draw table's direction cap binds for rank-1 populations."""
    from noise_b200.population import units_that_fit, workspace_bytes
    rows = 8 * 2048
    for budget in (workspace_bytes(rows), 16 << 30, 32 << 30):
        largest = 1
        while workspace_bytes(rows * (largest + 1)) <= budget:
            largest += 1
        for units in (1, 7, 1024, 4096):
            n = units_that_fit(rows, units, budget)
            assert workspace_bytes(rows * n) <= budget
            assert -(-units // n) == -(-units // min(units, largest)), (budget, units, n, largest)
            assert n == -(-units // -(-units // n))  # chunks of equal size, no short tail
    assert units_that_fit(rows, 5, 32 << 30) == 5
    assert units_that_fit(rows, 100, 1) == 1
    # rank-1 members: a chunk spans at most rows / 256 + 2 directions of the draw table
    short = 128
    n = units_that_fit(short, 4096, 32 << 30, pairs=2048)
    assert (n + 1) // 2 <= short * n // 256 + 2
