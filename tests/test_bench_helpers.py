"""CPU checks of bench.py's synthetic sparse-grid tables (the configs[3]
stand-in inputs of the SLat side measurements)."""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_neighbour_table_offsets_are_consistent():
    rng = np.random.default_rng(0)
    g = 12
    keys = np.sort(rng.choice(g ** 3, 200, replace=False))
    idx = bench.neighbour_table(keys, g)
    n = keys.size
    assert idx.shape == (27, n)
    assert np.array_equal(idx[13], np.arange(n))          # offset (0, 0, 0) is the cell itself
    for o in range(27):                                   # offset o and its mirror 26 - o are inverse maps
        hit = idx[o] >= 0
        assert np.array_equal(idx[26 - o][idx[o][hit]], np.nonzero(hit)[0])
    xyz = np.stack([keys // (g * g), (keys // g) % g, keys % g], 1)
    d = np.array([(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1)])
    for o in range(27):
        hit = idx[o] >= 0
        assert np.array_equal(xyz[idx[o][hit]] - xyz[hit], np.tile(d[o], (hit.sum(), 1)))


def test_slat_grid_tables_match_configs3():
    idx, cidx, rows, counts = bench.slat_grid_tables()
    fine, coarse = idx.shape[1], cidx.shape[1]
    assert fine == round(0.03 * 64 ** 3) and coarse == bench.slat_tokens()[1]
    assert rows.min() == 0 and rows.max() == coarse - 1
    assert np.array_equal(counts, np.bincount(rows, minlength=coarse) + 1)
    assert counts.max() <= 9                               # at most 8 children per 2x2x2 cell
