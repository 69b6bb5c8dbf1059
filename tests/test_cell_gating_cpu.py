"""Cell-level gating (gating.py:31-43) on the CPU: the oracle reproduces, bit for bit, the
masks the reference's own functions produced for the golden cases, and the cell-level
estimate is never looser than the block-level one."""
from pathlib import Path

import numpy as np

from oracle import sparse_oracle as so

GOLDEN = np.load(Path(__file__).parent / "golden" / "cells" / "cell_gating.npz")


def test_oracle_matches_reference_golden():
    radii, block = [int(r) for r in GOLDEN["radii"]], int(GOLDEN["block"])
    for i in range(int(GOLDEN["n_cases"])):
        cells = GOLDEN[f"c{i}_cells"].astype(bool)
        cell = int(GOLDEN[f"c{i}_cell"])
        for j, r in enumerate(radii):
            got_c = so.active_blocks_cell_level(cells, r, cell, block)
            got_b = so.active_blocks_block_level(cells, r, cell, block)
            np.testing.assert_array_equal(got_c, GOLDEN[f"c{i}_cell_level"][j].astype(bool), err_msg=f"case {i} r {r}")
            np.testing.assert_array_equal(got_b, GOLDEN[f"c{i}_block_level"][j].astype(bool), err_msg=f"case {i} r {r}")
            assert not (got_c & ~got_b).any()  # cell level is contained in block level


def test_cell_mode_oracle_is_tighter_and_consistent():
    """The engine's cell mode (``gate_cells`` + ``cell_group_masks``): at tau = 0 its
    changed blocks are the block gate's, its group masks are the reference's cell-level
    estimate and never exceed the block-level masks of the same groups."""
    rng = np.random.default_rng(2)
    n, h, w, block, cell = 2, 128, 192, 32, 8
    img = rng.integers(-3, 4, (n, h, w, 3)).astype(np.float16)
    f = img.copy()
    f[0, 40:45, 70:73] += 1
    f[1, 0:3, w - 2:] -= 2
    cells, changed = so.gate_cells(f, img, cell, block, 0.0)
    np.testing.assert_array_equal(changed, so.gate(f, img, block, 0.0))
    for r in (1, 11, 31, 55):
        rc = -(-r // cell)
        (got,) = so.cell_group_masks(cells, [rc], block // cell)
        np.testing.assert_array_equal(got, so.active_blocks_cell_level(cells, r, cell, block))
        assert not (got & ~so.dilate(changed, -(-r // block))).any()
    # extra forces every cell of its block
    extra = np.zeros((n, h // block, w // block), bool)
    extra[1, 2, 3] = True
    cells_x, changed_x = so.gate_cells(f, img, cell, block, 0.0, extra)
    assert cells_x[1, 8:12, 12:16].all() and changed_x[1, 2, 3]
