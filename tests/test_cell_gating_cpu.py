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
