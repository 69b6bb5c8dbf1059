"""Golden vectors for cell-level gating, made by the reference's own code.

Runs ``sarbon/sparse/gating.py`` of the reference checkout (its path is the first
argument) on seeded random change masks and writes ``cells/cell_gating.npz`` next to
this script.  The tests only read the ``.npz``; they never need the reference.

For each case the fixture holds the change mask of c x c-pixel cells ``[N, Hc, Wc]`` and,
for every receptive radius of the Sarbon-S stem, the block mask of
``active_blocks_cell_level`` (cells dilated by ceil(R / c), then any-pooled into blocks,
gating.py:42-43) and of ``active_blocks_block_level`` (gating.py:37-39).

Usage: python tests/golden/make_cell_golden.py /path/to/reference
"""
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "cells"
if len(sys.argv) < 2:
    sys.exit("usage: make_cell_golden.py /path/to/reference")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF))
from sarbon.sparse import gating  # noqa: E402

RADII = [1, 3, 7, 11, 15, 19, 23, 31, 39, 47, 55]  # Sarbon-S stem layers (image px)
BLOCK = 32


def main():
    rng = np.random.default_rng(7)
    cases = [  # (n, block rows, block cols, cell, density)
        (2, 4, 6, 8, 0.02),
        (1, 5, 7, 16, 0.05),
        (3, 3, 4, 4, 0.01),
        (1, 6, 9, 8, 0.0),
        (1, 2, 3, 8, 1.0),
        (2, 7, 5, 32, 0.15),
    ]
    out = {"radii": np.array(RADII, np.int32), "block": np.int32(BLOCK), "n_cases": np.int32(len(cases))}
    for i, (n, hb, wb, cell, dens) in enumerate(cases):
        k = BLOCK // cell
        cells = rng.random((n, hb * k, wb * k)) < dens
        if 0.0 < dens < 1.0:  # a change touching every image border too
            cells[0, 0, 0] = cells[-1, -1, -1] = True
        t = torch.from_numpy(cells)
        cl = np.stack([gating.active_blocks_cell_level(t, r, cell, BLOCK).numpy() for r in RADII])
        bl = np.stack([gating.active_blocks_block_level(t, r, cell, BLOCK).numpy() for r in RADII])
        out[f"c{i}_cells"] = cells.astype(np.uint8)
        out[f"c{i}_cell"] = np.int32(cell)
        out[f"c{i}_cell_level"] = cl.astype(np.uint8)
        out[f"c{i}_block_level"] = bl.astype(np.uint8)
    np.savez_compressed(OUT / "cell_gating.npz", **out)
    print("wrote", OUT / "cell_gating.npz", {k: v.shape for k, v in out.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()
