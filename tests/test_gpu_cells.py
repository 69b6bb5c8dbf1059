"""Cell-level gating on the GPU (``sb_cell_active_blocks``, gating.py:42-43 of the reference).

* the kernel reproduces, bit for bit, the block masks the reference's own
  ``active_blocks_cell_level`` produced for the golden cases (tests/golden/cells);
* on 16 cameras of 1080p cells (cell 8 and 16, block 32, every radius of the stem) it equals
  the oracle, and its masks never exceed the block-level ones;
* empty / full masks, radius 0 and argument errors.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sparse_oracle as so

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "cells" / "cell_gating.npz")
RADII = [int(r) for r in GOLDEN["radii"]]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def test_matches_reference_golden():
    from sarbon_b200 import cell_active_blocks
    block = int(GOLDEN["block"])
    for i in range(int(GOLDEN["n_cases"])):
        cells = torch.from_numpy(GOLDEN[f"c{i}_cells"]).cuda()
        got = cell_active_blocks(cells, RADII, int(GOLDEN[f"c{i}_cell"]), block).cpu().numpy()
        np.testing.assert_array_equal(got, GOLDEN[f"c{i}_cell_level"].astype(bool), err_msg=f"case {i}")


@pytest.mark.parametrize("cell", [8, 16])
def test_1080p_streams_vs_oracle(cell):
    from sarbon_b200 import cell_active_blocks
    block, n, h, w = 32, 16, 1088, 1920
    g = torch.Generator(device="cuda").manual_seed(cell)
    cells = torch.rand(n, h // cell, w // cell, device="cuda", generator=g) < 0.01
    got = cell_active_blocks(cells, RADII, cell, block).cpu().numpy()
    c = cells.cpu().numpy()
    for j, r in enumerate(RADII):
        exp = so.active_blocks_cell_level(c, r, cell, block)
        np.testing.assert_array_equal(got[j], exp, err_msg=f"radius {r}")
        assert not (got[j] & ~so.active_blocks_block_level(c, r, cell, block)).any()
    # two calls in a row give the same masks
    assert torch.equal(cell_active_blocks(cells, RADII, cell, block).cpu(), torch.from_numpy(got))


def test_edges_and_errors():
    from sarbon_b200 import SarbonLibraryError, cell_active_blocks
    for fill in (0, 1):
        cells = torch.full((2, 12, 20), fill, dtype=torch.uint8, device="cuda")
        got = cell_active_blocks(cells, [0, 5, 55], 8, 32).cpu().numpy()
        assert got.shape == (3, 2, 3, 5) and (got == bool(fill)).all()
    one = torch.zeros((1, 8, 8), dtype=torch.bool, device="cuda")
    one[0, 5, 2] = True  # cell (5, 2) of 16 px cells; blocks of 32 px = 2 x 2 cells: block (2, 1)
    got = cell_active_blocks(one, [0, 16, 17], 16, 32).cpu().numpy()
    own = np.zeros((4, 4), bool)
    own[2, 1] = True
    np.testing.assert_array_equal(got[0, 0], own)  # radius 0: the changed cell's own block only
    for j, r in enumerate([0, 16, 17]):
        np.testing.assert_array_equal(got[j], so.active_blocks_cell_level(one.cpu().numpy(), r, 16, 32))
    assert got[1].sum() < got[2].sum()  # 17 px reach one cell (and block) further than 16
    with pytest.raises(ValueError, match="multiple of cell"):
        cell_active_blocks(one, [1], 12, 32)
    with pytest.raises(SarbonLibraryError, match="hc and wc"):
        cell_active_blocks(torch.zeros((1, 6, 8), dtype=torch.bool, device="cuda"), [1], 8, 32)
    with pytest.raises(SarbonLibraryError, match="n_radii"):
        cell_active_blocks(one, list(range(17)), 16, 32)
    with pytest.raises(SarbonLibraryError, match="negative"):
        cell_active_blocks(one, [-1], 16, 32)


@pytest.mark.parametrize("wc,radius", [(2048, 1040), (2048, 24), (100, 2 ** 31 - 1)])
def test_wide_images_and_large_radii(wc, radius):
    """Both kernels behind the entry point: the bit-row kernel (bit rows of the cells a
    radius reaches fit in 48 KB of shared memory) and the byte-window kernel it falls back
    to (256 rows x 64 words at 130 cells of radius do not); a radius far past the image
    (capped to the image size inside) marks every block of a camera with any change."""
    from sarbon_b200 import cell_active_blocks
    cell, block, hc = 8, 32, 256
    g = torch.Generator(device="cuda").manual_seed(wc + radius % 1000)
    cells = torch.rand(2, hc, wc, device="cuda", generator=g) < 0.002
    cells[1] = False
    cells[1, 7, wc - 1] = True  # one change in the last column of camera 1
    got = cell_active_blocks(cells, [radius, 0], cell, block).cpu().numpy()
    c = cells.cpu().numpy()
    r_eq = min(radius, cell * (max(hc, wc) + 1))  # the oracle's loops need a finite radius
    np.testing.assert_array_equal(got[0], so.active_blocks_cell_level(c, r_eq, cell, block))
    np.testing.assert_array_equal(got[1], so.active_blocks_cell_level(c, 0, cell, block))
    if radius > cell * max(hc, wc):
        assert got[0].all()
