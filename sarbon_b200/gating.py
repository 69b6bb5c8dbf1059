"""Cell-level gating (the reference's ``sarbon/sparse/gating.py``), on the GPU.

``active_blocks_cell_level(cells, radius, cell, block)`` of the reference dilates a change
mask of cell x cell-pixel cells by ceil(radius / cell) cells and any-pools it into blocks
(gating.py:42-43).  It is a tighter estimate than dilating changed blocks
(``active_blocks_block_level``, gating.py:37-39): a change in the middle of a block no
longer activates the whole ring of neighbouring blocks.  Here one kernel
(``sb_cell_active_blocks``) computes the block masks of several radii at once; the masks
are bytes, so the result equals the reference's bit for bit.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import check, lib


@torch.no_grad()
def cell_active_blocks(cells: torch.Tensor, radii, cell: int, block: int) -> torch.Tensor:
    """Active blocks for each receptive radius in ``radii`` (image pixels).

    ``cells``: CUDA bool/uint8 ``[N, Hc, Wc]`` (nonzero = the cell changed).  Returns a bool
    ``[len(radii), N, Hc * cell // block, Wc * cell // block]`` tensor on the same device,
    written on the current stream.
    """
    if cells.dim() != 3 or not cells.is_cuda:
        raise ValueError("cells must be a CUDA [N, Hc, Wc] mask")
    radii = [int(r) for r in radii]
    k = block // cell if cell > 0 and block % cell == 0 else 0
    if k == 0:
        raise ValueError("block must be a positive multiple of cell")
    n, hc, wc = cells.shape
    src = cells.contiguous().view(torch.uint8) if cells.dtype == torch.bool else cells.to(torch.uint8).contiguous()
    out = torch.empty((len(radii), n, hc // k, wc // k), dtype=torch.uint8, device=cells.device)
    r = (C.c_int * max(1, len(radii)))(*radii)
    stream = torch.cuda.current_stream(cells.device).cuda_stream
    with torch.cuda.device(cells.device):
        check(lib().sb_cell_active_blocks(C.c_void_p(src.data_ptr()), n, hc, wc, cell, block, r, len(radii),
                                          C.c_void_p(out.data_ptr()), C.c_void_p(stream)),
              "sb_cell_active_blocks")
    return out.bool()
