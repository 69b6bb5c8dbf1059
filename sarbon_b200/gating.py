"""Cell-level gating (the reference's ``sarbon/sparse/gating.py``), on the GPU.

``active_blocks_cell_level(cells, radius, cell, block)`` of the reference dilates a change
mask of cell x cell-pixel cells by ceil(radius / cell) cells and any-pools it into blocks
(gating.py:42-43).  It is a tighter estimate than dilating changed blocks
(``active_blocks_block_level``, gating.py:37-39): a change in the middle of a block no
longer activates the whole ring of neighbouring blocks.  Here one kernel
(``sb_cell_active_blocks``) computes the block masks of several radii at once; the masks
are bytes, so the result equals the reference's bit for bit.

``boxes_to_block_mask`` / ``boxes_to_block_masks`` are the track-steered masks of the
reference's video loop (``sarbon/inference/video.py:26-34``, used by ``_steer`` at
:139-147): the blocks that the predicted track boxes touch, widened by ``margin`` blocks,
which the next step recomputes whether or not their pixels changed.  One kernel
(``sb_boxes_to_block_mask``) writes the masks of all cameras from the uploaded boxes.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
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


def _box_rows(boxes) -> np.ndarray:
    """One camera's boxes as float64 [k, 4]; ValueError where the reference's int(x // block) raises."""
    if isinstance(boxes, torch.Tensor):
        boxes = boxes.detach().cpu().numpy()
    b = np.asarray(boxes, dtype=np.float64)
    if b.size == 0:
        return np.zeros((0, 4), np.float64)
    if b.ndim != 2 or b.shape[1] != 4:
        raise ValueError(f"boxes must be [k, 4] xyxy, got shape {b.shape}")
    if not np.isfinite(b).all():  # x // block is NaN for NaN and +-inf: int() of it raises
        raise ValueError("box coordinates must be finite: cannot convert float NaN to integer")
    return b


@torch.no_grad()
def boxes_to_block_masks(boxes_per_cam, hb: int, wb: int, block: int, margin: int = 0,
                         device=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Blocks ``[N, hb, wb]`` touched by each camera's xyxy boxes (engine pixels), widened
    by ``margin`` blocks: video.py:26-34 for N cameras in one launch.

    ``boxes_per_cam``: a sequence of N box lists (each ``[k, 4]``, numpy / torch / lists,
    possibly empty).  The boxes go to the device as float64 (one copy, 32 bytes a box) and
    the mask is written into ``out`` (a CUDA bool or uint8 ``[N, hb, wb]``, e.g. an engine's
    ``extra`` mask) or a new bool tensor, on the current stream.
    """
    rows = [_box_rows(b) for b in boxes_per_cam]
    n = len(rows)
    if n == 0:
        raise ValueError("boxes_per_cam must hold one box list per camera")
    if block <= 0:
        raise ValueError("block must be positive")
    dev = torch.device(device) if device is not None else (out.device if out is not None else torch.device("cuda"))
    if out is None:
        out = torch.empty((n, hb, wb), dtype=torch.bool, device=dev)
    if tuple(out.shape) != (n, hb, wb) or out.dtype not in (torch.bool, torch.uint8) or not out.is_cuda \
            or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous CUDA bool/uint8 [{n}, {hb}, {wb}] tensor")
    offsets = np.zeros(n + 1, np.int32)
    np.cumsum([len(r) for r in rows], out=offsets[1:])
    total = int(offsets[-1])
    # boxes and offsets in one host buffer, one copy: float64 boxes, then the int32 offsets
    host = torch.empty(total * 32 + (n + 1) * 4, dtype=torch.uint8, pin_memory=True)
    hv = host.numpy()
    if total:
        hv[: total * 32] = np.concatenate(rows).view(np.uint8).reshape(-1)
    hv[total * 32:] = offsets.view(np.uint8)
    buf = host.to(out.device, non_blocking=True)
    stream = torch.cuda.current_stream(out.device).cuda_stream
    with torch.cuda.device(out.device):
        check(lib().sb_boxes_to_block_mask(C.c_void_p(buf.data_ptr() if total else None),
                                           C.c_void_p(buf.data_ptr() + total * 32), total, n, hb, wb,
                                           block, int(margin), C.c_void_p(out.data_ptr()), C.c_void_p(stream)),
              "sb_boxes_to_block_mask")
    return out


def boxes_to_block_mask(boxes, hb: int, wb: int, block: int, margin: int = 0, device=None) -> torch.Tensor:
    """One camera's ``[hb, wb]`` mask: the reference's ``boxes_to_block_mask`` (video.py:26-34)
    with the result a CUDA bool tensor instead of a numpy array."""
    return boxes_to_block_masks([boxes], hb, wb, block, margin, device=device)[0]
