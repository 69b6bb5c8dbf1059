"""The detector's multi-scale deformable attention core on the B200 (sb_ms_deform_attn).

Reference: Bahrombekk/Sarbon ``sarbon/models/deform_attn.py:14-28`` (``ms_deform_attn_core``,
grid_sample-based; "a fused kernel can replace `ms_deform_attn_core` later without
changing weights").  ``ms_deform_attn_core`` here has the same signature and result, as
one kernel: a warp per (batch, query, head), every level and point sampled bilinearly like
``grid_sample(align_corners=False, padding_mode="zeros")`` and summed with the attention
weights in fp32.  ``patch_reference(module)`` installs it into the reference's own
``MSDeformAttn`` (the reference's detector then runs it in its decoder layers).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, lib


def ms_deform_attn_core(value, shapes, loc, weights):
    """value [B, S, H, Dh]; shapes [(h, w)] per level; loc [B, Q, H, L, P, 2] in [0, 1];
    weights [B, Q, H, L, P] -> [B, Q, H * Dh] (deform_attn.py:14-28)."""
    if not value.is_cuda:
        raise ValueError("ms_deform_attn_core runs on CUDA tensors only")
    b, s, nh, dh = value.shape
    _, q, _, nl, npnt, _ = loc.shape
    # the reference returns (samples * weights).sum(-1): the promoted type of the two
    out_dtype = torch.promote_types(value.dtype, weights.dtype)
    if value.dtype not in (torch.float16, torch.float32):
        value = value.float()
    value = value.contiguous()
    if loc.dtype != torch.float32:
        # the reference forms grid = 2 * loc - 1 in loc's own type (fp16 under autocast) before
        # grid_sample; the kernel forms it in fp32 from loc, so pass the fp32 loc whose grid is
        # exactly that rounded grid ((g + 1) / 2 and back are exact for an fp16 g)
        loc = ((2 * loc - 1).float() + 1) / 2
    loc = loc.float().contiguous()
    weights = weights.float().contiguous()
    out = torch.empty(b, q, nh * dh, device=value.device, dtype=value.dtype)
    hw = [int(x) for hwl in shapes for x in hwl]
    arr = (C.c_int * len(hw))(*hw)
    check(lib().sb_ms_deform_attn(C.c_void_p(value.data_ptr()),
                                  _lib.SB_F16 if value.dtype == torch.float16 else _lib.SB_F32,
                                  b, s, nh, dh, arr, nl, C.c_void_p(loc.data_ptr()), C.c_void_p(weights.data_ptr()),
                                  q, npnt, C.c_void_p(out.data_ptr()),
                                  C.c_void_p(torch.cuda.current_stream(value.device).cuda_stream)),
          "sb_ms_deform_attn")
    return out if out.dtype == out_dtype else out.to(out_dtype)


def patch_reference(deform_attn_module):
    """Make the reference's ``MSDeformAttn`` (module ``sarbon.models.deform_attn``) call
    this kernel: its forward looks ``ms_deform_attn_core`` up in the module's globals."""
    deform_attn_module.ms_deform_attn_core = ms_deform_attn_core
