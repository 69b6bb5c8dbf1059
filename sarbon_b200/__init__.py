"""sarbon_b200: B200-native temporal block-sparse stem engine for Sarbon.

Public API (mirrors ``sarbon.sparse``):

* :class:`FusedSparseEngine` -- the engine (CUDA library ``libsarbon_sparse.so``).
* :class:`LocalBackbone`, :func:`stem_to_local`, :func:`fold` -- stem topology and BN folding.
* :func:`budget_buckets` -- the reference's budget schedule.
* :func:`cell_active_blocks` -- cell-level gating (``gating.py``) on the GPU.
* :func:`ms_deform_attn_core` -- the detector's deformable-attention core as one kernel.

Importing the package does not load the CUDA library; constructing an engine does, and
raises :class:`SarbonLibraryError` when it is missing.
"""
from ._lib import SarbonLibraryError
from .fused_engine import FusedSparseEngine, budget_buckets, fuse_layers
from .gating import boxes_to_block_mask, boxes_to_block_masks, cell_active_blocks
from .deform_attn import ms_deform_attn_core
from .local import LocalBackbone, Node, fold, stem_to_local

__all__ = ["FusedSparseEngine", "LocalBackbone", "Node", "SarbonLibraryError", "budget_buckets",
           "boxes_to_block_mask", "boxes_to_block_masks", "cell_active_blocks", "fold", "fuse_layers", "ms_deform_attn_core",
           "stem_to_local"]
