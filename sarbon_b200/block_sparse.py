"""The reference's first block-sparse engine API (M0, `BlockSparseEngine` in
sarbon/sparse/block_sparse.py:122-326) on the B200 engine.

M0 runs one camera: CHW frames, `full()` for the dense initialisation, `update()` with a
caller-given change mask, the sync-free `step(frame, capacity, tau)` returning an overflow
flag, and the helpers `changed_blocks` / `active_blocks` / `dilation`.  Here every one of
those calls runs the B200 engine (`FusedSparseEngine`, one stream) in its M0 mode
(`set_m0`): the whole frame enters the image cache every step, so the gate compares a
frame with the previous one (block_sparse.py:265,272-274); `step` recomputes exactly the
first `capacity` active blocks of every dilation, padded with block 0 like
`nonzero_static(size=capacity, fill_value=0)` (:268-271), leaves any further active block
as it was and raises the overflow flag (:271, count > capacity); `update` recomputes the
given blocks, dilated (:206-218).  The engine is created with single-block units so that
"the first `capacity` blocks" is exact for every layer.  The halo gather is the conv
kernels' TMA reads, the scatter their epilogue stores into the caches.

Differences from the reference, on purpose:
  * caches are the engine's NHWC caches without a border; `cache[name]` and the returned
    outputs are CHW *views* of them (M0 keeps CHW caches with a one-pixel zero border,
    block_sparse.py:22,135-140), and a conv + residual add is one fused layer (M0 also
    caches the conv output before the add);
  * the change test is the engine's: the exact per-block sum of |diff| against
    float32(tau * block^2 * 3), where M0 compares the fp32 mean (avg_pool of the channel
    mean, :323-326) with tau -- the same rule, which can differ only for a block whose sum
    lies within fp32 rounding of the threshold.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .fused_engine import FusedSparseEngine


def _bucket(n):
    """Active-block count rounded up to few distinct sizes (block_sparse.py:115-119)."""
    if n <= 16:
        return 16
    return 1 << math.ceil(math.log2(n))


class BlockSparseEngine:
    """Runs a LocalBackbone program densely once, then sparsely per frame (one camera)."""

    def __init__(self, net, block=32):
        self.net = net.eval()
        self.block = block
        self.nodes, self.outputs = net.program()
        for n in self.nodes:
            if not (n.stride <= block and block % n.stride == 0):
                raise ValueError("tile must be >= 1 px")
        self.cache = {}
        self._eng = None
        self._key = None

    # ---------- engine and cache views ----------
    def _engine(self, frame):
        if frame.dim() != 3 or frame.shape[0] != 3:
            raise ValueError("frames are [3, H, W]")
        _, h, w = frame.shape
        if h % self.block or w % self.block:
            raise ValueError("H and W must be multiples of the block")
        key = (h, w, frame.dtype, frame.device)
        if self._eng is None or self._key != key:
            self._eng = FusedSparseEngine(self.net, 1, h, w, block=self.block, dtype=frame.dtype, tau=0.0,
                                          refresh=0, dense_check_every=1, device=frame.device, block_units=True)
            self._key = key
            self._tau, self._m0 = 0.0, None
            self._buf = torch.empty(1, h, w, 3, dtype=frame.dtype, device=frame.device)
            self.cache = {name: v[0].permute(2, 0, 1) for name, v in self._eng.cache.items()}
        return self._eng

    def _configure(self, tau, capacity):
        """Threshold and M0 capacity of the next step (set only when they change: a new
        threshold drops the engine's captured step graphs)."""
        eng = self._eng
        if tau != self._tau:
            eng.set_tau(tau)
            self._tau = tau
        if self._m0 != capacity:
            eng.set_m0(True, capacity)
            self._m0 = capacity

    def _interior(self, name):
        return self.cache[name]

    def _stage(self, frame):
        self._buf[0].copy_(frame.permute(1, 2, 0))
        return self._buf

    def _outputs(self):
        return [self.cache[o] for o in self.outputs]

    # ---------- M0 API ----------
    @torch.no_grad()
    def full(self, frame):
        """Dense pass over a [3, H, W] frame that (re)initialises every cache."""
        eng = self._engine(frame)
        eng.reset(self._stage(frame))
        return self._outputs()

    def dilation(self, radius):
        return math.ceil(radius / self.block)

    def active_blocks(self, changed, radius):
        """Blocks whose receptive field (radius in image px) touches a changed block."""
        d = self.dilation(radius)
        m = changed.float()[None, None]
        if d:
            m = F.max_pool2d(m, 2 * d + 1, 1, d)
        return m[0, 0] > 0

    def changed_blocks(self, frame, prev, tau=0.0):
        """Per-block change mask from the mean absolute frame difference."""
        d = (frame - prev).abs().mean(0, keepdim=True)[None]
        return F.avg_pool2d(d, self.block)[0, 0] > tau

    @torch.no_grad()
    def update(self, frame, changed, graph=True):
        """Sparse update with a given [H/block, W/block] change mask (no gate)."""
        if self._eng is None:
            raise RuntimeError("call full() first")
        eng = self._engine(frame)
        self._configure(math.inf, 0)           # no block changes by its pixels ...
        eng.set_extra(changed.reshape(1, eng.hb, eng.wb).bool())  # ... only the given ones
        eng.step_async(self._stage(frame))
        return self._outputs()

    @torch.no_grad()
    def step(self, frame, capacity, tau=0.0):
        """Gate + sparse update for the next frame with no host sync (block_sparse.py:253-295).
        Returns (outputs, overflow): overflow is a 0-dim bool device tensor, True when more
        blocks were active than `capacity`; only the first `capacity` of them were
        recomputed, so the caller should schedule a dense refresh (`full`)."""
        if self._eng is None:
            raise RuntimeError("call full() first")
        if not 1 <= int(capacity) <= self._eng.n_blocks:
            raise ValueError(f"capacity must be in [1, {self._eng.n_blocks}]")
        eng = self._engine(frame)
        self._configure(float(tau), int(capacity))
        eng.extra.zero_()
        eng.step_async(self._stage(frame))
        over = eng.result_view()[1] > int(capacity)
        return self._outputs(), over

    def reset_prev(self, frame):
        """Make `frame` the reference the next step's gate compares against."""
        if self._eng is None:
            raise RuntimeError("call full() first")
        self._eng.cache["img"][0].copy_(frame.permute(1, 2, 0))
