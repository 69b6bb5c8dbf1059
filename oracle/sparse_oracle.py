"""CPU oracle for Sarbon's temporal block-sparse stem engine.

TEST INFRASTRUCTURE ONLY. This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product path (``sarbon_b200``) never calls it and fails loudly when its CUDA
library is missing.

It restates, in numpy, the algorithm of the reference engine
``sarbon/sparse/fused_engine.py`` (class ``FusedSparseEngine``) and its Triton
kernel ``sarbon/sparse/triton_conv.py`` (``_tile_conv_kernel``):

* gate            fused_engine.py:140-153
* img update      fused_engine.py:155-160
* block lists     fused_engine.py:161-165   (``nonzero_static``, ascending, pad 0)
* tile conv       triton_conv.py:15-61       (gather -> 3x3 conv -> bias -> +res -> ReLU)
* dense pass      fused_engine.py:172-185
* dispatch        fused_engine.py:214-240   (skip / sparse / dense, hysteresis)
* buckets         fused_engine.py:44-51, 188-193; triton_conv.py:64-69
* cell gating     gating.py:31-43           (cells dilated, then any-pooled into blocks)
* steered masks   video.py:26-34            (track boxes -> blocks, widened by a margin)

Number semantics (pinned against the reference by ``tests/golden``):

* The per-block change statistic is ``sum(|f16(f32(a) - f32(b))|)``; the reference
  sums it in fp32 in torch's reduction order.  The oracle sums exactly (float64 is
  exact here: every fp16 is a multiple of 2**-24 and 3*block**2 partial sums stay
  far below 2**53 * 2**-24).  Exact and fp32 sums can straddle the threshold only
  inside the fp32 rounding band; on integer-valued frames they are identical.
* The threshold is ``float32(tau * block * block * 3)`` (torch casts the Python
  scalar to the tensor dtype before comparing).
* Convolutions accumulate fp16 products in fp32, add the fp32 bias, add the
  residual (widened to fp32), apply ReLU and round to the cache dtype once.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import numpy as np

MODES = ("skip", "sparse", "dense")


# ----------------------------------------------------------------------------- host ints
def budget_buckets(n_blocks, unit=16, ratio=1.15):
    """Budgets ~15% apart, multiples of ``unit`` (fused_engine.py:44-51)."""
    out, b = [], unit
    while b < n_blocks:
        out.append(b)
        b = max(b + unit, int(math.ceil(b * ratio / unit)) * unit)
    out.append(int(math.ceil(n_blocks / unit)) * unit)
    return out


def tiles_per_program(t, block_m=64):
    """triton_conv.py:67-69: tiles whose pixels fill one 64-pixel program."""
    return max(1, block_m // (t * t))


def dilation(radius, block):
    """fused_engine.py:121-122."""
    return math.ceil(radius / block)


@dataclass
class OLayer:
    """One fused conv(+add) of the stem program (fused_engine.py:29-41)."""
    src: str
    dst: str
    res: str | None
    act: bool
    stride: int
    out_stride: int
    radius: int
    w: np.ndarray      # [3, 3, cin, cout] float32 (the tile kernel's layout)
    bias: np.ndarray   # [cout] float32

    @property
    def cin(self):
        return self.w.shape[2]

    @property
    def cout(self):
        return self.w.shape[3]


def fuse_program(nodes):
    """Fuse conv+add pairs into layers (fused_engine.py:99-119).

    ``nodes`` is a list of dicts with keys kind, src, dst, stride, radius, act and,
    for convs, ``w`` [cout, cin, 3, 3], ``b`` [cout], ``conv_stride``.
    """
    layers, i = [], 0
    while i < len(nodes):
        n = nodes[i]
        assert n["kind"] == "conv" and n["w"].shape[2] == 3
        nxt = nodes[i + 1] if i + 1 < len(nodes) else None
        fused = nxt is not None and nxt["kind"] == "add" and nxt["src"][0] == n["dst"]
        w = np.asarray(n["w"], np.float32)
        layers.append(OLayer(
            src=n["src"][0], dst=nxt["dst"] if fused else n["dst"],
            res=nxt["src"][1] if fused else None, act=True if fused else n["act"],
            stride=n["conv_stride"], out_stride=n["stride"],
            radius=nxt["radius"] if fused else n["radius"],
            w=np.ascontiguousarray(w.transpose(2, 3, 1, 0)),
            bias=np.asarray(n["b"], np.float32)))
        i += 2 if fused else 1
    return layers


# ----------------------------------------------------------------------------- gate
def block_change_sums(frames, img, block):
    """Exact per-block ``sum |f16(f32(f) - f32(i))|`` -> float64 [N, Hb, Wb].

    Restates fused_engine.py:142-143 with an exact (order-free) sum.
    """
    n, h, w, _ = frames.shape
    d = (frames.astype(np.float32) - img.astype(np.float32)).astype(frames.dtype)
    d = np.abs(d).astype(np.float64)
    return d.reshape(n, h // block, block, w // block, block, 3).sum(axis=(2, 4, 5))


def block_change_sums_fp32(frames, img, block):
    """The same statistic summed in float32 (numpy's pairwise order); diagnostic only."""
    n, h, w, _ = frames.shape
    d = np.abs((frames.astype(np.float32) - img.astype(np.float32)).astype(frames.dtype))
    d = d.astype(np.float32).reshape(n, h // block, block, w // block, block, 3)
    return d.transpose(0, 1, 3, 2, 4, 5).reshape(n, h // block, w // block, -1).sum(-1, dtype=np.float32)


def threshold(tau, block):
    """fp32 threshold the reference compares against (fused_engine.py:144)."""
    return np.float32(float(tau) * block * block * 3)


def gate(frames, img, block, tau, extra=None, refresh=0, tick=0):
    """Per-block change mask (fused_engine.py:140-148). Returns bool [N, Hb, Wb]."""
    sums = block_change_sums(frames, img, block)
    changed = sums > np.float64(threshold(tau, block))
    if extra is not None:
        changed |= extra.astype(bool)
    if refresh:
        lin = np.arange(changed.size, dtype=np.int64).reshape(changed.shape)
        changed |= (lin % refresh) == (tick % refresh)
    return changed


def dilate(mask, d):
    """``max_pool2d(k=2d+1, s=1, p=d)`` on a bool [N, Hb, Wb] mask (fused_engine.py:151)."""
    if d == 0:
        return mask.copy()
    n, hb, wb = mask.shape
    # a max over a (2d+1)^2 square is a max over rows of a max over columns (separable)
    p = np.zeros((n, hb, wb + 2 * d), bool)
    p[:, :, d:d + wb] = mask
    rows = np.zeros((n, hb + 2 * d, wb), bool)
    for dx in range(2 * d + 1):
        rows[:, d:d + hb] |= p[:, :, dx:dx + wb]
    out = np.zeros_like(mask)
    for dy in range(2 * d + 1):
        out |= rows[:, dy:dy + hb]
    return out


def cells_to_blocks(mask, k):
    """Any-pool k x k cells of a bool [N, Hc, Wc] mask into [N, Hc/k, Wc/k] blocks
    (gating.py:31-34)."""
    n, hc, wc = mask.shape
    return mask.reshape(n, hc // k, k, wc // k, k).any(axis=(2, 4))


def active_blocks_cell_level(cells, radius, cell, block):
    """Blocks whose cells, dilated by ceil(radius / cell) cells, hold a change
    (gating.py:42-43)."""
    return cells_to_blocks(dilate(cells, -(-radius // cell)), block // cell)


def active_blocks_block_level(cells, radius, cell, block):
    """Changed blocks dilated by ceil(radius / block) blocks (gating.py:37-39)."""
    return dilate(cells_to_blocks(cells, block // cell), -(-radius // block))



def gate_cells(frames, img, cell, block, tau, extra=None, refresh=0, tick=0):
    """Cell-level gate of the engine's optional cell mode: a cell changed when its exact
    sum of |diff| exceeds float32(tau * cell^2 * 3) (the block gate, fused_engine.py:140-148,
    applied per cell; gating.py:18-22 estimates cells the same way, as a mean) or when its
    block is forced by ``extra`` or the refresh phase.  Returns (cells [N, H/c, W/c],
    changed blocks [N, Hb, Wb]): a block changed when any of its cells did."""
    k = block // cell
    cells = block_change_sums(frames, img, cell) > np.float64(threshold(tau, cell))
    n, h, w, _ = frames.shape
    forced = np.zeros((n, h // block, w // block), bool)
    if extra is not None:
        forced |= extra.astype(bool)
    if refresh:
        lin = np.arange(forced.size, dtype=np.int64).reshape(forced.shape)
        forced |= (lin % refresh) == (tick % refresh)
    cells |= np.repeat(np.repeat(forced, k, axis=1), k, axis=2)
    return cells, cells_to_blocks(cells, k)


def cell_group_masks(cells, cell_radii, k):
    """Block masks of the cell mode: the changed cells dilated by each group's radius (in
    cells), any-pooled into blocks of k x k cells (gating.py:42-43)."""
    return [cells_to_blocks(dilate(cells, r), k) for r in cell_radii]


def boxes_to_block_mask(boxes, hb, wb, block, margin=0):
    """Track-steered mask of one camera (video.py:26-34): for each xyxy box in engine
    pixels, the block range from floor(lo / block) - margin to floor(hi / block) + margin,
    clipped to the grid, set when it is non-empty on both axes.  Python's float floor
    division is the exact floor of the real quotient; NaN and +-inf coordinates give a
    NaN quotient, whose ``int`` raises ValueError, as in the reference."""
    mask = np.zeros((hb, wb), bool)
    for x0, y0, x1, y1 in boxes:
        lo_r, hi_r = max(0, int(y0 // block) - margin), min(hb - 1, int(y1 // block) + margin)
        lo_c, hi_c = max(0, int(x0 // block) - margin), min(wb - 1, int(x1 // block) + margin)
        if lo_r <= hi_r and lo_c <= hi_c:
            mask[lo_r:hi_r + 1, lo_c:hi_c + 1] = True
    return mask


def block_lists(mask, cap=None):
    """``nonzero_static(mask.flatten(), size=cap, fill_value=0)`` split into
    (cam, by, bx) int32 (fused_engine.py:161-165). ``cap=None`` returns exactly k entries."""
    n, hb, wb = mask.shape
    flat = np.flatnonzero(mask.reshape(-1)).astype(np.int64)
    if cap is not None:
        pad = np.zeros(max(0, cap - len(flat)), np.int64)
        flat = np.concatenate([flat[:cap], pad])
    per = hb * wb
    r = flat % per
    return (flat // per).astype(np.int32), (r // wb).astype(np.int32), (r % wb).astype(np.int32)


def update_img(img, frames, changed, block):
    """``img = where(changed, frames, img)`` per block (fused_engine.py:157-160)."""
    n, h, w, c = img.shape
    m = np.repeat(np.repeat(changed, block, axis=1), block, axis=2)[..., None]
    return np.where(m, frames, img).astype(img.dtype)


# ----------------------------------------------------------------------------- tile conv
def conv_tiles(x, w, bias, y, cam, by, bx, t, stride, act, res=None, out_dtype=None):
    """Fused gather -> 3x3 conv (pad 1) -> bias -> (+res) -> ReLU -> scatter.

    Restates triton_conv.py:15-61 for the listed tiles (duplicates allowed: the
    reference pads lists with block 0). ``x``/``y``/``res`` are NHWC arrays;
    ``w`` is [3, 3, cin, cout]. ``y`` is updated in place and returned.
    Zero padding applies only at the image border (triton_conv.py:40).
    """
    out_dtype = out_dtype or y.dtype
    n, hx, wx, cin = x.shape
    cout = w.shape[3]
    if len(cam) == 0:
        return y
    # unique tiles: duplicate list entries write identical values
    key = np.unique(np.stack([cam, by, bx], 1).astype(np.int64), axis=0)
    cam, by, bx = key[:, 0], key[:, 1], key[:, 2]
    k = len(cam)
    py, px = np.divmod(np.arange(t * t), t)
    gy = by[:, None] * t + py[None]            # [k, t*t] output rows
    gx = bx[:, None] * t + px[None]
    xp = np.zeros((n, hx + 2, wx + 2, cin), np.float32)
    xp[:, 1:-1, 1:-1] = x.astype(np.float32)
    cols = []
    for ky in range(3):
        for kx in range(3):
            iy = gy * stride + ky          # +1 pad offset, -1 conv offset
            ix = gx * stride + kx
            cols.append(xp[cam[:, None], iy, ix])   # [k, t*t, cin]
    a = np.concatenate(cols, axis=-1).reshape(k * t * t, 9 * cin)
    acc = a @ w.reshape(9 * cin, cout).astype(np.float32)
    acc += bias.astype(np.float32)[None]
    cam_r = np.repeat(cam, t * t)
    gy_r, gx_r = gy.reshape(-1), gx.reshape(-1)
    if res is not None:
        acc += res[cam_r, gy_r, gx_r].astype(np.float32)
    if act:
        np.maximum(acc, 0.0, out=acc)
    y[cam_r, gy_r, gx_r] = acc.astype(out_dtype)
    return y


def conv_dense(x, w, bias, stride, act, res=None, out_dtype=np.float32):
    """Dense 3x3/pad-1 conv over the whole map: every tile of the output."""
    n, hx, wx, _ = x.shape
    ho, wo = hx // stride, wx // stride
    y = np.zeros((n, ho, wo, w.shape[3]), out_dtype)
    cam, gy, gx = np.meshgrid(np.arange(n), np.arange(ho), np.arange(wo), indexing="ij")
    return conv_tiles(x, w, bias, y, cam.reshape(-1), gy.reshape(-1), gx.reshape(-1),
                      1, stride, act, res, out_dtype)


# ----------------------------------------------------------------------------- engine
@dataclass
class OracleEngine:
    """numpy mirror of ``FusedSparseEngine`` (fused_engine.py:54-240).

    Dispatch follows the reference: k==0 -> skip; k <= fallback -> sparse at the
    budget bucket; otherwise dense; hysteresis keeps dense for
    ``dense_check_every`` steps without looking at the gate.
    """
    layers: list
    n: int
    h: int
    w: int
    block: int = 32
    dtype: type = np.float16
    tau: float = 0.0
    refresh: int = 0
    dense_check_every: int = 4
    outputs: tuple = ("t7", "t14")
    cache: dict = field(default_factory=dict)

    def __post_init__(self):
        assert self.h % self.block == 0 and self.w % self.block == 0
        # the tile kernel's weights are in the engine dtype, its bias in fp32
        # (fused_engine.py:114,116)
        self.layers = [replace(l, w=l.w.astype(self.dtype).astype(np.float32)) for l in self.layers]
        self.hb, self.wb = self.h // self.block, self.w // self.block
        self.n_blocks = self.n * self.hb * self.wb
        self.ds = sorted({dilation(l.radius, self.block) for l in self.layers})
        self.cache["img"] = np.zeros((self.n, self.h, self.w, 3), self.dtype)
        for l in self.layers:
            self.cache[l.dst] = np.zeros((self.n, self.h // l.out_stride, self.w // l.out_stride,
                                          l.cout), self.dtype)
        self.extra = np.zeros((self.n, self.hb, self.wb), bool)
        self.changed = np.zeros_like(self.extra)
        self.masks = {d: np.zeros_like(self.extra) for d in self.ds}
        # the reference warms its gate graph up once at construction (fused_engine.py:85,
        # 130-132), which runs `tick += 1` (:147): the first real step sees tick == 1
        self.tick = 1
        self.buckets = budget_buckets(self.n_blocks)
        self.fallback = self.buckets[-1]
        self._dense_run = 0
        self.stats = {m: 0 for m in MODES}
        self.last_lists = {}

    def bucket(self, k):
        """fused_engine.py:188-193."""
        lo = max(tiles_per_program(self.block // l.out_stride) for l in self.layers)
        for b in self.buckets:
            if b >= k and b % lo == 0:
                return b
        return self.buckets[-1]

    def _run_layers(self, lists):
        for l in self.layers:
            t = self.block // l.out_stride
            res = None if l.res is None else self.cache[l.res]
            if lists is None:
                self.cache[l.dst] = conv_dense(self.cache[l.src], l.w, l.bias, l.stride, l.act,
                                               res, self.dtype)
            else:
                cam, by, bx = lists[dilation(l.radius, self.block)]
                conv_tiles(self.cache[l.src], l.w, l.bias, self.cache[l.dst], cam, by, bx, t,
                           l.stride, l.act, res, self.dtype)

    def dense(self, frames):
        """fused_engine.py:172-185."""
        self.cache["img"] = np.array(frames, self.dtype, copy=True)
        self._run_layers(None)

    def reset(self, frames):
        """fused_engine.py:207-212."""
        self.dense(frames)
        self._dense_run = 0

    def gate(self, frames):
        """fused_engine.py:140-153: returns the active count of the widest dilation."""
        self.changed = gate(frames, self.cache["img"], self.block, self.tau, self.extra,
                            self.refresh, self.tick)
        if self.refresh:
            self.tick += 1
        for d in self.ds:
            self.masks[d] = dilate(self.changed, d)
        return int(self.masks[self.ds[-1]].sum())

    def sparse(self, frames, cap):
        """fused_engine.py:155-170."""
        self.cache["img"] = update_img(self.cache["img"], frames, self.changed, self.block)
        lists = {d: block_lists(self.masks[d], cap) for d in self.ds}
        self.last_lists = lists
        self._run_layers(lists)

    def step(self, frames):
        """fused_engine.py:214-240."""
        frames = np.asarray(frames, self.dtype)
        if 0 < self._dense_run < self.dense_check_every:
            self._dense_run += 1
            self.dense(frames)
            self.stats["dense"] += 1
            return "dense", -1
        k = self.gate(frames)
        if k == 0:
            mode = "skip"
        elif k <= self.fallback:
            self.sparse(frames, self.bucket(k))
            mode = "sparse"
        else:
            self.dense(frames)
            mode = "dense"
        self._dense_run = 1 if mode == "dense" else 0
        self.stats[mode] += 1
        return mode, k

    def outputs_nchw(self):
        return [self.cache[o].transpose(0, 3, 1, 2) for o in self.outputs]


# ----------------------------------------------------------------------------- e4m3 stage
# The engine's optional e4m3 stride-8 stage has no reference counterpart (the reference
# keeps its tile weights in the engine dtype, fused_engine.py:114); these restate its
# arithmetic so that each e4m3 layer can be checked against its own inputs.
def e4m3(x):
    """Nearest e4m3 (E4M3FN) values of float array `x`, ties to even, saturated to +-448,
    as float32 (torch's float8_e4m3fn type does the rounding)."""
    import torch
    t = torch.from_numpy(np.clip(np.asarray(x, np.float32), -448.0, 448.0))
    return t.to(torch.float8_e4m3fn).to(torch.float32).numpy()


def e4m3_codes(x):
    """e4m3 bit patterns (uint8) of the values nearest to `x` (as `e4m3`)."""
    import torch
    t = torch.from_numpy(np.clip(np.asarray(x, np.float32), -448.0, 448.0))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def conv_dense_e4m3(x, w, bias, stride, act, res, s_out, w_scale=None):
    """One layer of an e4m3 stage, densely: x and res are dequantised float inputs; with
    `w_scale` (per output channel) the weights are first quantised as the engine quantises
    them, code = e4m3(w / s), value = code * s.  Returns the e4m3 codes of y / s_out, or with
    s_out = None the fp32 result (for the layer whose output leaves the stage in fp16)."""
    w = np.asarray(w, np.float32)
    if w_scale is not None:
        w = e4m3(w / w_scale[None, None, None, :]) * w_scale[None, None, None, :]
    y = conv_dense(np.asarray(x, np.float32), w, bias, stride, act, None if res is None else np.asarray(res, np.float32),
                   np.float32)
    return y if s_out is None else e4m3_codes(y / np.float32(s_out))
