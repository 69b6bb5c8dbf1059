"""Drop-in ``FusedSparseEngine`` on the B200 CUDA library.

Same constructor, attributes and methods as the reference
(Bahrombekk/Sarbon ``sarbon/sparse/fused_engine.py:54-275``) so that
``sarbon.inference.video.SarbonVideo`` and ``tests/test_fused_engine.py`` use it
unchanged:

* ``FusedSparseEngine(net, n_cams, height, width, block=32, dtype=torch.float16,
  tau=0.0, refresh=0, dense_check_every=4, device="cuda")``  (:55-56)
* ``reset(frames)``, ``step(frames) -> (mode, k)``, ``calibrate(...)``,
  ``set_extra(mask)``, ``outputs_nchw()``, ``dilation(radius)``  (:121-275)
* added: ``steer(boxes_per_cam, margin=1)``, the caller's track steering
  (``sarbon/inference/video.py:139-147``) as one kernel writing ``extra``
* added: ``set_cell_gating(cell)``, cell-level gating (``sarbon/sparse/gating.py:42-43``)
  inside the step
* added: ``block_units=True`` and ``set_m0(on, capacity)``, the M0 engine's semantics
  (``sarbon/sparse/block_sparse.py:196-295``) on this engine
* added: ``fp8=True``: e4m3 caches and weights in the stride-8 stage, ``fp8="all"`` in the
  stride-4 stage too (p4 stays fp16); ``calibrate_fp8`` sets the activation scales,
  ``outputs_nchw`` dequantises
* attributes ``n, h, w, block, hb, wb, n_blocks, dtype, tau, refresh, layers, ds,
  outputs, cache, frames, changed, extra, masks, buckets, fallback,
  dense_check_every, dense_graph, stats``.

Every kernel runs in ``libsarbon_sparse.so`` (C ABI ``include/sarbon_sparse.h``);
tensors here are zero-copy views of engine-owned device memory.  There is no
PyTorch or CPU fallback: without the library the constructor raises.
"""
from __future__ import annotations

import ctypes as C
import math
import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib


@dataclass
class Layer:
    """One fused conv(+add) (fused_engine.py:29-41)."""
    src: str
    dst: str
    res: str | None
    act: bool
    stride: int
    out_stride: int
    radius: int
    w_tile: torch.Tensor   # [3, 3, cin, cout] float32 (host)
    bias: torch.Tensor     # [cout] float32 (host)


def budget_buckets(n_blocks, unit=16, ratio=1.15):
    """Budgets ~15% apart, multiples of ``unit`` (fused_engine.py:44-51)."""
    out, b = [], unit
    while b < n_blocks:
        out.append(b)
        b = max(b + unit, int(math.ceil(b * ratio / unit)) * unit)
    out.append(int(math.ceil(n_blocks / unit)) * unit)
    return out


def tiles_per_program(t, block_m=64):
    """Tiles whose pixels fill one 64-pixel program (triton_conv.py:67-69); kept for the
    reference's bucket rule."""
    return max(1, block_m // (t * t))


def fuse_layers(net):
    """Fuse each conv with a following residual add (fused_engine.py:99-119)."""
    nodes, _ = net.program()
    layers, i = [], 0
    while i < len(nodes):
        n = nodes[i]
        c = n.conv
        if n.kind != "conv" or c.kernel_size[0] != 3 or c.padding[0] != 1:
            raise ValueError("the engine runs 3x3 / padding-1 convolutions only")
        nxt = nodes[i + 1] if i + 1 < len(nodes) else None
        fused = nxt is not None and nxt.kind == "add" and nxt.src[0] == n.dst
        w = c.weight.detach().float().cpu()
        layers.append(Layer(
            src=n.src[0], dst=nxt.dst if fused else n.dst,
            res=nxt.src[1] if fused else None, act=True if fused else bool(n.act),
            stride=c.stride[0], out_stride=n.stride,
            radius=nxt.radius if fused else n.radius,
            w_tile=w.permute(2, 3, 1, 0).contiguous(),
            bias=c.bias.detach().float().cpu().contiguous()))
        i += 2 if fused else 1
    return layers


class _DeviceView:
    """``__cuda_array_interface__`` over engine-owned memory; keeps the engine alive."""

    def __init__(self, ptr, shape, typestr, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def _view(ptr, shape, typestr, owner, device):
    return torch.as_tensor(_DeviceView(ptr, shape, typestr, owner), device=device)


class _Handle:
    """Owns the C engine; destroyed when the last view / engine reference goes away."""

    def __init__(self, ptr):
        self.ptr = ptr

    def __del__(self):
        if self.ptr:
            try:
                lib().sb_destroy(self.ptr)
            except Exception:
                pass
            self.ptr = None


class _DenseGraph:
    """``dense_graph.replay()``: dense pass from ``engine.frames`` (fused_engine.py:88)."""

    def __init__(self, engine):
        self._e = engine

    def replay(self):
        e = self._e
        check(lib().sb_dense(e._h.ptr, C.c_void_p(e.frames.data_ptr()), e._stream()), "sb_dense")


class FusedSparseEngine:
    MODES = _lib.MODE_NAMES

    def __init__(self, net, n_cams, height, width, block=32, dtype=torch.float16, tau=0.0, refresh=0,
                 dense_check_every=4, device="cuda", block_units=False, fp8=False):
        assert height % block == 0 and width % block == 0
        if dtype not in (torch.float16, torch.float32):
            raise ValueError("dtype must be torch.float16 or torch.float32")
        self.n, self.h, self.w, self.block = n_cams, height, width, block
        self.cell, self.cell_radii = 0, None  # block-level gating (set_cell_gating)
        self.hb, self.wb = height // block, width // block
        self.n_blocks = n_cams * self.hb * self.wb
        self.dtype, self.tau, self.refresh = dtype, tau, refresh
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise ValueError("the engine runs on CUDA devices only")
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        self._net = net
        self.layers = fuse_layers(net)
        self.ds = sorted({self.dilation(l.radius) for l in self.layers})
        self.outputs = tuple(net.program()[1])
        L = lib()
        ids = {"img": 0}
        for i, l in enumerate(self.layers):
            ids[l.dst] = i + 1
        self._ids = ids
        descs = (_lib.LayerDesc * len(self.layers))()
        for i, l in enumerate(self.layers):
            descs[i] = _lib.LayerDesc(ids[l.src], -1 if l.res is None else ids[l.res], l.w_tile.shape[2],
                                      l.w_tile.shape[3], l.stride, l.out_stride, l.radius, int(l.act))
        handle = C.c_void_p()
        with torch.cuda.device(self.dev):
            check(L.sb_create_ex(descs, len(self.layers), n_cams, height, width, block,
                                 _lib.SB_F16 if dtype == torch.float16 else _lib.SB_F32, float(tau),
                                 int(refresh), int(dense_check_every),
                                 (_lib.SB_CREATE_BLOCK_UNITS if block_units else 0)
                                 | (_lib.SB_CREATE_FP8_S8 if fp8 else 0)
                                 | (_lib.SB_CREATE_FP8_S4 if fp8 == "all" else 0), C.byref(handle)), "sb_create_ex")
        self._h = _Handle(handle.value)
        for i, l in enumerate(self.layers):
            w = np.ascontiguousarray(l.w_tile.numpy(), np.float32)
            b = np.ascontiguousarray(l.bias.numpy(), np.float32)
            check(L.sb_upload_weights(self._h.ptr, i, w.ctypes.data_as(C.POINTER(C.c_float)),
                                      b.ctypes.data_as(C.POINTER(C.c_float))), "sb_upload_weights")
        typ = "<f2" if dtype == torch.float16 else "<f4"
        self.cache = {}
        self.fp8_caches = set()  # caches holding e4m3 codes (fp8=True: the stride-8 stage)
        for name, cid in ids.items():
            ptr, shape = C.c_void_p(), (C.c_int64 * 4)()
            check(L.sb_cache_ptr(self._h.ptr, cid, C.byref(ptr), shape), "sb_cache_ptr")
            dt = C.c_int()
            check(L.sb_cache_dtype(self._h.ptr, cid, C.byref(dt), None), "sb_cache_dtype")
            if dt.value == _lib.SB_F8:
                self.cache[name] = _view(ptr.value, list(shape), "|u1", self._h, self.dev).view(torch.float8_e4m3fn)
                self.fp8_caches.add(name)
            else:
                self.cache[name] = _view(ptr.value, list(shape), typ, self._h, self.dev)
        chg, masks, extra, nd, dl = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_int(), (C.c_int * 4)()
        check(L.sb_gate_buffers(self._h.ptr, C.byref(chg), C.byref(masks), C.byref(extra), C.byref(nd), dl),
              "sb_gate_buffers")
        assert list(dl)[:nd.value] == self.ds, (list(dl), self.ds)
        shp = (n_cams, self.hb, self.wb)
        self.changed = _view(chg.value, shp, "|b1", self._h, self.dev)
        mall = _view(masks.value, (nd.value, *shp), "|b1", self._h, self.dev)
        self.masks = {d: mall[i] for i, d in enumerate(self.ds)}
        self.extra = _view(extra.value, shp, "|b1", self._h, self.dev)
        self.frames = torch.zeros(n_cams, height, width, 3, device=self.dev, dtype=dtype)
        self.buckets = budget_buckets(self.n_blocks)
        self._fallback = self.buckets[-1]
        self._dense_check_every = dense_check_every
        self.dense_graph = _DenseGraph(self)
        self._host_stats = {m: 0 for m in self.MODES}

    # ---------- knobs that live on the device ----------
    @property
    def fallback(self):
        return self._fallback

    @fallback.setter
    def fallback(self, v):
        self._fallback = int(v)
        check(lib().sb_set_fallback(self._h.ptr, int(v), self._stream()), "sb_set_fallback")

    def set_m0(self, on, capacity=0):
        """M0 semantics for the next steps (block_sparse.py:196-295): the whole frame enters
        the image cache every step, no dense fallback, and with ``capacity`` > 0 every layer
        recomputes exactly the first ``capacity`` entries of its block list (padded with
        block 0).  Needs ``block_units=True`` (or an fp32 engine)."""
        check(lib().sb_set_m0(self._h.ptr, int(bool(on)), int(capacity)), "sb_set_m0")

    def set_step_graphs(self, on):
        """Replay each step's launch sequence as a captured CUDA graph (default) or launch
        every kernel from the host (``on=False``)."""
        check(lib().sb_set_step_graphs(self._h.ptr, int(bool(on))), "sb_set_step_graphs")

    def set_tau(self, tau):
        """Change threshold for the steps launched after this call (mean |diff| per block;
        an extension: the reference fixes `tau` at construction)."""
        self.tau = float(tau)
        check(lib().sb_set_tau(self._h.ptr, float(tau)), "sb_set_tau")

    @property
    def dense_check_every(self):
        return self._dense_check_every

    @dense_check_every.setter
    def dense_check_every(self, v):
        self._dense_check_every = int(v)
        check(lib().sb_set_dense_check_every(self._h.ptr, int(v), self._stream()), "sb_set_dense_check_every")

    @property
    def stats(self):
        s = _lib.Stats()
        check(lib().sb_stats(self._h.ptr, self._stream(), C.byref(s)), "sb_stats")
        return {"skip": s.skip, "sparse": s.sparse, "dense": s.dense}

    def device_stats(self):
        s = _lib.Stats()
        check(lib().sb_stats(self._h.ptr, self._stream(), C.byref(s)), "sb_stats")
        return s

    # ---------- helpers ----------
    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    def dilation(self, radius):
        return math.ceil(radius / self.block)

    def outputs_nchw(self):
        """p4, p8 as NCHW views of the caches; an e4m3 cache is returned dequantised (a new
        fp16 tensor: code * its activation scale)."""
        return [self.dequantized(o).permute(0, 3, 1, 2) for o in self.outputs]

    def act_scale(self, name):
        """Activation scale of an e4m3 cache (value = code * scale)."""
        dt, sc = C.c_int(), C.c_float()
        check(lib().sb_cache_dtype(self._h.ptr, self._ids[name], C.byref(dt), C.byref(sc)), "sb_cache_dtype")
        return float(sc.value)

    def set_act_scale(self, name, scale):
        """Activation scale of the e4m3 cache `name` for the next steps."""
        check(lib().sb_set_act_scale(self._h.ptr, self._ids[name], float(scale)), "sb_set_act_scale")

    def dequantized(self, name):
        """Cache `name` in the engine dtype: itself, or for an e4m3 cache code * scale."""
        c = self.cache[name]
        if name not in self.fp8_caches:
            return c
        return c.to(self.dtype) * self.act_scale(name)

    def weight_scales(self, layer):
        """Per-output-channel scales of layer `layer`'s e4m3 weights (fp8 engines)."""
        n = self.layers[layer].w_tile.shape[3]
        out = (C.c_float * n)()
        check(lib().sb_layer_wscale(self._h.ptr, int(layer), out, n), "sb_layer_wscale")
        return np.array(list(out), np.float32)

    @torch.no_grad()
    def calibrate_fp8(self, frames, net=None, headroom=2.0):
        """Activation scales of the e4m3 caches from a dense fp16 pass over `frames`:
        scale = the power of two at or above headroom * max|activation| / 448 (so that
        scaling is exact and a value `headroom` times the largest seen still fits e4m3).
        `net` is the stem the engine was built from (default: the one it was given)."""
        ref = FusedSparseEngine(net if net is not None else self._net, self.n, self.h, self.w, block=self.block,
                                dtype=torch.float16, device=self.dev)
        ref.reset(frames.to(torch.float16))
        out = {}
        for name in sorted(self.fp8_caches):
            amax = float(ref.cache[name].float().abs().max())
            sc = 2.0 ** math.ceil(math.log2(max(headroom * amax / 448.0, 2.0 ** -30)))
            self.set_act_scale(name, sc)
            out[name] = sc
        return out

    def _bucket(self, k):
        """fused_engine.py:188-193 (used by calibrate)."""
        lo = max(tiles_per_program(self.block // l.out_stride) for l in self.layers)
        for b in self.buckets:
            if b >= k and b % lo == 0:
                return b
        return self.buckets[-1]

    def set_extra(self, mask):
        """Blocks [N, Hb, Wb] recomputed next step regardless of pixel change (:201-205)."""
        self.extra.copy_(mask)  # a view of the engine's mask: the next gate reads it

    def set_cell_gating(self, cell):
        """Gate at cell level from the next step on (``cell`` px, a multiple of 8 dividing
        the block; 0 = block level, the reference's engine behaviour).

        The tighter estimate of the reference's gating analysis (gating.py:42-43): cells
        whose exact sum of |diff| exceeds float32(tau * cell^2 * 3) are dilated by
        ceil(R / cell) cells, R the largest receptive radius of each dilation group, and
        any-pooled into the group's block mask.  Lossless at tau = 0, like block level; a
        change in the middle of a block no longer activates its whole ring of neighbours.
        fp16 engines and ``step``/``step_async`` only (not ``step_u8``)."""
        if cell == 0:
            check(lib().sb_set_cell_gating(self._h.ptr, 0, None, 0), "sb_set_cell_gating")
            self.cell, self.cell_radii = 0, None
            return
        rc = [0] * len(self.ds)
        for l in self.layers:
            di = self.ds.index(self.dilation(l.radius))
            rc[di] = max(rc[di], -(-l.radius // cell))
        arr = (C.c_int * len(rc))(*rc)
        check(lib().sb_set_cell_gating(self._h.ptr, int(cell), arr, len(rc)), "sb_set_cell_gating")
        self.cell, self.cell_radii = int(cell), rc

    def steer(self, boxes_per_cam, margin=1):
        """Track steering (video.py:139-147): the blocks each camera's predicted boxes
        (xyxy, engine pixels) touch, widened by ``margin`` blocks, become the ``extra`` mask
        of the next step.  One kernel writes the engine's mask from the uploaded boxes."""
        from .gating import boxes_to_block_masks
        if len(boxes_per_cam) != self.n:
            raise ValueError(f"need one box list per camera ({self.n}), got {len(boxes_per_cam)}")
        boxes_to_block_masks(boxes_per_cam, self.hb, self.wb, self.block, margin, out=self.extra)

    def block_lists(self, d):
        """Active (cam, by, bx) int32 lists of dilation d from the last gated step."""
        di = self.ds.index(d)
        cam, by, bx, k = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_int64()
        check(lib().sb_debug_lists(self._h.ptr, di, C.byref(cam), C.byref(by), C.byref(bx), C.byref(k),
                                   self._stream()), "sb_debug_lists")
        n = int(k.value)
        if n == 0:
            return tuple(torch.zeros(0, dtype=torch.int32, device=self.dev) for _ in range(3))
        return tuple(_view(p.value, (n,), "<i4", self._h, self.dev).clone() for p in (cam, by, bx))

    # ---------- runtime ----------
    @torch.no_grad()
    def reset(self, frames):
        """Dense initialisation from [N, H, W, 3] frames (:207-212)."""
        self.frames.copy_(frames)
        check(lib().sb_reset(self._h.ptr, C.c_void_p(self.frames.data_ptr()), self._stream()), "sb_reset")

    @torch.no_grad()
    def step(self, frames):
        """Process one [N, H, W, 3] frame batch; returns (mode, active count) (:214-240).
        The count is -1 for dense steps taken without a gate look (hysteresis)."""
        self.frames.copy_(frames)
        mode, k = C.c_int(), C.c_int64()
        check(lib().sb_step(self._h.ptr, C.c_void_p(self.frames.data_ptr()), self._stream(), C.byref(mode),
                            C.byref(k)), "sb_step")
        name = self.MODES[mode.value]
        self._host_stats[name] += 1
        return name, int(k.value)

    @torch.no_grad()
    def step_async(self, frames):
        """Launch one step on ``frames`` (device tensor in the engine dtype, used in place)
        without a host sync; read the result later with :meth:`query`."""
        check(lib().sb_step(self._h.ptr, C.c_void_p(frames.data_ptr()), self._stream(), None, None), "sb_step")

    @torch.no_grad()
    def step_u8(self, frames_u8, mean, std, sync=True):
        """One step on uint8 BGR frames [N, h, w, 3] (device memory) with the caller's
        ``_prep`` (video.py:95-99) done by this library: BGR->RGB, (x - mean) / std in fp32,
        fp16 -- fused into the gate at engine size, or, for cameras of another size, one
        prep kernel that also resizes bilinearly (align_corners=False) to the engine size."""
        if frames_u8.dtype != torch.uint8 or frames_u8.dim() != 4 or frames_u8.shape[0] != self.n \
                or frames_u8.shape[3] != 3 or not frames_u8.is_contiguous():
            raise ValueError(f"need contiguous uint8 frames [{self.n}, h, w, 3]")
        mean = (C.c_float * 3)(*[float(np.float32(v)) for v in mean])
        std = (C.c_float * 3)(*[float(np.float32(v)) for v in std])
        mode, k = C.c_int(), C.c_int64()
        cam_h, cam_w = int(frames_u8.shape[1]), int(frames_u8.shape[2])
        if (cam_h, cam_w) == (self.h, self.w):
            check(lib().sb_step_u8(self._h.ptr, C.c_void_p(frames_u8.data_ptr()), mean, std, self._stream(),
                                   C.byref(mode) if sync else None, C.byref(k) if sync else None), "sb_step_u8")
        else:
            check(lib().sb_step_u8_resized(self._h.ptr, C.c_void_p(frames_u8.data_ptr()), cam_h, cam_w, mean, std,
                                           self._stream(), C.byref(mode) if sync else None,
                                           C.byref(k) if sync else None), "sb_step_u8_resized")
        if sync:
            return self.MODES[mode.value], int(k.value)
        return None

    @torch.no_grad()
    def step_profiled(self, frames):
        """One step on ``frames`` (used in place) with a CUDA event around every kernel;
        returns (mode, k, [ms per launch]) with launches ordered gate, lists, copy,
        conv per layer, finalize."""
        cap = 64
        ms, n = (C.c_float * cap)(), C.c_int()
        check(lib().sb_step_profiled(self._h.ptr, C.c_void_p(frames.data_ptr()), self._stream(), ms, cap,
                                     C.byref(n)), "sb_step_profiled")
        mode, k = self.query()
        return mode, k, [ms[i] for i in range(n.value)]

    @torch.no_grad()
    def dense_layers(self, first, last=None):
        """Recompute layers ``first..last`` densely from the caches as they are (the image
        cache and the gate untouched): one layer of this engine on inputs loaded from
        elsewhere, e.g. the reference's own caches."""
        last = first if last is None else last
        check(lib().sb_dense_layers(self._h.ptr, int(first), int(last), self._stream()), "sb_dense_layers")

    @torch.no_grad()
    def step_phases(self, frames):
        """One step on ``frames`` (used in place) with CUDA events only between its phases;
        returns (mode, k, {"gate", "lists", "copy", "conv", "finalize": ms}).  The conv
        phase is the whole layer sequence launched as in ``step`` (layers overlap their
        start-up with the previous layer's tail)."""
        ms = (C.c_float * 5)()
        check(lib().sb_step_phases(self._h.ptr, C.c_void_p(frames.data_ptr()), self._stream(), ms),
              "sb_step_phases")
        mode, k = self.query()
        return mode, k, dict(zip(("gate", "lists", "copy", "conv", "finalize"), list(ms)))

    def result_view(self):
        """int64 [2] device tensor {mode, count} written by every step's last kernel."""
        p = C.c_void_p()
        check(lib().sb_result_ptr(self._h.ptr, C.byref(p)), "sb_result_ptr")
        return _view(p.value, (2,), "<i8", self._h, self.dev)

    def query(self):
        mode, k = C.c_int(), C.c_int64()
        check(lib().sb_query(self._h.ptr, self._stream(), C.byref(mode), C.byref(k)), "sb_query")
        return self.MODES[mode.value], int(k.value)

    def launch_count(self):
        return lib().sb_last_launch_count(self._h.ptr)

    def layer_variants(self):
        """Per layer, the tile-conv variant it runs: window mode (0 per-tap boxes / first-layer
        gather, 1 row, 2 strided, 3 full windows) + 8 for CTA pairs + 16 * its e4m3 mode (1:
        e4m3 output, 2: e4m3 input and output); -1 on fp32 engines."""
        out = []
        for i in range(len(self.layers)):
            m = C.c_int()
            check(lib().sb_layer_variant(self._h.ptr, i, C.byref(m)), "sb_layer_variant")
            out.append(int(m.value))
        return out

    @torch.no_grad()
    def calibrate(self, reps=15, margin=0.95, dense_ref=None):
        """Time every budget bucket against the dense pass; set the crossover (:242-275).
        Sparse and dense runs are interleaved and compared by their best times."""
        def once(fn):
            torch.cuda.synchronize(self.dev)
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize(self.dev)
            return time.perf_counter() - t0

        dense = dense_ref or self.dense_graph.replay
        saved = {k: v.clone() for k, v in self.cache.items()}
        fp = C.c_void_p(self.frames.data_ptr())
        fallback, table, above = 0, [], 0
        for b in sorted({self._bucket(x) for x in self.buckets}):
            n = min(b, self.n_blocks)

            def sparse(n=n):
                check(lib().sb_run_sparse_forced(self._h.ptr, fp, n, self._stream()), "sb_run_sparse_forced")
            sparse()
            pairs = [(once(sparse), once(dense)) for _ in range(reps)]
            ratio = min(s for s, _ in pairs) / min(d for _, d in pairs)
            table.append((b, min(s for s, _ in pairs) * 1e3, ratio))
            if ratio > margin:
                above += 1
                if above == 2:
                    break
            else:
                above, fallback = 0, b
        for k, v in saved.items():
            self.cache[k].copy_(v)
        self.fallback = fallback
        return table
