"""Kernels of the detector after the stem (sarbon/models/sarbon_det.py:118-356), one call each.

Every op launches one kernel of ``libsarbon_sparse.so`` on the current CUDA stream, writes
into caller-provided (or freshly allocated) tensors and can be captured in a CUDA graph.
Feature maps are NHWC: a tensor ``[B, H, W, C]`` whose channels are contiguous; a
``[rows, C]`` matrix is the map ``[1, 1, rows, C]``.  Views whose pixels are ``ld``
elements apart (a channel slice of a wider map) and whose images are further apart than
``H * W`` pixels (one level inside the decoder's concatenated memory) are accepted as
sources, residuals and outputs.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, lib

ACT = {None: 0, "none": 0, "relu": 1, "gelu": 2}

# kernel launches issued through this module (each op is one launch)
LAUNCHES = [0]


def _stream(t):
    LAUNCHES[0] += 1
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def as_map(t: torch.Tensor) -> torch.Tensor:
    """A [rows, C] matrix as the 1 x rows map [1, 1, rows, C]; 4-D maps unchanged."""
    if t.dim() == 2:
        return t.unsqueeze(0).unsqueeze(0)
    if t.dim() != 4:
        raise ValueError(f"expected an NHWC map or a matrix, got shape {tuple(t.shape)}")
    return t


def _geometry(t: torch.Tensor, what: str):
    """(ld, img_stride) of an NHWC view: pixels ld elements apart, images img_stride pixels."""
    b, h, w, c = t.shape
    if t.stride(3) != 1:
        raise ValueError(f"{what}: channels must be contiguous")
    ld = t.stride(2)
    if h > 1 and t.stride(1) != w * ld:
        raise ValueError(f"{what}: rows of a map must follow each other")
    img = t.stride(0) // ld if b > 1 else h * w
    if b > 1 and t.stride(0) % ld != 0:
        raise ValueError(f"{what}: image stride is not a whole number of pixels")
    return ld, img


def gemm_conv(srcs, weight, bias=None, act=None, taps=1, stride=1, res=None, out=None, out_dtype=torch.float16):
    """out = act(conv_or_linear(cat(srcs, channels), weight) + bias + res) in one launch.

    srcs: one NHWC fp16 map or a list of two with the same B, H, W (their channels are
    concatenated); weight: fp16 [N, taps * sum(C)] with columns (tap = ky * 3 + kx, channel);
    bias: fp32 [N]; taps 1 (stride 1) or 9 (3x3, padding 1, stride 1 or 2).  Returns out
    [B, Ho, Wo, N] (matrix inputs give a [rows, N] matrix)."""
    if isinstance(srcs, torch.Tensor):
        srcs = [srcs]
    matrix = srcs[0].dim() == 2
    maps = [as_map(s) for s in srcs]
    b, h, w, _ = maps[0].shape
    for m in maps:
        if m.shape[:3] != (b, h, w) or m.dtype != torch.float16 or not m.is_cuda:
            raise ValueError("sources: fp16 CUDA maps of one size")
    arr = (_lib.GemmSrc * len(maps))()
    for i, m in enumerate(maps):
        ld, img = _geometry(m, "source")
        arr[i].ptr, arr[i].C, arr[i].ld, arr[i].img_stride = m.data_ptr(), m.shape[3], ld, img
    n = weight.shape[0]
    if weight.dtype != torch.float16 or not weight.is_contiguous():
        raise ValueError("weight: contiguous fp16 [N, K]")
    ho = (h - 1) // stride + 1 if taps == 9 else h
    wo = (w - 1) // stride + 1 if taps == 9 else w
    if out is None:
        out = torch.empty(b, ho, wo, n, device=maps[0].device, dtype=out_dtype)
        if matrix:
            out = out.view(ho * wo, n)
    om = as_map(out)
    if om.shape != (b, ho, wo, n):
        raise ValueError(f"out: expected {(b, ho, wo, n)}, got {tuple(om.shape)}")
    o_ld, o_img = _geometry(om, "out")
    r_ptr, r_dt, r_ld, r_img = None, _lib.SB_F16, 0, 0
    if res is not None:
        rm = as_map(res)
        if rm.shape != (b, ho, wo, n):
            raise ValueError(f"res: expected {(b, ho, wo, n)}, got {tuple(rm.shape)}")
        r_ld, r_img = _geometry(rm, "res")
        r_ptr, r_dt = rm.data_ptr(), (_lib.SB_F32 if rm.dtype == torch.float32 else _lib.SB_F16)
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise ValueError("bias: contiguous fp32 [N]")
    if taps == 1 and b * h * w > w:
        # a 1x1 conv whose operands are dense over the images is one [B*H*W, C] matrix product
        # (its tiles are then full 128-row blocks)
        dense = all(arr[i].img_stride == h * w for i in range(len(maps))) and o_img == h * w and \
            (res is None or r_img == h * w)
        if dense:
            for i in range(len(maps)):
                arr[i].img_stride = b * h * w
            b, h, w = 1, 1, b * h * w
            o_img = r_img = h * w
    check(lib().sb_gemm_conv(arr, len(maps), b, h, w, taps, stride, C.c_void_p(weight.data_ptr()), n,
                             C.c_void_p(bias.data_ptr() if bias is not None else None), ACT[act],
                             C.c_void_p(r_ptr), r_dt, r_ld, r_img, C.c_void_p(om.data_ptr()),
                             _lib.SB_F32 if om.dtype == torch.float32 else _lib.SB_F16, o_ld, o_img,
                             _stream(om)),
          "sb_gemm_conv")
    return out


def kernels_error(clear=True) -> int:
    """Sticky error flags of the detector kernels' bounded waits (0 = none); synchronises."""
    v = C.c_int(0)
    check(lib().sb_kernels_error(int(clear), C.byref(v)), "sb_kernels_error")
    return v.value


# ---------------------------------------------------------------- row ops
def _rows(t: torch.Tensor, what: str):
    """(ptr, ld, img) of [rows, D] or [B, T, D] rows with contiguous columns."""
    if t.stride(-1) != 1:
        raise ValueError(f"{what}: columns must be contiguous")
    ld = t.stride(-2)
    img = (t.stride(0) // ld) if t.dim() == 3 else t.shape[0]
    return t.data_ptr(), ld, img


def _dt(t):
    return _lib.SB_F32 if t.dtype == torch.float32 else _lib.SB_F16


def layernorm(a, weight, bias, eps, b=None, y32=None, y16=None, pos=None, sign=1.0, yp16=None, period=None):
    """nn.LayerNorm of the rows of a (+ b): fp32 statistics; fills the given outputs
    (y32 fp32, y16 fp16, yp16 = fp16(y + sign * pos[row % period]))."""
    rows, d = a.numel() // a.shape[-1], a.shape[-1]
    a2 = a.view(rows, d)  # views only: a copy would detach outputs from their storage
    b2 = b.view(rows, d) if b is not None else None
    pa, la, _ = _rows(a2, "a")
    pb, lb, _ = _rows(b2, "b") if b2 is not None else (None, 0, 0)
    out = {}
    for name, t in (("y32", y32), ("y16", y16), ("yp16", yp16)):
        out[name] = _rows(t.view(rows, d), name)[:2] if t is not None else (None, 0)
    pp, lp = (pos.data_ptr(), pos.stride(-2)) if pos is not None else (None, 0)
    check(lib().sb_layernorm(C.c_void_p(pa), _dt(a2), la, C.c_void_p(pb), _dt(b2) if b2 is not None else 0, lb,
                             C.c_void_p(weight.data_ptr()), C.c_void_p(bias.data_ptr()), float(eps), rows, d,
                             C.c_void_p(out["y32"][0]), out["y32"][1], C.c_void_p(out["y16"][0]), out["y16"][1],
                             C.c_void_p(pp), lp, int(period or rows), float(sign), C.c_void_p(out["yp16"][0]),
                             out["yp16"][1], _stream(a)),
          "sb_layernorm")


def add_rows(a, b, out, sign=1.0, period=None):
    """out (fp16) = fp16(a + sign * b[row % period]) over [rows, D]."""
    rows, d = a.numel() // a.shape[-1], a.shape[-1]
    pa, la, _ = _rows(a.view(rows, d), "a")
    pb, lb, _ = _rows(b.view(-1, d), "b")
    po, lo, _ = _rows(out.view(rows, d), "out")
    check(lib().sb_add_rows(C.c_void_p(pa), _dt(a), la, C.c_void_p(pb), _dt(b), lb, int(period or rows), float(sign),
                            rows, d, C.c_void_p(po), lo, _stream(a)),
          "sb_add_rows")
    return out


def dwconv3x3(x, w9c, bias, relu=True, out=None):
    """Depthwise 3x3 (padding 1) + bias + ReLU on an NHWC fp16 map; w9c fp32 [9, C]."""
    b, h, w, c = x.shape
    lx, ix = _geometry(x, "x")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format) if x.is_contiguous() else \
            torch.empty(b, h, w, c, device=x.device, dtype=x.dtype)
    ly, iy = _geometry(out, "out")
    check(lib().sb_dwconv3x3(C.c_void_p(x.data_ptr()), lx, ix, b, h, w, c, C.c_void_p(w9c.data_ptr()),
                             C.c_void_p(bias.data_ptr()), int(relu), C.c_void_p(out.data_ptr()), ly, iy, _stream(x)),
          "sb_dwconv3x3")
    return out


def upsample2x(x, out=None):
    b, h, w, c = x.shape
    lx, ix = _geometry(x, "x")
    if out is None:
        out = torch.empty(b, 2 * h, 2 * w, c, device=x.device, dtype=x.dtype)
    ly, iy = _geometry(out, "out")
    check(lib().sb_upsample2x(C.c_void_p(x.data_ptr()), lx, ix, b, h, w, c, C.c_void_p(out.data_ptr()), ly, iy,
                              _stream(x)),
          "sb_upsample2x")
    return out


def attention(q, k, v, heads, out=None):
    """softmax(q k^T / sqrt(32)) v per head for [B, T, heads*32] fp16 rows (views allowed)."""
    bq, tq, d = q.shape
    tk = k.shape[1]
    if out is None:
        out = torch.empty(bq, tq, d, device=q.device, dtype=torch.float16)
    pq, lq, iq = _rows(q, "q")
    pk, lk, ik = _rows(k, "k")
    pv, lv, iv = _rows(v, "v")
    po, lo, io = _rows(out, "out")
    check(lib().sb_attention(C.c_void_p(pq), lq, iq, C.c_void_p(pk), lk, ik, C.c_void_p(pv), lv, iv, bq, heads,
                             d // heads, tq, tk, C.c_void_p(po), lo, io, _stream(q)),
          "sb_attention")
    return out


def topk_rows(logits, k, valid=None, out=None):
    """[B, S, C] fp16 logits -> int32 [B, k] rows with the largest max-over-classes value."""
    b, s, c = logits.shape
    if out is None:
        out = torch.empty(b, k, device=logits.device, dtype=torch.int32)
    p, ld, img = _rows(logits, "logits")
    check(lib().sb_topk_rows(C.c_void_p(p), ld, img, b, s, c,
                             C.c_void_p(valid.data_ptr() if valid is not None else None), k,
                             C.c_void_p(out.data_ptr()), out.stride(0), _stream(logits)),
          "sb_topk_rows")
    return out


def gather_rows(src, idx, o32=None, o16=None):
    """o[b, i] = src[b, idx[b, i]] for [B, S, D] rows; fills o32 (fp32) and/or o16 (fp16)."""
    b, kk = idx.shape
    d = src.shape[-1]
    ps, ls, is_ = _rows(src, "src")
    a32 = _rows(o32, "o32") if o32 is not None else (None, 0, 0)
    a16 = _rows(o16, "o16") if o16 is not None else (None, 0, 0)
    rows = src.shape[-2]
    check(lib().sb_gather_rows(C.c_void_p(ps), _dt(src), ls, is_, rows, C.c_void_p(idx.data_ptr()), idx.stride(0), b,
                               kk, d, C.c_void_p(a32[0]), a32[1], a32[2], C.c_void_p(a16[0]), a16[1], a16[2],
                               _stream(src)),
          "sb_gather_rows")


def deform_sample(value, shapes, off, att, ref, heads, points, out=None):
    """MSDeformAttn between its projections: value [B, S, heads*32], off [B, Q, heads*L*P*2],
    att logits [B, Q, heads*L*P] (fp16), ref [B, Q, 4] (fp16 or fp32) -> fp16 [B, Q, heads*32]."""
    b, q = off.shape[:2]
    if out is None:
        out = torch.empty(b, q, value.shape[-1], device=value.device, dtype=torch.float16)
    hw = [int(x) for s in shapes for x in s]
    arr = (C.c_int * len(hw))(*hw)
    pv, lv, iv = _rows(value, "value")
    po_, lo_, io_ = _rows(off, "off")
    pa, la, ia = _rows(att, "att")
    pr, lr, ir = _rows(ref, "ref")
    pout, lout, iout = _rows(out, "out")
    check(lib().sb_deform_sample(C.c_void_p(pv), lv, iv, arr, len(shapes), C.c_void_p(po_), lo_, io_, C.c_void_p(pa),
                                 la, ia, C.c_void_p(pr), _dt(ref), lr, ir, b, q, heads, points, C.c_void_p(pout), lout,
                                 iout, _stream(value)),
          "sb_deform_sample")
    return out


def box_enc(encbox, anchors, idx, ref16, qin):
    b, kk = idx.shape
    check(lib().sb_box_enc(C.c_void_p(encbox.data_ptr()), encbox.stride(-2), C.c_void_p(anchors.data_ptr()),
                           anchors.shape[0], C.c_void_p(idx.data_ptr()), b, kk, C.c_void_p(ref16.data_ptr()),
                           C.c_void_p(qin.data_ptr()), qin.stride(-2), _stream(encbox)),
          "sb_box_enc")


def box_dec(first, head, corners, project, reg_scale, ref_init, box, prebox=None, ref16=None, qin=None):
    rows = corners.numel() // corners.shape[-1]
    r1 = project.numel()
    check(lib().sb_box_dec(int(first), C.c_void_p(prebox.data_ptr() if prebox is not None else None),
                           prebox.stride(-2) if prebox is not None else 0,
                           C.c_void_p(ref16.data_ptr() if ref16 is not None else None), C.c_void_p(head.data_ptr()),
                           head.stride(-2), C.c_void_p(corners.data_ptr()), corners.stride(-2), r1,
                           C.c_void_p(project.data_ptr()), float(reg_scale), C.c_void_p(ref_init.data_ptr()),
                           C.c_void_p(box.data_ptr()), C.c_void_p(qin.data_ptr() if qin is not None else None),
                           qin.stride(-2) if qin is not None else 0, rows, _stream(head)),
          "sb_box_dec")


def l2norm_rows(x, out):
    rows, d = x.numel() // x.shape[-1], x.shape[-1]
    check(lib().sb_l2norm_rows(C.c_void_p(x.data_ptr()), x.stride(-2), rows, d, C.c_void_p(out.data_ptr()),
                               out.stride(-2), _stream(x)),
          "sb_l2norm_rows")
    return out


def _time_one(argv):
    """Time one sb_gemm_conv shape with CUDA events (10 launches after 4 warm-up launches):
    ``python -m sarbon_b200.det_ops linear M K N`` or ``... conv B H W CIN COUT STRIDE``."""
    kind, dims = argv[0], [int(x) for x in argv[1:]]
    g = torch.Generator(device="cuda").manual_seed(0)
    if kind == "linear":
        m, k, n = dims
        x = torch.randn(m, k, device="cuda", generator=g).half()
        w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).half()
        out = torch.empty(m, n, device="cuda", dtype=torch.float16)
        taps, stride, flops, act = 1, 1, 2 * m * k * n, None
    else:
        b, h, wd, c, n, stride = dims
        x = torch.randn(b, h, wd, c, device="cuda", generator=g).half()
        w = (torch.randn(n, 9 * c, device="cuda", generator=g) / (9 * c) ** 0.5).half()
        ho, wo = (h - 1) // stride + 1, (wd - 1) // stride + 1
        out = torch.empty(b, ho, wo, n, device="cuda", dtype=torch.float16)
        taps, flops, act = 9, 2 * b * ho * wo * n * 9 * c, "relu"
    bias = torch.randn(n, device="cuda", generator=g)

    def run():
        gemm_conv(x, w, bias, act=act, taps=taps, stride=stride, out=out)

    for _ in range(4):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 10
    moved = (x.numel() + out.numel()) * 2
    print(f"{kind} {dims}: {ms * 1e3:.1f} us per launch, {flops / ms / 1e9:.1f} TFLOP/s, "
          f"{moved / ms / 1e6:.1f} GB/s of input + output; error flags {kernels_error()}")


if __name__ == "__main__":
    import sys
    _time_one(sys.argv[1:])
