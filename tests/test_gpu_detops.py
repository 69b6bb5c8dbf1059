"""The detector's row kernels against torch on the same inputs (sarbon_det.py, deform_attn.py,
box_ops.py semantics): LayerNorm with a residual and the pos outputs, depthwise conv,
nearest upsampling, attention, top-K selection, row gathers, deformable sampling and the
box heads."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def test_layernorm_outputs():
    from sarbon_b200 import det_ops as ops
    g = gen(1)
    rows, d = 600, 256
    a = torch.randn(rows, d, device="cuda", generator=g)
    b = torch.randn(rows, d, device="cuda", generator=g).half()
    pos = torch.randn(300, d, device="cuda", generator=g).half()
    w = torch.rand(d, device="cuda", generator=g) + 0.5
    bb = torch.randn(d, device="cuda", generator=g)
    y32 = torch.empty(rows, d, device="cuda")
    y16 = torch.empty(rows, d, device="cuda", dtype=torch.float16)
    yp = torch.empty(rows, d, device="cuda", dtype=torch.float16)
    ops.layernorm(a, w, bb, 1e-5, b=b, y32=y32, y16=y16, pos=pos, sign=-1.0, yp16=yp, period=300)
    ref = F.layer_norm(a + b.float(), (d,), w, bb, 1e-5)
    assert (y32 - ref).abs().max().item() < 1e-4
    assert torch.equal(y16, y32.half())
    assert torch.equal(yp, (y32 - pos.float().repeat(2, 1)).half())
    # fp16 + fp16: the sum is rounded to fp16 first
    a16 = a.half()
    ops.layernorm(a16, w, bb, 1e-5, b=b, y32=y32)
    ref = F.layer_norm((a16 + b).float(), (d,), w, bb, 1e-5)
    assert (y32 - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("b,h,w,c", [(2, 24, 40, 256), (1, 23, 7, 64), (3, 1, 5, 8)])
def test_dwconv_and_upsample(b, h, w, c):
    from sarbon_b200 import det_ops as ops
    g = gen(2 + h)
    x = torch.randn(b, h, w, c, device="cuda", generator=g).half()
    wt = torch.randn(c, 1, 3, 3, device="cuda", generator=g) / 3
    bias = torch.randn(c, device="cuda", generator=g)
    y = ops.dwconv3x3(x, wt.view(c, 9).t().contiguous(), bias, relu=True)
    ref = F.relu(F.conv2d(x.permute(0, 3, 1, 2).float(), wt, bias, padding=1, groups=c)).permute(0, 2, 3, 1)
    assert (y.float() - ref).abs().max().item() <= 2e-3 * ref.abs().max().item()
    up = ops.upsample2x(x)
    ref = F.interpolate(x.permute(0, 3, 1, 2), scale_factor=2.0).permute(0, 2, 3, 1)
    assert torch.equal(up, ref)


# (2341, 2333, 16): ragged query and key counts (37 CTAs x 16 heads x 2 images, 37 key tiles);
# (5, 1, 8): one key, 63 masked slots of its tile; (70, 64, 8) one full key tile; (64, 129, 2)
# a last tile with one key
@pytest.mark.parametrize("tq,tk,heads", [(300, 300, 8), (240, 240, 8), (2040, 2040, 8), (1, 77, 8), (130, 65, 4),
                                         (2341, 2333, 16), (5, 1, 8), (70, 64, 8), (64, 129, 2)])
def test_attention(tq, tk, heads):
    from sarbon_b200 import det_ops as ops
    g = gen(tq + tk)
    b, d = 2, heads * 32
    q = torch.randn(b, tq, d, device="cuda", generator=g).half()
    kv = torch.randn(b, tk, 2 * d, device="cuda", generator=g).half()
    k, v = kv[..., :d], kv[..., d:]
    out = ops.attention(q, k, v, heads)
    qh = q.float().view(b, tq, heads, 32).transpose(1, 2)
    kh = k.float().reshape(b, tk, heads, 32).transpose(1, 2)
    vh = v.float().reshape(b, tk, heads, 32).transpose(1, 2)
    ref = torch.softmax(qh @ kh.transpose(-1, -2) / math.sqrt(32), -1) @ vh
    ref = ref.transpose(1, 2).reshape(b, tq, d)
    assert (out.float() - ref).abs().max().item() < 2e-3


@pytest.mark.parametrize("s,k", [(5040, 300), (42840, 300), (300, 300), (5040, 1)])
def test_topk_rows(s, k):
    from sarbon_b200 import det_ops as ops
    g = gen(s + k)
    b, c = 2, 6
    logits = (torch.randn(b, s, c, device="cuda", generator=g) * 3).half()
    valid = (torch.rand(s, device="cuda", generator=g) > 0.1).to(torch.uint8)
    if k == s:
        valid.fill_(1)
    idx = ops.topk_rows(logits, k, valid)
    score = logits.max(-1).values.float().masked_fill(valid == 0, float("-inf"))
    # expected: value descending, then row ascending (a stable order of torch's selection)
    key = score * (s + 1) * 0  # placeholder to keep the device
    order = torch.stack([torch.tensor(sorted(range(s), key=lambda i: (-score[bb, i].item(), i))[:k])
                         for bb in range(b)]) if s <= 6000 else None
    got_vals = torch.gather(score, 1, idx.long())
    ref_vals = score.topk(k, 1).values
    assert torch.equal(got_vals, ref_vals)
    if order is not None:
        assert torch.equal(idx.long().cpu(), order)
    del key


def test_gather_rows():
    from sarbon_b200 import det_ops as ops
    g = gen(3)
    src = torch.randn(2, 500, 256, device="cuda", generator=g)
    idx = torch.randint(0, 500, (2, 300), device="cuda", generator=g, dtype=torch.int32)
    o32 = torch.empty(2, 300, 256, device="cuda")
    o16 = torch.empty(2, 300, 256, device="cuda", dtype=torch.float16)
    ops.gather_rows(src, idx, o32=o32, o16=o16)
    ref = torch.gather(src, 1, idx.long()[..., None].expand(-1, -1, 256))
    assert torch.equal(o32, ref) and torch.equal(o16, ref.half())
    # an index outside the image's rows gives a zero row, not a read past them
    idx[0, 0], idx[1, 5] = 500, -1
    ops.gather_rows(src, idx, o32=o32)
    assert not o32[0, 0].any() and not o32[1, 5].any()
    assert torch.equal(o32[0, 1:], ref[0, 1:])


@pytest.mark.parametrize("ref_dtype", [torch.float16, torch.float32])
def test_deform_sample_matches_grid_sample(ref_dtype):
    """deform_attn.py:57-66 + :14-28 written with torch ops on the same fp16 inputs."""
    from sarbon_b200 import det_ops as ops
    g = gen(4)
    b, q, nh, nl, npt = 2, 300, 8, 3, 4
    shapes = [(48, 80), (24, 40), (12, 20)]
    s = sum(h * w for h, w in shapes)
    value = torch.randn(b, s, nh * 32, device="cuda", generator=g).half()
    offatt = (torch.randn(b, q, nh * nl * npt * 3, device="cuda", generator=g) * 2).half()
    off, att = offatt[..., :nh * nl * npt * 2], offatt[..., nh * nl * npt * 2:]
    ref_box = torch.rand(b, q, 4, device="cuda", generator=g).to(ref_dtype)
    out = ops.deform_sample(value, shapes, off, att, ref_box, nh, npt)
    # torch restatement (fp32 sampling of the fp16 values; locations in the box's type)
    o = off.reshape(b, q, nh, nl, npt, 2)
    w = att.reshape(b, q, nh, nl * npt).float().softmax(-1).view(b, q, nh, nl, npt)
    r = ref_box[:, :, None, None, None]
    loc = r[..., :2] + o / npt * r[..., 2:] * 0.5
    grids = 2 * loc - 1
    splits = value.float().split([h * ww for h, ww in shapes], 1)
    sampled = []
    for lvl, (h, ww) in enumerate(shapes):
        v = splits[lvl].view(b, h * ww, nh, 32).permute(0, 2, 3, 1).reshape(b * nh, 32, h, ww)
        gg = grids[:, :, :, lvl].permute(0, 2, 1, 3, 4).reshape(b * nh, q, npt, 2).float()
        sampled.append(F.grid_sample(v, gg, mode="bilinear", padding_mode="zeros", align_corners=False))
    st = torch.stack(sampled, -2).flatten(-2)
    ww_ = w.permute(0, 2, 1, 3, 4).reshape(b * nh, 1, q, nl * npt)
    ref = (st * ww_).sum(-1).view(b, nh * 32, q).transpose(1, 2)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-3 * ref.abs().max().item(), err


def test_box_heads():
    """box_enc / box_dec against sarbon_det.py:316-350 and box_ops.py:78-106 in torch fp16/fp32."""
    from sarbon_b200 import det_ops as ops
    g = gen(5)
    B, K, s, r1 = 2, 300, 5040, 33
    encbox = (torch.randn(B, K, 4, device="cuda", generator=g)).half()
    anchors = (torch.randn(s, 4, device="cuda", generator=g) * 2).half()
    idx = torch.randint(0, s, (B, K), device="cuda", generator=g, dtype=torch.int32)
    ref16 = torch.empty(B, K, 4, device="cuda", dtype=torch.float16)
    qin = torch.zeros(B, K, 64, device="cuda", dtype=torch.float16)
    ops.box_enc(encbox.view(B * K, 4), anchors, idx, ref16, qin.view(B * K, 64))
    exp = (encbox + anchors[idx.long()]).sigmoid()
    assert torch.equal(ref16, exp) and torch.equal(qin[..., :4], exp)
    project = torch.linspace(-8, 8, r1, device="cuda")
    head = torch.randn(B, K, 4 * r1, device="cuda", generator=g).half()
    prebox = torch.randn(B, K, 4, device="cuda", generator=g).half()
    corners = torch.empty(B, K, 4 * r1, device="cuda", dtype=torch.float16)
    ref_init = torch.empty(B, K, 4, device="cuda")
    box = torch.empty(B, K, 4, device="cuda")
    ops.box_dec(True, head, corners, project, 4.0, ref_init, box, prebox=prebox, ref16=ref16, qin=qin)
    x = ref16.clamp(1e-5, 1 - 1e-5)
    pre = (prebox + torch.log((x / (1 - x)).float())).sigmoid()
    assert (ref_init - pre).abs().max().item() < 1e-6
    assert torch.equal(corners, head)

    def integral(c):
        p = c.view(B, K, 4, r1).float().softmax(-1)
        return (p.half().float() @ project.half().float()).half()

    def d2b(points, dist):
        cx, cy, w, h = points.unbind(-1)
        sw, sh = w / 4.0, h / 4.0
        x0 = cx - (2.0 + dist[..., 0]).float() * sw
        y0 = cy - (2.0 + dist[..., 1]).float() * sh
        x1 = cx + (2.0 + dist[..., 2]).float() * sw
        y1 = cy + (2.0 + dist[..., 3]).float() * sh
        return torch.stack([(x0 + x1) / 2, (y0 + y1) / 2, x1 - x0, y1 - y0], -1)

    exp_box = d2b(ref_init, integral(corners))
    assert (box - exp_box).abs().max().item() < 1e-5
    head2 = torch.randn(B, K, 4 * r1, device="cuda", generator=g).half()
    exp_c = head2 + corners
    ops.box_dec(False, head2, corners, project, 4.0, ref_init, box, qin=qin)
    assert torch.equal(corners, exp_c)
    assert (box - d2b(ref_init, integral(corners))).abs().max().item() < 1e-5
    assert torch.equal(qin[..., :4], box.half())
