"""sb_gemm_conv (tcgen05 implicit GEMM of the detector) against torch in fp32.

The inputs are fp16 (as under the reference's autocast, sarbon/inference/video.py:116-118);
the reference result is torch's fp32 conv / linear of the same fp16 values, so the only
differences are the accumulation order and the output rounding.  Shapes: the detector's
(sarbon_det.py:118-356 at 384x640 and 1088x1920 frames: 3x3 convs with stride 1 and 2 on
256-channel maps, 1x1 convs over two concatenated maps, linear layers with N = 6 ... 1024),
plus ragged sizes (maps narrower than a tile, N not a multiple of 16, one row).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _close(got, ref, tol=2e-3):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= tol * scale + 1e-4, (err, scale)
    return err / max(scale, 1e-30)


def _act(x, act):
    return {None: x, "relu": F.relu(x), "gelu": F.gelu(x)}[act]


@pytest.mark.parametrize("m,k,n,act", [(300, 256, 256, None), (300, 256, 768, None), (300, 256, 1024, "relu"),
                                       (300, 1024, 256, None), (5040, 256, 288, None), (5040, 256, 256, None),
                                       (1, 256, 6, None), (37, 64, 132, "relu"), (240, 256, 1024, "gelu"),
                                       (4096, 512, 256, "relu"), (300, 64, 512, "relu")])
def test_linear(m, k, n, act):
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    x = torch.randn(m, k, device="cuda", generator=g).half()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).half()
    b = torch.randn(n, device="cuda", generator=g)
    ref = _act(x.float() @ w.float().t() + b, act)
    got = gemm_conv(x, w, b, act=act, out_dtype=torch.float32)
    assert got.shape == (m, n)
    _close(got, ref, 1e-4)
    got16 = gemm_conv(x, w, b, act=act)
    _close(got16, ref, 2e-3)


@pytest.mark.parametrize("res_dtype", [torch.float16, torch.float32])
def test_linear_residual_and_strided_views(res_dtype):
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(5)
    m, k, n = 300, 256, 256
    big = torch.randn(m, 768, device="cuda", generator=g).half()  # q|k|v rows: read the middle third
    x = big[:, 256:512]
    w = (torch.randn(n, k, device="cuda", generator=g) / 16).half()
    b = torch.randn(n, device="cuda", generator=g)
    res = torch.randn(m, n, device="cuda", generator=g).to(res_dtype)
    out = torch.zeros(m, 512, device="cuda", dtype=torch.float32)  # write the second half of wider rows
    gemm_conv(x, w, b, res=res, out=out[:, 256:], out_dtype=torch.float32)
    ref = x.float() @ w.float().t() + b + res.float()
    _close(out[:, 256:], ref, 1e-4)
    assert not out[:, :256].any()
    # fp16 rows of a wider matrix (bulk tensor stores with a row pitch of 512)
    out16 = torch.zeros(m, 512, device="cuda", dtype=torch.float16)
    gemm_conv(x, w, b, res=res, out=out16[:, :256])
    _close(out16[:, :256], ref, 2e-3)
    assert not out16[:, 256:].any()


@pytest.mark.parametrize("b,h,w,cin,cout,stride", [(2, 24, 40, 128, 256, 2), (2, 24, 40, 256, 256, 1),
                                                   (1, 12, 20, 256, 256, 1), (2, 48, 80, 256, 256, 2),
                                                   (1, 7, 13, 64, 64, 1), (1, 7, 13, 64, 128, 2),
                                                   (1, 68, 120, 128, 256, 2), (1, 34, 60, 256, 256, 1),
                                                   (3, 5, 3, 128, 32, 1)])
def test_conv3x3(b, h, w, cin, cout, stride):
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(h * w + cin + stride)
    x = torch.randn(b, cin, h, w, device="cuda", generator=g).half()
    wt = (torch.randn(cout, cin, 3, 3, device="cuda", generator=g) / (9 * cin) ** 0.5).half()
    bias = torch.randn(cout, device="cuda", generator=g)
    ref = F.relu(F.conv2d(x.float(), wt.float(), bias, stride=stride, padding=1)).permute(0, 2, 3, 1)
    x_nhwc = x.permute(0, 2, 3, 1).contiguous()
    w_mat = wt.permute(0, 2, 3, 1).reshape(cout, 9 * cin).contiguous()
    got = gemm_conv(x_nhwc, w_mat, bias, act="relu", taps=9, stride=stride, out_dtype=torch.float32)
    assert got.shape == ref.shape
    _close(got, ref, 1e-4)


def test_conv3x3_residual_into_strided_output():
    """The Res block's second conv: act(bn(conv(x)) + x), written into one level of a
    concatenated [B, S, C] memory (image stride S > H * W)."""
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(11)
    b, h, w, c = 2, 24, 40, 256
    s_tot, off = 3840 + h * w + 240, 3840
    x = torch.randn(b, h, w, c, device="cuda", generator=g).half()
    wt = (torch.randn(c, c, 3, 3, device="cuda", generator=g) / (9 * c) ** 0.5).half()
    bias = torch.randn(c, device="cuda", generator=g)
    mem = torch.zeros(b, s_tot, c, device="cuda", dtype=torch.float16)
    out = mem[:, off:off + h * w].view(b, h, w, c)
    gemm_conv(x, wt.permute(0, 2, 3, 1).reshape(c, 9 * c).contiguous(), bias, act="relu", taps=9, res=x, out=out)
    ref = F.relu(F.conv2d(x.permute(0, 3, 1, 2).float(), wt.float(), bias, padding=1) + x.permute(0, 3, 1, 2).float())
    _close(out, ref.permute(0, 2, 3, 1), 2e-3)
    assert not mem[:, :off].any() and not mem[:, off + h * w:].any()


def test_conv1x1_over_two_sources():
    """fuse(): 1x1 conv over torch.cat([a, b], 1) (sarbon_det.py:73-77), with the second
    source one level of a concatenated memory and the first a channel slice."""
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(13)
    b, h, w = 2, 48, 80
    wide = torch.randn(b, h, w, 384, device="cuda", generator=g).half()
    a = wide[..., 128:]
    mem = torch.randn(b, h * w + 960, 256, device="cuda", generator=g).half()
    bb = mem[:, :h * w].view(b, h, w, 256)
    wt = (torch.randn(256, 512, device="cuda", generator=g) / 512 ** 0.5).half()
    bias = torch.randn(256, device="cuda", generator=g)
    got = gemm_conv([a, bb], wt, bias, act="relu", out_dtype=torch.float32)
    cat = torch.cat([a, bb], -1).float()
    ref = F.relu(cat @ wt.float().t() + bias)
    _close(got, ref, 1e-4)


def test_rejects_bad_arguments():
    from sarbon_b200._lib import SarbonLibraryError
    from sarbon_b200.det_ops import gemm_conv
    x = torch.randn(10, 48, device="cuda").half()  # C not a multiple of 64
    w = torch.randn(16, 48, device="cuda").half()
    with pytest.raises(SarbonLibraryError):
        gemm_conv(x, w)
    x = torch.randn(2, 8, 8, 64, device="cuda").half()
    w = torch.randn(16, 64, device="cuda").half()
    with pytest.raises(SarbonLibraryError):
        gemm_conv(x, w, taps=1, stride=2)


def test_conv1x1_dense_maps_as_one_matrix():
    """1x1 convs over dense maps (two sources, B > 1) run as one [B*H*W, C] product."""
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(17)
    b, h, w = 3, 17, 23
    a = torch.randn(b, h, w, 128, device="cuda", generator=g).half()
    c = torch.randn(b, h, w, 256, device="cuda", generator=g).half()
    wt = (torch.randn(256, 384, device="cuda", generator=g) / 384 ** 0.5).half()
    bias = torch.randn(256, device="cuda", generator=g)
    got = gemm_conv([a, c], wt, bias, act="relu")
    ref = F.relu(torch.cat([a, c], -1).float() @ wt.float().t() + bias)
    assert got.shape == (b, h, w, 256)
    _close(got, ref, 2e-3)


@pytest.mark.parametrize("m,k,n", [(40000, 256, 256), (20000, 256, 1024), (30001, 128, 96)])
def test_linear_weights_resident(m, k, n):
    """Many tiles per CTA with K * BN <= 1024: every CTA keeps one N tile's weights resident
    and streams only A (grid a multiple of the N tiles)."""
    from sarbon_b200.det_ops import gemm_conv
    g = torch.Generator(device="cuda").manual_seed(m + n)
    x = torch.randn(m, k, device="cuda", generator=g).half()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).half()
    b = torch.randn(n, device="cuda", generator=g)
    res = torch.randn(m, n, device="cuda", generator=g).half()
    ref = F.relu(x.float() @ w.float().t() + b + res.float())
    got = gemm_conv(x, w, b, act="relu", res=res, out_dtype=torch.float32)
    _close(got, ref, 1e-4)
