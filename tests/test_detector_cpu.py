"""Host-side pieces of B200Detector against the reference's own functions, on the CPU.

* BatchNorm folding (``_fold_conv_bn``) against conv -> BatchNorm of the reference's
  ``conv_bn_act`` modules (sarbon/models/block_local.py:24-28), fp32;
* the weight-matrix column order (tap = ky * 3 + kx, channel) against F.conv2d as an
  im2col product;
* ``anchors_of`` against ``SarbonDetector.anchors`` (sarbon_det.py:276-289) in fp16, and
  ``sincos_2d`` against the reference's ``sincos_2d`` (:109-115).
The reference package is the one installed under baseline/_ref (skipped when absent).
"""
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def sd():
    if not (REF / "sarbon").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    import sys
    sys.path.insert(0, str(REF))
    import sarbon.models.sarbon_det as m
    yield m
    sys.path.remove(str(REF))


def test_fold_conv_bn_matches_the_modules(sd):
    from sarbon.models.block_local import conv_bn_act

    from sarbon_b200.detector import _fold_conv_bn
    torch.manual_seed(0)
    m = conv_bn_act(64, 32, 2).eval()
    with torch.no_grad():
        bn = m[1]
        bn.running_mean.uniform_(-0.2, 0.2)
        bn.running_var.uniform_(0.5, 2.0)
        bn.weight.uniform_(0.5, 1.5)
        bn.bias.uniform_(-0.2, 0.2)
    x = torch.randn(2, 64, 17, 23)
    w, b = _fold_conv_bn(m[0], m[1])
    with torch.no_grad():
        ref = m[1](m[0](x))
    got = F.conv2d(x, w, b, stride=2, padding=1)
    assert (got - ref).abs().max().item() < 1e-4


def test_conv_matrix_column_order():
    from sarbon_b200.detector import _conv_mat
    torch.manual_seed(1)
    w = torch.randn(16, 8, 3, 3)
    x = torch.randn(1, 8, 6, 7)
    mat = _conv_mat(w).float()  # [16, 9 * 8], columns (tap, channel)
    pad = F.pad(x, (1, 1, 1, 1))
    cols = torch.stack([pad[0, :, ky:ky + 6, kx:kx + 7] for ky in range(3) for kx in range(3)])  # [9, 8, 6, 7]
    a = cols.permute(2, 3, 0, 1).reshape(42, 72)  # rows = pixels, columns (tap, channel)
    got = (a @ mat.t()).view(6, 7, 16).permute(2, 0, 1)
    ref = F.conv2d(x, w.half().float(), padding=1)[0]
    assert (got - ref).abs().max().item() < 1e-4


def test_anchors_and_positions(sd):
    from sarbon_b200.detector import anchors_of, sincos_2d
    shapes = [(48, 80), (24, 40), (12, 20)]
    ref_a, ref_v = sd.SarbonDetector.anchors(shapes, torch.device("cpu"), torch.float16)
    a, v = anchors_of(shapes, torch.device("cpu"))
    assert torch.equal(a, ref_a[0]) and torch.equal(v.bool(), ref_v[0, :, 0])
    assert torch.equal(sincos_2d(12, 20, 256, "cpu"), sd.sincos_2d(12, 20, 256, "cpu")[0])
